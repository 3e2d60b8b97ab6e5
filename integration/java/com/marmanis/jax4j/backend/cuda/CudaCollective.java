package com.marmanis.jax4j.backend.cuda;

import java.lang.foreign.Arena;
import java.lang.foreign.MemorySegment;
import java.util.Arrays;
import java.util.concurrent.BrokenBarrierException;
import java.util.concurrent.CyclicBarrier;
import java.util.concurrent.TimeUnit;
import java.util.concurrent.TimeoutException;

import static java.lang.foreign.ValueLayout.ADDRESS;
import static java.lang.foreign.ValueLayout.JAVA_INT;

/**
 * The CUDA build's replacement for api/SharedCollective.java: the same two
 * operations (psum, allGather) indexed by PmapContext.deviceIndex, as NCCL
 * collectives over one communicator per shard (j4c_comm_init_all for the
 * in-process pmap, one shard thread per GPU; j4c_comm_init_rank for one
 * process per GPU).  api/Pmap.java builds it where it built a
 * SharedCollective (Pmap.java:79, 99, 121).
 *
 * Differences from SharedCollective, on purpose:
 *  - every wait is bounded: the barrier that checks the shards' sizes has a
 *    timeout (SharedCollective's CyclicBarrier.await has none,
 *    SharedCollective.java:78-85), and the communicators carry a deadline
 *    after which a collective fails with J4C_E_TIMEOUT instead of hanging;
 *  - shards that deposit different sizes all fail with an exception before
 *    any device work is enqueued (SharedCollective.psum indexes every
 *    deposit with the caller's length, SharedCollective.java:44-54, so a
 *    shorter deposit throws on one shard and strands the others);
 *  - a shard that fails aborts the barrier and the communicators, so its
 *    peers fail at once.
 */
public final class CudaCollective {
    private final int numDevices;
    private final MemorySegment[] comms;   // one j4c_comm per shard (deviceIndex)
    private final int[] ordinals;          // CUDA device of each shard
    private final long[] deposited;
    private final CyclicBarrier barrier;
    private final long timeoutMs;

    /** One shard per GPU in this process (the reference's in-process pmap). */
    public CudaCollective(int[] deviceOrdinals, long timeoutMs) {
        this.numDevices = deviceOrdinals.length;
        this.ordinals = deviceOrdinals.clone();
        this.comms = new MemorySegment[numDevices];
        this.deposited = new long[numDevices];
        this.barrier = new CyclicBarrier(numDevices);
        this.timeoutMs = timeoutMs;
        try (Arena a = Arena.ofConfined()) {
            MemorySegment devs = a.allocateFrom(JAVA_INT, deviceOrdinals);
            MemorySegment out = a.allocate(ADDRESS, numDevices);
            J4C.check((int) J4C.COMM_INIT_ALL.invokeExact(devs, numDevices, timeoutMs, out), "j4c_comm_init_all");
            for (int i = 0; i < numDevices; i++) comms[i] = out.getAtIndex(ADDRESS, i);
        } catch (RuntimeException | Error e) {
            throw e;
        } catch (Throwable t) {
            throw new IllegalStateException(t);
        }
    }

    /**
     * One process per GPU: this process's rank of an nranks-wide group whose
     * id (j4c_comm_unique_id on rank 0) reached every rank out of band.  The
     * in-process size check does not apply (each process holds one shard);
     * the launcher checks sizes across processes before the first step.
     */
    public static CudaCollective forRank(byte[] uniqueId, int nranks, int rank, int device, long timeoutMs) {
        return new CudaCollective(uniqueId, nranks, rank, device, timeoutMs);
    }

    private CudaCollective(byte[] uniqueId, int nranks, int rank, int device, long timeoutMs) {
        this.numDevices = nranks;
        this.ordinals = new int[nranks];
        Arrays.fill(this.ordinals, device);
        this.comms = new MemorySegment[nranks];
        this.deposited = null;
        this.barrier = null;
        this.timeoutMs = timeoutMs;
        try (Arena a = Arena.ofConfined()) {
            MemorySegment id = a.allocate(uniqueId.length);
            id.copyFrom(MemorySegment.ofArray(uniqueId));
            MemorySegment out = a.allocate(ADDRESS);
            J4C.check((int) J4C.COMM_INIT_RANK.invokeExact(id, (long) uniqueId.length, nranks, rank, device,
                                                          timeoutMs, out), "j4c_comm_init_rank");
            Arrays.fill(comms, out.get(ADDRESS, 0));  // every index resolves to this rank's communicator
        } catch (RuntimeException | Error e) {
            throw e;
        } catch (Throwable t) {
            throw new IllegalStateException(t);
        }
    }

    /** In-process shards: all deposit their sizes, then each checks them. */
    private void checkSizes(String op, int deviceIndex, long count) {
        if (barrier == null) return;
        deposited[deviceIndex] = count;
        await();
        for (int d = 0; d < numDevices; d++)
            if (deposited[d] != count)
                throw new RuntimeException(op + ": shards deposited different sizes " + Arrays.toString(deposited));
        await();  // every shard has read the sizes before any deposits the next ones
    }

    private void await() {
        try {
            barrier.await(timeoutMs, TimeUnit.MILLISECONDS);
        } catch (InterruptedException e) {
            Thread.currentThread().interrupt();
            abort();
            throw new RuntimeException("Collective barrier interrupted", e);
        } catch (BrokenBarrierException | TimeoutException e) {
            abort();
            throw new RuntimeException("Collective barrier broken: a shard failed or timed out", e);
        }
    }

    /** All-reduce sum of a device-resident shard (Lax.psum, api/Lax.java:184-186). */
    public DeviceStorage psum(int deviceIndex, DeviceStorage x) {
        checkSizes("psum", deviceIndex, x.count());
        DeviceStorage out = DeviceStorage.allocate(x.count(), x.dtype(), x.device());
        try {
            J4C.check((int) J4C.PSUM.invokeExact(comms[deviceIndex], x.dtype().ordinal(), x.ptr(), out.ptr(),
                                                x.count(), MemorySegment.NULL), "j4c_psum");
        } catch (RuntimeException | Error e) {
            throw e;
        } catch (Throwable t) {
            throw new IllegalStateException(t);
        }
        return out;
    }

    /** SharedCollective.psum's signature: host arrays in and out. */
    public float[] psum(int deviceIndex, float[] data) {
        return psum(deviceIndex, DeviceStorage.of(data, ordinals[deviceIndex])).toFloatArray();
    }

    /** The shards stacked as [numDevices, *shard] on every shard (Lax.allGather, api/Lax.java:211-216). */
    public DeviceStorage allGather(int deviceIndex, DeviceStorage shard) {
        checkSizes("allGather", deviceIndex, shard.count());
        DeviceStorage out = DeviceStorage.allocate(numDevices * shard.count(), shard.dtype(), shard.device());
        try {
            J4C.check((int) J4C.ALL_GATHER.invokeExact(comms[deviceIndex], shard.dtype().ordinal(), shard.ptr(),
                                                      out.ptr(), shard.count(), MemorySegment.NULL), "j4c_all_gather");
        } catch (RuntimeException | Error e) {
            throw e;
        } catch (Throwable t) {
            throw new IllegalStateException(t);
        }
        return out;
    }

    public int numDevices() {
        return numDevices;
    }

    /** Ends every collective waiting on a peer; the communicators are unusable afterwards. */
    public void abort() {
        if (barrier != null) barrier.reset();
        for (MemorySegment c : comms) {
            try {
                int ignored = (int) J4C.COMM_ABORT.invokeExact(c);
            } catch (Throwable ignored) {
                // already aborted
            }
        }
    }

    /** Releases the communicators after the pmap call. */
    public void close() {
        MemorySegment last = null;
        for (MemorySegment c : comms) {
            if (c.equals(last)) continue;  // one process per GPU: one communicator behind every index
            last = c;
            try {
                J4C.check((int) J4C.COMM_DESTROY.invokeExact(c), "j4c_comm_destroy");
            } catch (RuntimeException | Error e) {
                throw e;
            } catch (Throwable t) {
                throw new IllegalStateException(t);
            }
        }
    }

    /**
     * Shards sharing one GPU (the reference's synthetic devices): the sum of
     * the deposits in slot order 0..D-1 on the device (j4c_psum_slots),
     * bit-identical to SharedCollective.psum's host loop.
     */
    public static DeviceStorage psumSlots(DeviceStorage[] slots) {
        DeviceStorage first = slots[0];
        for (DeviceStorage s : slots)
            if (s.count() != first.count() || s.dtype() != first.dtype())
                throw new RuntimeException("psum: shards deposited different sizes or dtypes");
        DeviceStorage out = DeviceStorage.allocate(first.count(), first.dtype(), first.device());
        try (Arena a = Arena.ofConfined()) {
            MemorySegment ptrs = a.allocate(ADDRESS, slots.length);
            for (int i = 0; i < slots.length; i++) ptrs.setAtIndex(ADDRESS, i, slots[i].ptr());
            J4C.check((int) J4C.PSUM_SLOTS.invokeExact(first.dtype().ordinal(), ptrs, slots.length, out.ptr(),
                                                      first.count(), MemorySegment.NULL), "j4c_psum_slots");
        } catch (RuntimeException | Error e) {
            throw e;
        } catch (Throwable t) {
            throw new IllegalStateException(t);
        }
        return out;
    }
}
