package com.marmanis.jax4j.backend.cuda;

import com.marmanis.jax4j.core.DType;

import java.lang.foreign.Arena;
import java.lang.foreign.MemorySegment;
import java.lang.ref.Cleaner;
import java.util.concurrent.ConcurrentHashMap;

import static java.lang.foreign.ValueLayout.ADDRESS;
import static java.lang.foreign.ValueLayout.JAVA_DOUBLE;
import static java.lang.foreign.ValueLayout.JAVA_FLOAT;
import static java.lang.foreign.ValueLayout.JAVA_INT;
import static java.lang.foreign.ValueLayout.JAVA_LONG;

/**
 * Device-resident storage of a ConcreteNDArray: the CUDA build's replacement
 * for the reference's host records F32Storage(float[]) / F64Storage(double[])
 * / I32Storage / I64Storage / BoolStorage (core/ConcreteNDArray.java:47-88).
 * The buffer belongs to the record and is released by a Cleaner when the
 * array is unreachable (j4c_free on the device's stream).  Arrays are
 * immutable, so the record is too; the host copy is made on demand
 * (toFloatArray / toDoubleArray), never kept.
 *
 * A FLOAT32 array that takes part in dot products may also hold its splits
 * (opaque device buffers of j4c_split_floats(rows, cols) floats each, one
 * pair per split kind) and its line maxima (rows + cols + 1 words from the
 * GEMM epilogue that produced it); both live and die with the storage.
 */
public record DeviceStorage(MemorySegment ptr, long count, DType dtype, int device, Extras extras) {
    private static final Cleaner CLEANER = Cleaner.create();

    /** Per-array device buffers derived from the data (splits, line maxima). */
    public static final class Extras {
        final ConcurrentHashMap<String, MemorySegment[]> splits = new ConcurrentHashMap<>();
        volatile MemorySegment lines;   // rows + cols + 1 uint32 words, or null
    }

    public static int elementBytes(DType dtype) {
        return switch (dtype) {
            case FLOAT32, INT32 -> 4;
            case FLOAT64, INT64 -> 8;
            case BOOL -> 1;
        };
    }

    public long bytes() {
        return count * elementBytes(dtype);
    }

    /** A new uninitialised device array of `count` elements on `device`. */
    public static DeviceStorage allocate(long count, DType dtype, int device) {
        MemorySegment p = malloc(Math.max(1, count * elementBytes(dtype)), device);
        Extras extras = new Extras();
        DeviceStorage s = new DeviceStorage(p, count, dtype, device, extras);
        long addr = p.address();
        CLEANER.register(s, () -> release(addr, device, extras));
        return s;
    }

    private static MemorySegment malloc(long bytes, int device) {
        try (Arena a = Arena.ofConfined()) {
            J4C.check((int) J4C.SET_DEVICE.invokeExact(device), "j4c_set_device");
            MemorySegment out = a.allocate(ADDRESS);
            J4C.check((int) J4C.MALLOC.invokeExact(bytes, out, MemorySegment.NULL), "j4c_malloc");
            return out.get(ADDRESS, 0).reinterpret(bytes);
        } catch (RuntimeException | Error e) {
            throw e;
        } catch (Throwable t) {
            throw new IllegalStateException(t);
        }
    }

    private static void release(long addr, int device, Extras extras) {
        try {
            J4C.check((int) J4C.SET_DEVICE.invokeExact(device), "j4c_set_device");
            for (MemorySegment[] pair : extras.splits.values())
                for (MemorySegment m : pair) J4C.check((int) J4C.FREE.invokeExact(m, MemorySegment.NULL), "j4c_free");
            if (extras.lines != null)
                J4C.check((int) J4C.FREE.invokeExact(extras.lines, MemorySegment.NULL), "j4c_free");
            J4C.check((int) J4C.FREE.invokeExact(MemorySegment.ofAddress(addr), MemorySegment.NULL), "j4c_free");
        } catch (Throwable ignored) {
            // a Cleaner action must not throw; the pool reclaims the memory at exit
        }
    }

    public static DeviceStorage of(float[] data, int device) {
        DeviceStorage s = allocate(data.length, DType.FLOAT32, device);
        s.upload(MemorySegment.ofArray(data));
        return s;
    }

    public static DeviceStorage of(double[] data, int device) {
        DeviceStorage s = allocate(data.length, DType.FLOAT64, device);
        s.upload(MemorySegment.ofArray(data));
        return s;
    }

    private void upload(MemorySegment heap) {
        try (Arena a = Arena.ofConfined()) {
            // FFM downcalls take native segments: stage the heap array once
            MemorySegment staging = a.allocate(bytes(), 16);
            staging.copyFrom(heap);
            J4C.check((int) J4C.MEMCPY_H2D.invokeExact(ptr, staging, bytes(), MemorySegment.NULL), "j4c_memcpy_h2d");
            J4C.check((int) J4C.STREAM_SYNCHRONIZE.invokeExact(MemorySegment.NULL), "j4c_stream_synchronize");
        } catch (RuntimeException | Error e) {
            throw e;
        } catch (Throwable t) {
            throw new IllegalStateException(t);
        }
    }

    private MemorySegment download(Arena a) {
        try {
            MemorySegment host = a.allocate(bytes(), 16);
            J4C.check((int) J4C.MEMCPY_D2H.invokeExact(host, ptr, bytes(), MemorySegment.NULL), "j4c_memcpy_d2h");
            J4C.check((int) J4C.STREAM_SYNCHRONIZE.invokeExact(MemorySegment.NULL), "j4c_stream_synchronize");
            return host;
        } catch (RuntimeException | Error e) {
            throw e;
        } catch (Throwable t) {
            throw new IllegalStateException(t);
        }
    }

    public float[] toFloatArray() {
        if (dtype != DType.FLOAT32) throw new IllegalStateException("storage is " + dtype + ", not FLOAT32");
        try (Arena a = Arena.ofConfined()) {
            return download(a).toArray(JAVA_FLOAT);
        }
    }

    public double[] toDoubleArray() {
        if (dtype != DType.FLOAT64) throw new IllegalStateException("storage is " + dtype + ", not FLOAT64");
        try (Arena a = Arena.ofConfined()) {
            return download(a).toArray(JAVA_DOUBLE);
        }
    }

    public int[] toIntArray() {
        if (dtype != DType.INT32) throw new IllegalStateException("storage is " + dtype + ", not INT32");
        try (Arena a = Arena.ofConfined()) {
            return download(a).toArray(JAVA_INT);
        }
    }

    public long[] toLongArray() {
        if (dtype != DType.INT64) throw new IllegalStateException("storage is " + dtype + ", not INT64");
        try (Arena a = Arena.ofConfined()) {
            return download(a).toArray(JAVA_LONG);
        }
    }

    /**
     * The split of kind `kind` ("r": one scale per row, "c": per column,
     * "t": transposed) of this [rows, cols] FLOAT32 array, made on first use
     * with j4c_split_f32 / j4c_split_f32_cols / j4c_split_f32_transposed.
     */
    public MemorySegment[] split(String kind, long rows, long cols) {
        return extras.splits.computeIfAbsent(kind, k -> {
            try {
                long r = k.equals("t") ? cols : rows, c = k.equals("t") ? rows : cols;
                long floats = (long) J4C.SPLIT_FLOATS.invokeExact(r, c);
                MemorySegment hi = malloc(4 * floats, device), lo = malloc(4 * floats, device);
                int rc = switch (k) {
                    case "r" -> (int) J4C.SPLIT_F32.invokeExact(ptr, rows, cols, hi, lo, MemorySegment.NULL);
                    case "c" -> (int) J4C.SPLIT_F32_COLS.invokeExact(ptr, rows, cols, hi, lo, MemorySegment.NULL);
                    case "t" -> (int) J4C.SPLIT_F32_TRANSPOSED.invokeExact(ptr, rows, cols, hi, lo, MemorySegment.NULL);
                    default -> throw new IllegalArgumentException("split kind " + k);
                };
                J4C.check(rc, "j4c_split_f32 (" + k + ")");
                return new MemorySegment[]{hi, lo};
            } catch (RuntimeException | Error e) {
                throw e;
            } catch (Throwable t) {
                throw new IllegalStateException(t);
            }
        });
    }
}
