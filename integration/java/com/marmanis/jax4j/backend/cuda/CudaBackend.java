package com.marmanis.jax4j.backend.cuda;

import com.marmanis.jax4j.backend.ExecutionBackend;
import com.marmanis.jax4j.core.DType;
import com.marmanis.jax4j.core.Device;
import com.marmanis.jax4j.ir.Primitive;

import java.lang.foreign.Arena;
import java.lang.foreign.MemorySegment;
import java.util.IdentityHashMap;
import java.util.List;
import java.util.Map;

import static java.lang.foreign.ValueLayout.JAVA_LONG;

/**
 * ExecutionBackend on libjax4j_cuda.so: the replacement for
 * backend/TornadoVMBackend.java.  Every method of the interface
 * (backend/ExecutionBackend.java:11-56) runs on the GPU, the FLOAT64
 * overloads included (the interface's defaults send those to HostBackend;
 * here they run the library's FP64 kernels, which keep the reference's
 * double arithmetic).  The float[] / double[] signatures stay for API
 * compatibility and copy through the device; a ConcreteNDArray backed by a
 * DeviceStorage calls the storage overloads and never leaves the GPU.
 *
 * Results equal the reference's: elementwise ops, comparisons and casts bit
 * for bit; tanh/sigmoid/exp/log/sin/cos within 1e-5 relative; reductions and
 * dot within 1e-4 relative of its sequential FP32 sums (a dot with a NaN or
 * an infinity in an operand is the sequential sum bit for bit).
 */
public final class CudaBackend implements ExecutionBackend {
    public static final CudaBackend INSTANCE = new CudaBackend();

    private final Map<Device, Integer> ordinals = new IdentityHashMap<>();

    private CudaBackend() {
        J4C.requireAbi();
        List<Device> devices = Device.getDevices();
        for (int i = 0; i < devices.size(); i++) ordinals.put(devices.get(i), i);
    }

    /** The CUDA ordinal of a reference Device (discovery order). */
    public int ordinal(Device device) {
        Integer i = ordinals.get(device);
        if (i == null) throw new IllegalArgumentException("not a CUDA device: " + device.getName());
        return i;
    }

    // ---------------------------------------------------------------- float[]
    @Override
    public float[] binary(Primitive primitive, float[] a, float[] b, Device device) {
        if (a.length != b.length)
            throw new IllegalArgumentException("binary: lengths " + a.length + " and " + b.length + " differ");
        int dev = ordinal(device);
        return binary(primitive, DeviceStorage.of(a, dev), DeviceStorage.of(b, dev)).toFloatArray();
    }

    @Override
    public float[] unary(Primitive primitive, float[] a, Device device) {
        return unary(primitive, DeviceStorage.of(a, ordinal(device))).toFloatArray();
    }

    @Override
    public float[] matmul(float[] a, float[] b, int m, int k, int n, Device device) {
        int dev = ordinal(device);
        return matmul(DeviceStorage.of(a, dev), DeviceStorage.of(b, dev), m, k, n).toFloatArray();
    }

    @Override
    public float[] reduce(Primitive primitive, float[] a, Device device) {
        return reduce(primitive, DeviceStorage.of(a, ordinal(device))).toFloatArray();
    }

    // --------------------------------------------------------------- double[]
    @Override
    public double[] reduce(Primitive primitive, double[] a, Device device) {
        return reduce(primitive, DeviceStorage.of(a, ordinal(device))).toDoubleArray();
    }

    @Override
    public double[] binary(Primitive primitive, double[] a, double[] b, Device device) {
        if (a.length != b.length)
            throw new IllegalArgumentException("binary: lengths " + a.length + " and " + b.length + " differ");
        int dev = ordinal(device);
        return binary(primitive, DeviceStorage.of(a, dev), DeviceStorage.of(b, dev)).toDoubleArray();
    }

    @Override
    public double[] unary(Primitive primitive, double[] a, Device device) {
        return unary(primitive, DeviceStorage.of(a, ordinal(device))).toDoubleArray();
    }

    @Override
    public double[] matmul(double[] a, double[] b, int m, int k, int n, Device device) {
        int dev = ordinal(device);
        return matmul(DeviceStorage.of(a, dev), DeviceStorage.of(b, dev), m, k, n).toDoubleArray();
    }

    // ------------------------------------------------ device-resident storage
    /** a (op) b over equal-length arrays of the same dtype (FLOAT32 or FLOAT64). */
    public DeviceStorage binary(Primitive primitive, DeviceStorage a, DeviceStorage b) {
        DeviceStorage out = DeviceStorage.allocate(a.count(), a.dtype(), a.device());
        try (Arena arena = Arena.ofConfined()) {
            MemorySegment dims = arena.allocateFrom(JAVA_LONG, a.count());
            J4C.check((int) J4C.BINARY.invokeExact(primitive.ordinal(), a.dtype().ordinal(), a.ptr(), dims, 1,
                                                  b.ptr(), dims, 1, out.ptr(), MemorySegment.NULL), "j4c_binary");
        } catch (RuntimeException | Error e) {
            throw e;
        } catch (Throwable t) {
            throw new IllegalStateException(t);
        }
        return out;
    }

    public DeviceStorage unary(Primitive primitive, DeviceStorage a) {
        DeviceStorage out = DeviceStorage.allocate(a.count(), a.dtype(), a.device());
        try {
            J4C.check((int) J4C.UNARY.invokeExact(primitive.ordinal(), a.dtype().ordinal(), a.ptr(), a.count(),
                                                 out.ptr(), MemorySegment.NULL), "j4c_unary");
        } catch (RuntimeException | Error e) {
            throw e;
        } catch (Throwable t) {
            throw new IllegalStateException(t);
        }
        return out;
    }

    /** SUM or MEAN of every element, as a one-element array (HostBackend.reduce). */
    public DeviceStorage reduce(Primitive primitive, DeviceStorage a) {
        if (primitive != Primitive.SUM && primitive != Primitive.MEAN)
            throw new IllegalArgumentException("reduce: " + primitive + " is not SUM or MEAN");
        DeviceStorage out = DeviceStorage.allocate(1, a.dtype(), a.device());
        try {
            J4C.check((int) J4C.REDUCE_ALL.invokeExact(primitive.ordinal(), a.dtype().ordinal(), a.ptr(), a.count(),
                                                      out.ptr(), MemorySegment.NULL), "j4c_reduce_all");
        } catch (RuntimeException | Error e) {
            throw e;
        } catch (Throwable t) {
            throw new IllegalStateException(t);
        }
        return out;
    }

    /**
     * (m x k) @ (k x n), row-major.  FLOAT32 goes through the tensor-core
     * split GEMM with each operand's split cached on its storage (A row
     * lines, B transposed: both read K-major); FLOAT64 through j4c_dot.
     */
    public DeviceStorage matmul(DeviceStorage a, DeviceStorage b, int m, int k, int n) {
        if (a.count() != (long) m * k || b.count() != (long) k * n)
            throw new IllegalArgumentException("matmul: operand sizes do not match " + m + "x" + k + " . " + k + "x" + n);
        DeviceStorage c = DeviceStorage.allocate((long) m * n, a.dtype(), a.device());
        try {
            if (a.dtype() == DType.FLOAT32) {
                MemorySegment[] sa = a.split("r", m, k);
                MemorySegment[] sb = b.split("t", k, n);  // B^T's rows: N lines, K-major
                J4C.check((int) J4C.DOT_SPLIT.invokeExact(sa[0], sa[1], sb[0], sb[1], c.ptr(), (long) m, (long) k,
                                                         (long) n, 0, 1, MemorySegment.NULL), "j4c_dot_split");
            } else {
                J4C.check((int) J4C.DOT.invokeExact(a.dtype().ordinal(), a.ptr(), b.ptr(), c.ptr(), (long) m,
                                                   (long) k, (long) n, 0, 0, MemorySegment.NULL), "j4c_dot");
            }
        } catch (RuntimeException | Error e) {
            throw e;
        } catch (Throwable t) {
            throw new IllegalStateException(t);
        }
        return c;
    }
}
