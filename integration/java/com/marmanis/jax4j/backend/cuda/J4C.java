package com.marmanis.jax4j.backend.cuda;

import java.lang.foreign.Arena;
import java.lang.foreign.FunctionDescriptor;
import java.lang.foreign.Linker;
import java.lang.foreign.MemorySegment;
import java.lang.foreign.SymbolLookup;
import java.lang.invoke.MethodHandle;

import static java.lang.foreign.ValueLayout.ADDRESS;
import static java.lang.foreign.ValueLayout.JAVA_DOUBLE;
import static java.lang.foreign.ValueLayout.JAVA_FLOAT;
import static java.lang.foreign.ValueLayout.JAVA_INT;
import static java.lang.foreign.ValueLayout.JAVA_LONG;

/**
 * Downcall handles for every entry point of libjax4j_cuda.so
 * (include/jax4j_cuda.h), through the Foreign Function & Memory API.  C
 * int / int32_t / uint32_t map to JAVA_INT, int64_t / uint64_t / size_t to
 * JAVA_LONG, double / float to JAVA_DOUBLE / JAVA_FLOAT, and every pointer
 * (streams and communicators included) to ADDRESS.  Primitive and DType
 * ordinals are passed unchanged: the library's J4C_* constants are those
 * ordinals.
 */
public final class J4C {
    private J4C() {}

    public static final int ABI_VERSION_EXPECTED = 2;
    public static final int OK = 0, E_INVALID = 1, E_UNSUPPORTED = 2, E_CUDA = 3, E_OOM = 4, E_NCCL = 5,
            E_TIMEOUT = 6, E_DEVICE = 7;
    public static final int FLOAT32 = 0, FLOAT64 = 1, INT32 = 2, INT64 = 3, BOOL = 4;

    private static final Linker LINKER = Linker.nativeLinker();
    private static final SymbolLookup LIB =
            SymbolLookup.libraryLookup(System.getProperty("jax4j.cuda.library", "libjax4j_cuda.so"), Arena.global());

    private static MethodHandle h(String name, FunctionDescriptor fd) {
        return LINKER.downcallHandle(LIB.find(name).orElseThrow(
                () -> new UnsatisfiedLinkError("libjax4j_cuda.so does not export " + name)), fd);
    }

    // ---- library and errors (runtime.cu) ----
    static final MethodHandle ABI_VERSION = h("j4c_abi_version", FunctionDescriptor.of(JAVA_INT));
    static final MethodHandle KERNEL_LAUNCHES = h("j4c_kernel_launches", FunctionDescriptor.of(JAVA_INT, ADDRESS));
    static final MethodHandle LAST_ERROR = h("j4c_last_error", FunctionDescriptor.of(ADDRESS));
    static final MethodHandle DEVICE_COUNT = h("j4c_device_count", FunctionDescriptor.of(JAVA_INT, ADDRESS));
    static final MethodHandle SET_DEVICE = h("j4c_set_device", FunctionDescriptor.of(JAVA_INT, JAVA_INT));
    static final MethodHandle GET_DEVICE = h("j4c_get_device", FunctionDescriptor.of(JAVA_INT, ADDRESS));
    static final MethodHandle ENABLE_PEER_ACCESS = h("j4c_enable_peer_access", FunctionDescriptor.of(
        JAVA_INT, JAVA_INT, JAVA_INT));
    static final MethodHandle STREAM_SYNCHRONIZE = h("j4c_stream_synchronize", FunctionDescriptor.of(
        JAVA_INT, ADDRESS));
    static final MethodHandle STREAM_CREATE = h("j4c_stream_create", FunctionDescriptor.of(JAVA_INT, ADDRESS));
    static final MethodHandle STREAM_DESTROY = h("j4c_stream_destroy", FunctionDescriptor.of(JAVA_INT, ADDRESS));
    static final MethodHandle DEVICE_STATUS = h("j4c_device_status", FunctionDescriptor.of(JAVA_INT, ADDRESS));
    static final MethodHandle SET_WAIT_LIMIT_NS = h("j4c_set_wait_limit_ns", FunctionDescriptor.of(
        JAVA_INT, JAVA_LONG, ADDRESS));

    // ---- memory: DeviceStorage (replaces F32Storage(float[]), core/ConcreteNDArray.java) ----
    static final MethodHandle MALLOC = h("j4c_malloc", FunctionDescriptor.of(
        JAVA_INT, JAVA_LONG, ADDRESS, ADDRESS));
    static final MethodHandle FREE = h("j4c_free", FunctionDescriptor.of(JAVA_INT, ADDRESS, ADDRESS));
    static final MethodHandle MEMCPY_H2D = h("j4c_memcpy_h2d", FunctionDescriptor.of(
        JAVA_INT, ADDRESS, ADDRESS, JAVA_LONG, ADDRESS));
    static final MethodHandle MEMCPY_D2H = h("j4c_memcpy_d2h", FunctionDescriptor.of(
        JAVA_INT, ADDRESS, ADDRESS, JAVA_LONG, ADDRESS));
    static final MethodHandle MEMCPY_D2D = h("j4c_memcpy_d2d", FunctionDescriptor.of(
        JAVA_INT, ADDRESS, ADDRESS, JAVA_LONG, ADDRESS));
    static final MethodHandle FILL = h("j4c_fill", FunctionDescriptor.of(
        JAVA_INT, JAVA_INT, ADDRESS, JAVA_LONG, JAVA_DOUBLE, ADDRESS));

    // ---- elementwise, casts, reductions (ConcreteNDArray.elementwise/compareElementwise/unary/astype/reduce*/argReduceAxis) ----
    static final MethodHandle BINARY = h("j4c_binary", FunctionDescriptor.of(
        JAVA_INT, JAVA_INT, JAVA_INT, ADDRESS, ADDRESS, JAVA_INT, ADDRESS, ADDRESS, JAVA_INT, ADDRESS, ADDRESS));
    static final MethodHandle COMPARE = h("j4c_compare", FunctionDescriptor.of(
        JAVA_INT, JAVA_INT, JAVA_INT, ADDRESS, ADDRESS, JAVA_INT, ADDRESS, ADDRESS, JAVA_INT, ADDRESS, ADDRESS));
    static final MethodHandle UNARY = h("j4c_unary", FunctionDescriptor.of(
        JAVA_INT, JAVA_INT, JAVA_INT, ADDRESS, JAVA_LONG, ADDRESS, ADDRESS));
    static final MethodHandle CAST = h("j4c_cast", FunctionDescriptor.of(
        JAVA_INT, JAVA_INT, JAVA_INT, ADDRESS, JAVA_LONG, ADDRESS, ADDRESS));
    static final MethodHandle REDUCE_ALL = h("j4c_reduce_all", FunctionDescriptor.of(
        JAVA_INT, JAVA_INT, JAVA_INT, ADDRESS, JAVA_LONG, ADDRESS, ADDRESS));
    static final MethodHandle REDUCE_AXIS = h("j4c_reduce_axis", FunctionDescriptor.of(
        JAVA_INT, JAVA_INT, JAVA_INT, ADDRESS, JAVA_LONG, JAVA_LONG, JAVA_LONG, ADDRESS, ADDRESS));
    static final MethodHandle REDUCE_AXIS_NOALLOC = h("j4c_reduce_axis_noalloc", FunctionDescriptor.of(
        JAVA_INT, JAVA_INT, JAVA_INT, ADDRESS, JAVA_LONG, JAVA_LONG, JAVA_LONG, ADDRESS, ADDRESS));
    static final MethodHandle ARGREDUCE = h("j4c_argreduce", FunctionDescriptor.of(
        JAVA_INT, JAVA_INT, JAVA_INT, ADDRESS, JAVA_LONG, JAVA_LONG, JAVA_LONG, ADDRESS, ADDRESS));

    // ---- Grad helpers and Numpy.take (api/Grad.java, api/Numpy.java) ----
    static final MethodHandle BROADCAST_LIKE = h("j4c_broadcast_like", FunctionDescriptor.of(
        JAVA_INT, JAVA_INT, ADDRESS, ADDRESS, JAVA_INT, ADDRESS, ADDRESS, JAVA_INT, ADDRESS));
    static final MethodHandle RELU_GRAD = h("j4c_relu_grad", FunctionDescriptor.of(
        JAVA_INT, JAVA_INT, ADDRESS, ADDRESS, JAVA_LONG, ADDRESS, ADDRESS));
    static final MethodHandle MAXMIN_GRAD = h("j4c_maxmin_grad", FunctionDescriptor.of(
        JAVA_INT, JAVA_INT, JAVA_INT, ADDRESS, ADDRESS, JAVA_INT, ADDRESS, ADDRESS, JAVA_INT, ADDRESS, ADDRESS,
        JAVA_INT, ADDRESS, ADDRESS, ADDRESS));
    static final MethodHandle TRANSPOSE = h("j4c_transpose", FunctionDescriptor.of(
        JAVA_INT, JAVA_INT, ADDRESS, JAVA_LONG, JAVA_LONG, ADDRESS, ADDRESS));
    static final MethodHandle GATHER_ROWS = h("j4c_gather_rows", FunctionDescriptor.of(
        JAVA_INT, JAVA_INT, ADDRESS, JAVA_LONG, JAVA_LONG, JAVA_INT, ADDRESS, JAVA_LONG, ADDRESS, ADDRESS));
    static final MethodHandle SCATTER_ADD_ROWS = h("j4c_scatter_add_rows", FunctionDescriptor.of(
        JAVA_INT, JAVA_INT, ADDRESS, JAVA_LONG, JAVA_LONG, JAVA_INT, ADDRESS, JAVA_LONG, ADDRESS, ADDRESS));

    // ---- dot (ConcreteNDArray.dot, core/ConcreteNDArray.java:452-459) and its splits ----
    static final MethodHandle DOT = h("j4c_dot", FunctionDescriptor.of(
        JAVA_INT, JAVA_INT, ADDRESS, ADDRESS, ADDRESS, JAVA_LONG, JAVA_LONG, JAVA_LONG, JAVA_INT, JAVA_INT,
        ADDRESS));
    static final MethodHandle DOT_WS = h("j4c_dot_ws", FunctionDescriptor.of(
        JAVA_INT, JAVA_INT, ADDRESS, ADDRESS, ADDRESS, JAVA_LONG, JAVA_LONG, JAVA_LONG, JAVA_INT, JAVA_INT,
        ADDRESS, JAVA_LONG, ADDRESS));
    static final MethodHandle DOT_WORKSPACE_SIZE = h("j4c_dot_workspace_size", FunctionDescriptor.of(
        JAVA_LONG, JAVA_INT, JAVA_LONG, JAVA_LONG, JAVA_LONG));
    static final MethodHandle DOT_SPLIT_KIND = h("j4c_dot_split_kind", FunctionDescriptor.of(JAVA_INT));
    static final MethodHandle SPLIT_PITCH = h("j4c_split_pitch", FunctionDescriptor.of(JAVA_LONG, JAVA_LONG));
    static final MethodHandle SPLIT_FLOATS = h("j4c_split_floats", FunctionDescriptor.of(
        JAVA_LONG, JAVA_LONG, JAVA_LONG));
    static final MethodHandle SPLIT_F32 = h("j4c_split_f32", FunctionDescriptor.of(
        JAVA_INT, ADDRESS, JAVA_LONG, JAVA_LONG, ADDRESS, ADDRESS, ADDRESS));
    static final MethodHandle SPLIT_F32_COLS = h("j4c_split_f32_cols", FunctionDescriptor.of(
        JAVA_INT, ADDRESS, JAVA_LONG, JAVA_LONG, ADDRESS, ADDRESS, ADDRESS));
    static final MethodHandle SPLIT_F32_TRANSPOSED = h("j4c_split_f32_transposed", FunctionDescriptor.of(
        JAVA_INT, ADDRESS, JAVA_LONG, JAVA_LONG, ADDRESS, ADDRESS, ADDRESS));
    static final MethodHandle SPLIT_F32_BOTH = h("j4c_split_f32_both", FunctionDescriptor.of(
        JAVA_INT, ADDRESS, JAVA_LONG, JAVA_LONG, ADDRESS, ADDRESS, ADDRESS, ADDRESS, ADDRESS));
    static final MethodHandle SPLIT_F32_EX = h("j4c_split_f32_ex", FunctionDescriptor.of(
        JAVA_INT, ADDRESS, JAVA_LONG, JAVA_LONG, ADDRESS, ADDRESS, ADDRESS, ADDRESS, ADDRESS, ADDRESS, ADDRESS,
        ADDRESS));
    static final MethodHandle SPLIT_LINES = h("j4c_split_lines", FunctionDescriptor.of(
        JAVA_INT, ADDRESS, JAVA_LONG, JAVA_LONG, ADDRESS, ADDRESS));
    static final MethodHandle SGD_UPDATE_LINES = h("j4c_sgd_update_lines", FunctionDescriptor.of(
        JAVA_INT, ADDRESS, ADDRESS, JAVA_LONG, JAVA_LONG, JAVA_FLOAT, JAVA_FLOAT, ADDRESS, ADDRESS, ADDRESS));
    static final MethodHandle DOT_SPLIT = h("j4c_dot_split", FunctionDescriptor.of(
        JAVA_INT, ADDRESS, ADDRESS, ADDRESS, ADDRESS, ADDRESS, JAVA_LONG, JAVA_LONG, JAVA_LONG, JAVA_INT,
        JAVA_INT, ADDRESS));
    static final MethodHandle DOT_SPLIT_BATCHED = h("j4c_dot_split_batched", FunctionDescriptor.of(
        JAVA_INT, ADDRESS, ADDRESS, ADDRESS, ADDRESS, ADDRESS, JAVA_LONG, JAVA_LONG, JAVA_LONG, JAVA_LONG,
        JAVA_INT, JAVA_INT, JAVA_INT, JAVA_INT, ADDRESS));
    static final MethodHandle DOT_SPLIT_EP = h("j4c_dot_split_ep", FunctionDescriptor.of(
        JAVA_INT, ADDRESS, ADDRESS, ADDRESS, ADDRESS, ADDRESS, JAVA_LONG, JAVA_LONG, JAVA_LONG, JAVA_INT,
        JAVA_INT, ADDRESS, ADDRESS, ADDRESS, ADDRESS));
    static final MethodHandle DOT_SPLIT_EP_MAX = h("j4c_dot_split_ep_max", FunctionDescriptor.of(
        JAVA_INT, ADDRESS, ADDRESS, ADDRESS, ADDRESS, ADDRESS, JAVA_LONG, JAVA_LONG, JAVA_LONG, JAVA_INT,
        JAVA_INT, ADDRESS, ADDRESS, ADDRESS, ADDRESS, ADDRESS));
    static final MethodHandle DOT_SPLIT_EP_BITS = h("j4c_dot_split_ep_bits", FunctionDescriptor.of(
        JAVA_INT, ADDRESS, ADDRESS, ADDRESS, ADDRESS, ADDRESS, JAVA_LONG, JAVA_LONG, JAVA_LONG, JAVA_INT,
        JAVA_INT, ADDRESS, ADDRESS, ADDRESS, ADDRESS, ADDRESS, ADDRESS, ADDRESS));

    // ---- Fft and Linalg (api/Fft.java, api/Linalg.java) ----
    static final MethodHandle FFT = h("j4c_fft", FunctionDescriptor.of(
        JAVA_INT, JAVA_INT, JAVA_INT, ADDRESS, ADDRESS, ADDRESS, ADDRESS, ADDRESS, JAVA_INT, ADDRESS));
    static final MethodHandle RFFT = h("j4c_rfft", FunctionDescriptor.of(
        JAVA_INT, JAVA_INT, JAVA_INT, ADDRESS, ADDRESS, ADDRESS, ADDRESS, ADDRESS));
    static final MethodHandle IRFFT = h("j4c_irfft", FunctionDescriptor.of(
        JAVA_INT, JAVA_INT, JAVA_INT, ADDRESS, ADDRESS, ADDRESS, ADDRESS, ADDRESS));
    static final MethodHandle DCT1 = h("j4c_dct1", FunctionDescriptor.of(
        JAVA_INT, JAVA_INT, JAVA_LONG, ADDRESS, ADDRESS, ADDRESS));
    static final MethodHandle LU_FACTOR = h("j4c_lu_factor", FunctionDescriptor.of(
        JAVA_INT, JAVA_INT, JAVA_LONG, ADDRESS, ADDRESS, ADDRESS, ADDRESS, ADDRESS, ADDRESS));
    static final MethodHandle LU_SOLVE = h("j4c_lu_solve", FunctionDescriptor.of(
        JAVA_INT, JAVA_LONG, JAVA_LONG, ADDRESS, ADDRESS, JAVA_INT, JAVA_INT, ADDRESS, ADDRESS, ADDRESS));
    static final MethodHandle LU_RCOND = h("j4c_lu_rcond", FunctionDescriptor.of(
        JAVA_INT, JAVA_LONG, ADDRESS, ADDRESS, JAVA_DOUBLE, ADDRESS, ADDRESS));
    static final MethodHandle EIG = h("j4c_eig", FunctionDescriptor.of(
        JAVA_INT, JAVA_INT, JAVA_LONG, ADDRESS, ADDRESS, ADDRESS, ADDRESS));
    static final MethodHandle SVD = h("j4c_svd", FunctionDescriptor.of(
        JAVA_INT, JAVA_INT, JAVA_LONG, JAVA_LONG, ADDRESS, ADDRESS, ADDRESS, ADDRESS, ADDRESS));

    // ---- JAX.jit fused chains (replaces backend/TornadoJitCompiler.java) ----
    static final MethodHandle FUSED_COMPILE = h("j4c_fused_compile", FunctionDescriptor.of(
        JAVA_INT, ADDRESS, ADDRESS));
    static final MethodHandle FUSED_SOURCE = h("j4c_fused_source", FunctionDescriptor.of(
        JAVA_INT, ADDRESS, JAVA_INT, ADDRESS, JAVA_LONG, ADDRESS));
    static final MethodHandle FUSED_LAUNCH = h("j4c_fused_launch", FunctionDescriptor.of(
        JAVA_INT, ADDRESS, JAVA_LONG, JAVA_LONG, ADDRESS, ADDRESS, ADDRESS, ADDRESS));

    // ---- Random (api/Random.java:86-140) ----
    static final MethodHandle RANDOM_PERMUTATION = h("j4c_random_permutation", FunctionDescriptor.of(
        JAVA_INT, JAVA_LONG, JAVA_LONG, ADDRESS, ADDRESS));
    static final MethodHandle RANDOM_UNIFORM = h("j4c_random_uniform", FunctionDescriptor.of(
        JAVA_INT, JAVA_LONG, JAVA_LONG, JAVA_LONG, JAVA_FLOAT, JAVA_FLOAT, ADDRESS, ADDRESS));
    static final MethodHandle RANDOM_NORMAL = h("j4c_random_normal", FunctionDescriptor.of(
        JAVA_INT, JAVA_LONG, JAVA_LONG, JAVA_LONG, ADDRESS, ADDRESS));

    // ---- collectives (replace api/SharedCollective.java) ----
    static final MethodHandle COMM_UNIQUE_ID = h("j4c_comm_unique_id", FunctionDescriptor.of(
        JAVA_INT, ADDRESS, JAVA_LONG));
    static final MethodHandle COMM_INIT_RANK = h("j4c_comm_init_rank", FunctionDescriptor.of(
        JAVA_INT, ADDRESS, JAVA_LONG, JAVA_INT, JAVA_INT, JAVA_INT, JAVA_LONG, ADDRESS));
    static final MethodHandle COMM_INIT_ALL = h("j4c_comm_init_all", FunctionDescriptor.of(
        JAVA_INT, ADDRESS, JAVA_INT, JAVA_LONG, ADDRESS));
    static final MethodHandle COMM_RANK = h("j4c_comm_rank", FunctionDescriptor.of(
        JAVA_INT, ADDRESS, ADDRESS, ADDRESS));
    static final MethodHandle COMM_DESTROY = h("j4c_comm_destroy", FunctionDescriptor.of(JAVA_INT, ADDRESS));
    static final MethodHandle COMM_ABORT = h("j4c_comm_abort", FunctionDescriptor.of(JAVA_INT, ADDRESS));
    static final MethodHandle PSUM = h("j4c_psum", FunctionDescriptor.of(
        JAVA_INT, ADDRESS, JAVA_INT, ADDRESS, ADDRESS, JAVA_LONG, ADDRESS));
    static final MethodHandle ALL_GATHER = h("j4c_all_gather", FunctionDescriptor.of(
        JAVA_INT, ADDRESS, JAVA_INT, ADDRESS, ADDRESS, JAVA_LONG, ADDRESS));
    static final MethodHandle REDUCE_SCATTER = h("j4c_reduce_scatter", FunctionDescriptor.of(
        JAVA_INT, ADDRESS, JAVA_INT, ADDRESS, ADDRESS, JAVA_LONG, ADDRESS));
    static final MethodHandle COMM_WAIT = h("j4c_comm_wait", FunctionDescriptor.of(JAVA_INT, ADDRESS, ADDRESS));
    static final MethodHandle PSUM_SLOTS = h("j4c_psum_slots", FunctionDescriptor.of(
        JAVA_INT, JAVA_INT, ADDRESS, JAVA_INT, ADDRESS, JAVA_LONG, ADDRESS));

    // ---- gradient all-reduce fused with the SGD update over peer memory (psum_sgd.cu) ----
    static final MethodHandle PEER_ALLOC = h("j4c_peer_alloc", FunctionDescriptor.of(
        JAVA_INT, JAVA_LONG, ADDRESS, ADDRESS, JAVA_LONG));
    static final MethodHandle PEER_OPEN = h("j4c_peer_open", FunctionDescriptor.of(
        JAVA_INT, ADDRESS, JAVA_LONG, ADDRESS));
    static final MethodHandle PEER_CLOSE = h("j4c_peer_close", FunctionDescriptor.of(JAVA_INT, ADDRESS));
    static final MethodHandle PEER_FREE = h("j4c_peer_free", FunctionDescriptor.of(JAVA_INT, ADDRESS));
    static final MethodHandle PSUM_SGD_FLAG_BYTES = h("j4c_psum_sgd_flag_bytes", FunctionDescriptor.of(JAVA_LONG));
    static final MethodHandle PSUM_SGD = h("j4c_psum_sgd", FunctionDescriptor.of(
        JAVA_INT, ADDRESS, ADDRESS, ADDRESS, JAVA_INT, JAVA_INT, JAVA_LONG, JAVA_INT, ADDRESS, ADDRESS,
        JAVA_FLOAT, JAVA_FLOAT, ADDRESS, ADDRESS, ADDRESS));

    /** The library's message for the last failed call on this thread. */
    public static String lastError() {
        try {
            return ((MemorySegment) LAST_ERROR.invokeExact()).reinterpret(4096).getString(0);
        } catch (Throwable t) {
            throw new IllegalStateException(t);
        }
    }

    /**
     * Status -> exception, mirroring the exception types the reference throws
     * for the same conditions: bad arguments are IllegalArgumentException
     * (as Shape/DType checks in core/ConcreteNDArray.java), unsupported
     * requests UnsupportedOperationException, device, collective and
     * timeout failures IllegalStateException / RuntimeException.
     */
    public static void check(int rc, String what) {
        if (rc == OK) return;
        String msg = what + ": " + lastError();
        switch (rc) {
            case E_INVALID -> throw new IllegalArgumentException(msg);
            case E_UNSUPPORTED -> throw new UnsupportedOperationException(msg);
            case E_OOM -> throw new OutOfMemoryError(msg);
            case E_NCCL, E_TIMEOUT -> throw new RuntimeException("Collective failed: " + msg);
            default -> throw new IllegalStateException(msg);
        }
    }

    /** Fails fast when the loaded library speaks a different ABI. */
    public static void requireAbi() {
        try {
            int v = (int) ABI_VERSION.invokeExact();
            if (v != ABI_VERSION_EXPECTED)
                throw new IllegalStateException("libjax4j_cuda.so ABI " + v + ", binding expects " + ABI_VERSION_EXPECTED);
        } catch (RuntimeException | Error e) {
            throw e;
        } catch (Throwable t) {
            throw new IllegalStateException(t);
        }
    }
}
