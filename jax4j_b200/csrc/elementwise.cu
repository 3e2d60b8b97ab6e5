// elementwise.cu -- broadcasting binary ops, comparisons, unary math, casts,
// fills and the Grad helpers that are pure elementwise maps.
//
// All kernels are HBM-bound: 16-byte vector loads/stores on the innermost
// contiguous dimension, a grid sized to a multiple of the SM count with a
// grid-stride loop, and index arithmetic on a collapsed broadcast shape (a
// same-shape op collapses to one dimension and does no division at all).
#include <type_traits>

#include "common.cuh"
#include "jmath.cuh"

namespace j4c {

// ---- op functors -------------------------------------------------------------
template <int OP, typename T>
__device__ __forceinline__ T binary_op(T a, T b) {
    if constexpr (OP == J4C_ADD) return r_add(a, b);
    else if constexpr (OP == J4C_SUB) return r_sub(a, b);
    else if constexpr (OP == J4C_MUL) return r_mul(a, b);
    else if constexpr (OP == J4C_DIV) return r_div(a, b);
    else if constexpr (OP == J4C_MAX) return java_max(a, b);
    else return java_min(a, b);
}

template <int OP, typename T>
__device__ __forceinline__ uint8_t compare_op(T a, T b) {
    if constexpr (OP == J4C_GT) return a > b;
    else if constexpr (OP == J4C_GE) return a >= b;
    else if constexpr (OP == J4C_LT) return a < b;
    else if constexpr (OP == J4C_LE) return a <= b;
    else if constexpr (OP == J4C_EQ) return a == b;
    else return a != b;
}

J4C_MATH_DEFS

// ConcreteNDArray.unary (core/ConcreteNDArray.java:657-664).  FP32 uses the
// CUDA single-precision functions (<= 2 ulp) for exp/log/sin/cos and the
// one-exponential tanh and sigmoid of jmath.cuh (<= 1.6e-6 relative for
// |x| <= 10); FP64 the double functions.
template <int OP>
__device__ __forceinline__ float unary_op(float x) {
    if constexpr (OP == J4C_EXP) return expf(x);
    else if constexpr (OP == J4C_LOG) return logf(x);
    else if constexpr (OP == J4C_SIN) return sinf(x);
    else if constexpr (OP == J4C_COS) return cosf(x);
    else if constexpr (OP == J4C_TANH) return j_tanh(x);
    else if constexpr (OP == J4C_RELU) return java_max(0.0f, x);
    else return j_sigmoid(x);  // SIGMOID: 1 / (1 + e^-x)
}
template <int OP>
__device__ __forceinline__ double unary_op(double x) {
    if constexpr (OP == J4C_EXP) return exp(x);
    else if constexpr (OP == J4C_LOG) return log(x);
    else if constexpr (OP == J4C_SIN) return sin(x);
    else if constexpr (OP == J4C_COS) return cos(x);
    else if constexpr (OP == J4C_TANH) return tanh(x);
    else if constexpr (OP == J4C_RELU) return java_max(0.0, x);
    else return __drcp_rn(__dadd_rn(1.0, exp(-x)));
}

// ---- vector helpers ------------------------------------------------------------
// A lane moves VEC consecutive elements as one 16-byte (or 8- / 4-byte)
// access, so each warp-wide access is contiguous; the streaming kernels below
// keep U such accesses per operand in flight per thread (grid-stride steps
// u * stride apart, all loads issued before any result is stored).
template <typename T, int N>
struct alignas(16) Pack {
    T v[N];
};

// N elements at p: consecutive (stride 1; p aligned to min(16, N*sizeof(T))
// bytes), N copies of p[0] (stride 0), or a strided gather.
template <typename T, int N>
__device__ __forceinline__ Pack<T, N> load_pack(const T *p, int64_t stride) {
    constexpr int BYTES = N * (int)sizeof(T);
    Pack<T, N> r;
    if (stride == 0) {
        const T x = p[0];
#pragma unroll
        for (int i = 0; i < N; i++) r.v[i] = x;
    } else if (stride == 1 && BYTES % 16 == 0) {
#pragma unroll
        for (int c = 0; c < BYTES / 16; c++)
            reinterpret_cast<uint4 *>(r.v)[c] = __ldg(reinterpret_cast<const uint4 *>(p) + c);
    } else if (stride == 1 && BYTES == 8) {
        *reinterpret_cast<uint2 *>(r.v) = __ldg(reinterpret_cast<const uint2 *>(p));
    } else if (stride == 1 && BYTES == 4) {
        *reinterpret_cast<unsigned int *>(r.v) = __ldg(reinterpret_cast<const unsigned int *>(p));
    } else {
#pragma unroll
        for (int i = 0; i < N; i++) r.v[i] = p[i * stride];
    }
    return r;
}

template <typename T, int N>
__device__ __forceinline__ void store_pack(T *p, const Pack<T, N> &r) {
    constexpr int BYTES = N * (int)sizeof(T);
    if constexpr (BYTES % 16 == 0) {
#pragma unroll
        for (int c = 0; c < BYTES / 16; c++)
            reinterpret_cast<uint4 *>(p)[c] = reinterpret_cast<const uint4 *>(r.v)[c];
    } else if constexpr (BYTES == 8) {
        *reinterpret_cast<uint2 *>(p) = *reinterpret_cast<const uint2 *>(r.v);
    } else if constexpr (BYTES == 4) {
        *reinterpret_cast<unsigned int *>(p) = *reinterpret_cast<const unsigned int *>(r.v);
    } else {
#pragma unroll
        for (int i = 0; i < N; i++) p[i] = r.v[i];
    }
}

// Offsets of output element i in each operand (rank-1 shapes need no division).
__device__ __forceinline__ void elem_offsets(const Indexer &ix, int64_t i, int64_t (&off)[3]) {
    if (ix.rank == 1) {
        off[0] = i * ix.stride[0][0];
        off[1] = i * ix.stride[1][0];
        off[2] = i * ix.stride[2][0];
    } else {
        index_offsets(ix, i, off);
    }
}

// Whether VEC consecutive outputs per thread step may use vector accesses:
// the innermost collapsed dim is a multiple of VEC and every contiguous
// operand (and the output) is 16-byte aligned.
inline bool vec_ok(const Indexer &ix, int vec, const void *a, const void *b, const void *out,
                   int out_align = 16) {
    const int last = ix.rank - 1;
    return ix.size[last] % vec == 0 && (reinterpret_cast<uintptr_t>(out) % out_align == 0) &&
           (ix.stride[0][last] != 1 || aligned16(a)) && (ix.stride[1][last] != 1 || aligned16(b));
}

// ---- binary -----------------------------------------------------------------
// VEC consecutive outputs per lane access (see vec_ok), U accesses in flight.
template <typename T, int OP, int VEC, int U>
__global__ void __launch_bounds__(256) binary_kernel(Indexer ix, const T *__restrict__ a,
                                                     const T *__restrict__ b, T *__restrict__ out,
                                                     int64_t n) {
    const int64_t nvec = n / VEC, stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t sa0 = ix.stride[0][ix.rank - 1], sb0 = ix.stride[1][ix.rank - 1];
    for (int64_t v0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v0 < nvec; v0 += U * stride) {
        Pack<T, VEC> pa[U], pb[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t v = v0 + u * stride;
            if (v < nvec) {
                int64_t off[3];
                elem_offsets(ix, v * VEC, off);
                pa[u] = load_pack<T, VEC>(a + off[0], sa0);
                pb[u] = load_pack<T, VEC>(b + off[1], sb0);
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t v = v0 + u * stride;
            if (v < nvec) {
                Pack<T, VEC> r;
#pragma unroll
                for (int k = 0; k < VEC; k++) r.v[k] = binary_op<OP, T>(pa[u].v[k], pb[u].v[k]);
                store_pack<T, VEC>(out + v * VEC, r);
            }
        }
    }
}

template <typename T, int OP>
static int launch_binary(const Indexer &ix, const void *a, const void *b, void *out, int64_t n,
                         cudaStream_t s) {
    constexpr int V = 16 / sizeof(T), U = 1;  // U = 2 measured slower for a scalar operand
    if (vec_ok(ix, V, a, b, out)) {
        binary_kernel<T, OP, V, U><<<grid_for(ceil_div(n / V, U), 256), 256, 0, s>>>(
            ix, (const T *)a, (const T *)b, (T *)out, n);
    } else {
        binary_kernel<T, OP, 1, U><<<grid_for(ceil_div(n, U), 256), 256, 0, s>>>(ix, (const T *)a, (const T *)b,
                                                                                  (T *)out, n);
    }
    J4C_LAUNCH_CHECK("binary_kernel");
    return J4C_OK;
}

template <typename T>
static int dispatch_binary(int prim, const Indexer &ix, const void *a, const void *b, void *out,
                           int64_t n, cudaStream_t s) {
    switch (prim) {
    case J4C_ADD: return launch_binary<T, J4C_ADD>(ix, a, b, out, n, s);
    case J4C_SUB: return launch_binary<T, J4C_SUB>(ix, a, b, out, n, s);
    case J4C_MUL: return launch_binary<T, J4C_MUL>(ix, a, b, out, n, s);
    case J4C_DIV: return launch_binary<T, J4C_DIV>(ix, a, b, out, n, s);
    case J4C_MAX: return launch_binary<T, J4C_MAX>(ix, a, b, out, n, s);
    case J4C_MIN: return launch_binary<T, J4C_MIN>(ix, a, b, out, n, s);
    default: return set_error(J4C_E_INVALID, "j4c_binary: primitive %d is not a binary op", prim);
    }
}

// ---- compare ----------------------------------------------------------------
// VEC outputs per lane access; 16 (one 16-byte store of BOOLs per lane, the
// operands read as 4 (8) consecutive 16-byte pieces) measured fastest.
template <typename T, int OP, int VEC, int U>
__global__ void __launch_bounds__(256) compare_kernel(Indexer ix, const T *__restrict__ a,
                                                      const T *__restrict__ b,
                                                      uint8_t *__restrict__ out, int64_t n) {
    const int64_t nvec = n / VEC, stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t sa0 = ix.stride[0][ix.rank - 1], sb0 = ix.stride[1][ix.rank - 1];
    for (int64_t v0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v0 < nvec; v0 += U * stride) {
        Pack<T, VEC> pa[U], pb[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t v = v0 + u * stride;
            if (v < nvec) {
                int64_t off[3];
                elem_offsets(ix, v * VEC, off);
                pa[u] = load_pack<T, VEC>(a + off[0], sa0);
                pb[u] = load_pack<T, VEC>(b + off[1], sb0);
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t v = v0 + u * stride;
            if (v < nvec) {
                Pack<uint8_t, VEC> r;
#pragma unroll
                for (int k = 0; k < VEC; k++) r.v[k] = compare_op<OP, T>(pa[u].v[k], pb[u].v[k]);
                store_pack<uint8_t, VEC>(out + v * VEC, r);
            }
        }
    }
}

template <typename T, int OP>
static void launch_compare(const Indexer &ix, const void *a, const void *b, uint8_t *out, int64_t n,
                           cudaStream_t s) {
    constexpr int U = 1;
    if (vec_ok(ix, 16, a, b, out, 16))
        compare_kernel<T, OP, 16, U><<<grid_for(n / 16, 256), 256, 0, s>>>(ix, (const T *)a, (const T *)b, out, n);
    else if (vec_ok(ix, 4, a, b, out, 4))
        compare_kernel<T, OP, 4, U><<<grid_for(n / 4, 256), 256, 0, s>>>(ix, (const T *)a, (const T *)b, out, n);
    else
        compare_kernel<T, OP, 1, U><<<grid_for(ceil_div(n, U), 256), 256, 0, s>>>(ix, (const T *)a,
                                                                                   (const T *)b, out, n);
}

template <typename T>
static int dispatch_compare(int prim, const Indexer &ix, const void *a, const void *b, uint8_t *out,
                            int64_t n, cudaStream_t s) {
    switch (prim) {
    case J4C_GT: launch_compare<T, J4C_GT>(ix, a, b, out, n, s); break;
    case J4C_GE: launch_compare<T, J4C_GE>(ix, a, b, out, n, s); break;
    case J4C_LT: launch_compare<T, J4C_LT>(ix, a, b, out, n, s); break;
    case J4C_LE: launch_compare<T, J4C_LE>(ix, a, b, out, n, s); break;
    case J4C_EQ: launch_compare<T, J4C_EQ>(ix, a, b, out, n, s); break;
    case J4C_NE: launch_compare<T, J4C_NE>(ix, a, b, out, n, s); break;
    default: return set_error(J4C_E_INVALID, "j4c_compare: primitive %d is not a comparison", prim);
    }
    J4C_LAUNCH_CHECK("compare_kernel");
    return J4C_OK;
}

// ---- unary ------------------------------------------------------------------
// VEC consecutive elements per lane access, U accesses in flight, then a
// scalar tail (fewer than VEC elements).
template <typename T, int OP, int VEC, int U>
__global__ void __launch_bounds__(256) unary_kernel(const T *__restrict__ in, T *__restrict__ out,
                                                    int64_t n) {
    const int64_t nvec = n / VEC, stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t v0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v0 < nvec; v0 += U * stride) {
        Pack<T, VEC> p[U];
#pragma unroll
        for (int u = 0; u < U; u++)
            if (v0 + u * stride < nvec) p[u] = load_pack<T, VEC>(in + (v0 + u * stride) * VEC, 1);
#pragma unroll
        for (int u = 0; u < U; u++) {
            if (v0 + u * stride < nvec) {
#pragma unroll
                for (int k = 0; k < VEC; k++) p[u].v[k] = unary_op<OP>(p[u].v[k]);
                store_pack<T, VEC>(out + (v0 + u * stride) * VEC, p[u]);
            }
        }
    }
    const int64_t t = nvec * VEC + blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (VEC > 1 && t < n) out[t] = unary_op<OP>(in[t]);  // n - nvec*VEC < VEC <= threads
}

template <typename T, int OP>
static int launch_unary(const void *in, void *out, int64_t n, cudaStream_t s) {
    constexpr int V = 16 / sizeof(T), U = 4;
    if (aligned16(in) && aligned16(out) && n >= V)
        unary_kernel<T, OP, V, U><<<grid_for(ceil_div(ceil_div(n, V), U), 256), 256, 0, s>>>((const T *)in,
                                                                                            (T *)out, n);
    else
        unary_kernel<T, OP, 1, U><<<grid_for(ceil_div(n, U), 256), 256, 0, s>>>((const T *)in, (T *)out, n);
    J4C_LAUNCH_CHECK("unary_kernel");
    return J4C_OK;
}

template <typename T>
static int dispatch_unary(int prim, const void *in, void *out, int64_t n, cudaStream_t s) {
    switch (prim) {
    case J4C_EXP: return launch_unary<T, J4C_EXP>(in, out, n, s);
    case J4C_LOG: return launch_unary<T, J4C_LOG>(in, out, n, s);
    case J4C_SIN: return launch_unary<T, J4C_SIN>(in, out, n, s);
    case J4C_COS: return launch_unary<T, J4C_COS>(in, out, n, s);
    case J4C_TANH: return launch_unary<T, J4C_TANH>(in, out, n, s);
    case J4C_RELU: return launch_unary<T, J4C_RELU>(in, out, n, s);
    case J4C_SIGMOID: return launch_unary<T, J4C_SIGMOID>(in, out, n, s);
    default: return set_error(J4C_E_INVALID, "j4c_unary: primitive %d is not a unary op", prim);
    }
}

// ---- cast ---------------------------------------------------------------------
// Java conversion rules (core/ConcreteNDArray.java:666-730, JLS 5.1.2/5.1.3).

template <typename S, typename D>
__device__ __forceinline__ D java_cast(S v) {
    if constexpr (std::is_same<D, uint8_t>::value) {
        if constexpr (std::is_same<S, uint8_t>::value) return v ? 1 : 0;
        else return v != S(0) ? 1 : 0;
    } else if constexpr (std::is_same<S, uint8_t>::value) {
        return v ? D(1) : D(0);
    } else if constexpr (std::is_same<D, int32_t>::value) {
        if constexpr (std::is_floating_point<S>::value) return java_d2i((double)v);
        else return (int32_t)(uint32_t)(uint64_t)(int64_t)v;  // long->int wraps
    } else if constexpr (std::is_same<D, int64_t>::value) {
        if constexpr (std::is_floating_point<S>::value) return java_d2l((double)v);
        else return (int64_t)v;
    } else {
        return (D)v;  // to float/double: round to nearest (cvt.rn)
    }
}

template <typename S, typename D, int VEC, int U>
__global__ void __launch_bounds__(256) cast_kernel(const S *__restrict__ in, D *__restrict__ out,
                                                   int64_t n) {
    const int64_t nvec = n / VEC, stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t v0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v0 < nvec; v0 += U * stride) {
        Pack<S, VEC> p[U];
#pragma unroll
        for (int u = 0; u < U; u++)
            if (v0 + u * stride < nvec) p[u] = load_pack<S, VEC>(in + (v0 + u * stride) * VEC, 1);
#pragma unroll
        for (int u = 0; u < U; u++) {
            if (v0 + u * stride < nvec) {
                Pack<D, VEC> r;
#pragma unroll
                for (int k = 0; k < VEC; k++) r.v[k] = java_cast<S, D>(p[u].v[k]);
                store_pack<D, VEC>(out + (v0 + u * stride) * VEC, r);
            }
        }
    }
    const int64_t t = nvec * VEC + blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (VEC > 1 && t < n) out[t] = java_cast<S, D>(in[t]);
}

template <typename S, typename D>
static void launch_cast(const void *in, void *out, int64_t n, cudaStream_t s) {
    // 4 elements per lane access: 4 B (bool) .. 32 B (8-byte types) per side
    constexpr int U = 4;
    if (aligned16(in) && aligned16(out) && n >= 4)
        cast_kernel<S, D, 4, U><<<grid_for(ceil_div(ceil_div(n, 4), U), 256), 256, 0, s>>>((const S *)in,
                                                                                           (D *)out, n);
    else
        cast_kernel<S, D, 1, U><<<grid_for(ceil_div(n, U), 256), 256, 0, s>>>((const S *)in, (D *)out, n);
}

template <typename S>
static int cast_from(int dst, const void *in, void *out, int64_t n, cudaStream_t s) {
    switch (dst) {
    case J4C_FLOAT32: launch_cast<S, float>(in, out, n, s); break;
    case J4C_FLOAT64: launch_cast<S, double>(in, out, n, s); break;
    case J4C_INT32: launch_cast<S, int32_t>(in, out, n, s); break;
    case J4C_INT64: launch_cast<S, int64_t>(in, out, n, s); break;
    case J4C_BOOL: launch_cast<S, uint8_t>(in, out, n, s); break;
    default: return set_error(J4C_E_INVALID, "j4c_cast: bad target dtype %d", dst);
    }
    J4C_LAUNCH_CHECK("cast_kernel");
    return J4C_OK;
}

// ---- fill / relu_grad / maxmin_grad / transpose / broadcast -------------------
template <typename T>
__global__ void fill_kernel(T *out, int64_t n, T v) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = v;
}

template <typename T, int VEC, int U>
__global__ void __launch_bounds__(256) relu_grad_kernel(const T *__restrict__ g,
                                                        const T *__restrict__ x,
                                                        T *__restrict__ out, int64_t n) {
    const int64_t nvec = n / VEC, stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t v0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v0 < nvec; v0 += U * stride) {
        Pack<T, VEC> pg[U], px[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            if (v0 + u * stride < nvec) {
                pg[u] = load_pack<T, VEC>(g + (v0 + u * stride) * VEC, 1);
                px[u] = load_pack<T, VEC>(x + (v0 + u * stride) * VEC, 1);
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            if (v0 + u * stride < nvec) {
#pragma unroll
                for (int k = 0; k < VEC; k++) pg[u].v[k] = px[u].v[k] > T(0) ? pg[u].v[k] : T(0);
                store_pack<T, VEC>(out + (v0 + u * stride) * VEC, pg[u]);
            }
        }
    }
    const int64_t t = nvec * VEC + blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (VEC > 1 && t < n) out[t] = x[t] > T(0) ? g[t] : T(0);
}

template <typename T>
__global__ void __launch_bounds__(256) maxmin_grad_kernel(Indexer ix, int is_max,
                                                          const T *__restrict__ g,
                                                          const T *__restrict__ a,
                                                          const T *__restrict__ b,
                                                          T *__restrict__ ga, T *__restrict__ gb,
                                                          int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t off[3];
        index_offsets(ix, i, off);
        T va = a[off[0]], vb = b[off[1]];
        bool a_wins = is_max ? va >= vb : va <= vb;
        T gv = g[i];
        ga[i] = a_wins ? gv : T(0);
        gb[i] = a_wins ? T(0) : gv;
    }
}

template <typename T>
__global__ void transpose_kernel(const T *__restrict__ in, int64_t rows, int64_t cols,
                                 T *__restrict__ out) {
    __shared__ T tile[32][33];
    int64_t bx = blockIdx.x * 32, by = blockIdx.y * 32;
    for (int j = threadIdx.y; j < 32; j += 8) {
        int64_t r = by + j, c = bx + threadIdx.x;
        if (r < rows && c < cols) tile[j][threadIdx.x] = in[r * cols + c];
    }
    __syncthreads();
    for (int j = threadIdx.y; j < 32; j += 8) {
        int64_t r = bx + j, c = by + threadIdx.x;  // out is [cols, rows]
        if (r < cols && c < rows) out[r * rows + c] = tile[threadIdx.x][j];
    }
}

// out[i] = g[broadcast index]: the expand branch of Grad.broadcastLike.
template <typename T, int VEC>
__global__ void __launch_bounds__(256) expand_kernel(Indexer ix, const T *__restrict__ g,
                                                     T *__restrict__ out, int64_t n) {
    const int64_t s0 = ix.stride[0][ix.rank - 1];
    for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < n / VEC;
         v += (int64_t)gridDim.x * blockDim.x) {
        int64_t off[3];
        index_offsets(ix, v * VEC, off);
        store_pack<T, VEC>(out + v * VEC, load_pack<T, VEC>(g + off[0], s0));
    }
}

// ---- Numpy.take (GATHER) and its VJP -----------------------------------------------
// out[p, :] = table[idx[p], :]; rows are copied 16 bytes at a time when aligned.
// Indices outside [0, rows) write zeros (the host validates them first).
template <typename T, typename I>
__global__ void __launch_bounds__(256) gather_rows_kernel(const T *__restrict__ table, int64_t rows, int64_t dim,
                                                          const I *__restrict__ idx, int64_t n,
                                                          T *__restrict__ out) {
    const int64_t total = n * dim;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t p = e / dim, d = e - p * dim;
        const int64_t r = (int64_t)idx[p];
        out[e] = (r >= 0 && r < rows) ? table[r * dim + d] : T(0);
    }
}

// gtable[idx[p], :] += g[p, :] (gtable zeroed by the caller); repeated
// indices accumulate with atomic adds.
template <typename T, typename I>
__global__ void __launch_bounds__(256) scatter_add_rows_kernel(const T *__restrict__ g, int64_t rows, int64_t dim,
                                                               const I *__restrict__ idx, int64_t n,
                                                               T *__restrict__ gtable) {
    const int64_t total = n * dim;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t p = e / dim, d = e - p * dim;
        const int64_t r = (int64_t)idx[p];
        if (r >= 0 && r < rows) atomicAdd(gtable + r * dim + d, g[e]);
    }
}

// ---- Random (api/Random.java:39-113) ----------------------------------------------
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}
__device__ __forceinline__ float raw_uniform01(uint64_t state, uint64_t i) {
    const uint64_t kGamma = 0x9E3779B97F4A7C15ULL, kSample = 0x2545F4914F6CDD1DULL;
    uint64_t bits = mix64(state ^ kSample ^ (kGamma * (i + 1)));
    return __fdiv_rn((float)(int32_t)(bits >> 40), 16777216.0f);
}

__global__ void uniform_kernel(uint64_t key, int64_t offset, int64_t n, float lo, float hi,
                               float *out) {
    float span = __fsub_rn(hi, lo);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        float u = raw_uniform01(key, (uint64_t)(offset + i));
        out[i] = __fadd_rn(lo, __fmul_rn(u, span));
    }
}

__global__ void normal_kernel(uint64_t key, int64_t offset, int64_t n, float *out) {
    const double two_pi = 2.0 * 3.141592653589793;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        uint64_t k = (uint64_t)(offset + i);
        float u1 = raw_uniform01(key, 2 * k);
        if (!(u1 >= 1e-7f)) u1 = 1e-7f;
        float u2 = raw_uniform01(key, 2 * k + 1);
        double r = __dmul_rn(sqrt(__dmul_rn(-2.0, log((double)u1))), cos(__dmul_rn(two_pi, (double)u2)));
        out[i] = (float)r;
    }
}

// Random.permutation (Random.java:130-140): Fisher-Yates from the top, swap
// index j = min((int)(u_i * (i + 1)), i) with u_i the i-th uniform draw.  The
// swaps are sequential, so one thread performs them after a parallel fill.
__global__ void iota_kernel(int32_t *out, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = (int32_t)i;
}

__global__ void fisher_yates_kernel(uint64_t key, int64_t n, int32_t *out) {
    for (int64_t i = n - 1; i > 0; i--) {
        const float u = raw_uniform01(key, (uint64_t)i);
        int64_t j = (int64_t)(int32_t)__fmul_rn(u, (float)(i + 1));  // Java: (int) (u * (i + 1)), float product
        if (j > i) j = i;
        const int32_t t = out[i];
        out[i] = out[j];
        out[j] = t;
    }
}

// ---- in-process psum over slots (api/SharedCollective.java:44-54) -----------------
struct SlotPtrs {
    const void *p[16];
};

template <typename T>
__global__ void __launch_bounds__(256) psum_slots_kernel(SlotPtrs slots, int nslots,
                                                         T *__restrict__ out, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        T acc = T(0);
        for (int d = 0; d < nslots; d++) acc = r_add(acc, static_cast<const T *>(slots.p[d])[i]);
        out[i] = acc;
    }
}

}  // namespace j4c

using namespace j4c;

extern "C" {

int j4c_binary(int prim, int dtype, const void *a, const int64_t *a_dims, int a_rank,
               const void *b, const int64_t *b_dims, int b_rank, void *out, j4c_stream stream) {
    J4C_REQUIRE(a_rank >= 0 && b_rank >= 0 && a_rank <= kMaxDims && b_rank <= kMaxDims,
                "j4c_binary: rank out of range");
    if (dtype != J4C_FLOAT32 && dtype != J4C_FLOAT64)
        return set_error(J4C_E_INVALID, "%d requires FLOAT32 or FLOAT64 operands, got %s", prim,
                         dtype_name(dtype));
    int64_t od[kMaxDims];
    int orank = 0;
    if (!broadcast_shape(a_dims, a_rank, b_dims, b_rank, od, &orank))
        return set_error(J4C_E_INVALID, "j4c_binary: shapes are not broadcast-compatible");
    int64_t n = shape_numel(od, orank);
    if (n == 0) return J4C_OK;
    J4C_REQUIRE(a && b && out, "j4c_binary: NULL pointer");
    Indexer ix;
    const int64_t *dims[2] = {a_dims, b_dims};
    int ranks[2] = {a_rank, b_rank};
    if (!make_indexer(ix, od, orank, 2, dims, ranks))
        return set_error(J4C_E_INVALID, "j4c_binary: bad broadcast");
    cudaStream_t s = as_stream(stream);
    return dtype == J4C_FLOAT32 ? dispatch_binary<float>(prim, ix, a, b, out, n, s)
                                : dispatch_binary<double>(prim, ix, a, b, out, n, s);
}

int j4c_compare(int prim, int dtype, const void *a, const int64_t *a_dims, int a_rank,
                const void *b, const int64_t *b_dims, int b_rank, uint8_t *out,
                j4c_stream stream) {
    J4C_REQUIRE(a_rank >= 0 && b_rank >= 0 && a_rank <= kMaxDims && b_rank <= kMaxDims,
                "j4c_compare: rank out of range");
    int64_t od[kMaxDims];
    int orank = 0;
    if (!broadcast_shape(a_dims, a_rank, b_dims, b_rank, od, &orank))
        return set_error(J4C_E_INVALID, "j4c_compare: shapes are not broadcast-compatible");
    int64_t n = shape_numel(od, orank);
    if (n == 0) return J4C_OK;
    J4C_REQUIRE(a && b && out, "j4c_compare: NULL pointer");
    Indexer ix;
    const int64_t *dims[2] = {a_dims, b_dims};
    int ranks[2] = {a_rank, b_rank};
    if (!make_indexer(ix, od, orank, 2, dims, ranks))
        return set_error(J4C_E_INVALID, "j4c_compare: bad broadcast");
    cudaStream_t s = as_stream(stream);
    switch (dtype) {
    case J4C_FLOAT32: return dispatch_compare<float>(prim, ix, a, b, out, n, s);
    case J4C_FLOAT64: return dispatch_compare<double>(prim, ix, a, b, out, n, s);
    case J4C_INT32: return dispatch_compare<int32_t>(prim, ix, a, b, out, n, s);
    case J4C_INT64: return dispatch_compare<int64_t>(prim, ix, a, b, out, n, s);
    default:
        return set_error(J4C_E_INVALID,
                         "%d requires FLOAT32, INT32, FLOAT64, or INT64 operands, got %s", prim,
                         dtype_name(dtype));
    }
}

int j4c_unary(int prim, int dtype, const void *in, int64_t n, void *out, j4c_stream stream) {
    J4C_REQUIRE(n >= 0, "j4c_unary: negative size");
    if (n == 0) return J4C_OK;
    J4C_REQUIRE(in && out, "j4c_unary: NULL pointer");
    cudaStream_t s = as_stream(stream);
    if (dtype == J4C_FLOAT32) return dispatch_unary<float>(prim, in, out, n, s);
    if (dtype == J4C_FLOAT64) return dispatch_unary<double>(prim, in, out, n, s);
    return set_error(J4C_E_INVALID, "%d requires FLOAT32 or FLOAT64 operands, got %s", prim,
                     dtype_name(dtype));
}

int j4c_cast(int src_dtype, int dst_dtype, const void *in, int64_t n, void *out,
             j4c_stream stream) {
    J4C_REQUIRE(n >= 0, "j4c_cast: negative size");
    if (n == 0) return J4C_OK;
    J4C_REQUIRE(in && out, "j4c_cast: NULL pointer");
    cudaStream_t s = as_stream(stream);
    switch (src_dtype) {
    case J4C_FLOAT32: return cast_from<float>(dst_dtype, in, out, n, s);
    case J4C_FLOAT64: return cast_from<double>(dst_dtype, in, out, n, s);
    case J4C_INT32: return cast_from<int32_t>(dst_dtype, in, out, n, s);
    case J4C_INT64: return cast_from<int64_t>(dst_dtype, in, out, n, s);
    case J4C_BOOL: return cast_from<uint8_t>(dst_dtype, in, out, n, s);
    default: return set_error(J4C_E_INVALID, "j4c_cast: bad source dtype %d", src_dtype);
    }
}

int j4c_fill(int dtype, void *out, int64_t n, double value, j4c_stream stream) {
    J4C_REQUIRE(n >= 0, "j4c_fill: negative size");
    if (n == 0) return J4C_OK;
    J4C_REQUIRE(out, "j4c_fill: NULL pointer");
    cudaStream_t s = as_stream(stream);
    unsigned g = grid_for(n, 256);
    switch (dtype) {
    case J4C_FLOAT32: fill_kernel<float><<<g, 256, 0, s>>>((float *)out, n, (float)value); break;
    case J4C_FLOAT64: fill_kernel<double><<<g, 256, 0, s>>>((double *)out, n, value); break;
    case J4C_INT32: fill_kernel<int32_t><<<g, 256, 0, s>>>((int32_t *)out, n, (int32_t)value); break;
    case J4C_INT64: fill_kernel<int64_t><<<g, 256, 0, s>>>((int64_t *)out, n, (int64_t)value); break;
    case J4C_BOOL: fill_kernel<uint8_t><<<g, 256, 0, s>>>((uint8_t *)out, n, value != 0.0); break;
    default: return set_error(J4C_E_INVALID, "j4c_fill: bad dtype %d", dtype);
    }
    J4C_LAUNCH_CHECK("fill_kernel");
    return J4C_OK;
}

int j4c_relu_grad(int dtype, const void *g, const void *x, int64_t n, void *out,
                  j4c_stream stream) {
    J4C_REQUIRE(n >= 0, "j4c_relu_grad: negative size");
    if (n == 0) return J4C_OK;
    J4C_REQUIRE(g && x && out, "j4c_relu_grad: NULL pointer");
    cudaStream_t s = as_stream(stream);
    const bool vec = aligned16(g) && aligned16(x) && aligned16(out) && n >= 4;
    if (dtype == J4C_FLOAT32) {
        if (vec)
            relu_grad_kernel<float, 4, 2><<<grid_for(ceil_div(ceil_div(n, 4), 2), 256), 256, 0, s>>>(
                (const float *)g, (const float *)x, (float *)out, n);
        else
            relu_grad_kernel<float, 1, 2><<<grid_for(ceil_div(n, 2), 256), 256, 0, s>>>(
                (const float *)g, (const float *)x, (float *)out, n);
    } else if (dtype == J4C_FLOAT64) {
        if (vec)
            relu_grad_kernel<double, 2, 2><<<grid_for(ceil_div(ceil_div(n, 2), 2), 256), 256, 0, s>>>(
                (const double *)g, (const double *)x, (double *)out, n);
        else
            relu_grad_kernel<double, 1, 2><<<grid_for(ceil_div(n, 2), 256), 256, 0, s>>>(
                (const double *)g, (const double *)x, (double *)out, n);
    } else {
        return set_error(J4C_E_INVALID, "j4c_relu_grad: dtype %s", dtype_name(dtype));
    }
    J4C_LAUNCH_CHECK("relu_grad_kernel");
    return J4C_OK;
}

int j4c_maxmin_grad(int is_max, int dtype, const void *g, const int64_t *g_dims, int g_rank,
                    const void *a, const int64_t *a_dims, int a_rank, const void *b,
                    const int64_t *b_dims, int b_rank, void *ga_full, void *gb_full,
                    j4c_stream stream) {
    int64_t n = shape_numel(g_dims, g_rank);
    if (n == 0) return J4C_OK;
    J4C_REQUIRE(g && a && b && ga_full && gb_full, "j4c_maxmin_grad: NULL pointer");
    Indexer ix;
    const int64_t *dims[2] = {a_dims, b_dims};
    int ranks[2] = {a_rank, b_rank};
    if (!make_indexer(ix, g_dims, g_rank, 2, dims, ranks))
        return set_error(J4C_E_INVALID, "j4c_maxmin_grad: operands do not broadcast to g");
    cudaStream_t s = as_stream(stream);
    unsigned gr = grid_for(n, 256);
    if (dtype == J4C_FLOAT32)
        maxmin_grad_kernel<float><<<gr, 256, 0, s>>>(ix, is_max, (const float *)g, (const float *)a,
                                                     (const float *)b, (float *)ga_full,
                                                     (float *)gb_full, n);
    else if (dtype == J4C_FLOAT64)
        maxmin_grad_kernel<double><<<gr, 256, 0, s>>>(ix, is_max, (const double *)g,
                                                      (const double *)a, (const double *)b,
                                                      (double *)ga_full, (double *)gb_full, n);
    else
        return set_error(J4C_E_INVALID, "j4c_maxmin_grad: dtype %s", dtype_name(dtype));
    J4C_LAUNCH_CHECK("maxmin_grad_kernel");
    return J4C_OK;
}

int j4c_transpose(int dtype, const void *in, int64_t rows, int64_t cols, void *out,
                  j4c_stream stream) {
    J4C_REQUIRE(rows >= 0 && cols >= 0, "j4c_transpose: negative size");
    if (rows == 0 || cols == 0) return J4C_OK;
    J4C_REQUIRE(in && out && in != out, "j4c_transpose: bad pointers");
    J4C_REQUIRE(ceil_div(rows, 32) < 65536, "j4c_transpose: too many rows");
    dim3 grid((unsigned)ceil_div(cols, 32), (unsigned)ceil_div(rows, 32));
    dim3 block(32, 8);
    cudaStream_t s = as_stream(stream);
    switch (dtype_size(dtype)) {
    case 4: transpose_kernel<float><<<grid, block, 0, s>>>((const float *)in, rows, cols, (float *)out); break;
    case 8: transpose_kernel<double><<<grid, block, 0, s>>>((const double *)in, rows, cols, (double *)out); break;
    case 1: transpose_kernel<uint8_t><<<grid, block, 0, s>>>((const uint8_t *)in, rows, cols, (uint8_t *)out); break;
    default: return set_error(J4C_E_INVALID, "j4c_transpose: bad dtype %d", dtype);
    }
    J4C_LAUNCH_CHECK("transpose_kernel");
    return J4C_OK;
}

int j4c_gather_rows(int dtype, const void *table, int64_t rows, int64_t dim, int idx_dtype, const void *idx,
                    int64_t n, void *out, j4c_stream stream) {
    J4C_REQUIRE(rows >= 0 && dim >= 0 && n >= 0, "j4c_gather_rows: negative size");
    if (n == 0 || dim == 0) return J4C_OK;
    J4C_REQUIRE(table && idx && out, "j4c_gather_rows: NULL pointer");
    J4C_REQUIRE(idx_dtype == J4C_INT32 || idx_dtype == J4C_INT64, "j4c_gather_rows: indices must be INT32 or INT64");
    cudaStream_t s = as_stream(stream);
    const unsigned g = grid_for(n * dim, 256);
#define J4C_GATHER(T)                                                                                          \
    if (idx_dtype == J4C_INT32)                                                                              \
        gather_rows_kernel<T, int32_t><<<g, 256, 0, s>>>((const T *)table, rows, dim, (const int32_t *)idx, n, \
                                                        (T *)out);                                            \
    else                                                                                                       \
        gather_rows_kernel<T, int64_t><<<g, 256, 0, s>>>((const T *)table, rows, dim, (const int64_t *)idx, n, \
                                                        (T *)out);
    switch (dtype_size(dtype)) {
    case 4: J4C_GATHER(float) break;
    case 8: J4C_GATHER(double) break;
    case 1: J4C_GATHER(uint8_t) break;
    default: return set_error(J4C_E_INVALID, "j4c_gather_rows: bad dtype %d", dtype);
    }
#undef J4C_GATHER
    J4C_LAUNCH_CHECK("gather_rows_kernel");
    return J4C_OK;
}

int j4c_scatter_add_rows(int dtype, const void *g, int64_t rows, int64_t dim, int idx_dtype, const void *idx,
                         int64_t n, void *gtable, j4c_stream stream) {
    J4C_REQUIRE(rows >= 0 && dim >= 0 && n >= 0, "j4c_scatter_add_rows: negative size");
    if (n == 0 || dim == 0) return J4C_OK;
    J4C_REQUIRE(g && idx && gtable, "j4c_scatter_add_rows: NULL pointer");
    J4C_REQUIRE(idx_dtype == J4C_INT32 || idx_dtype == J4C_INT64,
                "j4c_scatter_add_rows: indices must be INT32 or INT64");
    J4C_REQUIRE(dtype == J4C_FLOAT32 || dtype == J4C_FLOAT64, "j4c_scatter_add_rows: dtype %s", dtype_name(dtype));
    cudaStream_t s = as_stream(stream);
    const unsigned gr = grid_for(n * dim, 256);
    if (dtype == J4C_FLOAT32) {
        if (idx_dtype == J4C_INT32)
            scatter_add_rows_kernel<float, int32_t><<<gr, 256, 0, s>>>((const float *)g, rows, dim,
                                                                       (const int32_t *)idx, n, (float *)gtable);
        else
            scatter_add_rows_kernel<float, int64_t><<<gr, 256, 0, s>>>((const float *)g, rows, dim,
                                                                       (const int64_t *)idx, n, (float *)gtable);
    } else {
        if (idx_dtype == J4C_INT32)
            scatter_add_rows_kernel<double, int32_t><<<gr, 256, 0, s>>>((const double *)g, rows, dim,
                                                                        (const int32_t *)idx, n, (double *)gtable);
        else
            scatter_add_rows_kernel<double, int64_t><<<gr, 256, 0, s>>>((const double *)g, rows, dim,
                                                                        (const int64_t *)idx, n, (double *)gtable);
    }
    J4C_LAUNCH_CHECK("scatter_add_rows_kernel");
    return J4C_OK;
}

int j4c_random_permutation(uint64_t key, int64_t n, int32_t *out, j4c_stream stream) {
    J4C_REQUIRE(n >= 0 && n < (1ll << 31), "j4c_random_permutation: n out of range");
    if (n == 0) return J4C_OK;
    J4C_REQUIRE(out, "j4c_random_permutation: NULL pointer");
    cudaStream_t s = as_stream(stream);
    iota_kernel<<<grid_for(n, 256), 256, 0, s>>>(out, n);
    J4C_LAUNCH_CHECK("iota_kernel");
    fisher_yates_kernel<<<1, 1, 0, s>>>(key, n, out);
    J4C_LAUNCH_CHECK("fisher_yates_kernel");
    return J4C_OK;
}

int j4c_random_uniform(uint64_t key, int64_t offset, int64_t n, float lo, float hi, float *out,
                       j4c_stream stream) {
    J4C_REQUIRE(n >= 0 && offset >= 0, "j4c_random_uniform: negative size/offset");
    if (n == 0) return J4C_OK;
    J4C_REQUIRE(out, "j4c_random_uniform: NULL pointer");
    uniform_kernel<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(key, offset, n, lo, hi, out);
    J4C_LAUNCH_CHECK("uniform_kernel");
    return J4C_OK;
}

int j4c_random_normal(uint64_t key, int64_t offset, int64_t n, float *out, j4c_stream stream) {
    J4C_REQUIRE(n >= 0 && offset >= 0, "j4c_random_normal: negative size/offset");
    if (n == 0) return J4C_OK;
    J4C_REQUIRE(out, "j4c_random_normal: NULL pointer");
    normal_kernel<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(key, offset, n, out);
    J4C_LAUNCH_CHECK("normal_kernel");
    return J4C_OK;
}

int j4c_psum_slots(int dtype, const void *const *slots, int nslots, void *out, int64_t n,
                   j4c_stream stream) {
    J4C_REQUIRE(slots && out, "j4c_psum_slots: NULL pointer");
    J4C_REQUIRE(nslots >= 1 && nslots <= 16, "j4c_psum_slots: 1..16 slots supported, got %d",
                nslots);
    if (n == 0) return J4C_OK;
    SlotPtrs sp;
    for (int i = 0; i < 16; i++) sp.p[i] = i < nslots ? slots[i] : nullptr;
    cudaStream_t s = as_stream(stream);
    unsigned g = grid_for(n, 256);
    if (dtype == J4C_FLOAT32) psum_slots_kernel<float><<<g, 256, 0, s>>>(sp, nslots, (float *)out, n);
    else if (dtype == J4C_FLOAT64) psum_slots_kernel<double><<<g, 256, 0, s>>>(sp, nslots, (double *)out, n);
    else return set_error(J4C_E_INVALID, "j4c_psum_slots: dtype %s", dtype_name(dtype));
    J4C_LAUNCH_CHECK("psum_slots_kernel");
    return J4C_OK;
}

}  // extern "C"

// expand is shared with reduce.cu's broadcast_like.
namespace j4c {
int launch_expand(int dtype, const Indexer &ix, const void *g, void *out, int64_t n, cudaStream_t s) {
    size_t es = dtype_size(dtype);
    bool vec = aligned16(out) && (ix.stride[0][ix.rank - 1] != 1 || aligned16(g));
    if (es == 4) {
        if (vec && ix.size[ix.rank - 1] % 4 == 0)
            expand_kernel<float, 4><<<grid_for(n / 4, 256), 256, 0, s>>>(ix, (const float *)g, (float *)out, n);
        else
            expand_kernel<float, 1><<<grid_for(n, 256), 256, 0, s>>>(ix, (const float *)g, (float *)out, n);
    } else if (es == 8) {
        if (vec && ix.size[ix.rank - 1] % 2 == 0)
            expand_kernel<double, 2><<<grid_for(n / 2, 256), 256, 0, s>>>(ix, (const double *)g, (double *)out, n);
        else
            expand_kernel<double, 1><<<grid_for(n, 256), 256, 0, s>>>(ix, (const double *)g, (double *)out, n);
    } else {
        return set_error(J4C_E_INVALID, "broadcast: unsupported dtype %d", dtype);
    }
    J4C_LAUNCH_CHECK("expand_kernel");
    return J4C_OK;
}
}  // namespace j4c
