// reduce.cu -- deterministic reductions: full sum/mean, per-axis sum/mean,
// argmax/argmin, and Grad.broadcastLike's sum-down.
//
// All are HBM-bound streaming reads.  The order of every tree is a function
// of the shape and the device's SM count only, so repeated runs on the same
// device return identical bits.  Rows (inner == 1) use a CTA or a warp per
// row with 16-byte loads; columns (inner > 1) give each thread a run of
// adjacent columns (coalesced) and split long axes across CTAs, combining the
// partials in a second deterministic pass.
#include <algorithm>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace j4c {

int launch_expand(int dtype, const Indexer &ix, const void *g, void *out, int64_t n,
                  cudaStream_t s);

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = r_add(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum in a fixed order; result valid in thread 0.
template <typename T, int THREADS>
__device__ __forceinline__ T block_sum(T v) {
    __shared__ T smem[THREADS / 32];
    v = warp_sum(v);
    int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (THREADS > 32) {
        if (lane == 0) smem[warp] = v;
        __syncthreads();
        if (warp == 0) {
            v = lane < THREADS / 32 ? smem[lane] : T(0);
            v = warp_sum(v);
        }
        __syncthreads();
    }
    return v;
}

template <typename T>
__device__ __forceinline__ T to_mean(T sum, int64_t n) {
    return r_div(sum, (T)n);  // Java: total / axisSize with the int widened to T
}

// ---- row reduction: [rows, len] -> [rows] -------------------------------------
// TPR threads per row (32: a warp per row, 256: a CTA per row).
template <typename T, int TPR, bool VEC4>
__global__ void __launch_bounds__(256) row_reduce_kernel(const T *__restrict__ in, int64_t rows,
                                                         int64_t len, T *__restrict__ out,
                                                         int mean) {
    constexpr int ROWS_PER_CTA = 256 / TPR;
    const int sub = threadIdx.x % TPR;
    for (int64_t r0 = (int64_t)blockIdx.x * ROWS_PER_CTA; r0 < rows;
         r0 += (int64_t)gridDim.x * ROWS_PER_CTA) {
        int64_t row = r0 + threadIdx.x / TPR;
        T acc = T(0);
        if (row < rows) {
            const T *p = in + row * len;
            if (VEC4) {
                const float4 *p4 = reinterpret_cast<const float4 *>(p);
                int64_t n4 = len / 4;
                for (int64_t j = sub; j < n4; j += TPR) {
                    float4 v = __ldg(p4 + j);
                    acc = r_add(acc, r_add(r_add(v.x, v.y), r_add(v.z, v.w)));
                }
            } else {
                for (int64_t j = sub; j < len; j += TPR) acc = r_add(acc, p[j]);
            }
        }
        if (TPR == 32) {
            acc = warp_sum(acc);
            if (sub == 0 && row < rows) out[row] = mean ? to_mean(acc, len) : acc;
        } else {
            acc = block_sum<T, 256>(acc);
            if (threadIdx.x == 0 && row < rows) out[row] = mean ? to_mean(acc, len) : acc;
        }
    }
}

// ---- column reduction: [outer, axis, inner] -> [outer, inner] ------------------
// grid: x over column groups, y over outer, z over axis splits.  With
// splits > 1 the partial sums go to part[z][outer*inner].
// Column reduction (inner > 1): each thread owns VEC adjacent columns (one
// 16-byte load per row for FLOAT32) of one outer slice and sums a chunk of
// the axis with four independent accumulators per column (rows a, a+1, a+2,
// a+3), combined at the end; with more than one chunk the partial sums go to
// `part` and combine_parts_kernel adds them in chunk order.
template <typename T, int VEC>
__global__ void __launch_bounds__(256) col_reduce_kernel(const T *__restrict__ in, int64_t outer,
                                                         int64_t axis, int64_t inner,
                                                         int64_t chunk, T *__restrict__ out,
                                                         T *__restrict__ part, int mean) {
    const int64_t i = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) * VEC;
    if (i >= inner) return;
    for (int64_t o = blockIdx.y; o < outer; o += gridDim.y) {
        const int64_t a0 = blockIdx.z * chunk, a1 = std::min<int64_t>(axis, a0 + chunk);
        const T *p = in + o * axis * inner + i;
        T acc[4][VEC];
#pragma unroll
        for (int u = 0; u < 4; u++)
#pragma unroll
            for (int k = 0; k < VEC; k++) acc[u][k] = T(0);
        int64_t a = a0;
        // eight rows' loads in flight before their adds; row a+u still goes
        // to accumulator u % 4 in row order, so the sums are unchanged
        for (; a + 8 <= a1; a += 8) {
            T v[8][VEC];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                if constexpr (VEC == 4 && sizeof(T) == 4) {
                    const float4 q = __ldg(reinterpret_cast<const float4 *>(p + (a + u) * inner));
                    v[u][0] = q.x; v[u][1] = q.y; v[u][2] = q.z; v[u][3] = q.w;
                } else {
#pragma unroll
                    for (int k = 0; k < VEC; k++) v[u][k] = p[(a + u) * inner + k];
                }
            }
#pragma unroll
            for (int u = 0; u < 8; u++)
#pragma unroll
                for (int k = 0; k < VEC; k++) acc[u & 3][k] = r_add(acc[u & 3][k], v[u][k]);
        }
        for (; a + 4 <= a1; a += 4) {
#pragma unroll
            for (int u = 0; u < 4; u++) {
                T v[VEC];
                if constexpr (VEC == 4 && sizeof(T) == 4) {
                    const float4 q = __ldg(reinterpret_cast<const float4 *>(p + (a + u) * inner));
                    v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
                } else {
#pragma unroll
                    for (int k = 0; k < VEC; k++) v[k] = p[(a + u) * inner + k];
                }
#pragma unroll
                for (int k = 0; k < VEC; k++) acc[u][k] = r_add(acc[u][k], v[k]);
            }
        }
        for (; a < a1; a++)
#pragma unroll
            for (int k = 0; k < VEC; k++) acc[0][k] = r_add(acc[0][k], p[a * inner + k]);
#pragma unroll
        for (int k = 0; k < VEC; k++) {
            const T r = r_add(r_add(acc[0][k], acc[1][k]), r_add(acc[2][k], acc[3][k]));
            if (gridDim.z == 1) out[o * inner + i + k] = mean ? to_mean(r, axis) : r;
            else part[(int64_t)blockIdx.z * outer * inner + o * inner + i + k] = r;
        }
    }
}

// The launch shape of a column reduction, shared by j4c_reduce_axis and
// j4c_reduce_axis_noalloc so both add in the same order.
constexpr int kMaxColSplits = 64;  // most chunks col_plan cuts an axis into

struct ColPlan {
    int vec;
    int64_t gx, gy, splits, chunk;
};
template <typename T>
static ColPlan col_plan(const T *in, int64_t outer, int64_t axis, int64_t inner) {
    ColPlan c;
    c.vec = (sizeof(T) == 4 && inner % 4 == 0 && aligned16(in)) ? 4 : 1;
    c.gx = ceil_div(inner, 256 * c.vec);
    c.gy = std::min<int64_t>(outer, 65535);
    const int64_t ctas = c.gx * c.gy, want = (int64_t)sm_count() * 4;
    c.splits = 1;
    if (ctas < want && axis >= 64)
        c.splits = std::min<int64_t>({ceil_div(want, ctas), axis / 32, (int64_t)kMaxColSplits});
    c.chunk = ceil_div(axis, c.splits);
    c.splits = ceil_div(axis, c.chunk);
    return c;
}

template <typename T>
static void launch_col_reduce(const ColPlan &c, const T *in, int64_t outer, int64_t axis, int64_t inner, T *out,
                              T *part, int mean, cudaStream_t s) {
    dim3 grid((unsigned)c.gx, (unsigned)c.gy, (unsigned)c.splits);
    if (c.vec == 4) col_reduce_kernel<T, 4><<<grid, 256, 0, s>>>(in, outer, axis, inner, c.chunk, out, part, mean);
    else col_reduce_kernel<T, 1><<<grid, 256, 0, s>>>(in, outer, axis, inner, c.chunk, out, part, mean);
}

template <typename T>
__global__ void __launch_bounds__(256) combine_parts_kernel(const T *__restrict__ part, int splits,
                                                            int64_t n, int64_t axis,
                                                            T *__restrict__ out, int mean) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        T acc = T(0);
        if (splits <= kMaxColSplits) {
            // all the loads first (independent), then the adds in chunk order
            T v[kMaxColSplits];
#pragma unroll
            for (int s = 0; s < kMaxColSplits; s++)
                if (s < splits) v[s] = part[(int64_t)s * n + i];
#pragma unroll
            for (int s = 0; s < kMaxColSplits; s++)
                if (s < splits) acc = r_add(acc, v[s]);
        } else {
            for (int s = 0; s < splits; s++) acc = r_add(acc, part[(int64_t)s * n + i]);
        }
        out[i] = mean ? to_mean(acc, axis) : acc;
    }
}

// ---- full reduction ----------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) partial_sum_kernel(const T *__restrict__ in, int64_t n,
                                                          T *__restrict__ part) {
    T acc = T(0);
    const bool vec = sizeof(T) == 4 && (reinterpret_cast<uintptr_t>(in) & 15) == 0;
    if (vec) {
        const float4 *p4 = reinterpret_cast<const float4 *>(in);
        int64_t n4 = n / 4;
        for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < n4;
             j += (int64_t)gridDim.x * blockDim.x) {
            float4 v = __ldg(p4 + j);
            acc = r_add(acc, (T)r_add(r_add(v.x, v.y), r_add(v.z, v.w)));
        }
        int64_t t = n4 * 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
        if (t < n) acc = r_add(acc, in[t]);
    } else {
        for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < n;
             j += (int64_t)gridDim.x * blockDim.x)
            acc = r_add(acc, in[j]);
    }
    acc = block_sum<T, 256>(acc);
    if (threadIdx.x == 0) part[blockIdx.x] = acc;
}

template <typename T>
__global__ void __launch_bounds__(256) final_sum_kernel(const T *__restrict__ part, int nparts,
                                                        int64_t n, T *__restrict__ out, int mean) {
    T acc = T(0);
    for (int j = threadIdx.x; j < nparts; j += 256) acc = r_add(acc, part[j]);
    acc = block_sum<T, 256>(acc);
    if (threadIdx.x == 0) out[0] = mean ? to_mean(acc, n) : acc;
}

// ---- argmax / argmin ------------------------------------------------------------
// The reference scans sequentially and replaces the best only on a strict
// improvement (core/ConcreteNDArray.java:606-613), so: the earliest of equal
// extremes wins, a NaN never replaces the best, and a NaN in the first slot
// is never replaced.  Equivalent parallel form: if element 0 is NaN the answer
// is 0; otherwise NaNs are skipped and candidates combine by (value, -index).
template <typename T, bool MAX>
__device__ __forceinline__ bool arg_better(T v, int32_t i, T best, int32_t bi) {
    if (MAX ? v > best : v < best) return true;
    return v == best && i < bi;
}

template <typename T, bool MAX>
__device__ __forceinline__ void arg_warp(T &best, int32_t &bi) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        T v = __shfl_xor_sync(0xffffffffu, best, o);
        int32_t i = __shfl_xor_sync(0xffffffffu, bi, o);
        if (arg_better<T, MAX>(v, i, best, bi)) {
            best = v;
            bi = i;
        }
    }
}

template <typename T, bool MAX, int TPR, int VEC>
__global__ void __launch_bounds__(256) row_arg_kernel(const T *__restrict__ in, int64_t rows,
                                                      int64_t len, int32_t *__restrict__ out) {
    constexpr int ROWS_PER_CTA = 256 / TPR;
    __shared__ T sv[256 / 32];
    __shared__ int32_t si[256 / 32];
    const int sub = threadIdx.x % TPR;
    const T none = MAX ? -INFINITY : INFINITY;
    for (int64_t r0 = (int64_t)blockIdx.x * ROWS_PER_CTA; r0 < rows;
         r0 += (int64_t)gridDim.x * ROWS_PER_CTA) {
        int64_t row = r0 + threadIdx.x / TPR;
        T best = none;
        int32_t bi = INT32_MAX;
        bool first_nan = false;
        if (row < rows) {
            const T *p = in + row * len;
            first_nan = p[0] != p[0];
            // VEC consecutive elements per step (one 16-byte load when VEC > 1;
            // the launcher checks alignment and len % VEC), U steps' loads
            // issued before any is compared (more bytes in flight per thread);
            // each lane still visits its elements in increasing index order.
            constexpr int U = 4;
            constexpr int64_t STEP = (int64_t)TPR * VEC;
            for (int64_t j00 = (int64_t)sub * VEC; j00 < len; j00 += U * STEP) {
                T v[U][VEC];
#pragma unroll
                for (int u = 0; u < U; u++) {
                    const int64_t j0 = j00 + u * STEP;
                    if (j0 < len) {
                        if constexpr (VEC == 4 && sizeof(T) == 4) {
                            const float4 q = __ldg(reinterpret_cast<const float4 *>(p + j0));
                            v[u][0] = q.x; v[u][1] = q.y; v[u][2] = q.z; v[u][3] = q.w;
                        } else {
                            v[u][0] = p[j0];
                        }
                    }
                }
#pragma unroll
                for (int u = 0; u < U; u++) {
                    const int64_t j0 = j00 + u * STEP;
                    if (j0 >= len) break;
#pragma unroll
                    for (int k = 0; k < VEC; k++) {
                        if (v[u][k] == v[u][k] && arg_better<T, MAX>(v[u][k], (int32_t)(j0 + k), best, bi)) {
                            best = v[u][k];
                            bi = (int32_t)(j0 + k);
                        }
                    }
                }
            }
        }
        arg_warp<T, MAX>(best, bi);
        if (TPR == 256) {
            int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
            if (lane == 0) {
                sv[warp] = best;
                si[warp] = bi;
            }
            __syncthreads();
            if (warp == 0) {
                best = lane < 8 ? sv[lane] : none;
                bi = lane < 8 ? si[lane] : INT32_MAX;
                arg_warp<T, MAX>(best, bi);
            }
            __syncthreads();
            if (threadIdx.x == 0 && row < rows) out[row] = first_nan || bi == INT32_MAX ? 0 : bi;
        } else {
            if (sub == 0 && row < rows) out[row] = first_nan || bi == INT32_MAX ? 0 : bi;
        }
    }
}

// Columns: one thread per (outer, inner) pair runs the reference's own scan.
template <typename T, bool MAX>
__global__ void __launch_bounds__(256) col_arg_kernel(const T *__restrict__ in, int64_t outer,
                                                      int64_t axis, int64_t inner,
                                                      int32_t *__restrict__ out) {
    int64_t total = outer * inner;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        int64_t o = t / inner, i = t % inner;
        const T *p = in + o * axis * inner + i;
        int32_t bi = 0;
        T best = p[0];
        for (int64_t a = 1; a < axis; a++) {
            T v = p[a * inner];
            if (MAX ? v > best : v < best) {
                best = v;
                bi = (int32_t)a;
            }
        }
        out[t] = bi;
    }
}

// ---- host-side launchers ----------------------------------------------------------
template <typename T>
static int reduce_axis_t(const T *in, int64_t outer, int64_t axis, int64_t inner, T *out,
                         int mean, cudaStream_t s) {
    if (inner == 1) {
        bool vec4 = sizeof(T) == 4 && axis % 4 == 0 && aligned16(in);
        if (axis >= 2048) {
            unsigned g = (unsigned)std::min<int64_t>(outer, (int64_t)sm_count() * 16);
            if (vec4) row_reduce_kernel<T, 256, true><<<g, 256, 0, s>>>(in, outer, axis, out, mean);
            else row_reduce_kernel<T, 256, false><<<g, 256, 0, s>>>(in, outer, axis, out, mean);
        } else {
            unsigned g = (unsigned)std::min<int64_t>(ceil_div(outer, 8), (int64_t)sm_count() * 16);
            if (vec4) row_reduce_kernel<T, 32, true><<<g, 256, 0, s>>>(in, outer, axis, out, mean);
            else row_reduce_kernel<T, 32, false><<<g, 256, 0, s>>>(in, outer, axis, out, mean);
        }
        J4C_LAUNCH_CHECK("row_reduce_kernel");
        return J4C_OK;
    }
    // columns
    const ColPlan c = col_plan<T>(in, outer, axis, inner);
    T *part = nullptr;
    if (c.splits > 1) {
        int rc = scratch_alloc(sizeof(T) * (size_t)(c.splits * outer * inner), (void **)&part, s);
        if (rc) return rc;
    }
    launch_col_reduce<T>(c, in, outer, axis, inner, out, part, mean, s);
    J4C_LAUNCH_CHECK("col_reduce_kernel");
    if (c.splits > 1) {
        int64_t n = outer * inner;
        combine_parts_kernel<T><<<grid_for(n, 256), 256, 0, s>>>(part, (int)c.splits, n, axis, out, mean);
        J4C_LAUNCH_CHECK("combine_parts_kernel");
        return scratch_free(part, s);
    }
    return J4C_OK;
}

template <typename T>
static int reduce_all_t(const T *in, int64_t n, T *out, int mean, cudaStream_t s) {
    int nparts = (int)std::min<int64_t>(std::max<int64_t>(ceil_div(n, 256 * 16), 1),
                                        (int64_t)sm_count() * 4);
    T *part = nullptr;
    int rc = scratch_alloc(sizeof(T) * (size_t)nparts, (void **)&part, s);
    if (rc) return rc;
    partial_sum_kernel<T><<<nparts, 256, 0, s>>>(in, n, part);
    J4C_LAUNCH_CHECK("partial_sum_kernel");
    final_sum_kernel<T><<<1, 256, 0, s>>>(part, nparts, n, out, mean);
    J4C_LAUNCH_CHECK("final_sum_kernel");
    return scratch_free(part, s);
}

template <typename T, bool MAX>
static int argreduce_t(const T *in, int64_t outer, int64_t axis, int64_t inner, int32_t *out,
                       cudaStream_t s) {
    if (inner == 1) {
        constexpr int V = sizeof(T) == 4 ? 4 : 1;  // 16-byte loads for FLOAT32
        const bool v4 = V == 4 && axis % 4 == 0 && aligned16(in);
        if (axis >= 2048) {
            unsigned g = (unsigned)std::min<int64_t>(outer, (int64_t)sm_count() * 16);
            if (v4) row_arg_kernel<T, MAX, 256, V><<<g, 256, 0, s>>>(in, outer, axis, out);
            else row_arg_kernel<T, MAX, 256, 1><<<g, 256, 0, s>>>(in, outer, axis, out);
        } else {
            unsigned g = (unsigned)std::min<int64_t>(ceil_div(outer, 8), (int64_t)sm_count() * 16);
            if (v4) row_arg_kernel<T, MAX, 32, V><<<g, 256, 0, s>>>(in, outer, axis, out);
            else row_arg_kernel<T, MAX, 32, 1><<<g, 256, 0, s>>>(in, outer, axis, out);
        }
    } else {
        col_arg_kernel<T, MAX><<<grid_for(outer * inner, 256), 256, 0, s>>>(in, outer, axis, inner, out);
    }
    J4C_LAUNCH_CHECK("argreduce kernel");
    return J4C_OK;
}

int reduce_axis_any(int dtype, const void *in, int64_t outer, int64_t axis, int64_t inner,
                    void *out, int mean, cudaStream_t s) {
    if (dtype == J4C_FLOAT32)
        return reduce_axis_t<float>((const float *)in, outer, axis, inner, (float *)out, mean, s);
    if (dtype == J4C_FLOAT64)
        return reduce_axis_t<double>((const double *)in, outer, axis, inner, (double *)out, mean, s);
    return set_error(J4C_E_INVALID, "reduction requires FLOAT32 or FLOAT64 operands, got %s",
                     dtype_name(dtype));
}

int reduce_all_any(int dtype, const void *in, int64_t n, void *out, int mean, cudaStream_t s) {
    if (dtype == J4C_FLOAT32) return reduce_all_t<float>((const float *)in, n, (float *)out, mean, s);
    if (dtype == J4C_FLOAT64)
        return reduce_all_t<double>((const double *)in, n, (double *)out, mean, s);
    return set_error(J4C_E_INVALID, "reduction requires FLOAT32 or FLOAT64 operands, got %s",
                     dtype_name(dtype));
}

// ---- j4c_reduce_axis_noalloc: the same reduction with static scratch ----------------
// The only scratch a per-axis reduction needs is the partial sums of a split
// axis (splits x outer x inner values).  This array holds them for the
// allocation-free entry point.  It lives in the library's device image, so
// every GPU that loads the library keeps these bytes until the process
// exits.  Host code must not pass the symbol itself to a kernel: on the host
// it is only a stand-in, not a device address.
static __device__ __align__(256) unsigned char g_reduce_noalloc_scratch[J4C_REDUCE_NOALLOC_SCRATCH_BYTES];

// Device address of the array on the current device, looked up once per
// device (the first call on a device does this; it allocates nothing itself,
// but under lazy module loading the lookup may load the library's device
// image, whose memory -- this array included -- the driver then reserves).
static int noalloc_scratch(void **out) {
    static std::mutex mu;
    static std::vector<void *> ptrs;
    int dev = 0;
    J4C_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(mu);
    if ((int)ptrs.size() <= dev) ptrs.resize(dev + 1, nullptr);
    if (!ptrs[dev]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_reduce_noalloc_scratch);
        if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(g_reduce_noalloc_scratch)");
        ptrs[dev] = p;
    }
    *out = ptrs[dev];
    return J4C_OK;
}

// Same kernels and the same split of the axis as reduce_axis_t, so the result
// is bit-identical to j4c_reduce_axis; only the partial-sum buffer differs.
template <typename T>
static int reduce_axis_noalloc_t(const T *in, int64_t outer, int64_t axis, int64_t inner, T *out,
                                 int mean, cudaStream_t s) {
    if (inner == 1) return reduce_axis_t<T>(in, outer, axis, inner, out, mean, s);  // no scratch
    const ColPlan c = col_plan<T>(in, outer, axis, inner);
    if (c.splits == 1) return reduce_axis_t<T>(in, outer, axis, inner, out, mean, s);  // no scratch
    const int64_t splits = c.splits;
    const size_t need = sizeof(T) * (size_t)(splits * outer * inner);
    if (need > (size_t)J4C_REDUCE_NOALLOC_SCRATCH_BYTES)
        return set_error(J4C_E_INVALID,
                         "j4c_reduce_axis_noalloc: this reduction needs %zu bytes of scratch, more "
                         "than the %d-byte static maximum; call j4c_reduce_axis instead",
                         need, (int)J4C_REDUCE_NOALLOC_SCRATCH_BYTES);
    void *part = nullptr;
    int rc = noalloc_scratch(&part);
    if (rc) return rc;
    // Every partial is written before it is read, so the array's previous
    // contents never matter and nothing is cleared.
    launch_col_reduce<T>(c, in, outer, axis, inner, out, (T *)part, mean, s);
    J4C_LAUNCH_CHECK("col_reduce_kernel");
    int64_t n = outer * inner;
    combine_parts_kernel<T><<<grid_for(n, 256), 256, 0, s>>>((const T *)part, (int)splits, n, axis, out, mean);
    J4C_LAUNCH_CHECK("combine_parts_kernel");
    return J4C_OK;
}

}  // namespace j4c

using namespace j4c;

extern "C" {

int j4c_reduce_all(int prim, int dtype, const void *in, int64_t n, void *out, j4c_stream stream) {
    J4C_REQUIRE(prim == J4C_SUM || prim == J4C_MEAN, "j4c_reduce_all: primitive %d", prim);
    J4C_REQUIRE(in && out && n >= 0, "j4c_reduce_all: bad arguments");
    cudaStream_t s = as_stream(stream);
    if (n == 0) return j4c_fill(dtype, out, 1, prim == J4C_MEAN ? NAN : 0.0, stream);
    return reduce_all_any(dtype, in, n, out, prim == J4C_MEAN, s);
}

int j4c_reduce_axis(int prim, int dtype, const void *in, int64_t outer, int64_t axis_len,
                    int64_t inner, void *out, j4c_stream stream) {
    J4C_REQUIRE(prim == J4C_SUM_AXIS || prim == J4C_MEAN_AXIS, "j4c_reduce_axis: primitive %d", prim);
    J4C_REQUIRE(in && out && outer >= 0 && axis_len >= 0 && inner >= 0,
                "j4c_reduce_axis: bad arguments");
    if (outer * inner == 0) return J4C_OK;
    if (axis_len == 0)
        return j4c_fill(dtype, out, outer * inner, prim == J4C_MEAN_AXIS ? NAN : 0.0, stream);
    return reduce_axis_any(dtype, in, outer, axis_len, inner, out, prim == J4C_MEAN_AXIS,
                           as_stream(stream));
}

// See include/jax4j_cuda.h: allocation-free variant of j4c_reduce_axis.
int j4c_reduce_axis_noalloc(int prim, int dtype, const void *in, int64_t outer, int64_t axis_len,
                            int64_t inner, void *out, j4c_stream stream) {
    J4C_REQUIRE(prim == J4C_SUM_AXIS || prim == J4C_MEAN_AXIS, "j4c_reduce_axis_noalloc: primitive %d",
                prim);
    J4C_REQUIRE(in && out && outer >= 0 && axis_len >= 0 && inner >= 0,
                "j4c_reduce_axis_noalloc: bad arguments");
    if (outer * inner == 0) return J4C_OK;
    if (axis_len == 0)
        return j4c_fill(dtype, out, outer * inner, prim == J4C_MEAN_AXIS ? NAN : 0.0, stream);
    cudaStream_t s = as_stream(stream);
    const int mean = prim == J4C_MEAN_AXIS;
    if (dtype == J4C_FLOAT32)
        return reduce_axis_noalloc_t<float>((const float *)in, outer, axis_len, inner, (float *)out, mean, s);
    if (dtype == J4C_FLOAT64)
        return reduce_axis_noalloc_t<double>((const double *)in, outer, axis_len, inner, (double *)out, mean, s);
    return set_error(J4C_E_INVALID, "reduction requires FLOAT32 or FLOAT64 operands, got %s",
                     dtype_name(dtype));
}

int j4c_argreduce(int prim, int dtype, const void *in, int64_t outer, int64_t axis_len,
                  int64_t inner, int32_t *out, j4c_stream stream) {
    J4C_REQUIRE(prim == J4C_ARGMAX || prim == J4C_ARGMIN, "j4c_argreduce: primitive %d", prim);
    J4C_REQUIRE(in && out && outer >= 0 && axis_len >= 1 && inner >= 0,
                "j4c_argreduce: bad arguments (axis_len must be >= 1)");
    if (outer * inner == 0) return J4C_OK;
    cudaStream_t s = as_stream(stream);
    bool mx = prim == J4C_ARGMAX;
    if (dtype == J4C_FLOAT32)
        return mx ? argreduce_t<float, true>((const float *)in, outer, axis_len, inner, out, s)
                  : argreduce_t<float, false>((const float *)in, outer, axis_len, inner, out, s);
    if (dtype == J4C_FLOAT64)
        return mx ? argreduce_t<double, true>((const double *)in, outer, axis_len, inner, out, s)
                  : argreduce_t<double, false>((const double *)in, outer, axis_len, inner, out, s);
    return set_error(J4C_E_INVALID, "argmax/argmin requires FLOAT32 or FLOAT64 operands, got %s",
                     dtype_name(dtype));
}

// Grad.broadcastLike (api/Grad.java:539-582).
int j4c_broadcast_like(int dtype, const void *g, const int64_t *g_dims, int g_rank, void *out,
                       const int64_t *t_dims, int t_rank, j4c_stream stream) {
    J4C_REQUIRE(g && out, "j4c_broadcast_like: NULL pointer");
    J4C_REQUIRE(g_rank <= kMaxDims && t_rank <= kMaxDims, "j4c_broadcast_like: rank too large");
    J4C_REQUIRE(dtype == J4C_FLOAT32 || dtype == J4C_FLOAT64, "j4c_broadcast_like: dtype %s",
                dtype_name(dtype));
    cudaStream_t s = as_stream(stream);
    int64_t gs = shape_numel(g_dims, g_rank), ts = shape_numel(t_dims, t_rank);
    size_t es = dtype_size(dtype);
    if (gs == ts) {  // equal shapes or a pure reshape
        if (g != out) J4C_CUDA(cudaMemcpyAsync(out, g, es * (size_t)gs, cudaMemcpyDeviceToDevice, s));
        return J4C_OK;
    }
    if (ts == 0) return J4C_OK;
    if (gs < ts) {  // broadcast g out to the target
        Indexer ix;
        const int64_t *dims[1] = {g_dims};
        int ranks[1] = {g_rank};
        if (!make_indexer(ix, t_dims, t_rank, 1, dims, ranks))
            return set_error(J4C_E_INVALID, "j4c_broadcast_like: g does not broadcast to target");
        return launch_expand(dtype, ix, g, out, ts, s);
    }
    // Sum-down: the target broadcasts to g.  Classify g's dims as kept (K) or
    // reduced (R), merge runs, then reduce R groups innermost-first.
    if (t_rank > g_rank) return set_error(J4C_E_INVALID, "j4c_broadcast_like: target rank > g rank");
    std::vector<std::pair<char, int64_t>> groups;  // ('K'|'R', size)
    for (int i = 0; i < g_rank; i++) {
        int j = i - (g_rank - t_rank);
        int64_t td = j >= 0 ? t_dims[j] : 1;
        int64_t gd = g_dims[i];
        if (gd == 1) continue;
        char kind;
        if (td == gd) kind = 'K';
        else if (td == 1) kind = 'R';
        else return set_error(J4C_E_INVALID, "j4c_broadcast_like: target does not broadcast to g");
        if (!groups.empty() && groups.back().first == kind) groups.back().second *= gd;
        else groups.push_back({kind, gd});
    }
    if (groups.empty()) return set_error(J4C_E_INVALID, "j4c_broadcast_like: nothing to reduce");
    const void *cur = g;
    void *tmp = nullptr;
    int rc = J4C_OK;
    while (true) {
        int last_r = -1, nr = 0;
        for (int i = 0; i < (int)groups.size(); i++)
            if (groups[i].first == 'R') {
                last_r = i;
                nr++;
            }
        int64_t outer = 1, inner = 1;
        for (int i = 0; i < last_r; i++) outer *= groups[i].second;
        for (int i = last_r + 1; i < (int)groups.size(); i++) inner *= groups[i].second;
        int64_t axis = groups[last_r].second;
        void *dst = out;
        void *next_tmp = nullptr;
        if (nr > 1) {
            rc = scratch_alloc(es * (size_t)(outer * inner), &next_tmp, s);
            if (rc) break;
            dst = next_tmp;
        }
        rc = reduce_axis_any(dtype, cur, outer, axis, inner, dst, 0, s);
        if (tmp) scratch_free(tmp, s);
        tmp = next_tmp;
        if (rc || nr == 1) break;
        cur = dst;
        groups.erase(groups.begin() + last_r);
        // merge neighbours of the same kind
        std::vector<std::pair<char, int64_t>> merged;
        for (auto &gp : groups) {
            if (!merged.empty() && merged.back().first == gp.first) merged.back().second *= gp.second;
            else merged.push_back(gp);
        }
        groups.swap(merged);
    }
    if (tmp) scratch_free(tmp, s);
    return rc;
}

}  // extern "C"
