// common.cuh -- shared helpers of libjax4j_cuda.so: status/error reporting,
// dtype dispatch, launch geometry and the Java arithmetic rules the kernels
// must reproduce (java.lang.Math.max/min, JLS 5.1.3 narrowing casts).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/jax4j_cuda.h"

namespace j4c {

constexpr int kMaxDims = 8;

// ---- status / last error ---------------------------------------------------
int set_error(int code, const char *fmt, ...);
void clear_error();
int cuda_status(cudaError_t e, const char *what);
void count_launch();

#define J4C_CUDA(expr)                                                   \
    do {                                                                 \
        cudaError_t _e = (expr);                                         \
        if (_e != cudaSuccess) return ::j4c::cuda_status(_e, #expr);     \
    } while (0)

// Every kernel launch site ends with this check; it also counts launches
// (j4c_kernel_launches) so callers can report how many kernels ran.
#define J4C_LAUNCH_CHECK(what)                                           \
    do {                                                                 \
        ::j4c::count_launch();                                           \
        cudaError_t _e = cudaGetLastError();                             \
        if (_e != cudaSuccess) return ::j4c::cuda_status(_e, what);      \
    } while (0)

#define J4C_REQUIRE(cond, ...)                                           \
    do {                                                                 \
        if (!(cond)) return ::j4c::set_error(J4C_E_INVALID, __VA_ARGS__); \
    } while (0)

// ---- device properties -----------------------------------------------------
int sm_count();  // SMs of the current device (cached per device)
inline cudaStream_t as_stream(j4c_stream s) { return reinterpret_cast<cudaStream_t>(s); }

// Stream-ordered scratch from the device pool (released with scratch_free).
int scratch_alloc(size_t bytes, void **out, cudaStream_t s);
int scratch_free(void *p, cudaStream_t s);

// Device status word (one int per device, allocated on first use): kernels
// that give up a bounded wait or reject their input record a code there
// instead of trapping; j4c_device_status reads and clears it.  Returns NULL
// if the word cannot be allocated.
int *device_status_ptr();

// The limit, in ns without progress, after which a pipeline wait of a
// persistent kernel gives up and records its status (j4c_set_wait_limit_ns;
// 2 s unless set).
uint64_t wait_limit_ns();

inline size_t dtype_size(int dtype) {
    switch (dtype) {
    case J4C_FLOAT32: return 4;
    case J4C_FLOAT64: return 8;
    case J4C_INT32: return 4;
    case J4C_INT64: return 8;
    case J4C_BOOL: return 1;
    default: return 0;
    }
}

inline const char *dtype_name(int dtype) {
    switch (dtype) {
    case J4C_FLOAT32: return "float32";
    case J4C_FLOAT64: return "float64";
    case J4C_INT32: return "int32";
    case J4C_INT64: return "int64";
    case J4C_BOOL: return "bool";
    default: return "?";
    }
}

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Grid size for a grid-stride elementwise kernel: enough CTAs to fill every
// SM several times over, never more than the work needs.
inline unsigned grid_for(int64_t work_items, int threads, int waves = 8) {
    int64_t need = ceil_div(work_items, threads);
    int64_t cap = (int64_t)sm_count() * waves;
    if (need < 1) need = 1;
    return (unsigned)(need < cap ? need : cap);
}

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---- Java arithmetic rules ---------------------------------------------------
// java.lang.Math.max(double,double): NaN if either is NaN, max(-0,+0)=+0.
template <typename T>
__device__ __forceinline__ T java_max(T a, T b) {
    if (a != a) return a;
    if (a == T(0) && b == T(0) && signbit(a)) return b;
    return (a >= b) ? a : b;
}
// java.lang.Math.min(double,double): NaN if either is NaN, min(+0,-0)=-0.
template <typename T>
__device__ __forceinline__ T java_min(T a, T b) {
    if (a != a) return a;
    if (a == T(0) && b == T(0) && signbit(b)) return b;
    return (a <= b) ? a : b;
}

// IEEE round-to-nearest arithmetic without contraction into FMA.
__device__ __forceinline__ float r_add(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float r_sub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float r_mul(float a, float b) { return __fmul_rn(a, b); }
// IEEE division.  A zero dividend over a non-zero, non-NaN divisor (an
// infinity included) is a zero whose sign is the XOR of the operands' signs;
// that case is answered directly (gradients through a division are mostly
// zeros, e.g. a one-hot target's log-softmax VJP), everything else is the
// correctly rounded quotient.
__device__ __forceinline__ float r_div(float a, float b) {
    if (a == 0.0f && b == b && b != 0.0f)
        return __int_as_float((__float_as_int(a) ^ __float_as_int(b)) & (int)0x80000000);
    return __fdiv_rn(a, b);
}
__device__ __forceinline__ double r_add(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double r_sub(double a, double b) { return __dsub_rn(a, b); }
__device__ __forceinline__ double r_mul(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ double r_div(double a, double b) { return __ddiv_rn(a, b); }

// JLS 5.1.3 narrowing of a floating value: NaN -> 0, saturate, truncate.
__device__ __forceinline__ int32_t java_d2i(double v) {
    if (v != v) return 0;
    if (v >= 2147483647.0) return INT32_MAX;
    if (v <= -2147483648.0) return INT32_MIN;
    return (int32_t)v;
}
__device__ __forceinline__ int64_t java_d2l(double v) {
    if (v != v) return 0;
    if (v >= 9223372036854775807.0) return INT64_MAX;
    if (v <= -9223372036854775808.0) return INT64_MIN;
    return (int64_t)v;
}

// ---- broadcast indexing ------------------------------------------------------
// Output shape collapsed to at most kMaxDims dims, with per-operand element
// strides (0 along broadcast dims).  Adjacent dims merge when every operand
// is contiguous (or uniformly broadcast) across them.
struct Indexer {
    int rank;
    int nops;
    int64_t size[kMaxDims];
    int64_t stride[3][kMaxDims];
};

// Builds an Indexer for out_dims with up to three operands; returns false if
// the operand shapes do not broadcast to out_dims.
bool make_indexer(Indexer &ix, const int64_t *out_dims, int out_rank, int nops,
                  const int64_t *const *op_dims, const int *op_ranks);

// Broadcast shape of two shapes (core/Shape.java:37-49); false if incompatible.
bool broadcast_shape(const int64_t *a, int ar, const int64_t *b, int br, int64_t *out,
                     int *orank);
int64_t shape_numel(const int64_t *d, int r);

__device__ __forceinline__ void index_offsets(const Indexer &ix, int64_t flat, int64_t *off) {
    // ix.rank >= 1; the innermost dimension is last.
    int64_t o0 = 0, o1 = 0, o2 = 0;
#pragma unroll
    for (int d = kMaxDims - 1; d >= 0; d--) {
        if (d < ix.rank) {
            int64_t sz = ix.size[d];
            int64_t c = (d == 0) ? flat : flat % sz;
            flat = (d == 0) ? 0 : flat / sz;
            o0 += c * ix.stride[0][d];
            o1 += c * ix.stride[1][d];
            o2 += c * ix.stride[2][d];
        }
    }
    off[0] = o0;
    off[1] = o1;
    off[2] = o2;
}

}  // namespace j4c
