// dot_simt.cu -- CUDA-core GEMM for FLOAT64 and for FLOAT32 shapes the
// tensor-core kernel does not take (it is never a host fallback).
//
// C[M,N] = op(A)[M,K] . op(B)[K,N] with op = identity or transpose, so the
// DOT VJP (api/Grad.java:385-390) reads the stored operands directly instead
// of materialising Grad.transpose (api/Grad.java:643-664).
// 128x128 CTA tile, BK = 8, 256 threads, an 8x8 register tile per thread,
// register-prefetched double buffering through shared memory.
#include "common.cuh"

namespace j4c {

template <typename T>
__global__ void __launch_bounds__(256) simt_gemm_kernel(const T *__restrict__ A,
                                                        const T *__restrict__ B, T *__restrict__ Cm,
                                                        int64_t M, int64_t K, int64_t N,
                                                        int trans_a, int trans_b) {
    constexpr int BM = 128, BN = 128, BK = 8;
    __shared__ T As[2][BK][BM];
    __shared__ T Bs[2][BK][BN];
    const int tid = threadIdx.x;
    const int tx = tid % 16, ty = tid / 16;
    const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;

    T ra[4], rb[4];
    auto load_a = [&](int64_t k0) {
#pragma unroll
        for (int r = 0; r < 4; r++) {
            int e = tid + 256 * r;
            int m, k;
            if (!trans_a) { m = e / BK; k = e % BK; } else { k = e / BM; m = e % BM; }
            int64_t gm = m0 + m, gk = k0 + k;
            T v = T(0);
            if (gm < M && gk < K) v = trans_a ? A[gk * M + gm] : A[gm * K + gk];
            ra[r] = v;
        }
    };
    auto load_b = [&](int64_t k0) {
#pragma unroll
        for (int r = 0; r < 4; r++) {
            int e = tid + 256 * r;
            int n, k;
            if (!trans_b) { k = e / BN; n = e % BN; } else { n = e / BK; k = e % BK; }
            int64_t gn = n0 + n, gk = k0 + k;
            T v = T(0);
            if (gn < N && gk < K) v = trans_b ? B[gn * K + gk] : B[gk * N + gn];
            rb[r] = v;
        }
    };
    auto store = [&](int buf) {
#pragma unroll
        for (int r = 0; r < 4; r++) {
            int e = tid + 256 * r;
            int m, k;
            if (!trans_a) { m = e / BK; k = e % BK; } else { k = e / BM; m = e % BM; }
            As[buf][k][m] = ra[r];
            int n, kb;
            if (!trans_b) { kb = e / BN; n = e % BN; } else { n = e / BK; kb = e % BK; }
            Bs[buf][kb][n] = rb[r];
        }
    };

    T acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = T(0);

    const int64_t ktiles = ceil_div(K, BK);
    load_a(0);
    load_b(0);
    store(0);
    __syncthreads();
    for (int64_t kt = 0; kt < ktiles; kt++) {
        int buf = (int)(kt & 1);
        if (kt + 1 < ktiles) {
            load_a((kt + 1) * BK);
            load_b((kt + 1) * BK);
        }
#pragma unroll
        for (int k = 0; k < BK; k++) {
            T av[8], bv[8];
#pragma unroll
            for (int i = 0; i < 8; i++) av[i] = As[buf][k][ty + 16 * i];
#pragma unroll
            for (int j = 0; j < 8; j++) bv[j] = Bs[buf][k][tx + 16 * j];
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) acc[i][j] = fma(av[i], bv[j], acc[i][j]);
        }
        if (kt + 1 < ktiles) store(buf ^ 1);
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 8; i++) {
        int64_t gm = m0 + ty + 16 * i;
        if (gm >= M) continue;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            int64_t gn = n0 + tx + 16 * j;
            if (gn < N) Cm[gm * N + gn] = acc[i][j];
        }
    }
}

int simt_gemm(int dtype, const void *a, const void *b, void *c, int64_t M, int64_t K, int64_t N,
              int trans_a, int trans_b, cudaStream_t s) {
    J4C_REQUIRE(ceil_div(M, 128) < 65536, "dot: M too large for the CUDA-core kernel");
    dim3 grid((unsigned)ceil_div(N, 128), (unsigned)ceil_div(M, 128));
    if (dtype == J4C_FLOAT32)
        simt_gemm_kernel<float><<<grid, 256, 0, s>>>((const float *)a, (const float *)b, (float *)c,
                                                      M, K, N, trans_a, trans_b);
    else
        simt_gemm_kernel<double><<<grid, 256, 0, s>>>((const double *)a, (const double *)b,
                                                       (double *)c, M, K, N, trans_a, trans_b);
    J4C_LAUNCH_CHECK("simt_gemm_kernel");
    return J4C_OK;
}

}  // namespace j4c
