// dot_dmma.cu -- FLOAT64 GEMM on the FP64 tensor path (DMMA).
//
// C[M,N] = op(A)[M,K] . op(B)[K,N], op = identity or transpose, in FP64:
// the reference's FLOAT64 dot (core/ConcreteNDArray.java:452-459 in double;
// ExecutionBackend.matmul(double[]), backend/ExecutionBackend.java:50-55).
// tcgen05 has no FP64 kind, so the FP64 tensor instruction is
// mma.sync.aligned.m8n8k4.row.col.f64 (each an exact-product, fused
// 8 x 8 x 4 multiply-add per warp).  The sum of a C element is taken in
// k-groups of 4 inside the instruction and the groups in k order, so the
// result differs from a sequential FMA chain only by rounding (tests: 1e-12
// relative).
//
// Tiling: 64 x 128 CTA tile, 8 warps as 2 (M) x 4 (N) of 32 x 32 each (4 x 4
// DMMA tiles, 32 FP64 accumulators per thread), BK = 8 k-values per stage,
// two shared-memory stages filled through registers one stage ahead.  The
// operands are read as stored (row-major, or transposed for the DOT VJP).
#include "common.cuh"

namespace j4c {

namespace {

constexpr int DBM = 64, DBN = 128, DBK = 8;
constexpr int PAD = 4;  // doubles of padding per shared row: fewer bank conflicts on fragment loads

__device__ __forceinline__ void dmma_8x8x4(double (&d)[2], double a, double b) {
    asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};"
                 : "+d"(d[0]), "+d"(d[1])
                 : "d"(a), "d"(b));
}

__global__ void __launch_bounds__(256) dmma_gemm_kernel(const double *__restrict__ A, const double *__restrict__ B,
                                                        double *__restrict__ Cm, int64_t M, int64_t K, int64_t N,
                                                        int trans_a, int trans_b) {
    __shared__ double As[2][DBK][DBM + PAD];  // [k][m]
    __shared__ double Bs[2][DBK][DBN + PAD];  // [k][n]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int wm = warp >> 2, wn = warp & 3;  // warp tile origin: rows wm * 32, columns wn * 32
    const int64_t m0 = (int64_t)blockIdx.y * DBM, n0 = (int64_t)blockIdx.x * DBN;

    // stage loads: A 64 x 8 (2 per thread), B 8 x 128 (4 per thread)
    double ra[2], rb[4];
    auto load = [&](int64_t k0) {
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const int e = tid + 256 * r;
            int m, k;
            if (!trans_a) { m = e / DBK; k = e % DBK; } else { k = e / DBM; m = e % DBM; }
            const int64_t gm = m0 + m, gk = k0 + k;
            ra[r] = (gm < M && gk < K) ? (trans_a ? A[gk * M + gm] : A[gm * K + gk]) : 0.0;
        }
#pragma unroll
        for (int r = 0; r < 4; r++) {
            const int e = tid + 256 * r;
            int n, k;
            if (!trans_b) { k = e / DBN; n = e % DBN; } else { n = e / DBK; k = e % DBK; }
            const int64_t gn = n0 + n, gk = k0 + k;
            rb[r] = (gn < N && gk < K) ? (trans_b ? B[gn * K + gk] : B[gk * N + gn]) : 0.0;
        }
    };
    auto store = [&](int buf) {
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const int e = tid + 256 * r;
            int m, k;
            if (!trans_a) { m = e / DBK; k = e % DBK; } else { k = e / DBM; m = e % DBM; }
            As[buf][k][m] = ra[r];
        }
#pragma unroll
        for (int r = 0; r < 4; r++) {
            const int e = tid + 256 * r;
            int n, k;
            if (!trans_b) { k = e / DBN; n = e % DBN; } else { n = e / DBK; k = e % DBK; }
            Bs[buf][k][n] = rb[r];
        }
    };

    double acc[4][4][2];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j][0] = acc[i][j][1] = 0.0;

    // fragment coordinates (m8n8k4, row.col): A element (row lane / 4, k lane % 4),
    // B element (k lane % 4, column lane / 4), C elements (row lane / 4,
    // columns 2 (lane % 4) and 2 (lane % 4) + 1)
    const int fr = lane >> 2, fk = lane & 3;
    const int64_t ktiles = ceil_div(K, DBK);
    load(0);
    store(0);
    __syncthreads();
    for (int64_t kt = 0; kt < ktiles; kt++) {
        const int buf = (int)(kt & 1);
        if (kt + 1 < ktiles) load((kt + 1) * DBK);
#pragma unroll
        for (int kk = 0; kk < DBK; kk += 4) {
            double a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; i++) a[i] = As[buf][kk + fk][wm * 32 + i * 8 + fr];
#pragma unroll
            for (int j = 0; j < 4; j++) b[j] = Bs[buf][kk + fk][wn * 32 + j * 8 + fr];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) dmma_8x8x4(acc[i][j], a[i], b[j]);
        }
        if (kt + 1 < ktiles) store(buf ^ 1);
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int64_t gm = m0 + wm * 32 + i * 8 + fr;
        if (gm >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int64_t gn = n0 + wn * 32 + j * 8 + 2 * fk;
            if (gn < N) Cm[gm * N + gn] = acc[i][j][0];
            if (gn + 1 < N) Cm[gm * N + gn + 1] = acc[i][j][1];
        }
    }
}

}  // namespace

int dmma_gemm(const double *a, const double *b, double *c, int64_t M, int64_t K, int64_t N, int trans_a, int trans_b,
              cudaStream_t s) {
    J4C_REQUIRE(ceil_div(M, DBM) < 65536, "dot: M too large for the FP64 tensor kernel");
    dim3 grid((unsigned)ceil_div(N, DBN), (unsigned)ceil_div(M, DBM));
    dmma_gemm_kernel<<<grid, 256, 0, s>>>(a, b, c, M, K, N, trans_a, trans_b);
    J4C_LAUNCH_CHECK("dmma_gemm_kernel");
    return J4C_OK;
}

}  // namespace j4c
