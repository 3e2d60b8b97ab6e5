// dot_tcgen05.cu -- FP32 GEMM on the B200's 5th-generation tensor cores.
//
// C[M,N] = op(A)[M,K] . op(B)[K,N] in FP32 accuracy from TF32 tensor-core
// products (the "3xTF32" split): every operand x is split as
//     hi = tf32_round(x),  lo = tf32_round(x - hi)      (x - hi is exact)
// and  a.b ~= lo_a.hi_b + hi_a.lo_b + hi_a.hi_b, accumulated in FP32 in
// tensor memory (TMEM).  The dropped lo_a.lo_b term and the TF32 rounding
// of lo are ~2^-22 relative, so the result matches an FP32 dot to within
// the reordering of its sum (the reference's dot is a sequential FP32 sum,
// core/ConcreteNDArray.java:452-459; backend/HostBackend.java:56-66).
//
// Pipeline:
//  1. split pass (HBM-bound): op(A) and op(B) are written K-major as hi/lo
//     pairs [rows, Kp] (Kp = K rounded up to 32, zero padded); a transposed
//     operand (the DOT VJP's A^T / B^T, api/Grad.java:385-390) is transposed
//     on the way through shared memory, so the GEMM sees one layout.
//  2. GEMM: a persistent kernel, one CTA per SM, three warp roles:
//     warp 0 lane 0 issues TMA loads (cp.async.bulk.tensor, 128B swizzle)
//     into a STAGES-deep shared-memory ring; warp 1 lane 0 issues
//     tcgen05.mma.kind::tf32 (M=128, N=BN, K=8) and tcgen05.commit's the
//     ring slots back; warps 2..9 accumulate and store C.
//  Promotion: the tensor core's FP32 accumulation does not round to nearest,
//  so its error grows linearly with the number of accumulating MMAs.  The
//  K loop is therefore cut into chunks of CHUNK_KB k-blocks; each chunk's
//  partial product goes to one of two TMEM buffers, and the epilogue warps
//  add it into FP32 registers with round-to-nearest while the MMA warp
//  fills the other buffer.  The error then grows with sqrt(K) like an FP32
//  sum.
//  Every mbarrier wait is bounded: after kWaitLimitNs without progress the
//  kernel records J4C status kStatusTimeout, stops all roles, waits
//  (bounded) for its own TMA and MMA work in flight, frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace j4c {
namespace tc {

constexpr int BM = 128;           // rows of a CTA tile (TMEM lanes)
constexpr int KPAD = 32;          // K is zero-padded to a multiple of this in the split
constexpr int UMMA_K = 8;         // K of one tf32 MMA instruction (32 bytes)
constexpr int CHUNK_K = 256;      // K accumulated in TMEM before promotion to registers
constexpr int kEpiWarps = 8;      // two warps per TMEM lane quadrant
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kStatusTimeout = 0x7C05;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s without progress

// BK = FP32 elements per smem row of a stage: 32 (128-byte swizzle) or 16
// (64-byte swizzle, half the bytes per stage, so twice the stages fit).
template <int BN, int STAGES, int BK>
struct Cfg {
    static_assert(BK == 32 || BK == 16, "BK is 32 (SW128) or 16 (SW64)");
    static constexpr int CHUNK_KB = CHUNK_K / BK;
    static constexpr int A_BYTES = BM * BK * 4;
    static constexpr int B_BYTES = BN * BK * 4;
    static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
    static constexpr int TMEM_COLS = 2 * BN;  // two partial-sum buffers
    static constexpr int COLS_PER_WARP = BN / 2;  // each epilogue warp owns half the columns
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
    static_assert(TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM allocation must be a power of 2");
    static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

template <int STAGES>
struct Ctl {
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    uint64_t tfull[2];
    uint64_t tempty[2];
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
};

// ---- PTX wrappers ----------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity; false if the CTA is aborting or
// no progress was seen for kWaitLimitNs (then records the status and aborts).
__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, volatile int *abort,
                                         int *status, bool honour_abort = true) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = now_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63) == 0) {
            if (honour_abort && *abort) return false;
            if (now_ns() - t0 > kWaitLimitNs) {
                *abort = 1;
                if (status) atomicCAS(status, 0, kStatusTimeout);
                return false;
            }
        }
    }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// K-major operand tile with a BK*4-byte swizzle: 8-row core-matrix groups are
// 8 rows * row bytes apart (SBO); the leading-dimension offset is unused for
// swizzled K-major.  Layout type 2 = 128-byte swizzle, 4 = 64-byte swizzle.
template <int BK>
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
    constexpr uint64_t row_bytes = BK * 4;
    constexpr uint64_t layout = BK == 32 ? 2 : 4;
    uint64_t d = 0;
    d |= (uint64_t)((addr & 0x3FFFF) >> 4);
    d |= (uint64_t)1 << 16;                      // LBO (unused here)
    d |= (uint64_t)((8 * row_bytes) >> 4) << 32; // SBO
    d |= (uint64_t)1 << 46;                      // descriptor version for sm_100
    d |= layout << 61;
    return d;
}

// kind::tf32 instruction descriptor: D f32, A/B tf32, both K-major.
__host__ __device__ constexpr uint32_t idesc_tf32(int m, int n) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Grouped raster: 8 M-tiles share each run of N-tiles so operand tiles are
// reused out of L2 by CTAs running at the same time.
__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int &mt, int &nt) {
    constexpr int G = 8;
    const int per_group = G * num_n;
    const int first_m = (t / per_group) * G;
    const int gsize = min(G, num_m - first_m);
    const int r = t % per_group;
    mt = first_m + r % gsize;
    nt = r / gsize;
}

template <int BN, int STAGES, int BK>
__global__ void __launch_bounds__(kThreads, 1)
gemm_3xtf32_kernel(const __grid_constant__ CUtensorMap tAh, const __grid_constant__ CUtensorMap tAl,
                   const __grid_constant__ CUtensorMap tBh, const __grid_constant__ CUtensorMap tBl,
                   float *__restrict__ C, int M, int N, int num_kb, int vec_store, int *status) {
    using Q = Cfg<BN, STAGES, BK>;
    constexpr int CHUNK_KB = Q::CHUNK_KB;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Ctl<STAGES> *ctl = reinterpret_cast<Ctl<STAGES> *>(smem + STAGES * Q::STAGE_BYTES);
    volatile int *abort = &ctl->abort;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int num_m = (M + BM - 1) / BM, num_n = (N + BN - 1) / BN;
    const int num_tiles = num_m * num_n;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(smem_u32(&ctl->full[s]), 1);
            mbar_init(smem_u32(&ctl->empty[s]), 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(smem_u32(&ctl->tfull[b]), 1);
            mbar_init(smem_u32(&ctl->tempty[b]), kEpiWarps);
        }
        mbar_init(smem_u32(&ctl->drain), 1);
        ctl->abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&ctl->tmem_base)),
                     "r"(Q::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int issued = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < num_tiles; t += gridDim.x) {
                int mt, nt;
                tile_coords(t, num_m, num_n, mt, nt);
                for (int kb = 0; kb < num_kb; kb++) {
                    if (!wait_bar(smem_u32(&ctl->empty[stage]), phase ^ 1, abort, status)) {
                        ok = false;
                        break;
                    }
                    const uint32_t sb = smem_u32(smem + stage * Q::STAGE_BYTES);
                    const uint32_t fb = smem_u32(&ctl->full[stage]);
                    mbar_expect_tx(fb, Q::STAGE_BYTES);
                    const int kx = kb * BK;
                    tma_load_2d(sb, &tAh, kx, mt * BM, fb);
                    tma_load_2d(sb + Q::A_BYTES, &tAl, kx, mt * BM, fb);
                    tma_load_2d(sb + 2 * Q::A_BYTES, &tBh, kx, nt * BN, fb);
                    tma_load_2d(sb + 2 * Q::A_BYTES + Q::B_BYTES, &tBl, kx, nt * BN, fb);
                    issued++;
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            // Every load this thread issued must land before the CTA exits:
            // wait (bounded, even when aborting) on the last STAGES slots.
            for (int i = 0; i < STAGES && i < issued; i++) {
                if (--stage < 0) {
                    stage = STAGES - 1;
                    phase ^= 1;
                }
                wait_bar(smem_u32(&ctl->full[stage]), phase, abort, status, false);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_tf32(BM, BN);
            int stage = 0;
            uint32_t phase = 0;
            int ci = 0;  // chunk counter across tiles: selects the TMEM buffer
            bool ok = true;
            for (int t = blockIdx.x; ok && t < num_tiles; t += gridDim.x) {
                for (int kb0 = 0; ok && kb0 < num_kb; kb0 += CHUNK_KB, ci++) {
                    const int buf = ci & 1;
                    const uint32_t bph = (ci >> 1) & 1;
                    if (!wait_bar(smem_u32(&ctl->tempty[buf]), bph ^ 1, abort, status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t dcol = tmem + buf * BN;
                    const int kb1 = min(num_kb, kb0 + CHUNK_KB);
                    for (int kb = kb0; kb < kb1; kb++) {
                        if (!wait_bar(smem_u32(&ctl->full[stage]), phase, abort, status)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t sa_hi = smem_u32(smem + stage * Q::STAGE_BYTES);
                        const uint32_t sa_lo = sa_hi + Q::A_BYTES;
                        const uint32_t sb_hi = sa_hi + 2 * Q::A_BYTES;
                        const uint32_t sb_lo = sb_hi + Q::B_BYTES;
#pragma unroll
                        for (int kk = 0; kk < BK / UMMA_K; kk++) {
                            const uint32_t off = kk * UMMA_K * 4;
                            const uint64_t ah = smem_desc<BK>(sa_hi + off), al = smem_desc<BK>(sa_lo + off);
                            const uint64_t bh = smem_desc<BK>(sb_hi + off), bl = smem_desc<BK>(sb_lo + off);
                            mma_tf32(dcol, al, bh, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
                            mma_tf32(dcol, ah, bl, idesc, 1u);
                            mma_tf32(dcol, ah, bh, idesc, 1u);
                        }
                        mma_commit(smem_u32(&ctl->empty[stage]));
                        if (++stage == STAGES) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                    if (!ok) break;
                    mma_commit(smem_u32(&ctl->tfull[buf]));
                }
            }
            // All MMAs this thread issued complete before TMEM is released.
            mma_commit(smem_u32(&ctl->drain));
            wait_bar(smem_u32(&ctl->drain), 0, abort, status, false);
        }
    } else {
        // ---------------- epilogue: promote partials, store C ----------------
        const int ew = warp - 2;
        const int q = warp & 3;                      // TMEM lane quadrant this warp may access
        const int half = ew >> 2;                    // which half of the BN columns
        const int cbase = half * Q::COLS_PER_WARP;
        const uint32_t lane_off = (uint32_t)(q * 32) << 16;
        int ci = 0;
        bool ok = true;
        for (int t = blockIdx.x; ok && t < num_tiles; t += gridDim.x) {
            int mt, nt;
            tile_coords(t, num_m, num_n, mt, nt);
            float acc[Q::COLS_PER_WARP];
#pragma unroll
            for (int j = 0; j < Q::COLS_PER_WARP; j++) acc[j] = 0.0f;
            for (int kb0 = 0; kb0 < num_kb; kb0 += CHUNK_KB, ci++) {
                const int buf = ci & 1;
                const uint32_t bph = (ci >> 1) & 1;
                if (!wait_bar(smem_u32(&ctl->tfull[buf]), bph, abort, status)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < Q::COLS_PER_WARP / 32; c++) {
                    uint32_t r[32];
                    tmem_ld32(tmem + (uint32_t)(buf * BN + cbase + c * 32) + lane_off, r);
#pragma unroll
                    for (int j = 0; j < 32; j++) acc[c * 32 + j] = __fadd_rn(acc[c * 32 + j], __uint_as_float(r[j]));
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&ctl->tempty[buf]));
            }
            if (!ok) break;
            const int row = mt * BM + q * 32 + lane;
            const int col0 = nt * BN + cbase;
            if (row < M && col0 < N) {
                float *crow = C + (size_t)row * (size_t)N + col0;
                if (vec_store && col0 + Q::COLS_PER_WARP <= N) {
                    float4 *dst = reinterpret_cast<float4 *>(crow);
#pragma unroll
                    for (int v = 0; v < Q::COLS_PER_WARP / 4; v++)
                        dst[v] = make_float4(acc[4 * v], acc[4 * v + 1], acc[4 * v + 2], acc[4 * v + 3]);
                } else {
#pragma unroll
                    for (int j = 0; j < Q::COLS_PER_WARP; j++)
                        if (col0 + j < N) crow[j] = acc[j];
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        __syncwarp();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Q::TMEM_COLS)
                     : "memory");
    }
}

// ---- operand split: op(X) -> K-major hi/lo pairs [rows, Kp] ---------------------------
__device__ __forceinline__ float tf32_round(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r & 0xFFFFE000u);
}

// Direct operand ([rows, K] row-major): 4 consecutive k per thread step,
// 16-byte loads when K allows, 16-byte stores of hi and lo (Kp % 4 == 0).
__global__ void __launch_bounds__(256) split_direct_kernel(const float *__restrict__ src, int64_t rows,
                                                           int64_t K, int64_t Kp, int vec,
                                                           float *__restrict__ hi,
                                                           float *__restrict__ lo) {
    const int64_t q = Kp / 4;
    const int64_t n = rows * q;
    for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < n;
         v += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = v / q, k = (v - r * q) * 4;
        float x[4];
        const float *p = src + r * K + k;
        if (vec && k + 4 <= K) {
            const float4 t = __ldg(reinterpret_cast<const float4 *>(p));
            x[0] = t.x; x[1] = t.y; x[2] = t.z; x[3] = t.w;
        } else {
#pragma unroll
            for (int j = 0; j < 4; j++) x[j] = (k + j < K) ? p[j] : 0.0f;
        }
        float h[4], l[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            h[j] = tf32_round(x[j]);
            l[j] = tf32_round(x[j] - h[j]);
        }
        *reinterpret_cast<float4 *>(hi + r * Kp + k) = make_float4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<float4 *>(lo + r * Kp + k) = make_float4(l[0], l[1], l[2], l[3]);
    }
}

// Transposed operand (stored [K, rows] row-major): 64 x 64 tiles through
// shared memory, reads coalesced along rows, writes coalesced along k.
__global__ void __launch_bounds__(256) split_transpose_kernel(const float *__restrict__ src, int64_t rows,
                                                              int64_t K, int64_t Kp,
                                                              float *__restrict__ hi,
                                                              float *__restrict__ lo) {
    __shared__ float tile[64][65];
    const int64_t k0 = (int64_t)blockIdx.x * 64, r0 = (int64_t)blockIdx.y * 64;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
    for (int j = ty; j < 64; j += 8) {  // tile[r][k] <- src[k][r]
        const int64_t k = k0 + j;
        for (int i = tx; i < 64; i += 32) {
            const int64_t r = r0 + i;
            tile[i][j] = (r < rows && k < K) ? src[k * rows + r] : 0.0f;
        }
    }
    __syncthreads();
    for (int j = ty; j < 64; j += 8) {
        const int64_t r = r0 + j;
        if (r >= rows) continue;
        for (int i = tx; i < 64; i += 32) {
            const int64_t k = k0 + i;
            if (k < Kp) {
                const float x = tile[j][i];
                const float h = tf32_round(x);
                hi[r * Kp + k] = h;
                lo[r * Kp + k] = tf32_round(x - h);
            }
        }
    }
}

// ---- host side -------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

static int make_map(CUtensorMap *map, const float *base, int64_t rows, int64_t Kp, int box_rows, int bk) {
    auto fn = encode_fn();
    if (!fn) return set_error(J4C_E_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[2] = {(cuuint64_t)Kp, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)Kp * 4};
    cuuint32_t box[2] = {(cuuint32_t)bk, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), dims, strides, box,
                    estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    bk == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(J4C_E_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return J4C_OK;
}

template <int BN, int STAGES, int BK>
static int launch_gemm(const float *ah, const float *al, const float *bh, const float *bl, float *c,
                       int64_t M, int64_t N, int64_t Kp, cudaStream_t s) {
    using Q = Cfg<BN, STAGES, BK>;
    static std::mutex mu;
    static std::vector<char> configured;
    int dev = 0;
    J4C_CUDA(cudaGetDevice(&dev));
    {
        std::lock_guard<std::mutex> lock(mu);
        if ((int)configured.size() <= dev) configured.resize(dev + 1, 0);
        if (!configured[dev]) {
            J4C_CUDA(cudaFuncSetAttribute(gemm_3xtf32_kernel<BN, STAGES, BK>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, Q::SMEM_BYTES));
            configured[dev] = 1;
        }
    }
    CUtensorMap mAh, mAl, mBh, mBl;
    int rc;
    if ((rc = make_map(&mAh, ah, M, Kp, BM, BK)) || (rc = make_map(&mAl, al, M, Kp, BM, BK)) ||
        (rc = make_map(&mBh, bh, N, Kp, BN, BK)) || (rc = make_map(&mBl, bl, N, Kp, BN, BK)))
        return rc;
    int *status = device_status_ptr();
    if (!status) return set_error(J4C_E_OOM, "no device status word");
    const int64_t tiles = ceil_div(M, BM) * ceil_div(N, BN);
    const int grid = (int)std::min<int64_t>(tiles, sm_count());
    const int vec = (N % 4 == 0) && aligned16(c);
    gemm_3xtf32_kernel<BN, STAGES, BK><<<grid, kThreads, Q::SMEM_BYTES, s>>>(
        mAh, mAl, mBh, mBl, c, (int)M, (int)N, (int)(Kp / BK), vec, status);
    J4C_LAUNCH_CHECK("gemm_3xtf32_kernel");
    return J4C_OK;
}

static int launch_split(const float *src, int64_t rows, int64_t K, int64_t Kp, int kr, float *hi,
                        float *lo, cudaStream_t s) {
    if (!kr) {
        const int vec = (K % 4 == 0) && aligned16(src);
        split_direct_kernel<<<grid_for(rows * (Kp / 4), 256), 256, 0, s>>>(src, rows, K, Kp, vec, hi, lo);
        J4C_LAUNCH_CHECK("split_direct_kernel");
    } else {
        dim3 grid((unsigned)ceil_div(Kp, 64), (unsigned)ceil_div(rows, 64));
        split_transpose_kernel<<<grid, 256, 0, s>>>(src, rows, K, Kp, hi, lo);
        J4C_LAUNCH_CHECK("split_transpose_kernel");
    }
    return J4C_OK;
}

}  // namespace tc

bool tc_gemm_supported(int64_t M, int64_t K, int64_t N) {
    // int32 coordinates/extents in the kernel and the split grid's y limit
    return M >= 1 && N >= 1 && K >= 1 && M < (1ll << 31) && N < (1ll << 31) &&
           ceil_div(M, 64) < 65536 && ceil_div(N, 64) < 65536 && K < (1ll << 30);
}

int tc_gemm_workspace(int64_t M, int64_t K, int64_t N, size_t *bytes) {
    const int64_t Kp = ceil_div(K, tc::KPAD) * tc::KPAD;
    *bytes = (size_t)(M + N) * (size_t)Kp * 2 * sizeof(float);
    return J4C_OK;
}

int tc_gemm_f32(const float *a, const float *b, float *c, int64_t M, int64_t K, int64_t N,
                int trans_a, int trans_b, void *ws, size_t ws_bytes, cudaStream_t s) {
    const int64_t Kp = ceil_div(K, tc::KPAD) * tc::KPAD;
    float *ah = static_cast<float *>(ws);
    float *al = ah + M * Kp;
    float *bh = al + M * Kp;
    float *bl = bh + N * Kp;
    J4C_REQUIRE(aligned16(ws), "dot: workspace must be 16-byte aligned");
    int rc;
    // op(A) = A [M,K] (trans_a = 0) or A^T with A stored [K,M]
    if ((rc = tc::launch_split(a, M, K, Kp, trans_a ? 1 : 0, ah, al, s))) return rc;
    // op(B) = B [K,N]: the GEMM wants it K-major [N,K]
    if ((rc = tc::launch_split(b, N, K, Kp, trans_b ? 0 : 1, bh, bl, s))) return rc;
    static const int variant = [] {
        const char *v = getenv("J4C_GEMM_VARIANT");
        return v ? atoi(v) : 1;
    }();
    if (variant == 0) return tc::launch_gemm<256, 2, 32>(ah, al, bh, bl, c, M, N, Kp, s);
    return tc::launch_gemm<256, 4, 16>(ah, al, bh, bl, c, M, N, Kp, s);
}

}  // namespace j4c
