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
//  1. split pass (HBM-bound): each operand is split elementwise in its own
//     row-major layout into hi/lo arrays whose rows are padded to a multiple
//     of 4 floats (16-byte TMA strides).  No transpose is needed: the GEMM
//     reads an operand K-major (K contiguous) or MN-major (M or N
//     contiguous, the DOT VJP's A^T / B^T, api/Grad.java:385-390) as it lies,
//     so one split of a tensor serves all the products it takes part in.
//  2. GEMM: a persistent kernel, one CTA per SM, three warp roles:
//     warp 0 lane 0 issues TMA loads (cp.async.bulk.tensor; K-major tiles
//     with a BK*4-byte swizzle, MN-major tiles as 32-float-wide column
//     blocks in the 128-byte/32-byte-atom swizzle) into a STAGES-deep
//     shared-memory ring; warp 1 lane 0 issues
//     tcgen05.mma.kind::tf32 (M=128, N=BN, K=8) and tcgen05.commit's the
//     ring slots back; warps 2..9 accumulate and store C.
//  Promotion: the tensor core's FP32 accumulation does not round to nearest,
//  so its error grows linearly with the number of accumulating MMAs.  The
//  K loop is therefore cut into chunks of CHUNK_KB k-blocks; each chunk's
//  partial product goes to one of two TMEM buffers, and the epilogue warps
//  add it into FP32 registers with round-to-nearest while the MMA warp
//  fills the other buffer.  The error then grows with sqrt(K) like an FP32
//  sum.
//  Split mode 3xFP16 (the default; J4C_GEMM_SPLIT=tf32 selects 3xTF32): the same three products from
//  FP16 operands, at twice the tensor rate of TF32.  FP16 has TF32's 11-bit
//  significand but a 5-bit exponent, so every operand is first scaled by a
//  power of two 2^e chosen from its largest finite magnitude (max |x| 2^e in
//  [2^14, 2^15)): hi = fp16(x 2^e), lo = fp16(x 2^e - hi), stored as 2-byte
//  halves with the max in a word after the hi array, and the
//  epilogue multiplies the accumulator by 2^-(e_a + e_b) (exact).  Elements
//  below 2^-24 of the tensor's max lose digits (FP16 subnormals): an
//  absolute error of at most ~2^-38 max |x| per element, on top of the
//  2^-22 relative error of the split.
//  Every mbarrier wait is bounded: after kWaitLimitNs without progress the
//  kernel records J4C status kStatusTimeout, stops all roles, waits
//  (bounded) for its own TMA and MMA work in flight, frees TMEM and returns.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace j4c {
namespace tc {

constexpr int BM = 128;           // rows of a CTA tile (TMEM lanes)
constexpr int CHUNK_K = 256;      // K accumulated in TMEM before promotion (3xTF32; 512 for 3xFP16)
constexpr int kEpiWarps = 8;      // two warps per TMEM lane quadrant
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kStatusTimeout = 0x7C05;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s without progress
constexpr int kMaxTailSplits = 4; // parts along K of a tile of the last wave

// Operand element of a split mode: 3xTF32 (4-byte tf32 values) or 3xFP16.
template <bool F16>
struct Elt {
    static constexpr int SIZE = F16 ? 2 : 4;     // bytes per element
    static constexpr int UMMA_K = F16 ? 16 : 8;  // K of one MMA instruction (32 bytes either way)
    static constexpr int MNW = F16 ? 64 : 32;    // MN-major tiles: elements per 128-byte swizzle row
};

// BK = 32-bit words per smem row of a stage: 32 (128-byte swizzle) or 16
// (64-byte swizzle, half the bytes per stage, so twice the stages fit);
// BKE = the K elements those bytes hold.
template <int BN, int STAGES, int BK, bool F16 = false>
struct Cfg {
    static_assert(BK == 32 || BK == 16, "BK is 32 (SW128) or 16 (SW64)");
    static constexpr int BKE = BK * 4 / Elt<F16>::SIZE;
    // FP16 MMAs take half the time of TF32 ones per K, so the FP16 chunk is
    // twice as deep: the same number of MMAs accumulate in TMEM either way,
    // and the epilogue keeps a chunk's worth of MMA time to store a tile.
    static constexpr int CHUNK_KB = (F16 ? 2 * CHUNK_K : CHUNK_K) / BKE;
    static constexpr int A_BYTES = BM * BK * 4;
    static constexpr int B_BYTES = BN * BK * 4;
    static constexpr int MN_BOX_BYTES = 128 * BKE;  // one MN-major column block (BKE rows x 128 B)
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

// 3-D tile load {x, y, z}: z selects the batch entry (0 for an unbatched operand).
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, int x, int y, int z,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
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

// MN-major operand tile: 128-byte rows along M/N, one row per k, in column
// blocks BKE rows deep and MN_BOX_BYTES apart (LBO = the distance between
// column blocks along M/N; SBO = the distance between groups of k-rows).
//   tf32: the tensor core reads 32-bit MN-major data only in the "128-byte
//   swizzle with 32-byte atoms" layout (descriptor layout type 1; the TMA
//   writes it with CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B): rows of 32 floats
//   whose four 32-byte pieces are permuted by (row mod 4); SBO = 4 k-rows.
//   fp16: the plain 128-byte swizzle (layout type 2, the TMA's
//   CU_TENSOR_MAP_SWIZZLE_128B): rows of 64 halves; SBO = 8 k-rows.
template <int BK, bool F16>
__device__ __forceinline__ uint64_t smem_desc_mn(uint32_t addr) {
    constexpr uint64_t box_bytes = 128 * (BK * 4 / Elt<F16>::SIZE);
    constexpr uint64_t group_rows = F16 ? 8 : 4;
    uint64_t d = 0;
    d |= (uint64_t)((addr & 0x3FFFF) >> 4);
    d |= (uint64_t)(box_bytes >> 4) << 16;           // LBO: next column block
    d |= (uint64_t)((group_rows * 128) >> 4) << 32;  // SBO: next group of k-rows
    d |= (uint64_t)1 << 46;                          // descriptor version for sm_100
    d |= (uint64_t)(F16 ? 2 : 1) << 61;              // swizzle mode
    return d;
}

// Instruction descriptor of kind::tf32 (A/B format 2) or kind::f16 with
// fp16 A/B (format 0): D f32; a_mn / b_mn select the MN-major operand layout
// (bits 15 / 16).
template <bool F16>
__host__ __device__ constexpr uint32_t idesc_mma(int m, int n, bool a_mn, bool b_mn) {
    return (1u << 4) | ((F16 ? 0u : 2u) << 7) | ((F16 ? 0u : 2u) << 10) | ((a_mn ? 1u : 0u) << 15) |
           ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

template <bool F16>
__device__ __forceinline__ void mma_issue(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                          uint32_t accumulate) {
    if constexpr (F16) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
            : "memory");
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
            : "memory");
    }
}

// The scale exponent e of an fp16 split from the bits of its max |x|
// (finite, non-negative): max 2^e in [2^14, 2^15); 0 for a zero max;
// clamped to [-100, 100] so that 2^-e is a normal float.
__host__ __device__ __forceinline__ int split_exp(uint32_t maxbits) {
    if (maxbits == 0) return 0;
    const int e = 14 - ((int)((maxbits >> 23) & 0xFF) - 127);
    return e < -100 ? -100 : (e > 100 ? 100 : e);
}

// 2^k as a float, |k| <= 100.
__device__ __forceinline__ float pow2f(int k) { return __uint_as_float((uint32_t)(127 + k) << 23); }

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

// Work units.  The tiles of the full waves are units of their own; the tiles
// of a last, partial wave are cut into `splits` parts along K (k-blocks
// [num_kb*p/splits, num_kb*(p+1)/splits)), so that wave takes 1/splits of a
// tile's time.  Each part leaves its FP32 partial in `part`; the last part of
// a tile to finish adds the partials in part order and stores the tile.
struct Unit {
    int tile, kb0, kb1, part;  // part < 0: a whole tile
};

__device__ __forceinline__ Unit unit_of(int u, int full_tiles, int splits, int num_kb) {
    if (u < full_tiles) return Unit{u, 0, num_kb, -1};
    const int r = u - full_tiles, part = r % splits;
    return Unit{full_tiles + r / splits, (int)((int64_t)num_kb * part / splits),
                (int)((int64_t)num_kb * (part + 1) / splits), part};
}

// Elementwise work fused into the GEMM's store (each part optional), in the
// coordinates of the stored C [rows, cols]:
//   v = acc + bias[col]            (a bias add broadcast along rows)
//   v = mask[row][col] > 0 ? v : 0 (relu' given the saved pre-activation)
//   C[row][col] = v,  act[row][col] = max(0, v)  (Java Math.max rules)
// and, with out_max set (zeroed by the launch), the bits of the largest
// finite |value| written to act (or to C when there is no act): the max word
// a later 3xFP16 split of that output takes instead of its own max pass.
struct Epilogue {
    const float *bias;
    const float *mask;
    float *act;
    uint32_t *out_max;
};

// m = the bits of max(m, |v|) over finite v.
__device__ __forceinline__ void track_max(uint32_t &m, float v) {
    const uint32_t b = __float_as_uint(v) & 0x7FFFFFFFu;
    if (b < 0x7F800000u && b > m) m = b;
}

__device__ __forceinline__ float ep_relu(float v) { return (0.0f >= v) ? 0.0f : v; }

// Loads one operand's hi or lo tile (ROWS of M or N, BKE of K) into smem.
template <int ROWS, int BK, bool MN, bool F16>
__device__ __forceinline__ void load_operand(uint32_t dst, const CUtensorMap *map, int kx, int row0, int z,
                                             uint32_t bar) {
    if constexpr (!MN) {
        tma_load_3d(dst, map, kx, row0, z, bar);  // box {BKE, ROWS, 1} of a [batch][rows, K] array
    } else {
        constexpr int W = Elt<F16>::MNW, BOX = 128 * (BK * 4 / Elt<F16>::SIZE);
#pragma unroll
        for (int i = 0; i < ROWS / W; i++)        // boxes {MNW, BKE, 1} of a [batch][K, rows] array
            tma_load_3d(dst + i * BOX, map, row0 + i * W, kx, z, bar);
    }
}

// F16: the 3xFP16 split; amax / bmax are then the operands' max words.
template <int BN, int STAGES, int BK, bool A_MN, bool B_MN, bool F16>
__global__ void __launch_bounds__(kThreads, 1)
gemm_3xtf32_kernel(const __grid_constant__ CUtensorMap tAh, const __grid_constant__ CUtensorMap tAl,
                   const __grid_constant__ CUtensorMap tBh, const __grid_constant__ CUtensorMap tBl,
                   float *__restrict__ C, int M, int N, int num_kb, int vec_store, int store_t,
                   Epilogue ep, int batch, int a_batched, int b_batched, int *status, int full_tiles,
                   int splits, float *__restrict__ part, int *__restrict__ arrivals,
                   const uint32_t *__restrict__ amax, const uint32_t *__restrict__ bmax) {
    using Q = Cfg<BN, STAGES, BK, F16>;
    constexpr int UMMA_K = Elt<F16>::UMMA_K;
    constexpr int CHUNK_KB = Q::CHUNK_KB;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Ctl<STAGES> *ctl = reinterpret_cast<Ctl<STAGES> *>(smem + STAGES * Q::STAGE_BYTES);
    volatile int *abort = &ctl->abort;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int num_m = (M + BM - 1) / BM, num_n = (N + BN - 1) / BN;
    const int tiles_per_batch = num_m * num_n;
    const int num_tiles = tiles_per_batch * batch;  // batch entries one after another
    const int num_units = full_tiles + (num_tiles - full_tiles) * splits;

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
            for (int u = blockIdx.x; ok && u < num_units; u += gridDim.x) {
                const Unit w = unit_of(u, full_tiles, splits, num_kb);
                const int t = w.tile;
                int mt, nt;
                const int bidx = t / tiles_per_batch;
                tile_coords(t - bidx * tiles_per_batch, num_m, num_n, mt, nt);
                const int za = a_batched ? bidx : 0, zb = b_batched ? bidx : 0;
                for (int kb = w.kb0; kb < w.kb1; kb++) {
                    if (!wait_bar(smem_u32(&ctl->empty[stage]), phase ^ 1, abort, status)) {
                        ok = false;
                        break;
                    }
                    const uint32_t sb = smem_u32(smem + stage * Q::STAGE_BYTES);
                    const uint32_t fb = smem_u32(&ctl->full[stage]);
                    mbar_expect_tx(fb, Q::STAGE_BYTES);
                    const int kx = kb * Q::BKE;
                    load_operand<BM, BK, A_MN, F16>(sb, &tAh, kx, mt * BM, za, fb);
                    load_operand<BM, BK, A_MN, F16>(sb + Q::A_BYTES, &tAl, kx, mt * BM, za, fb);
                    load_operand<BN, BK, B_MN, F16>(sb + 2 * Q::A_BYTES, &tBh, kx, nt * BN, zb, fb);
                    load_operand<BN, BK, B_MN, F16>(sb + 2 * Q::A_BYTES + Q::B_BYTES, &tBl, kx, nt * BN, zb, fb);
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
            constexpr uint32_t idesc = idesc_mma<F16>(BM, BN, A_MN, B_MN);
            int stage = 0;
            uint32_t phase = 0;
            int ci = 0;  // chunk counter across tiles: selects the TMEM buffer
            bool ok = true;
            for (int u = blockIdx.x; ok && u < num_units; u += gridDim.x) {
                const Unit w = unit_of(u, full_tiles, splits, num_kb);
                for (int kb0 = w.kb0; ok && kb0 < w.kb1; kb0 += CHUNK_KB, ci++) {
                    const int buf = ci & 1;
                    const uint32_t bph = (ci >> 1) & 1;
                    if (!wait_bar(smem_u32(&ctl->tempty[buf]), bph ^ 1, abort, status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t dcol = tmem + buf * BN;
                    const int kb1 = min(w.kb1, kb0 + CHUNK_KB);
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
                        for (int kk = 0; kk < Q::BKE / UMMA_K; kk++) {
                            // next UMMA_K: 32 bytes along a K-major row, UMMA_K rows of 128 B in an MN-major block
                            const uint32_t oa = A_MN ? kk * UMMA_K * 128 : kk * 32;
                            const uint32_t ob = B_MN ? kk * UMMA_K * 128 : kk * 32;
                            const uint64_t ah = A_MN ? smem_desc_mn<BK, F16>(sa_hi + oa) : smem_desc<BK>(sa_hi + oa);
                            const uint64_t al = A_MN ? smem_desc_mn<BK, F16>(sa_lo + oa) : smem_desc<BK>(sa_lo + oa);
                            const uint64_t bh = B_MN ? smem_desc_mn<BK, F16>(sb_hi + ob) : smem_desc<BK>(sb_hi + ob);
                            const uint64_t bl = B_MN ? smem_desc_mn<BK, F16>(sb_lo + ob) : smem_desc<BK>(sb_lo + ob);
                            mma_issue<F16>(dcol, al, bh, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
                            mma_issue<F16>(dcol, ah, bl, idesc, 1u);
                            mma_issue<F16>(dcol, ah, bh, idesc, 1u);
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
        for (int u = blockIdx.x; ok && u < num_units; u += gridDim.x) {
            const Unit w = unit_of(u, full_tiles, splits, num_kb);
            const int t = w.tile;
            int mt, nt;
            const int bidx = t / tiles_per_batch;
            tile_coords(t - bidx * tiles_per_batch, num_m, num_n, mt, nt);
            // this batch entry's C (and mask / act): [M, N], or [N, M] when stored transposed
            const size_t boff = (size_t)bidx * (size_t)M * (size_t)N;
            float *const Cb = C ? C + boff : nullptr;  // NULL: only the relu output is stored
            const float *const mask_b = ep.mask ? ep.mask + boff : nullptr;
            float *const act_b = ep.act ? ep.act + boff : nullptr;
            float acc[Q::COLS_PER_WARP];
#pragma unroll
            for (int j = 0; j < Q::COLS_PER_WARP; j++) acc[j] = 0.0f;
            for (int kb0 = w.kb0; kb0 < w.kb1; kb0 += CHUNK_KB, ci++) {
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
            if (w.part >= 0) {
                // A part of a split tile.  Each epilogue warp owns 32 rows x
                // COLS_PER_WARP columns of the tile and settles them alone (no
                // wait on other warps): it leaves its partial (a column j of the
                // region is 32 consecutive floats), counts its arrival, and the
                // warp of the last part to arrive adds all partials in part order.
                constexpr int RF = 32 * Q::COLS_PER_WARP;  // floats of one warp's region
                const size_t tix = (size_t)(t - full_tiles);
                float *mine = part + ((tix * splits + w.part) * kEpiWarps + ew) * (size_t)RF + lane;
#pragma unroll
                for (int j = 0; j < Q::COLS_PER_WARP; j++) mine[(size_t)j * 32] = acc[j];
                __threadfence();
                __syncwarp();
                int before = 0;
                if (lane == 0) before = atomicAdd(arrivals + tix * kEpiWarps + ew, 1);
                before = __shfl_sync(0xffffffffu, before, 0);
                if (before != splits - 1) continue;  // a later part settles the region
                __threadfence();
                // every partial (this part's too) is read back through L2
                const float *rp = part + (tix * splits * kEpiWarps + ew) * (size_t)RF + lane;
#pragma unroll
                for (int j = 0; j < Q::COLS_PER_WARP; j++) {
                    float v = __ldcg(rp + (size_t)j * 32);
#pragma unroll
                    for (int p = 1; p < kMaxTailSplits; p++)
                        if (p < splits) v = __fadd_rn(v, __ldcg(rp + (size_t)p * kEpiWarps * RF + (size_t)j * 32));
                    acc[j] = v;
                }
            }
            if constexpr (F16) {
                // the accumulator is in units of 2^(e_a + e_b): two exact power-of-two scalings
                const int E = split_exp(__ldg(amax)) + split_exp(__ldg(bmax));
                const float f1 = pow2f(-(E >> 1)), f2 = pow2f(-(E - (E >> 1)));
#pragma unroll
                for (int j = 0; j < Q::COLS_PER_WARP; j++) acc[j] = acc[j] * f1 * f2;
            }
            const int row = mt * BM + q * 32 + lane;
            const int col0 = nt * BN + cbase;
            uint32_t mloc = 0;  // max of the values this lane stores (ep.out_max)
            if (store_t) {
                // C holds the transpose of this product ([N, M]): for each
                // column the warp's 32 lanes write 32 consecutive floats.
                // Stored C's column index is `row`, so the bias is one value.
                if (row < M) {
                    const float b = ep.bias ? __ldg(ep.bias + row) : 0.0f;
#pragma unroll
                    for (int j = 0; j < Q::COLS_PER_WARP; j++) {
                        if (col0 + j < N) {
                            const size_t idx = (size_t)(col0 + j) * (size_t)M + row;
                            float v = ep.bias ? __fadd_rn(acc[j], b) : acc[j];
                            if (mask_b) v = __ldg(mask_b + idx) > 0.0f ? v : 0.0f;
                            if (Cb) Cb[idx] = v;
                            if (act_b) act_b[idx] = ep_relu(v);
                            if (ep.out_max) track_max(mloc, act_b ? ep_relu(v) : v);
                        }
                    }
                }
            } else if (row < M && col0 < N) {
                const size_t base = (size_t)row * (size_t)N + col0;
                if (vec_store && col0 + Q::COLS_PER_WARP <= N) {
#pragma unroll
                    for (int v4 = 0; v4 < Q::COLS_PER_WARP / 4; v4++) {
                        float x[4] = {acc[4 * v4], acc[4 * v4 + 1], acc[4 * v4 + 2], acc[4 * v4 + 3]};
                        if (ep.bias) {
                            const float4 b = __ldg(reinterpret_cast<const float4 *>(ep.bias + col0) + v4);
                            x[0] = __fadd_rn(x[0], b.x); x[1] = __fadd_rn(x[1], b.y);
                            x[2] = __fadd_rn(x[2], b.z); x[3] = __fadd_rn(x[3], b.w);
                        }
                        if (mask_b) {
                            const float4 m = __ldg(reinterpret_cast<const float4 *>(mask_b + base) + v4);
                            x[0] = m.x > 0.0f ? x[0] : 0.0f; x[1] = m.y > 0.0f ? x[1] : 0.0f;
                            x[2] = m.z > 0.0f ? x[2] : 0.0f; x[3] = m.w > 0.0f ? x[3] : 0.0f;
                        }
                        if (Cb) reinterpret_cast<float4 *>(Cb + base)[v4] = make_float4(x[0], x[1], x[2], x[3]);
                        if (act_b)
                            reinterpret_cast<float4 *>(act_b + base)[v4] =
                                make_float4(ep_relu(x[0]), ep_relu(x[1]), ep_relu(x[2]), ep_relu(x[3]));
                        if (ep.out_max) {
#pragma unroll
                            for (int i = 0; i < 4; i++) track_max(mloc, act_b ? ep_relu(x[i]) : x[i]);
                        }
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < Q::COLS_PER_WARP; j++) {
                        if (col0 + j < N) {
                            float v = ep.bias ? __fadd_rn(acc[j], __ldg(ep.bias + col0 + j)) : acc[j];
                            if (mask_b) v = __ldg(mask_b + base + j) > 0.0f ? v : 0.0f;
                            if (Cb) Cb[base + j] = v;
                            if (act_b) act_b[base + j] = ep_relu(v);
                            if (ep.out_max) track_max(mloc, act_b ? ep_relu(v) : v);
                        }
                    }
                }
            }
            if (ep.out_max) {  // uniform: every lane of the warp gets here
                for (int o = 16; o > 0; o >>= 1) mloc = max(mloc, __shfl_xor_sync(0xffffffffu, mloc, o));
                if (lane == 0 && mloc) atomicMax(ep.out_max, mloc);
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

// ---- operand split: X [rows, cols] -> hi/lo [rows, pitch], pitch = cols rounded up to 4 ----
__device__ __forceinline__ float tf32_round(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r & 0xFFFFE000u);
}

// 4 consecutive columns per thread step: 16-byte loads when the source
// allows, 16-byte stores of hi and lo; padding columns are written as zero.
__global__ void __launch_bounds__(256) split_kernel(const float *__restrict__ src, int64_t rows, int64_t cols,
                                                    int64_t pitch, int vec, float *__restrict__ hi,
                                                    float *__restrict__ lo) {
    const int64_t q = pitch / 4;
    const int64_t n = rows * q;
    for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < n;
         v += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = v / q, k = (v - r * q) * 4;
        float x[4];
        const float *p = src + r * cols + k;
        if (vec && k + 4 <= cols) {
            const float4 t = __ldg(reinterpret_cast<const float4 *>(p));
            x[0] = t.x; x[1] = t.y; x[2] = t.z; x[3] = t.w;
        } else {
#pragma unroll
            for (int j = 0; j < 4; j++) x[j] = (k + j < cols) ? p[j] : 0.0f;
        }
        float h[4], l[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            h[j] = tf32_round(x[j]);
            l[j] = tf32_round(x[j] - h[j]);
        }
        *reinterpret_cast<float4 *>(hi + r * pitch + k) = make_float4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<float4 *>(lo + r * pitch + k) = make_float4(l[0], l[1], l[2], l[3]);
    }
}

// Transposed split: X [rows, cols] -> hi/lo of X^T, [cols, pitch] with
// pitch = rows rounded up to 4.  64 x 64 tiles through shared memory; each
// lane reads 4 consecutive floats of an X row (16 bytes when X's rows allow)
// and writes 4 consecutive floats of an X^T row to hi and to lo (16 bytes;
// pitch is a multiple of 4 and the tile origin a multiple of 64).
// With phi / plo set it also writes the split in the stored layout
// ([rows, ppitch], zero padding), from the values it loads: both splits of
// an operand for one read of it.
__global__ void __launch_bounds__(256) split_t_kernel(const float *__restrict__ src, int64_t rows, int64_t cols,
                                                      int64_t pitch, int64_t tiles_c, int vec_in,
                                                      float *__restrict__ hi, float *__restrict__ lo,
                                                      float *__restrict__ phi, float *__restrict__ plo,
                                                      int64_t ppitch) {
    __shared__ float tile[64][65];
    const int64_t c0 = (blockIdx.x % tiles_c) * 64, r0 = (blockIdx.x / tiles_c) * 64;
    const int q = threadIdx.x & 15, w = threadIdx.x >> 4;  // 16 lanes per 64-float row, 16 rows per pass
#pragma unroll
    for (int pass = 0; pass < 4; pass++) {  // tile[i][4q..4q+3] = X[r0 + i][c0 + 4q ..]
        const int i = pass * 16 + w;
        const int64_t r = r0 + i, c = c0 + 4 * q;
        float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (r < rows) {
            if (vec_in && c + 4 <= cols) {
                const float4 t = __ldg(reinterpret_cast<const float4 *>(src + r * cols + c));
                v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
            } else {
#pragma unroll
                for (int k = 0; k < 4; k++) v[k] = (c + k < cols) ? src[r * cols + c + k] : 0.0f;
            }
        }
#pragma unroll
        for (int k = 0; k < 4; k++) tile[i][4 * q + k] = v[k];
        if (phi && r < rows && c < ppitch) {  // columns past `cols` were loaded as zero
            float h[4], l[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                h[k] = tf32_round(v[k]);
                l[k] = tf32_round(v[k] - h[k]);
            }
            *reinterpret_cast<float4 *>(phi + r * ppitch + c) = make_float4(h[0], h[1], h[2], h[3]);
            *reinterpret_cast<float4 *>(plo + r * ppitch + c) = make_float4(l[0], l[1], l[2], l[3]);
        }
    }
    __syncthreads();
#pragma unroll
    for (int pass = 0; pass < 4; pass++) {  // X^T[c0 + j][r0 + 4q ..] = tile[4q..4q+3][j]
        const int j = pass * 16 + w;
        const int64_t c = c0 + j, r = r0 + 4 * q;
        if (c >= cols || r >= pitch) continue;
        float h[4], l[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const float x = tile[4 * q + k][j];  // rows >= `rows` were loaded as zero
            h[k] = tf32_round(x);
            l[k] = tf32_round(x - h[k]);
        }
        *reinterpret_cast<float4 *>(hi + c * pitch + r) = make_float4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<float4 *>(lo + c * pitch + r) = make_float4(l[0], l[1], l[2], l[3]);
    }
}

// ---- 3xFP16 operand split --------------------------------------------------------------
// *word = the bits of max |x| over the finite elements of X [n] (zeroed beforehand):
// non-negative floats order like their bits as unsigned integers.
__global__ void __launch_bounds__(256) absmax_kernel(const float *__restrict__ src, int64_t n, int vec,
                                                     uint32_t *__restrict__ word) {
    uint32_t m = 0;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t t0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    int64_t done = 0;
    if (vec) {
        // four independent 16-byte loads in flight per thread
        const uint4 *s4 = reinterpret_cast<const uint4 *>(src);
        const int64_t n4 = n / 4;
        int64_t v = t0;
        for (; v + 3 * stride < n4; v += 4 * stride) {
            uint4 u[4];
#pragma unroll
            for (int i = 0; i < 4; i++) u[i] = __ldg(s4 + v + i * stride);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const uint32_t b[4] = {u[i].x & 0x7FFFFFFFu, u[i].y & 0x7FFFFFFFu, u[i].z & 0x7FFFFFFFu,
                                       u[i].w & 0x7FFFFFFFu};
#pragma unroll
                for (int j = 0; j < 4; j++)
                    if (b[j] < 0x7F800000u && b[j] > m) m = b[j];
            }
        }
        for (; v < n4; v += stride) {
            const uint4 u = __ldg(s4 + v);
            const uint32_t b[4] = {u.x & 0x7FFFFFFFu, u.y & 0x7FFFFFFFu, u.z & 0x7FFFFFFFu, u.w & 0x7FFFFFFFu};
#pragma unroll
            for (int j = 0; j < 4; j++)
                if (b[j] < 0x7F800000u && b[j] > m) m = b[j];
        }
        done = n4 * 4;
    }
    for (int64_t i = done + t0; i < n; i += stride) {
        const uint32_t b = __float_as_uint(src[i]) & 0x7FFFFFFFu;
        if (b < 0x7F800000u && b > m) m = b;
    }
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0 && m) atomicMax(word, m);
}

// hi = fp16(x 2^e), lo = fp16(x 2^e - hi) of 8 consecutive values.
__device__ __forceinline__ void split8_f16(const float (&x)[8], float sc, uint4 &h, uint4 &l) {
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const float a = x[2 * j] * sc, b = x[2 * j + 1] * sc;
        const __half ha = __float2half_rn(a), hb = __float2half_rn(b);
        const __half la = __float2half_rn(a - __half2float(ha)), lb = __float2half_rn(b - __half2float(hb));
        hw[j] = (uint32_t)__half_as_ushort(ha) | ((uint32_t)__half_as_ushort(hb) << 16);
        lw[j] = (uint32_t)__half_as_ushort(la) | ((uint32_t)__half_as_ushort(lb) << 16);
    }
    h = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    l = make_uint4(lw[0], lw[1], lw[2], lw[3]);
}

// X [rows, cols] -> fp16 hi/lo [rows, pitch] (pitch = cols rounded up to 8,
// padding written as zero), scaled by 2^e from the max word.  8 columns per
// thread step: 32-byte loads when the source allows, 16-byte stores.
__global__ void __launch_bounds__(256) split16_kernel(const float *__restrict__ src, int64_t rows, int64_t cols,
                                                      int64_t pitch, int vec, const uint32_t *__restrict__ word,
                                                      __half *__restrict__ hi, __half *__restrict__ lo) {
    const float sc = pow2f(split_exp(*word));
    const int64_t q = pitch / 8;
    const int64_t n = rows * q;
    for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < n;
         v += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = v / q, k = (v - r * q) * 8;
        float x[8];
        const float *p = src + r * cols + k;
        if (vec && k + 8 <= cols) {
            const float4 t0 = __ldg(reinterpret_cast<const float4 *>(p));
            const float4 t1 = __ldg(reinterpret_cast<const float4 *>(p) + 1);
            x[0] = t0.x; x[1] = t0.y; x[2] = t0.z; x[3] = t0.w;
            x[4] = t1.x; x[5] = t1.y; x[6] = t1.z; x[7] = t1.w;
        } else {
#pragma unroll
            for (int j = 0; j < 8; j++) x[j] = (k + j < cols) ? p[j] : 0.0f;
        }
        uint4 h, l;
        split8_f16(x, sc, h, l);
        *reinterpret_cast<uint4 *>(hi + r * pitch + k) = h;
        *reinterpret_cast<uint4 *>(lo + r * pitch + k) = l;
    }
}

// hi = fp16(x 2^e), lo = fp16(x 2^e - hi) of 4 consecutive values, packed.
__device__ __forceinline__ void split4_f16(const float (&x)[4], float sc, uint2 &h, uint2 &l) {
    uint32_t hw[2], lw[2];
#pragma unroll
    for (int j = 0; j < 2; j++) {
        const float a = x[2 * j] * sc, b = x[2 * j + 1] * sc;
        const __half ha = __float2half_rn(a), hb = __float2half_rn(b);
        const __half la = __float2half_rn(a - __half2float(ha)), lb = __float2half_rn(b - __half2float(hb));
        hw[j] = (uint32_t)__half_as_ushort(ha) | ((uint32_t)__half_as_ushort(hb) << 16);
        lw[j] = (uint32_t)__half_as_ushort(la) | ((uint32_t)__half_as_ushort(lb) << 16);
    }
    h = make_uint2(hw[0], hw[1]);
    l = make_uint2(lw[0], lw[1]);
}

// The fp16 split of X^T ([cols, pitch], pitch = rows rounded up to 8) and,
// with phi / plo set, of X in its stored layout ([rows, ppitch], ppitch =
// cols rounded up to 8) from the same loads; split_t_kernel's tiling, 8-byte
// stores of 4 halves.  The first thread copies the max word to pword.
__global__ void __launch_bounds__(256) split16_t_kernel(const float *__restrict__ src, int64_t rows, int64_t cols,
                                                        int64_t pitch, int64_t tiles_c, int vec_in,
                                                        const uint32_t *__restrict__ word, __half *__restrict__ hi,
                                                        __half *__restrict__ lo, __half *__restrict__ phi,
                                                        __half *__restrict__ plo, int64_t ppitch,
                                                        uint32_t *__restrict__ pword) {
    __shared__ float tile[64][65];
    const uint32_t mw = *word;
    const float sc = pow2f(split_exp(mw));
    if (pword && blockIdx.x == 0 && threadIdx.x == 0) *pword = mw;
    const int64_t c0 = (blockIdx.x % tiles_c) * 64, r0 = (blockIdx.x / tiles_c) * 64;
    const int q = threadIdx.x & 15, w = threadIdx.x >> 4;
#pragma unroll
    for (int pass = 0; pass < 4; pass++) {
        const int i = pass * 16 + w;
        const int64_t r = r0 + i, c = c0 + 4 * q;
        float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (r < rows) {
            if (vec_in && c + 4 <= cols) {
                const float4 t = __ldg(reinterpret_cast<const float4 *>(src + r * cols + c));
                v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
            } else {
#pragma unroll
                for (int k = 0; k < 4; k++) v[k] = (c + k < cols) ? src[r * cols + c + k] : 0.0f;
            }
        }
#pragma unroll
        for (int k = 0; k < 4; k++) tile[i][4 * q + k] = v[k];
        if (phi && r < rows && c < ppitch) {  // columns past `cols` were loaded as zero
            uint2 h, l;
            split4_f16(v, sc, h, l);
            *reinterpret_cast<uint2 *>(phi + r * ppitch + c) = h;
            *reinterpret_cast<uint2 *>(plo + r * ppitch + c) = l;
        }
    }
    __syncthreads();
#pragma unroll
    for (int pass = 0; pass < 4; pass++) {
        const int j = pass * 16 + w;
        const int64_t c = c0 + j, r = r0 + 4 * q;
        if (c >= cols || r >= pitch) continue;
        const float x[4] = {tile[4 * q][j], tile[4 * q + 1][j], tile[4 * q + 2][j], tile[4 * q + 3][j]};
        uint2 h, l;
        split4_f16(x, sc, h, l);
        *reinterpret_cast<uint2 *>(hi + c * pitch + r) = h;
        *reinterpret_cast<uint2 *>(lo + c * pitch + r) = l;
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

// The operand split mode, fixed for the process: 3xFP16 unless
// J4C_GEMM_SPLIT is "tf32" (3xTF32).  Splits and GEMMs must agree, so it is
// read once.
bool split_fp16() {
    static const bool f16 = [] {
        const char *v = getenv("J4C_GEMM_SPLIT");
        return !(v && (v[0] == 't' || v[0] == 'T') && (v[1] == 'f' || v[1] == 'F') && v[2] == '3' && v[3] == '2');
    }();
    return f16;
}

// Elements per row of a split array: cols rounded up to a 16-byte multiple.
inline int64_t split_pitch(int64_t cols) { return split_fp16() ? ceil_div(cols, 8) * 8 : ceil_div(cols, 4) * 4; }
inline int64_t split_esize() { return split_fp16() ? 2 : 4; }

// Bytes of one hi or lo array of an operand [rows, cols]; an fp16 hi array is
// followed by its 32-bit max word (16 bytes reserved).
inline int64_t split_bytes(int64_t rows, int64_t cols) {
    return rows * split_pitch(cols) * split_esize() + (split_fp16() ? 16 : 0);
}

// The max word of an fp16 hi array of an operand [rows, cols].
inline uint32_t *split_word(const float *hi, int64_t rows, int64_t cols) {
    return reinterpret_cast<uint32_t *>(reinterpret_cast<char *>(const_cast<float *>(hi)) +
                                        rows * split_pitch(cols) * 2);
}

// Tensor map of a hi or lo array [rows, pitch] (pitch * esize bytes per row).
//   K-major use (rows = M or N, cols = K): box {BKE, box_rows}, BK*4-byte swizzle.
//   MN-major use (rows = K, cols = M or N): box {MNW, BKE}; tf32: 128-byte
//   swizzle of 32-byte atoms, fp16: 128-byte swizzle.
// Columns past `cols` and rows past `rows` read as zero (TMA fill).
static int make_map(CUtensorMap *map, const float *base, int64_t rows, int64_t cols, bool mn, int box_rows,
                    int bk, int64_t batch) {
    auto fn = encode_fn();
    if (!fn) return set_error(J4C_E_CUDA, "cuTensorMapEncodeTiled is unavailable");
    const bool f16 = split_fp16();
    const int64_t es = split_esize();
    const int bke = bk * 4 / (int)es;
    // [batch][rows, pitch]: batch entries back to back (batch = 1 for an operand shared by all)
    cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)batch};
    cuuint64_t strides[2] = {(cuuint64_t)(split_pitch(cols) * es), (cuuint64_t)(rows * split_pitch(cols) * es)};
    cuuint32_t box[3];
    CUtensorMapSwizzle sw;
    if (mn) {
        box[0] = f16 ? 64 : 32;
        box[1] = (cuuint32_t)bke;
        sw = f16 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
    } else {
        box[0] = (cuuint32_t)bke;
        box[1] = (cuuint32_t)box_rows;
        sw = bk == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    }
    box[2] = 1;
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3,
                    const_cast<float *>(base), dims, strides, box,
                    estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(J4C_E_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return J4C_OK;
}

// The tail split of a GEMM (Unit): the tiles of the full waves stay whole;
// the rest are cut into as many parts along K (up to 4) as still fit one
// wave, each part keeping at least one promotion chunk of k-blocks.
struct TailPlan {
    int64_t full_tiles;
    int splits;
};

static TailPlan tail_plan(int64_t tiles, int64_t num_kb, int64_t chunk_kb, int64_t sms) {
    const int64_t full = tiles / sms * sms, rem = tiles - full;
    if (rem == 0) return TailPlan{tiles, 1};
    int64_t sp = std::min<int64_t>(kMaxTailSplits, sms / rem);
    while (sp > 1 && num_kb / sp < chunk_kb) sp--;
    return sp < 2 ? TailPlan{tiles, 1} : TailPlan{full, (int)sp};
}

// Scratch of a tail split: the parts' FP32 partial tiles, then one arrival
// counter per (split tile, epilogue warp).
static size_t tail_scratch_bytes(int64_t tiles, const TailPlan &p, int bn) {
    if (p.splits < 2) return 0;
    const int64_t rem = tiles - p.full_tiles;
    return (size_t)(rem * p.splits * BM * bn) * sizeof(float) + (size_t)(rem * kEpiWarps) * sizeof(int);
}

// An upper bound of tail_scratch_bytes for an [m, n] product in either
// orientation (the K condition only lowers the number of parts).
size_t tail_scratch_bound(int64_t m, int64_t n, int64_t batch) {
    size_t most = 0;
    for (int o = 0; o < 2; o++) {
        const int64_t tiles = ceil_div(o ? n : m, BM) * ceil_div(o ? m : n, 256) * batch;
        most = std::max(most, tail_scratch_bytes(tiles, tail_plan(tiles, 1ll << 40, 1, sm_count()), 256));
    }
    return most;
}

template <int BN, int STAGES, int BK, bool A_MN, bool B_MN, bool F16>
static int launch_gemm(const float *ah, const float *al, const float *bh, const float *bl, float *c,
                       int64_t M, int64_t N, int64_t K, bool store_t, const Epilogue &ep, int64_t batch,
                       bool a_bat, bool b_bat, void *tail_ws, cudaStream_t s) {
    using Q = Cfg<BN, STAGES, BK, F16>;
    auto kernel = gemm_3xtf32_kernel<BN, STAGES, BK, A_MN, B_MN, F16>;
    static std::mutex mu;
    static std::vector<char> configured;
    int dev = 0;
    J4C_CUDA(cudaGetDevice(&dev));
    {
        std::lock_guard<std::mutex> lock(mu);
        if ((int)configured.size() <= dev) configured.resize(dev + 1, 0);
        if (!configured[dev]) {
            J4C_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Q::SMEM_BYTES));
            configured[dev] = 1;
        }
    }
    CUtensorMap mAh, mAl, mBh, mBl;
    int rc;
    // op(A) [M, K]: stored [M, K] (K-major) or [K, M] (MN-major); likewise op(B)^T [N, K].
    const int64_t ar = A_MN ? K : M, ac = A_MN ? M : K;
    const int64_t br = B_MN ? K : N, bc = B_MN ? N : K;
    const int64_t ab = a_bat ? batch : 1, bb = b_bat ? batch : 1;
    if ((rc = make_map(&mAh, ah, ar, ac, A_MN, BM, BK, ab)) || (rc = make_map(&mAl, al, ar, ac, A_MN, BM, BK, ab)) ||
        (rc = make_map(&mBh, bh, br, bc, B_MN, BN, BK, bb)) || (rc = make_map(&mBl, bl, br, bc, B_MN, BN, BK, bb)))
        return rc;
    int *status = device_status_ptr();
    if (!status) return set_error(J4C_E_OOM, "no device status word");
    const int64_t tiles = ceil_div(M, BM) * ceil_div(N, BN) * batch;
    if (tiles >= (1ll << 30)) return set_error(J4C_E_UNSUPPORTED, "dot: too many output tiles");
    const int64_t num_kb = ceil_div(K, Q::BKE);
    const TailPlan tp = tail_plan(tiles, num_kb, Q::CHUNK_KB, sm_count());
    const int64_t units = tp.full_tiles + (tiles - tp.full_tiles) * tp.splits;
    const int grid = (int)std::min<int64_t>(units, sm_count());
    const int vec = (N % 4 == 0) && aligned16(c) && (!ep.bias || aligned16(ep.bias)) &&
                    (!ep.mask || aligned16(ep.mask)) && (!ep.act || aligned16(ep.act));
    float *part = nullptr;
    int *arrivals = nullptr;
    void *owned = nullptr;
    if (tp.splits > 1) {
        const size_t bytes = tail_scratch_bytes(tiles, tp, BN);
        if (!tail_ws) {
            if ((rc = scratch_alloc(bytes, &owned, s))) return rc;
            tail_ws = owned;
        }
        part = static_cast<float *>(tail_ws);
        arrivals = reinterpret_cast<int *>(part + (tiles - tp.full_tiles) * tp.splits * BM * BN);
        J4C_CUDA(cudaMemsetAsync(arrivals, 0, (size_t)((tiles - tp.full_tiles) * kEpiWarps) * sizeof(int), s));
    }
    if (ep.out_max) J4C_CUDA(cudaMemsetAsync(ep.out_max, 0, sizeof(uint32_t), s));
    const uint32_t *amax = F16 ? split_word(ah, ar * ab, ac) : nullptr;
    const uint32_t *bmax = F16 ? split_word(bh, br * bb, bc) : nullptr;
    kernel<<<grid, kThreads, Q::SMEM_BYTES, s>>>(mAh, mAl, mBh, mBl, c, (int)M, (int)N, (int)num_kb,
                                                 store_t ? 0 : vec, store_t ? 1 : 0, ep, (int)batch, a_bat ? 1 : 0,
                                                 b_bat ? 1 : 0, status, (int)tp.full_tiles, tp.splits, part, arrivals,
                                                 amax, bmax);
    J4C_LAUNCH_CHECK("gemm_3xtf32_kernel");
    if (owned) return scratch_free(owned, s);
    return J4C_OK;
}

template <int BN, int STAGES, int BK, bool F16>
static int launch_gemm_any(const float *ah, const float *al, const float *bh, const float *bl, float *c,
                           int64_t M, int64_t N, int64_t K, bool a_mn, bool b_mn, const Epilogue &ep,
                           int64_t batch, bool a_bat, bool b_bat, void *tail_ws, cudaStream_t s) {
    if (!a_mn && !b_mn)
        return launch_gemm<BN, STAGES, BK, false, false, F16>(ah, al, bh, bl, c, M, N, K, false, ep, batch, a_bat, b_bat, tail_ws, s);
    if (a_mn && !b_mn)
        return launch_gemm<BN, STAGES, BK, true, false, F16>(ah, al, bh, bl, c, M, N, K, false, ep, batch, a_bat, b_bat, tail_ws, s);
    // The wide (BN = 256) operand is read MN-major at a smem cost that
    // throttles the tensor pipe, so a K-major A with an MN-major B runs as
    // C^T = op(B)^T . op(A)^T: B's split becomes the (MN-major) A operand,
    // A's the (K-major) B operand, and the epilogue stores transposed.
    if (!a_mn && b_mn)
        return launch_gemm<BN, STAGES, BK, true, false, F16>(bh, bl, ah, al, c, N, M, K, true, ep, batch, b_bat, a_bat, tail_ws, s);
    return launch_gemm<BN, STAGES, BK, true, true, F16>(ah, al, bh, bl, c, M, N, K, false, ep, batch, a_bat, b_bat, tail_ws, s);
}

// *word = the bits of X's max finite |x| (n elements).
static int absmax(const float *src, int64_t n, uint32_t *word, cudaStream_t s) {
    J4C_CUDA(cudaMemsetAsync(word, 0, sizeof(uint32_t), s));
    const int vec = aligned16(src);
    absmax_kernel<<<grid_for(vec ? ceil_div(n, 16) : n, 256, 8), 256, 0, s>>>(src, n, vec, word);
    J4C_LAUNCH_CHECK("absmax_kernel");
    return J4C_OK;
}

// The split of X^T, and with phi / plo also X's own split, in one pass.
// max_in (3xFP16 only): X's max word computed already (a GEMM epilogue's
// out_max), copied instead of a max pass.
int split_t(const float *src, int64_t rows, int64_t cols, float *hi, float *lo, cudaStream_t s,
            float *phi = nullptr, float *plo = nullptr, const uint32_t *max_in = nullptr) {
    if (rows == 0 || cols == 0) return J4C_OK;
    J4C_REQUIRE(aligned16(hi) && aligned16(lo), "split: hi/lo must be 16-byte aligned");
    J4C_REQUIRE(!phi == !plo && (!phi || (aligned16(phi) && aligned16(plo))),
                "split: both stored-layout outputs, 16-byte aligned");
    const int64_t pitch = split_pitch(rows);
    const int64_t tiles_c = ceil_div(cols, 64), tiles_r = ceil_div(pitch, 64);
    J4C_REQUIRE(tiles_c * tiles_r < (1ll << 31), "split: array too large");
    const int vec_in = (cols % 4 == 0) && aligned16(src);
    if (split_fp16()) {
        uint32_t *word = split_word(hi, cols, rows);
        if (max_in) {
            J4C_CUDA(cudaMemcpyAsync(word, max_in, sizeof(uint32_t), cudaMemcpyDeviceToDevice, s));
        } else {
            const int rc = absmax(src, rows * cols, word, s);
            if (rc) return rc;
        }
        split16_t_kernel<<<(unsigned)(tiles_c * tiles_r), 256, 0, s>>>(
            src, rows, cols, pitch, tiles_c, vec_in, word, reinterpret_cast<__half *>(hi),
            reinterpret_cast<__half *>(lo), reinterpret_cast<__half *>(phi), reinterpret_cast<__half *>(plo),
            split_pitch(cols), phi ? split_word(phi, rows, cols) : nullptr);
        J4C_LAUNCH_CHECK("split16_t_kernel");
        return J4C_OK;
    }
    split_t_kernel<<<(unsigned)(tiles_c * tiles_r), 256, 0, s>>>(src, rows, cols, pitch, tiles_c, vec_in, hi, lo,
                                                                 phi, plo, split_pitch(cols));
    J4C_LAUNCH_CHECK("split_t_kernel");
    return J4C_OK;
}

int split(const float *src, int64_t rows, int64_t cols, float *hi, float *lo, cudaStream_t s,
          const uint32_t *max_in = nullptr) {
    if (rows == 0 || cols == 0) return J4C_OK;
    J4C_REQUIRE(aligned16(hi) && aligned16(lo), "split: hi/lo must be 16-byte aligned");
    const int64_t pitch = split_pitch(cols);
    const int vec = (cols % 4 == 0) && aligned16(src);
    if (split_fp16()) {
        uint32_t *word = split_word(hi, rows, cols);
        if (max_in) {
            J4C_CUDA(cudaMemcpyAsync(word, max_in, sizeof(uint32_t), cudaMemcpyDeviceToDevice, s));
        } else {
            const int rc = absmax(src, rows * cols, word, s);
            if (rc) return rc;
        }
        split16_kernel<<<grid_for(rows * (pitch / 8), 256), 256, 0, s>>>(
            src, rows, cols, pitch, vec, word, reinterpret_cast<__half *>(hi), reinterpret_cast<__half *>(lo));
        J4C_LAUNCH_CHECK("split16_kernel");
        return J4C_OK;
    }
    split_kernel<<<grid_for(rows * (pitch / 4), 256), 256, 0, s>>>(src, rows, cols, pitch, vec, hi, lo);
    J4C_LAUNCH_CHECK("split_kernel");
    return J4C_OK;
}

}  // namespace tc

bool tc_gemm_supported(int64_t M, int64_t K, int64_t N) {
    // int32 coordinates and extents in the kernel and the tensor maps
    return M >= 1 && N >= 1 && K >= 1 && M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31);
}

// Bytes of one hi or lo array of an operand stored [rows, cols], 256-byte aligned.
static int64_t split_buf(int64_t rows, int64_t cols) { return ceil_div(tc::split_bytes(rows, cols), 256) * 256; }

// Floats per row that a caller allocates for one hi or lo array of an
// operand with `cols` columns: rows * this floats hold split_bytes(rows, cols)
// for every rows >= 1 (3xFP16: 2-byte halves plus the 16-byte max word).
int64_t tc_split_alloc_pitch(int64_t cols) {
    return tc::split_fp16() ? tc::split_pitch(cols) / 2 + 4 : tc::split_pitch(cols);
}

// 1 for the 3xFP16 split, 0 for 3xTF32.
int tc_split_kind() { return tc::split_fp16() ? 1 : 0; }

int tc_gemm_workspace(int64_t M, int64_t K, int64_t N, size_t *bytes) {
    // hi and lo of the larger of the two storage orders of each operand,
    // then the scratch of a tail split
    const int64_t a = 2 * std::max(split_buf(M, K), split_buf(K, M));
    const int64_t b = 2 * std::max(split_buf(K, N), split_buf(N, K));
    *bytes = (size_t)(a + b) + tc::tail_scratch_bound(M, N, 1);
    return J4C_OK;
}

int tc_split_f32(const float *x, int64_t rows, int64_t cols, float *hi, float *lo, cudaStream_t s) {
    return tc::split(x, rows, cols, hi, lo, s);
}

int tc_split_f32_t(const float *x, int64_t rows, int64_t cols, float *hi, float *lo, cudaStream_t s) {
    return tc::split_t(x, rows, cols, hi, lo, s);
}

int tc_split_f32_both(const float *x, int64_t rows, int64_t cols, float *hi, float *lo, float *hi_t, float *lo_t,
                      cudaStream_t s) {
    return tc::split_t(x, rows, cols, hi_t, lo_t, s, hi, lo);
}

// Any of the splits (stored layout: hi/lo; transposed: hi_t/lo_t; both in
// one pass), with X's max word given (3xFP16) or NULL.
int tc_split_f32_ex(const float *x, int64_t rows, int64_t cols, float *hi, float *lo, float *hi_t, float *lo_t,
                    const uint32_t *max_in, cudaStream_t s) {
    if (hi_t) return tc::split_t(x, rows, cols, hi_t, lo_t, s, hi, lo, max_in);
    return tc::split(x, rows, cols, hi, lo, s, max_in);
}

// tail_ws: scratch of at least tc::tail_scratch_bound bytes, or NULL to take it
// from the library's pool when the product splits its last wave.
static int gemm_presplit_ws(const float *ah, const float *al, const float *bh, const float *bl, float *c, int64_t M,
                            int64_t K, int64_t N, int trans_a, int trans_b, const float *bias, const float *mask,
                            float *act, int64_t batch, int a_batched, int b_batched, void *tail_ws,
                            cudaStream_t s, uint32_t *out_max = nullptr) {
    J4C_REQUIRE(aligned16(ah) && aligned16(al) && aligned16(bh) && aligned16(bl),
                "dot: split operands must be 16-byte aligned");
    // op(A) = A [M,K] is read K-major; A^T (A stored [K,M]) MN-major.
    // op(B) = B [K,N] is read MN-major; B^T (B stored [N,K]) K-major.
    const bool a_mn = trans_a != 0, b_mn = trans_b == 0;
    static const int variant = [] {
        const char *v = getenv("J4C_GEMM_VARIANT");
        return v ? atoi(v) : 1;
    }();
    const tc::Epilogue ep{bias, mask, act, out_max};
    const bool ab = a_batched != 0, bb = b_batched != 0;
    if (tc::split_fp16())
        return tc::launch_gemm_any<256, 4, 16, true>(ah, al, bh, bl, c, M, N, K, a_mn, b_mn, ep, batch, ab, bb, tail_ws, s);
    if (variant == 0)
        return tc::launch_gemm_any<256, 2, 32, false>(ah, al, bh, bl, c, M, N, K, a_mn, b_mn, ep, batch, ab, bb, tail_ws, s);
    return tc::launch_gemm_any<256, 4, 16, false>(ah, al, bh, bl, c, M, N, K, a_mn, b_mn, ep, batch, ab, bb, tail_ws, s);
}

int tc_gemm_presplit(const float *ah, const float *al, const float *bh, const float *bl, float *c, int64_t M,
                     int64_t K, int64_t N, int trans_a, int trans_b, const float *bias, const float *mask,
                     float *act, int64_t batch, int a_batched, int b_batched, cudaStream_t s,
                     uint32_t *out_max) {
    return gemm_presplit_ws(ah, al, bh, bl, c, M, K, N, trans_a, trans_b, bias, mask, act, batch, a_batched,
                            b_batched, nullptr, s, out_max);
}

int tc_gemm_f32(const float *a, const float *b, float *c, int64_t M, int64_t K, int64_t N,
                int trans_a, int trans_b, void *ws, size_t ws_bytes, cudaStream_t s) {
    J4C_REQUIRE(aligned16(ws), "dot: workspace must be 16-byte aligned");
    const int64_t ar = trans_a ? K : M, ac = trans_a ? M : K;  // A as stored
    const int64_t br = trans_b ? N : K, bc = trans_b ? K : N;  // B as stored
    const bool b_transposed = trans_a && !trans_b;  // B is split as B^T: [bc, pitch(br)]
    char *w = static_cast<char *>(ws);
    float *ah = reinterpret_cast<float *>(w);
    float *al = reinterpret_cast<float *>(w + split_buf(ar, ac));
    float *bh = reinterpret_cast<float *>(w + 2 * split_buf(ar, ac));
    float *bl = reinterpret_cast<float *>(w + 2 * split_buf(ar, ac) +
                                          (b_transposed ? split_buf(bc, br) : split_buf(br, bc)));
    // the tail-split scratch follows the largest layout of both splits
    void *tail_ws = w + 2 * std::max(split_buf(M, K), split_buf(K, M)) + 2 * std::max(split_buf(K, N), split_buf(N, K));
    int rc;
    if ((rc = tc::split(a, ar, ac, ah, al, s))) return rc;
    if (b_transposed) {
        // both stored K-leading: B goes in as the split of B^T (K-major)
        if ((rc = tc::split_t(b, br, bc, bh, bl, s))) return rc;
        return gemm_presplit_ws(ah, al, bh, bl, c, M, K, N, trans_a, 1, nullptr, nullptr, nullptr, 1, 0, 0, tail_ws, s);
    }
    if ((rc = tc::split(b, br, bc, bh, bl, s))) return rc;
    return gemm_presplit_ws(ah, al, bh, bl, c, M, K, N, trans_a, trans_b, nullptr, nullptr, nullptr, 1, 0, 0, tail_ws,
                            s);
}

}  // namespace j4c
