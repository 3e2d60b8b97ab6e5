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
//  Promotion: the tensor core's FP32 accumulation does not round to nearest
//  (it truncates), so its error grows linearly with the number of
//  accumulating MMAs and is biased toward zero.  The K loop is therefore cut
//  into chunks (Cfg::CHUNK_KB, CHUNK2_KB); each chunk's partial product goes
//  to one of two TMEM buffers, and the epilogue warps add it into FP32
//  registers with round-to-nearest while the MMA warp fills the other
//  buffer.  The error then grows with sqrt(K) like an FP32 sum, plus a
//  relative bias of about 3.6e-8 per MMA of a chunk (-1.6e-6 for 3xFP16).
//  Split mode 3xFP16 (the default; J4C_GEMM_SPLIT=tf32 selects 3xTF32): the
//  same three products from FP16 operands, at twice the tensor rate of TF32.
//  FP16 has TF32's 11-bit significand but a 5-bit exponent, so every line of
//  an operand -- a row of op(A) (one of the M rows) or a column of op(B) (one
//  of the N columns) -- is scaled by its own power of two 2^e, chosen from
//  the line's largest finite magnitude m so that m 2^e lies in [2^14, 2^15):
//  hi = fp16(x 2^e), lo = fp16(x 2^e - hi).  The scale of a line is constant
//  along K, so it factors out of the line's dot products, and the epilogue
//  multiplies C[i][j] by 2^-(e_i + e_j) (exact, one rounding at most when the
//  result is subnormal).  e spans [-113, 127]: every finite FP32 line is
//  brought into FP16's normal range, whatever the line's magnitude or how far
//  it lies below the rest of the tensor.  Within a line, elements more than
//  2^24 below the line's max fall into FP16 subnormals: their split carries
//  an absolute error of at most ~2^-39 of the line's max.
//  Special values.  The hi/lo decomposition cannot carry an infinity (inf -
//  inf = NaN in lo, 0 * inf = NaN against a partner whose lo is zero), so a
//  split records whether its source holds a NaN or an infinity, and where the
//  source is.  A GEMM either of whose operands does runs its exact path: every
//  output is the reference's sequential FP32 sum (float products added from
//  k = 0 in order, no fused multiply-add, core/ConcreteNDArray.java:452-459)
//  of the FP32 sources, on the CUDA cores -- slow, but the reference's result
//  bit for bit, special values included.
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
// K accumulated in TMEM before promotion: the first two chunks of a work
// unit, then the rest (see Cfg).
// Measured on a B200 (positive operands, where the truncation bias cannot
// cancel): 3xFP16 with 512-deep chunks -3.4e-6 relative at 448 TFLOP/s
// (4096^3), 256-deep -1.6e-6 at 431, 128-deep -0.7e-6 at 400; 3xTF32 at K =
// 8192 -2.3e-6 (256 throughout) and -1.4e-6 (256 then 128) at the same speed.
constexpr int CHUNK_F16_FIRST = 256, CHUNK_F16_REST = 256;
constexpr int CHUNK_TF32_FIRST = 256, CHUNK_TF32_REST = 128;
constexpr int kEpiWarps = 8;      // two warps per TMEM lane quadrant
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kStatusTimeout = 0x7C05;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s without progress
constexpr int kMaxTailSplits = 4; // parts along K of a tile of the last wave
constexpr int kStatusBadSplit = 0x7C06;  // an operand is not a split of the layout its use needs

// ---- split format ----------------------------------------------------------------
// A split of a FLOAT32 array X is two device arrays, hi and lo.  Each holds a
// data matrix [rd, cd] -- X as stored, or X^T for a transposed split -- in
// rows of split_pitch(cd) elements (2-byte halves under 3xFP16, 4-byte tf32
// values under 3xTF32; padding columns zero).  The hi array continues after
// its data (a multiple of 16 bytes) with a SplitHeader and the line words:
// one per data row (a split read K-major, whose rows are M or N) or one per
// data column (read MN-major), each the bits of the largest finite |x| of
// its line, from which the line's scale follows (split_exp).  Both split
// kinds scale: FP16 needs it for range, TF32 for FP32 subnormals, which its
// products do not keep.
constexpr uint32_t kLayoutT = 1;      // the data is X^T
constexpr uint32_t kLayoutCols = 2;   // one line word per data column (MN-major use)
constexpr uint32_t kSplitMagic = 0x53433449u;

struct SplitHeader {
    unsigned long long src;  // X as stored (FP32): what the exact path reads
    unsigned int nonfinite;  // nonzero: X holds a NaN or an infinity
    unsigned int layout;     // kLayoutT | kLayoutCols
    unsigned int lines;      // line words after the header
    unsigned int magic;      // kSplitMagic once a split has been written
    unsigned long long reserved;
};
static_assert(sizeof(SplitHeader) == 32, "split header size");

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
// PAIR: a CTA pair (cluster of 2) computes a 256 x BN tile with
// tcgen05.mma.cta_group::2: each CTA holds 128 rows of op(A) and BN / 2 rows
// of op(B)^T in its shared memory and 128 rows x BN columns of the result in
// its tensor memory, so each SM reads half of B's tile per MMA.
template <int BN, int STAGES, int BK, bool F16 = false, bool PAIR = false>
struct Cfg {
    static_assert(BK == 32 || BK == 16, "BK is 32 (SW128) or 16 (SW64)");
    static constexpr int BKE = BK * 4 / Elt<F16>::SIZE;
    // Promotion chunks: the first two of a work unit are CHUNK_KB k-blocks
    // deep -- while the MMAs fill them the epilogue warps are still storing
    // the previous tile, so they must last as long as that store -- and the
    // rest CHUNK2_KB, shorter, since the tensor core's truncating accumulation
    // biases a partial sum toward zero by about 3.6e-8 per MMA it adds.
    static constexpr int CHUNK_KB = (F16 ? CHUNK_F16_FIRST : CHUNK_TF32_FIRST) / BKE;
    static constexpr int CHUNK2_KB = (F16 ? CHUNK_F16_REST : CHUNK_TF32_REST) / BKE;
    static constexpr int TM = PAIR ? 2 * BM : BM;  // rows of an output tile
    static constexpr int BROWS = PAIR ? BN / 2 : BN;  // rows of op(B)^T in one CTA's stage
    static constexpr int A_BYTES = BM * BK * 4;
    static constexpr int B_BYTES = BROWS * BK * 4;
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

// Non-blocking probe of the phase with the given parity.
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

constexpr uint64_t kShortLimitNs = 1000000ull;  // below this a wait polls without suspending

// Waits for the phase with the given parity; false if the CTA is aborting or
// no progress was seen for limit_ns (then records the status and aborts).
// The pipeline's waits take the launch's limit (j4c_set_wait_limit_ns); the
// drains before exit (honour_abort false) always take kWaitLimitNs, so
// every load and MMA a CTA issued lands before it releases its memory.
__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, volatile int *abort,
                                         int *status, bool honour_abort = true,
                                         uint64_t limit_ns = kWaitLimitNs) {
    if (limit_ns < kShortLimitNs) {
        // A short limit (set for a test of this path): try_wait may suspend
        // the thread until the phase completes, so probe without suspending
        // and read the clock at every probe.
        const uint64_t t0 = now_ns();
        for (;;) {
            if (mbar_test_wait(bar, parity)) return true;
            if (honour_abort && *abort) return false;
            if (now_ns() - t0 > limit_ns) {
                *abort = 1;
                if (status) atomicCAS(status, 0, kStatusTimeout);
                return false;
            }
        }
    }
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = now_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63) == 0) {
            if (honour_abort && *abort) return false;
            if (now_ns() - t0 > limit_ns) {
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

// The CTA pair's TMA load: data into this CTA's shared memory, completion
// bytes to the barrier at `bar`, a shared::cluster address (the pair
// leader's barrier).  No multicast.
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap *map, int x, int y, int z,
                                                 uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
        : "memory");
}
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// The shared::cluster address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
// Every thread of both CTAs of the pair: nothing is left to wait for here
// (the pair's CTAs run together), so the hardware barrier cannot stall.
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
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

// The scale exponent e of a line of an fp16 split from the bits of its
// largest finite |x|: max 2^e in [2^14, 2^15); 0 for a zero line.  A finite
// max is below 2^128, so e >= -113; a max below 2^-112 takes e = 126, which
// still keeps the line's values to 22 significant bits in hi + lo (and
// represents an FP32 subnormal, at most 23 bits above 2^-149, exactly).
// 2^e and 2^-e are then normal floats.
__host__ __device__ __forceinline__ int split_exp(uint32_t maxbits) {
    if (maxbits == 0) return 0;
    const int e = 14 - ((int)((maxbits >> 23) & 0xFF) - 127);
    return e > 126 ? 126 : e;
}

// 2^k as a float, -149 <= k <= 127 (a subnormal below -126).
__device__ __forceinline__ float pow2f(int k) {
    return __uint_as_float(k >= -126 ? (uint32_t)(127 + k) << 23 : 1u << (k + 149));
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// The pair's MMA (issued by the leader CTA for both) and its commits: to the
// barrier at the same offset in both CTAs, or to the leader's alone.
template <bool F16>
__device__ __forceinline__ void mma_issue_pair(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                               uint32_t accumulate) {
    if constexpr (F16) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
            : "memory");
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
            : "memory");
    }
}
__device__ __forceinline__ void mma_commit_pair_both(uint32_t bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
        "h"((uint16_t)3)
        : "memory");
}
__device__ __forceinline__ void mma_commit_pair_leader(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// 16 consecutive TMEM columns of this warp's 32 lanes (tcgen05.ld 32x32b.x16).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
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
// and, with out_lines set (zeroed by the launch), the line words of the
// stored output: out_lines[r] (r < out_rows) the bits of the largest finite
// |value| of stored row r, out_lines[out_rows + c] of stored column c, taken
// over what is written to act (or to C when there is no act), and *out_flag
// nonzero when a written value is a NaN or an infinity -- what a later split
// of that output takes instead of its own max pass.
// The relu' mask may come as bits instead (mask_bits, one bit per element:
// bit c & 31 of word c / 32 of a row of bits_words words, set where the
// mask is > 0), and the relu output's bits (act > 0) may be written the same
// way (act_bits): 1/32 of the bytes.  Bits need C stored untransposed.
struct Epilogue {
    const float *bias;
    const float *mask;
    float *act;
    uint32_t *out_lines;
    int out_rows;
    uint32_t *out_flag;
    const uint32_t *mask_bits;
    uint32_t *act_bits;
    int bits_words;
};

// The bits of |v| for finite v, else 0.
__device__ __forceinline__ uint32_t finite_bits(float v) {
    const uint32_t b = __float_as_uint(v) & 0x7FFFFFFFu;
    return b < 0x7F800000u ? b : 0u;
}

__device__ __forceinline__ float ep_relu(float v) { return (0.0f >= v) ? 0.0f : v; }

// The exact path, for operands one of which holds a NaN or an infinity: each
// output of this CTA's tiles is the reference's dot -- float products of the
// FP32 sources added in k order from 0.0f, no fused multiply-add
// (core/ConcreteNDArray.java:452-459) -- then the epilogue, one element per
// thread step.  A source element (line l, k) of an operand whose data rows
// are its lines (read K-major, not transposed) is src[(z * L + l) * K + k];
// otherwise (MN-major, or a transposed split) src[(z * K + k) * L + l], with
// z the batch entry of a batched operand and L = M for A, N for B.
template <int BN>
__device__ void exact_tiles(const float *__restrict__ A, bool a_col, const float *__restrict__ B, bool b_col,
                            float *__restrict__ C, int M, int N, int K, int store_t, const Epilogue &ep,
                            int batch, int a_batched, int b_batched) {
    const int num_m = (M + BM - 1) / BM, num_n = (N + BN - 1) / BN;
    const int tiles_per_batch = num_m * num_n, num_tiles = tiles_per_batch * batch;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
        const int bidx = t / tiles_per_batch;
        int mt, nt;
        tile_coords(t - bidx * tiles_per_batch, num_m, num_n, mt, nt);
        const float *Ab = A + (a_batched ? (size_t)bidx * M * K : 0);
        const float *Bb = B + (b_batched ? (size_t)bidx * N * K : 0);
        const size_t boff = (size_t)bidx * (size_t)M * (size_t)N;
        if (ep.act_bits) {  // this tile's words start at zero, then take each element's bit
            for (int e = threadIdx.x; e < BM * (BN / 32); e += blockDim.x) {
                const int i = mt * BM + e / (BN / 32), wd = nt * (BN / 32) + e % (BN / 32);
                if (i < M && wd < ep.bits_words) ep.act_bits[(size_t)i * ep.bits_words + wd] = 0u;
            }
            __syncthreads();
        }
        for (int e = threadIdx.x; e < BM * BN; e += blockDim.x) {
            const int i = mt * BM + e / BN, j = nt * BN + e % BN;
            if (i >= M || j >= N) continue;
            float s = 0.0f;
            for (int k = 0; k < K; k++) {
                const float a = a_col ? Ab[(size_t)k * M + i] : Ab[(size_t)i * K + k];
                const float b = b_col ? Bb[(size_t)k * N + j] : Bb[(size_t)j * K + k];
                s = __fadd_rn(s, __fmul_rn(a, b));
            }
            const size_t idx = boff + (store_t ? (size_t)j * M + i : (size_t)i * N + j);
            float v = ep.bias ? __fadd_rn(s, __ldg(ep.bias + (store_t ? i : j))) : s;
            if (ep.mask_bits)
                v = (__ldg(ep.mask_bits + (size_t)i * ep.bits_words + (j >> 5)) >> (j & 31)) & 1u ? v : 0.0f;
            else if (ep.mask)
                v = __ldg(ep.mask + idx) > 0.0f ? v : 0.0f;
            if (C) C[idx] = v;
            if (ep.act) ep.act[idx] = ep_relu(v);
            if (ep.act_bits && ep_relu(v) > 0.0f)
                atomicOr(ep.act_bits + (size_t)i * ep.bits_words + (j >> 5), 1u << (j & 31));
            if (ep.out_lines) {
                const float tv = ep.act ? ep_relu(v) : v;
                const uint32_t m = finite_bits(tv);
                const int sr = store_t ? j : i, sc = store_t ? i : j;
                if (m) {
                    atomicMax(ep.out_lines + sr, m);
                    atomicMax(ep.out_lines + ep.out_rows + sc, m);
                }
                if ((__float_as_uint(tv) & 0x7F800000u) == 0x7F800000u) atomicOr(ep.out_flag, 1u);
            }
        }
        if (ep.act_bits) __syncthreads();  // the tile's bits are settled before the next tile zeroes its own
    }
}

// Loads one operand's hi or lo tile (ROWS of M or N, BKE of K) into smem.
template <int ROWS, int BK, bool MN, bool F16, bool PAIR = false>
__device__ __forceinline__ void load_operand(uint32_t dst, const CUtensorMap *map, int kx, int row0, int z,
                                             uint32_t bar) {
    auto load = [&](uint32_t d, int x, int y) {
        if constexpr (PAIR) tma_load_3d_pair(d, map, x, y, z, bar);
        else tma_load_3d(d, map, x, y, z, bar);
    };
    if constexpr (!MN) {
        load(dst, kx, row0);  // box {BKE, ROWS, 1} of a [batch][rows, K] array
    } else {
        constexpr int W = Elt<F16>::MNW, BOX = 128 * (BK * 4 / Elt<F16>::SIZE);
#pragma unroll
        for (int i = 0; i < ROWS / W; i++)        // boxes {MNW, BKE, 1} of a [batch][K, rows] array
            load(dst + i * BOX, row0 + i * W, kx);
    }
}

// F16: the 3xFP16 split (else 3xTF32).  ahdr / bhdr: the headers of the
// operands' hi arrays, whose line words give the scales.
template <int BN, int STAGES, int BK, bool A_MN, bool B_MN, bool F16, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
gemm_3xtf32_kernel(const __grid_constant__ CUtensorMap tAh, const __grid_constant__ CUtensorMap tAl,
                   const __grid_constant__ CUtensorMap tBh, const __grid_constant__ CUtensorMap tBl,
                   float *__restrict__ C, int M, int N, int K, int num_kb, int vec_store, int store_t,
                   Epilogue ep, int batch, int a_batched, int b_batched, int *status, uint64_t wait_ns, int full_tiles,
                   int splits, float *__restrict__ part, int *__restrict__ arrivals,
                   const SplitHeader *__restrict__ ahdr, const SplitHeader *__restrict__ bhdr) {
    using Q = Cfg<BN, STAGES, BK, F16, PAIR>;
    constexpr int UMMA_K = Elt<F16>::UMMA_K;
    constexpr int NPAIR = PAIR ? 2 : 1;
    // end of chunk n of a unit that starts at k-block kb0 and ends at end
    auto chunk_end = [](int kb0, int n, int end) { return min(end, kb0 + (n < 2 ? Q::CHUNK_KB : Q::CHUNK2_KB)); };
    {
        // What the operands' splits say, the same for every thread: a split
        // must match its use (under 3xFP16 its lines are the rows of a
        // K-major operand, the columns of an MN-major one), and a source
        // with a NaN or an infinity sends the whole product down the exact path.
        const uint32_t a_layout = ahdr->layout, b_layout = bhdr->layout;
        const bool bad = ahdr->magic != kSplitMagic || bhdr->magic != kSplitMagic ||
                         ((a_layout & kLayoutCols) != 0) != A_MN || ((b_layout & kLayoutCols) != 0) != B_MN;
        if (bad) {
            if (threadIdx.x == 0 && status) atomicCAS(status, 0, kStatusBadSplit);
            return;
        }
        if (ahdr->nonfinite | bhdr->nonfinite) {
            exact_tiles<BN>(reinterpret_cast<const float *>(ahdr->src), A_MN || (a_layout & kLayoutT),
                            reinterpret_cast<const float *>(bhdr->src), B_MN || (b_layout & kLayoutT), C, M, N, K,
                            store_t, ep, batch, a_batched, b_batched);
            return;
        }
    }
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Ctl<STAGES> *ctl = reinterpret_cast<Ctl<STAGES> *>(smem + STAGES * Q::STAGE_BYTES);
    volatile int *abort = &ctl->abort;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    // A pair shares its work units: unit u goes to pair u mod (pairs); this
    // CTA holds rows crank * 128.. of each tile and of B's tile rows.
    const uint32_t crank = PAIR ? cluster_ctarank() : 0u;
    const bool leader = crank == 0;
    const int u0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
    const int ustep = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
    const int num_m = (M + Q::TM - 1) / Q::TM, num_n = (N + BN - 1) / BN;
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
            mbar_init(smem_u32(&ctl->tempty[b]), NPAIR * kEpiWarps);  // the leader's counts both CTAs' warps
        }
        mbar_init(smem_u32(&ctl->drain), 1);
        ctl->abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        if constexpr (PAIR) {
            // both CTAs' warp 1, the same destination offset
            asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                             smem_u32(&ctl->tmem_base)),
                         "r"(Q::TMEM_COLS)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
        } else {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                             smem_u32(&ctl->tmem_base)),
                         "r"(Q::TMEM_COLS)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        }
    }
    tc_fence_before();
    if constexpr (PAIR) cluster_sync();  // both CTAs' barriers exist before either signals the other's
    else __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int issued = 0;
            bool ok = true;
            for (int u = u0; ok && u < num_units; u += ustep) {
                const Unit w = unit_of(u, full_tiles, splits, num_kb);
                const int t = w.tile;
                int mt, nt;
                const int bidx = t / tiles_per_batch;
                tile_coords(t - bidx * tiles_per_batch, num_m, num_n, mt, nt);
                const int za = a_batched ? bidx : 0, zb = b_batched ? bidx : 0;
                const int arow = mt * Q::TM + (int)crank * BM, brow = nt * BN + (int)crank * Q::BROWS;
                for (int kb = w.kb0; kb < w.kb1; kb++) {
                    if (!wait_bar(smem_u32(&ctl->empty[stage]), phase ^ 1, abort, status, true, wait_ns)) {
                        ok = false;
                        break;
                    }
                    const uint32_t sb = smem_u32(smem + stage * Q::STAGE_BYTES);
                    // both CTAs' bytes complete the leader's full barrier, which
                    // the leader alone arms with the pair's total
                    const uint32_t fb_local = smem_u32(&ctl->full[stage]);
                    const uint32_t fb = PAIR ? mapa_shared(fb_local, 0) : fb_local;
                    if (leader) mbar_expect_tx(fb_local, NPAIR * Q::STAGE_BYTES);
                    const int kx = kb * Q::BKE;
                    load_operand<BM, BK, A_MN, F16, PAIR>(sb, &tAh, kx, arow, za, fb);
                    load_operand<BM, BK, A_MN, F16, PAIR>(sb + Q::A_BYTES, &tAl, kx, arow, za, fb);
                    load_operand<Q::BROWS, BK, B_MN, F16, PAIR>(sb + 2 * Q::A_BYTES, &tBh, kx, brow, zb, fb);
                    load_operand<Q::BROWS, BK, B_MN, F16, PAIR>(sb + 2 * Q::A_BYTES + Q::B_BYTES, &tBl, kx, brow, zb,
                                                                fb);
                    issued++;
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            // Every load this thread issued must land before the CTA exits:
            // wait (bounded, even when aborting) on the last STAGES slots.  In
            // a pair the leader's full barriers count both CTAs' loads; the
            // follower's land before the pair's final barrier.
            for (int i = 0; leader && i < STAGES && i < issued; i++) {
                if (--stage < 0) {
                    stage = STAGES - 1;
                    phase ^= 1;
                }
                wait_bar(smem_u32(&ctl->full[stage]), phase, abort, status, false);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0 && leader) {
            constexpr uint32_t idesc = idesc_mma<F16>(Q::TM, BN, A_MN, B_MN);
            int stage = 0;
            uint32_t phase = 0;
            int ci = 0;  // chunk counter across tiles: selects the TMEM buffer
            bool ok = true;
            for (int u = u0; ok && u < num_units; u += ustep) {
                const Unit w = unit_of(u, full_tiles, splits, num_kb);
                for (int kb0 = w.kb0, n = 0; ok && kb0 < w.kb1; kb0 = chunk_end(kb0, n, w.kb1), n++, ci++) {
                    const int buf = ci & 1;
                    const uint32_t bph = (ci >> 1) & 1;
                    if (!wait_bar(smem_u32(&ctl->tempty[buf]), bph ^ 1, abort, status, true, wait_ns)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t dcol = tmem + buf * BN;
                    const int kb1 = chunk_end(kb0, n, w.kb1);
                    for (int kb = kb0; kb < kb1; kb++) {
                        if (!wait_bar(smem_u32(&ctl->full[stage]), phase, abort, status, true, wait_ns)) {
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
                            if constexpr (PAIR) {
                                mma_issue_pair<F16>(dcol, al, bh, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
                                mma_issue_pair<F16>(dcol, ah, bl, idesc, 1u);
                                mma_issue_pair<F16>(dcol, ah, bh, idesc, 1u);
                            } else {
                                mma_issue<F16>(dcol, al, bh, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
                                mma_issue<F16>(dcol, ah, bl, idesc, 1u);
                                mma_issue<F16>(dcol, ah, bh, idesc, 1u);
                            }
                        }
                        if constexpr (PAIR) mma_commit_pair_both(smem_u32(&ctl->empty[stage]));
                        else mma_commit(smem_u32(&ctl->empty[stage]));
                        if (++stage == STAGES) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                    if (!ok) break;
                    if constexpr (PAIR) mma_commit_pair_both(smem_u32(&ctl->tfull[buf]));
                    else mma_commit(smem_u32(&ctl->tfull[buf]));
                }
            }
            // All MMAs this thread issued complete before TMEM is released (in
            // a pair, before the pair's final barrier releases the follower).
            if constexpr (PAIR) mma_commit_pair_leader(smem_u32(&ctl->drain));
            else mma_commit(smem_u32(&ctl->drain));
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
        // the leader's tempty barrier counts both CTAs' epilogue warps
        const uint32_t tempty_addr[2] = {
            PAIR && !leader ? mapa_shared(smem_u32(&ctl->tempty[0]), 0) : smem_u32(&ctl->tempty[0]),
            PAIR && !leader ? mapa_shared(smem_u32(&ctl->tempty[1]), 0) : smem_u32(&ctl->tempty[1])};
        for (int u = u0; ok && u < num_units; u += ustep) {
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
            for (int kb0 = w.kb0, n = 0; kb0 < w.kb1; kb0 = chunk_end(kb0, n, w.kb1), n++, ci++) {
                const int buf = ci & 1;
                const uint32_t bph = (ci >> 1) & 1;
                if (!wait_bar(smem_u32(&ctl->tfull[buf]), bph, abort, status, true, wait_ns)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < Q::COLS_PER_WARP / 16; c++) {
                    // 16 columns at a time: fewer registers live beside the 128 accumulators
                    uint32_t r[16];
                    tmem_ld16(tmem + (uint32_t)(buf * BN + cbase + c * 16) + lane_off, r);
#pragma unroll
                    for (int j = 0; j < 16; j++) acc[c * 16 + j] = __fadd_rn(acc[c * 16 + j], __uint_as_float(r[j]));
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    if (PAIR && !leader) mbar_arrive_cluster(tempty_addr[buf]);
                    else mbar_arrive(tempty_addr[buf]);
                }
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
                float *mine = part + (((tix * splits + w.part) * NPAIR + crank) * kEpiWarps + ew) * (size_t)RF + lane;
#pragma unroll
                for (int j = 0; j < Q::COLS_PER_WARP; j++) mine[(size_t)j * 32] = acc[j];
                __threadfence();
                __syncwarp();
                int before = 0;
                if (lane == 0) before = atomicAdd(arrivals + (tix * NPAIR + crank) * kEpiWarps + ew, 1);
                before = __shfl_sync(0xffffffffu, before, 0);
                if (before != splits - 1) continue;  // a later part settles the region
                __threadfence();
                // every partial (this part's too) is read back through L2
                const float *rp = part + ((tix * splits * NPAIR + crank) * kEpiWarps + ew) * (size_t)RF + lane;
#pragma unroll
                for (int j = 0; j < Q::COLS_PER_WARP; j++) {
                    float v = __ldcg(rp + (size_t)j * 32);
#pragma unroll
                    for (int p = 1; p < kMaxTailSplits; p++)
                        if (p < splits)
                            v = __fadd_rn(v, __ldcg(rp + (size_t)p * NPAIR * kEpiWarps * RF + (size_t)j * 32));
                    acc[j] = v;
                }
            }
            const int row = mt * Q::TM + (int)crank * BM + q * 32 + lane;
            const int col0 = nt * BN + cbase;
            const bool row_ok = row < M;
            // The accumulator of C[row][col] is in units of
            // 2^(e_a(row) + e_b(col)), the scales of op(A)'s row line and op(B)'s
            // column line.  A K-major batched operand has lines per batch entry; an
            // MN-major one shares its column lines (taken over all entries).
            const uint32_t *al = reinterpret_cast<const uint32_t *>(ahdr + 1) +
                                 ((!A_MN && a_batched) ? (size_t)bidx * M : 0);
            const uint32_t *bl = reinterpret_cast<const uint32_t *>(bhdr + 1) +
                                 ((!B_MN && b_batched) ? (size_t)bidx * N : 0);
            const int ea = row_ok ? split_exp(__ldg(al + row)) : 0;
            const bool vec_full = row_ok && !store_t && vec_store && col0 + Q::COLS_PER_WARP <= N;
            // relu' mask bits and the relu output's bits of this lane's row, one
            // 32-column word at a time (C stored untransposed): word j / 32 of
            // the lane's columns is at bits + row * bits_words + col0 / 32 + j / 32
            const size_t bits_row = (size_t)row * ep.bits_words + (col0 >> 5);
            uint32_t mword = 0u, aword = 0u;
            const float bias_t = (store_t && ep.bias && row_ok) ? __ldg(ep.bias + row) : 0.0f;
            {
                // lane l reads the line word of column g*32 + l; the warp shares it
                // 2^-(ea + eb) as (2^(nea1) 2^(neb1)) (2^(nea - nea1) 2^(neb - neb1)) with
                // nea = -ea, neb = -eb (each in [-126, 113]) and x1 = x >> 1: every
                // factor and both products are normal floats (exponents in [-126, 114]),
                // the two products differ by at most a factor 4, so the intermediate
                // lies within a factor 4 of the path from v to the result -- exact
                // whenever the result is a normal float.
                const int nea = -ea, nea1 = nea >> 1;
                const float pa1 = __uint_as_float((uint32_t)(127 + nea1) << 23);
                const float pa2 = __uint_as_float((uint32_t)(127 + nea - nea1) << 23);
#pragma unroll
                for (int g = 0; g < Q::COLS_PER_WARP / 32; g++) {
                    const int mycol = col0 + g * 32 + lane;
                    const int neb = mycol < N ? -split_exp(__ldg(bl + mycol)) : 0, neb1 = neb >> 1;
                    const float pb1 = __uint_as_float((uint32_t)(127 + neb1) << 23);
                    const float pb2 = __uint_as_float((uint32_t)(127 + neb - neb1) << 23);
#pragma unroll
                    for (int jj = 0; jj < 32; jj++)
                        acc[g * 32 + jj] = acc[g * 32 + jj] * (pa1 * __shfl_sync(0xffffffffu, pb1, jj)) *
                                           (pa2 * __shfl_sync(0xffffffffu, pb2, jj));
                }
            }
            // Store; afterwards acc[j] holds the stored value (the relu output
            // when act is written; 0 outside C), from which the line maxima are
            // taken.
            if (vec_full) {
                const size_t base = (size_t)row * (size_t)N + col0;
#pragma unroll
                for (int v4 = 0; v4 < Q::COLS_PER_WARP / 4; v4++) {
                    float x[4] = {acc[4 * v4], acc[4 * v4 + 1], acc[4 * v4 + 2], acc[4 * v4 + 3]};
                    if ((v4 & 7) == 0) {  // a new 32-column word
                        mword = ep.mask_bits ? __ldg(ep.mask_bits + bits_row + (v4 >> 3)) : 0u;
                        aword = 0u;
                    }
                    if (ep.bias) {
                        const float4 b = __ldg(reinterpret_cast<const float4 *>(ep.bias + col0) + v4);
                        x[0] = __fadd_rn(x[0], b.x); x[1] = __fadd_rn(x[1], b.y);
                        x[2] = __fadd_rn(x[2], b.z); x[3] = __fadd_rn(x[3], b.w);
                    }
                    if (ep.mask_bits) {
#pragma unroll
                        for (int e = 0; e < 4; e++) x[e] = (mword >> ((4 * v4 + e) & 31)) & 1u ? x[e] : 0.0f;
                    } else if (mask_b) {
                        const float4 m = __ldg(reinterpret_cast<const float4 *>(mask_b + base) + v4);
                        x[0] = m.x > 0.0f ? x[0] : 0.0f; x[1] = m.y > 0.0f ? x[1] : 0.0f;
                        x[2] = m.z > 0.0f ? x[2] : 0.0f; x[3] = m.w > 0.0f ? x[3] : 0.0f;
                    }
                    if (Cb) reinterpret_cast<float4 *>(Cb + base)[v4] = make_float4(x[0], x[1], x[2], x[3]);
                    if (act_b) {
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            x[e] = ep_relu(x[e]);
                            if (x[e] > 0.0f) aword |= 1u << ((4 * v4 + e) & 31);
                        }
                        reinterpret_cast<float4 *>(act_b + base)[v4] = make_float4(x[0], x[1], x[2], x[3]);
                    }
                    if ((v4 & 7) == 7 && ep.act_bits) ep.act_bits[bits_row + (v4 >> 3)] = aword;
#pragma unroll
                    for (int e = 0; e < 4; e++) acc[4 * v4 + e] = x[e];
                }
            } else if (store_t) {
                if (row_ok) {
#pragma unroll
                    for (int j = 0; j < Q::COLS_PER_WARP; j++) {
                        if (col0 + j < N) {
                            const size_t idx = (size_t)(col0 + j) * (size_t)M + row;
                            float v = ep.bias ? __fadd_rn(acc[j], bias_t) : acc[j];
                            if (mask_b) v = __ldg(mask_b + idx) > 0.0f ? v : 0.0f;
                            if (Cb) Cb[idx] = v;
                            if (act_b) {
                                v = ep_relu(v);
                                act_b[idx] = v;
                            }
                            acc[j] = v;
                        }
                    }
                }
            } else {
                const size_t base = (size_t)row * (size_t)N + col0;
#pragma unroll
                for (int j = 0; j < Q::COLS_PER_WARP; j++) {
                    float v = 0.0f;
                    const bool word_in = row_ok && (col0 >> 5) + (j >> 5) < ep.bits_words;
                    if ((j & 31) == 0) {
                        mword = (ep.mask_bits && word_in) ? __ldg(ep.mask_bits + bits_row + (j >> 5)) : 0u;
                        aword = 0u;
                    }
                    if (row_ok && col0 + j < N) {
                        v = ep.bias ? __fadd_rn(acc[j], __ldg(ep.bias + col0 + j)) : acc[j];
                        if (ep.mask_bits)
                            v = (mword >> (j & 31)) & 1u ? v : 0.0f;
                        else if (mask_b)
                            v = __ldg(mask_b + base + j) > 0.0f ? v : 0.0f;
                        if (Cb) Cb[base + j] = v;
                        if (act_b) {
                            v = ep_relu(v);
                            act_b[base + j] = v;
                            if (v > 0.0f) aword |= 1u << (j & 31);
                        }
                    }
                    acc[j] = v;
                    if ((j & 31) == 31 && ep.act_bits && word_in) ep.act_bits[bits_row + (j >> 5)] = aword;
                }
            }
            uint32_t rmax = 0;  // over this lane's values: a stored row (a stored column when store_t)
            if (ep.out_lines) {  // uniform: every lane of the warp gets here
                bool nonfinite = false;
#pragma unroll
                for (int j = 0; j < Q::COLS_PER_WARP; j++) {
                    const bool in_c = row_ok && col0 + j < N;
                    nonfinite |= in_c && (__float_as_uint(acc[j]) & 0x7F800000u) == 0x7F800000u;
                    const uint32_t b = in_c ? finite_bits(acc[j]) : 0u;
                    rmax = max(rmax, b);
                    acc[j] = __uint_as_float(b);
                }
                if (__any_sync(0xffffffffu, nonfinite) && lane == 0) atomicOr(ep.out_flag, 1u);
#pragma unroll
                for (int g = 0; g < Q::COLS_PER_WARP / 32; g++) {
                    // Column maxima over the warp's 32 rows: a butterfly that halves
                    // the group each step, after which lane l holds column g*32 + l.
#pragma unroll
                    for (int off = 16; off >= 1; off >>= 1) {
                        const bool up = (lane & off) != 0;
#pragma unroll
                        for (int i = 0; i < off; i++) {
                            const uint32_t lo_v = __float_as_uint(acc[g * 32 + i]);
                            const uint32_t hi_v = __float_as_uint(acc[g * 32 + i + off]);
                            const uint32_t got = __shfl_xor_sync(0xffffffffu, up ? lo_v : hi_v, off);
                            acc[g * 32 + i] = __uint_as_float(max(up ? hi_v : lo_v, got));
                        }
                    }
                    const int col = col0 + g * 32 + lane;
                    const uint32_t m = __float_as_uint(acc[g * 32]);
                    if (col < N && m) atomicMax(ep.out_lines + (store_t ? col : ep.out_rows + col), m);
                }
            }
            if (ep.out_lines && row_ok && rmax) atomicMax(ep.out_lines + (store_t ? ep.out_rows + row : row), rmax);
        }
    }

    tc_fence_before();
    // a pair: the leader's MMAs (which write the follower's tensor memory and
    // read its shared memory) are drained, and neither CTA signals the other
    // any more, before either releases its memory
    if constexpr (PAIR) cluster_sync();
    else __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        __syncwarp();
        if constexpr (PAIR)
            asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Q::TMEM_COLS)
                         : "memory");
        else
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Q::TMEM_COLS)
                         : "memory");
    }
}

// ---- operand splits ---------------------------------------------------------------------
__device__ __forceinline__ float tf32_round(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r & 0xFFFFE000u);
}

__device__ __forceinline__ bool is_finite_f(float x) { return (__float_as_uint(x) & 0x7F800000u) != 0x7F800000u; }

// A non-finite source element is split as zero (the exact path computes
// every output of a product whose operand holds one); `bad` records it.
__device__ __forceinline__ float finite_or_zero(float x, bool &bad) {
    if (is_finite_f(x)) return x;
    bad = true;
    return 0.0f;
}

// Block 0 thread 0 writes a split's header.  nf: the source's NaN/Inf flag
// as the pass that computed its line maxima left it, written here; or NULL
// when the header was zeroed beforehand and the split's own threads OR in
// what they see (flag_nonfinite).
__device__ __forceinline__ void write_header(SplitHeader *h, const float *src, uint32_t layout, uint32_t lines,
                                             const uint32_t *nf) {
    h->src = reinterpret_cast<unsigned long long>(src);
    if (nf) {
        h->nonfinite = *nf;
        h->reserved = 0;
    }
    h->layout = layout;
    h->lines = lines;
    h->magic = kSplitMagic;
}

// Every warp ORs `bad` into the headers' nonfinite words (when no flag came
// with the line maxima).
__device__ __forceinline__ void flag_nonfinite(bool bad, SplitHeader *h0, SplitHeader *h1, const uint32_t *nf) {
    if (!nf && __any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) {
        if (h0) atomicOr(&h0->nonfinite, 1u);
        if (h1) atomicOr(&h1->nonfinite, 1u);
    }
}

// Line maxima of X [R, C]: rowmax[r] / colmax[c] = the bits of the largest
// finite |x| of row r / column c (each array optional, zeroed beforehand;
// non-negative floats order like their bits as unsigned integers).  Work
// unit (s, g): the 512-column strip s of the rows [g R / G, (g + 1) R / G);
// lane l reads the four columns 4l.. of each 128-column quarter of the strip
// (16-byte loads when X allows), warp w every 8th row from w, four rows per
// step (16 independent loads in flight per thread).  A row's max over the
// strip is reduced over the warp (redux.sync) and added with one atomic; a
// column's over the unit's rows is kept in registers, reduced over the 8
// warps in shared memory and added with one atomic per unit.
// SGD: src is a parameter w and each element first becomes
// w - ((gsrc * scale) * lr), written to out; the maxima are those of the result
// (the SGD update of a weight leaving the line words its next splits take).
template <bool ROWS, bool COLS, bool SGD = false>
__global__ void __launch_bounds__(256) lines_max_kernel(const float *__restrict__ src, int64_t R, int64_t C, int vec,
                                                        int64_t groups, uint32_t *__restrict__ rowmax,
                                                        uint32_t *__restrict__ colmax, uint32_t *__restrict__ flag,
                                                        const float *__restrict__ gsrc = nullptr, float scale = 0.0f,
                                                        float lr = 0.0f, float *__restrict__ out = nullptr) {
    constexpr int TC = 512, RW = 4;
    __shared__ uint32_t cm[COLS ? 8 : 1][COLS ? TC : 1];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t strips = (C + TC - 1) / TC;
    bool bad = false;
    for (int64_t unit = blockIdx.x; unit < strips * groups; unit += gridDim.x) {
        const int64_t s = unit % strips, g = unit / strips;
        const int64_t c0 = s * TC, r_begin = g * R / groups, r_end = (g + 1) * R / groups;
        uint32_t cmx[16];
#pragma unroll
        for (int k = 0; k < 16; k++) cmx[k] = 0;
        for (int64_t rb = r_begin + warp; rb < r_end; rb += 8 * RW) {
            uint32_t b[RW][16];
#pragma unroll
            for (int i = 0; i < RW; i++) {
                const int64_t r = rb + 8 * i;
                const float *p = src + r * C;
#pragma unroll
                for (int qq = 0; qq < 4; qq++) {
                    const int64_t c = c0 + qq * 128 + 4 * lane;
                    if (r < r_end && vec && c + 4 <= C) {
                        const uint4 u = __ldg(reinterpret_cast<const uint4 *>(p + c));
                        b[i][4 * qq] = u.x; b[i][4 * qq + 1] = u.y; b[i][4 * qq + 2] = u.z; b[i][4 * qq + 3] = u.w;
                        if constexpr (SGD) {
                            const float4 gv = __ldg(reinterpret_cast<const float4 *>(gsrc + r * C + c));
                            const float gg[4] = {gv.x, gv.y, gv.z, gv.w};
                            float o[4];
#pragma unroll
                            for (int e = 0; e < 4; e++) {
                                o[e] = __fsub_rn(__uint_as_float(b[i][4 * qq + e]),
                                                 __fmul_rn(__fmul_rn(gg[e], scale), lr));
                                b[i][4 * qq + e] = __float_as_uint(o[e]);
                            }
                            *reinterpret_cast<float4 *>(out + r * C + c) = make_float4(o[0], o[1], o[2], o[3]);
                        }
                    } else {
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            const bool in = r < r_end && c + e < C;
                            b[i][4 * qq + e] = in ? __float_as_uint(p[c + e]) : 0u;
                            if constexpr (SGD) {
                                if (in) {
                                    const float o = __fsub_rn(__uint_as_float(b[i][4 * qq + e]),
                                                              __fmul_rn(__fmul_rn(gsrc[r * C + c + e], scale), lr));
                                    out[r * C + c + e] = o;
                                    b[i][4 * qq + e] = __float_as_uint(o);
                                }
                            }
                        }
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < RW; i++) {
                uint32_t rmx = 0;
#pragma unroll
                for (int k = 0; k < 16; k++) {
                    bad |= (b[i][k] & 0x7F800000u) == 0x7F800000u;
                    const uint32_t m = finite_bits(__uint_as_float(b[i][k]));
                    rmx = max(rmx, m);
                    cmx[k] = max(cmx[k], m);
                }
                if (ROWS) {
                    rmx = __reduce_max_sync(0xffffffffu, rmx);
                    const int64_t r = rb + 8 * i;
                    if (lane == 0 && r < r_end && rmx) atomicMax(rowmax + r, rmx);
                }
            }
        }
        if (COLS) {
#pragma unroll
            for (int k = 0; k < 16; k++) cm[warp][(k >> 2) * 128 + 4 * lane + (k & 3)] = cmx[k];
            __syncthreads();
            for (int cc = threadIdx.x; cc < TC; cc += blockDim.x) {
                uint32_t m = 0;
#pragma unroll
                for (int w = 0; w < 8; w++) m = max(m, cm[w][cc]);
                if (m && c0 + cc < C) atomicMax(colmax + c0 + cc, m);
            }
            __syncthreads();
        }
    }
    if (flag && __any_sync(0xffffffffu, bad) && lane == 0) atomicOr(flag, 1u);
}

// The scale 2^e of a line from its max word.
__device__ __forceinline__ float line_scale(const uint32_t *lines, int64_t i) {
    return pow2f(split_exp(__ldg(lines + i)));
}

// 3xTF32 split of X [rows, cols] in its stored layout -> hi/lo [rows, pitch]
// (pitch = cols rounded up to 4): with row scales from rmax into hr/lr (a
// split for K-major use) and/or column scales from cmax into hc/lc (for
// MN-major use).  The scales keep FP32 subnormals, which TF32 products do
// not, exact.  4 consecutive columns per thread step: 16-byte loads when the
// source allows, 16-byte stores; padding columns are written as zero.
__global__ void __launch_bounds__(256) split_kernel(const float *__restrict__ src, int64_t rows, int64_t cols,
                                                    int64_t pitch, int vec, const uint32_t *__restrict__ rmax,
                                                    const uint32_t *__restrict__ cmax, float *__restrict__ hr,
                                                    float *__restrict__ lr, float *__restrict__ hc,
                                                    float *__restrict__ lc, SplitHeader *hdr_r, SplitHeader *hdr_c,
                                                    uint32_t *__restrict__ copy_r, uint32_t *__restrict__ copy_c,
                                                    const uint32_t *nf) {
    const int64_t q = pitch / 4;
    const int64_t n = rows * q;
    const int64_t t0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x, stride = (int64_t)gridDim.x * blockDim.x;
    if (t0 == 0) {
        if (hdr_r) write_header(hdr_r, src, 0, (uint32_t)rows, nf);
        if (hdr_c) write_header(hdr_c, src, kLayoutCols, (uint32_t)cols, nf);
    }
    if (copy_r)
        for (int64_t i = t0; i < rows; i += stride) copy_r[i] = rmax[i];
    if (copy_c)
        for (int64_t i = t0; i < cols; i += stride) copy_c[i] = cmax[i];
    bool bad = false;
    for (int64_t v = t0; v < n; v += stride) {
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
#pragma unroll
        for (int j = 0; j < 4; j++) x[j] = finite_or_zero(x[j], bad);
        float h[4], l[4];
        if (hr) {
            const float sc = line_scale(rmax, r);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                h[j] = tf32_round(x[j] * sc);
                l[j] = tf32_round(x[j] * sc - h[j]);
            }
            *reinterpret_cast<float4 *>(hr + r * pitch + k) = make_float4(h[0], h[1], h[2], h[3]);
            *reinterpret_cast<float4 *>(lr + r * pitch + k) = make_float4(l[0], l[1], l[2], l[3]);
        }
        if (hc) {
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float sc = k + j < cols ? line_scale(cmax, k + j) : 1.0f;
                h[j] = tf32_round(x[j] * sc);
                l[j] = tf32_round(x[j] * sc - h[j]);
            }
            *reinterpret_cast<float4 *>(hc + r * pitch + k) = make_float4(h[0], h[1], h[2], h[3]);
            *reinterpret_cast<float4 *>(lc + r * pitch + k) = make_float4(l[0], l[1], l[2], l[3]);
        }
    }
    flag_nonfinite(bad, hdr_r, hdr_c, nf);
}

// Transposed 3xTF32 split: X [rows, cols] -> hi/lo of X^T, [cols, pitch] with
// pitch = rows rounded up to 4.  64 x 64 tiles through shared memory; each
// lane reads 4 consecutive floats of an X row (16 bytes when X's rows allow)
// and writes 4 consecutive floats of an X^T row to hi and to lo (16 bytes;
// pitch is a multiple of 4 and the tile origin a multiple of 64).
// With phi / plo set it also writes the split in the stored layout
// ([rows, ppitch], zero padding), from the values it loads: both splits of
// an operand for one read of it.
__global__ void __launch_bounds__(256) split_t_kernel(const float *__restrict__ src, int64_t rows, int64_t cols,
                                                      int64_t pitch, int64_t tiles_c, int vec_in,
                                                      const uint32_t *__restrict__ rmax,
                                                      const uint32_t *__restrict__ cmax, float *__restrict__ hi,
                                                      float *__restrict__ lo, float *__restrict__ phi,
                                                      float *__restrict__ plo, int64_t ppitch, SplitHeader *ht,
                                                      SplitHeader *hp, uint32_t *__restrict__ copy_t,
                                                      uint32_t *__restrict__ copy_p, const uint32_t *nf) {
    __shared__ float tile[64][65];
    const int64_t t0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x, stride = (int64_t)gridDim.x * blockDim.x;
    if (t0 == 0) {
        write_header(ht, src, kLayoutT, (uint32_t)cols, nf);
        if (hp) write_header(hp, src, 0, (uint32_t)rows, nf);
    }
    if (copy_t)
        for (int64_t i = t0; i < cols; i += stride) copy_t[i] = cmax[i];
    if (copy_p)
        for (int64_t i = t0; i < rows; i += stride) copy_p[i] = rmax[i];
    const int64_t c0 = (blockIdx.x % tiles_c) * 64, r0 = (blockIdx.x / tiles_c) * 64;
    const int q = threadIdx.x & 15, w = threadIdx.x >> 4;  // 16 lanes per 64-float row, 16 rows per pass
    bool bad = false;
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
        for (int k = 0; k < 4; k++) {
            v[k] = finite_or_zero(v[k], bad);
            tile[i][4 * q + k] = v[k];
        }
        if (phi && r < rows && c < ppitch) {  // columns past `cols` were loaded as zero
            const float sc = line_scale(rmax, r);
            float h[4], l[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                h[k] = tf32_round(v[k] * sc);
                l[k] = tf32_round(v[k] * sc - h[k]);
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
        const float sc = line_scale(cmax, c);
        float h[4], l[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const float x = tile[4 * q + k][j] * sc;  // rows >= `rows` were loaded as zero
            h[k] = tf32_round(x);
            l[k] = tf32_round(x - h[k]);
        }
        *reinterpret_cast<float4 *>(hi + c * pitch + r) = make_float4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<float4 *>(lo + c * pitch + r) = make_float4(l[0], l[1], l[2], l[3]);
    }
    flag_nonfinite(bad, ht, hp, nf);
}

// ---- 3xFP16 splits ----------------------------------------------------------------------
// hi = fp16(x s), lo = fp16(x s - hi) of a finite x (x s - hi is exact in FP32).
__device__ __forceinline__ uint32_t split2_f16(float a, float b, float sa, float sb, uint32_t &lw) {
    const float xa = a * sa, xb = b * sb;
    const __half ha = __float2half_rn(xa), hb = __float2half_rn(xb);
    const __half la = __float2half_rn(xa - __half2float(ha)), lb = __float2half_rn(xb - __half2float(hb));
    lw = (uint32_t)__half_as_ushort(la) | ((uint32_t)__half_as_ushort(lb) << 16);
    return (uint32_t)__half_as_ushort(ha) | ((uint32_t)__half_as_ushort(hb) << 16);
}

// X [rows, cols] -> fp16 hi/lo [rows, pitch] (pitch = cols rounded up to 8,
// padding written as zero) in the stored layout: with row scales from rmax
// into hr/lr (a split for K-major use) and/or with column scales from cmax
// into hc/lc (for MN-major use).  8 columns per thread step: 32-byte loads
// when the source allows, 16-byte stores.  copy_r / copy_c, when given,
// receive rmax / cmax (the outputs' own line words, when the maxima came
// from elsewhere).
__global__ void __launch_bounds__(256) split16_kernel(const float *__restrict__ src, int64_t rows, int64_t cols,
                                                      int64_t pitch, int vec, const uint32_t *__restrict__ rmax,
                                                      const uint32_t *__restrict__ cmax, __half *__restrict__ hr,
                                                      __half *__restrict__ lr, __half *__restrict__ hc,
                                                      __half *__restrict__ lc, SplitHeader *hdr_r,
                                                      SplitHeader *hdr_c, uint32_t *__restrict__ copy_r,
                                                      uint32_t *__restrict__ copy_c, const uint32_t *nf) {
    const int64_t q = pitch / 8;
    const int64_t n = rows * q;
    const int64_t t0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x, stride = (int64_t)gridDim.x * blockDim.x;
    if (t0 == 0) {
        if (hdr_r) write_header(hdr_r, src, 0, (uint32_t)rows, nf);
        if (hdr_c) write_header(hdr_c, src, kLayoutCols, (uint32_t)cols, nf);
    }
    if (copy_r)
        for (int64_t i = t0; i < rows; i += stride) copy_r[i] = rmax[i];
    if (copy_c)
        for (int64_t i = t0; i < cols; i += stride) copy_c[i] = cmax[i];
    bool bad = false;
    // the column scales of a thread's 8 columns, kept while its columns stay
    // the same (the grid stride is usually a multiple of a row's vectors)
    int64_t sc_k = -1;
    float csc[8];
    // two vectors per thread per step, both loaded before either is split
    for (int64_t v0 = t0; v0 < n; v0 += 2 * stride) {
        float xx[2][8];
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int64_t v = v0 + u * stride;
            if (v >= n) break;
            const int64_t r = v / q, k = (v - r * q) * 8;
            const float *p = src + r * cols + k;
            if (vec && k + 8 <= cols) {
                const float4 t0v = __ldg(reinterpret_cast<const float4 *>(p));
                const float4 t1v = __ldg(reinterpret_cast<const float4 *>(p) + 1);
                xx[u][0] = t0v.x; xx[u][1] = t0v.y; xx[u][2] = t0v.z; xx[u][3] = t0v.w;
                xx[u][4] = t1v.x; xx[u][5] = t1v.y; xx[u][6] = t1v.z; xx[u][7] = t1v.w;
            } else {
#pragma unroll
                for (int j = 0; j < 8; j++) xx[u][j] = (k + j < cols) ? p[j] : 0.0f;
            }
        }
#pragma unroll
        for (int u = 0; u < 2; u++) {
        const int64_t v = v0 + u * stride;
        if (v >= n) break;
        const int64_t r = v / q, k = (v - r * q) * 8;
        float *x = xx[u];
#pragma unroll
        for (int j = 0; j < 8; j++) x[j] = finite_or_zero(x[j], bad);
        if (hr) {
            const float sc = line_scale(rmax, r);
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int j = 0; j < 4; j++) hw[j] = split2_f16(x[2 * j], x[2 * j + 1], sc, sc, lw[j]);
            *reinterpret_cast<uint4 *>(hr + r * pitch + k) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *reinterpret_cast<uint4 *>(lr + r * pitch + k) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
        if (hc) {
            if (k != sc_k) {
#pragma unroll
                for (int j = 0; j < 8; j++) csc[j] = k + j < cols ? line_scale(cmax, k + j) : 1.0f;
                sc_k = k;
            }
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int j = 0; j < 4; j++)
                hw[j] = split2_f16(x[2 * j], x[2 * j + 1], csc[2 * j], csc[2 * j + 1], lw[j]);
            *reinterpret_cast<uint4 *>(hc + r * pitch + k) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *reinterpret_cast<uint4 *>(lc + r * pitch + k) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
        }
    }
    flag_nonfinite(bad, hdr_r, hdr_c, nf);
}

// The fp16 split of X^T ([cols, pitch], pitch = rows rounded up to 8; its
// rows are X's columns, scaled by cmax) and, with phi / plo set, the
// row-scaled split of X in its stored layout ([rows, ppitch], ppitch = cols
// rounded up to 8, scaled by rmax) from the same loads; split_t_kernel's
// tiling, 8-byte stores of 4 halves.
__global__ void __launch_bounds__(256) split16_t_kernel(const float *__restrict__ src, int64_t rows, int64_t cols,
                                                        int64_t pitch, int64_t tiles_c, int vec_in,
                                                        const uint32_t *__restrict__ rmax,
                                                        const uint32_t *__restrict__ cmax, __half *__restrict__ hi,
                                                        __half *__restrict__ lo, __half *__restrict__ phi,
                                                        __half *__restrict__ plo, int64_t ppitch, SplitHeader *ht,
                                                        SplitHeader *hp, uint32_t *__restrict__ copy_t,
                                                        uint32_t *__restrict__ copy_p, const uint32_t *nf) {
    __shared__ float tile[64][65];
    const int64_t t0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x, stride = (int64_t)gridDim.x * blockDim.x;
    if (t0 == 0) {
        write_header(ht, src, kLayoutT, (uint32_t)cols, nf);
        if (hp) write_header(hp, src, 0, (uint32_t)rows, nf);
    }
    if (copy_t)
        for (int64_t i = t0; i < cols; i += stride) copy_t[i] = cmax[i];
    if (copy_p)
        for (int64_t i = t0; i < rows; i += stride) copy_p[i] = rmax[i];
    const int64_t c0 = (blockIdx.x % tiles_c) * 64, r0 = (blockIdx.x / tiles_c) * 64;
    const int q = threadIdx.x & 15, w = threadIdx.x >> 4;
    bool bad = false;
    // all four rows' loads in flight before any of them is used
    float vv[4][4];
#pragma unroll
    for (int pass = 0; pass < 4; pass++) {
        const int64_t r = r0 + pass * 16 + w, c = c0 + 4 * q;
#pragma unroll
        for (int k = 0; k < 4; k++) vv[pass][k] = 0.0f;
        if (r < rows) {
            if (vec_in && c + 4 <= cols) {
                const float4 t = __ldg(reinterpret_cast<const float4 *>(src + r * cols + c));
                vv[pass][0] = t.x; vv[pass][1] = t.y; vv[pass][2] = t.z; vv[pass][3] = t.w;
            } else {
#pragma unroll
                for (int k = 0; k < 4; k++) vv[pass][k] = (c + k < cols) ? src[r * cols + c + k] : 0.0f;
            }
        }
    }
#pragma unroll
    for (int pass = 0; pass < 4; pass++) {
        const int i = pass * 16 + w;
        const int64_t r = r0 + i, c = c0 + 4 * q;
        float *v = vv[pass];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            v[k] = finite_or_zero(v[k], bad);
            tile[i][4 * q + k] = v[k];
        }
        if (phi && r < rows && c < ppitch) {  // columns past `cols` were loaded as zero
            const float sc = line_scale(rmax, r);
            uint32_t lw0, lw1;
            const uint32_t h0 = split2_f16(v[0], v[1], sc, sc, lw0), h1 = split2_f16(v[2], v[3], sc, sc, lw1);
            *reinterpret_cast<uint2 *>(phi + r * ppitch + c) = make_uint2(h0, h1);
            *reinterpret_cast<uint2 *>(plo + r * ppitch + c) = make_uint2(lw0, lw1);
        }
    }
    __syncthreads();
#pragma unroll
    for (int pass = 0; pass < 4; pass++) {
        const int j = pass * 16 + w;
        const int64_t c = c0 + j, r = r0 + 4 * q;
        if (c >= cols || r >= pitch) continue;
        const float sc = line_scale(cmax, c);
        uint32_t lw0, lw1;
        const uint32_t h0 = split2_f16(tile[4 * q][j], tile[4 * q + 1][j], sc, sc, lw0);
        const uint32_t h1 = split2_f16(tile[4 * q + 2][j], tile[4 * q + 3][j], sc, sc, lw1);
        *reinterpret_cast<uint2 *>(hi + c * pitch + r) = make_uint2(h0, h1);
        *reinterpret_cast<uint2 *>(lo + c * pitch + r) = make_uint2(lw0, lw1);
    }
    flag_nonfinite(bad, ht, hp, nf);
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

// Elements per row of a split's data: cols rounded up to a 16-byte multiple.
inline int64_t split_pitch(int64_t cols) { return split_fp16() ? ceil_div(cols, 8) * 8 : ceil_div(cols, 4) * 4; }
inline int64_t split_esize() { return split_fp16() ? 2 : 4; }

// Bytes of a split's data [rd, cd] (a multiple of 16).
inline int64_t split_data_bytes(int64_t rd, int64_t cd) { return rd * split_pitch(cd) * split_esize(); }

// Bytes of one hi or lo array of a split whose data is [rd, cd], for either
// line axis: the data, the header and max(rd, cd) line words.
inline int64_t split_bytes(int64_t rd, int64_t cd) {
    return ceil_div(split_data_bytes(rd, cd) + (int64_t)sizeof(SplitHeader) + 4 * std::max(rd, cd), 16) * 16;
}

// The header of a hi array whose data is [rd, cd], and its line words.
inline SplitHeader *split_header(const float *hi, int64_t rd, int64_t cd) {
    return reinterpret_cast<SplitHeader *>(reinterpret_cast<char *>(const_cast<float *>(hi)) + split_data_bytes(rd, cd));
}
inline uint32_t *split_lines(const float *hi, int64_t rd, int64_t cd) {
    return reinterpret_cast<uint32_t *>(split_header(hi, rd, cd) + 1);
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

// slots: the work units that run at once (one per SM, one per pair of SMs).
static TailPlan tail_plan(int64_t tiles, int64_t num_kb, int64_t chunk_kb, int64_t slots) {
    const int64_t full = tiles / slots * slots, rem = tiles - full;
    if (rem == 0) return TailPlan{tiles, 1};
    int64_t sp = std::min<int64_t>(kMaxTailSplits, slots / rem);
    while (sp > 1 && num_kb / sp < chunk_kb) sp--;
    return sp < 2 ? TailPlan{tiles, 1} : TailPlan{full, (int)sp};
}

// Scratch of a tail split: the parts' FP32 partial tiles (tm x bn each), then
// one arrival counter per (split tile, CTA of the tile, epilogue warp).
static size_t tail_scratch_bytes(int64_t tiles, const TailPlan &p, int tm, int bn) {
    if (p.splits < 2) return 0;
    const int64_t rem = tiles - p.full_tiles;
    return (size_t)(rem * p.splits * tm * bn) * sizeof(float) + (size_t)(rem * (tm / BM) * kEpiWarps) * sizeof(int);
}

// An upper bound of tail_scratch_bytes for an [m, n] product in either
// orientation (the K condition only lowers the number of parts).
size_t tail_scratch_bound(int64_t m, int64_t n, int64_t batch) {
    size_t most = 0;
    for (int o = 0; o < 2; o++)
        for (int tm : {BM, 2 * BM}) {
            const int64_t tiles = ceil_div(o ? n : m, tm) * ceil_div(o ? m : n, 256) * batch;
            const int64_t slots = tm == BM ? sm_count() : sm_count() / 2;
            most = std::max(most, tail_scratch_bytes(tiles, tail_plan(tiles, 1ll << 40, 1, slots), tm, 256));
        }
    return most;
}

template <int BN, int STAGES, int BK, bool A_MN, bool B_MN, bool F16, bool PAIR>
static int launch_gemm(const float *ah, const float *al, const float *bh, const float *bl, float *c,
                       int64_t M, int64_t N, int64_t K, bool store_t, const Epilogue &ep, int64_t batch,
                       bool a_bat, bool b_bat, void *tail_ws, cudaStream_t s) {
    using Q = Cfg<BN, STAGES, BK, F16, PAIR>;
    auto kernel = gemm_3xtf32_kernel<BN, STAGES, BK, A_MN, B_MN, F16, PAIR>;
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
        (rc = make_map(&mBh, bh, br, bc, B_MN, Q::BROWS, BK, bb)) ||
        (rc = make_map(&mBl, bl, br, bc, B_MN, Q::BROWS, BK, bb)))
        return rc;
    int *status = device_status_ptr();
    if (!status) return set_error(J4C_E_OOM, "no device status word");
    const int64_t tiles = ceil_div(M, Q::TM) * ceil_div(N, BN) * batch;
    if (tiles >= (1ll << 30)) return set_error(J4C_E_UNSUPPORTED, "dot: too many output tiles");
    const int64_t num_kb = ceil_div(K, Q::BKE);
    const int64_t slots = PAIR ? sm_count() / 2 : sm_count();
    const TailPlan tp = tail_plan(tiles, num_kb, Q::CHUNK_KB, slots);
    const int64_t units = tp.full_tiles + (tiles - tp.full_tiles) * tp.splits;
    const int grid = (int)std::min<int64_t>(units, slots) * (PAIR ? 2 : 1);
    const int vec = (N % 4 == 0) && aligned16(c) && (!ep.bias || aligned16(ep.bias)) &&
                    (!ep.mask || aligned16(ep.mask)) && (!ep.act || aligned16(ep.act));
    float *part = nullptr;
    int *arrivals = nullptr;
    void *owned = nullptr;
    if (tp.splits > 1) {
        const size_t bytes = tail_scratch_bytes(tiles, tp, Q::TM, BN);
        if (!tail_ws) {
            if ((rc = scratch_alloc(bytes, &owned, s))) return rc;
            tail_ws = owned;
        }
        part = static_cast<float *>(tail_ws);
        arrivals = reinterpret_cast<int *>(part + (tiles - tp.full_tiles) * tp.splits * Q::TM * BN);
        J4C_CUDA(cudaMemsetAsync(arrivals, 0,
                                 (size_t)((tiles - tp.full_tiles) * (Q::TM / BM) * kEpiWarps) * sizeof(int), s));
    }
    if (ep.out_lines) J4C_CUDA(cudaMemsetAsync(ep.out_lines, 0, (size_t)(M + N + 1) * sizeof(uint32_t), s));
    const SplitHeader *ahdr = split_header(ah, ar * ab, ac);
    const SplitHeader *bhdr = split_header(bh, br * bb, bc);
    if constexpr (PAIR) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)grid);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = Q::SMEM_BYTES;
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        const int mi = (int)M, ni = (int)N, ki = (int)K, kbi = (int)num_kb, vs = store_t ? 0 : vec,
                  st = store_t ? 1 : 0, bt = (int)batch, abi = a_bat ? 1 : 0, bbi = b_bat ? 1 : 0,
                  ft = (int)tp.full_tiles;
        J4C_CUDA(cudaLaunchKernelEx(&cfg, kernel, mAh, mAl, mBh, mBl, c, mi, ni, ki, kbi, vs, st, ep, bt, abi, bbi,
                                    status, wait_limit_ns(), ft, tp.splits, part, arrivals, ahdr, bhdr));
        count_launch();
    } else {
        kernel<<<grid, kThreads, Q::SMEM_BYTES, s>>>(mAh, mAl, mBh, mBl, c, (int)M, (int)N, (int)K, (int)num_kb,
                                                     store_t ? 0 : vec, store_t ? 1 : 0, ep, (int)batch,
                                                     a_bat ? 1 : 0, b_bat ? 1 : 0, status, wait_limit_ns(),
                                                     (int)tp.full_tiles, tp.splits, part, arrivals, ahdr, bhdr);
        J4C_LAUNCH_CHECK("gemm_3xtf32_kernel");
    }
    if (owned) return scratch_free(owned, s);
    return J4C_OK;
}

template <int BN, int STAGES, int BK, bool F16, bool PAIR = false>
static int launch_gemm_any(const float *ah, const float *al, const float *bh, const float *bl, float *c,
                           int64_t M, int64_t N, int64_t K, bool a_mn, bool b_mn, const Epilogue &ep,
                           int64_t batch, bool a_bat, bool b_bat, void *tail_ws, cudaStream_t s) {
    if (!a_mn && !b_mn)
        return launch_gemm<BN, STAGES, BK, false, false, F16, PAIR>(ah, al, bh, bl, c, M, N, K, false, ep, batch, a_bat, b_bat, tail_ws, s);
    if (a_mn && !b_mn)
        return launch_gemm<BN, STAGES, BK, true, false, F16, PAIR>(ah, al, bh, bl, c, M, N, K, false, ep, batch, a_bat, b_bat, tail_ws, s);
    // The wide (BN = 256) operand is read MN-major at a smem cost that
    // throttles the tensor pipe, so a K-major A with an MN-major B runs as
    // C^T = op(B)^T . op(A)^T: B's split becomes the (MN-major) A operand,
    // A's the (K-major) B operand, and the epilogue stores transposed.
    if (!a_mn && b_mn)
        return launch_gemm<BN, STAGES, BK, true, false, F16, PAIR>(bh, bl, ah, al, c, N, M, K, true, ep, batch, b_bat, a_bat, tail_ws, s);
    return launch_gemm<BN, STAGES, BK, true, true, F16, PAIR>(ah, al, bh, bl, c, M, N, K, false, ep, batch, a_bat, b_bat, tail_ws, s);
}

// rowmax[r] / colmax[c] (either may be NULL): the bits of the largest finite
// |x| of each row / column of X [rows, cols]; *flag (may be NULL) nonzero
// when X holds a NaN or an infinity.  All three start at zero: the caller
// zeroes them (one memset when they lie back to back).
static int lines_max(const float *src, int64_t rows, int64_t cols, uint32_t *rowmax, uint32_t *colmax,
                     uint32_t *flag, cudaStream_t s) {
    if (!rowmax && !colmax && !flag) return J4C_OK;
    const int vec = (cols % 4 == 0) && aligned16(src);
    // units: 512-column strips times row groups of at least 32 rows, about
    // four per SM
    const int64_t strips = ceil_div(cols, 512);
    const int64_t groups = std::max<int64_t>(1, std::min<int64_t>(ceil_div(rows, 32),
                                                                  ceil_div((int64_t)sm_count() * 4, strips)));
    const unsigned grid = (unsigned)std::min<int64_t>(strips * groups, (int64_t)sm_count() * 8);
    if (rowmax && colmax)
        lines_max_kernel<true, true><<<grid, 256, 0, s>>>(src, rows, cols, vec, groups, rowmax, colmax, flag);
    else if (rowmax)
        lines_max_kernel<true, false><<<grid, 256, 0, s>>>(src, rows, cols, vec, groups, rowmax, colmax, flag);
    else
        lines_max_kernel<false, true><<<grid, 256, 0, s>>>(src, rows, cols, vec, groups, rowmax, colmax, flag);
    J4C_LAUNCH_CHECK("lines_max_kernel");
    return J4C_OK;
}

// out = w - ((g * scale) * lr) over W [rows, cols], with out's line words
// (rows, columns, NaN/Inf flag) in lines, zeroed here: the SGD update of a
// weight that leaves what its next splits take instead of a max pass.
int sgd_update_lines(const float *w, const float *g, int64_t rows, int64_t cols, float scale, float lr, float *out,
                     uint32_t *lines, cudaStream_t s) {
    J4C_REQUIRE(w && g && out && lines, "j4c_sgd_update_lines: NULL argument");
    J4C_REQUIRE(rows > 0 && cols > 0 && rows < (1ll << 31) && cols < (1ll << 31), "j4c_sgd_update_lines: bad extent");
    J4C_CUDA(cudaMemsetAsync(lines, 0, (size_t)(rows + cols + 1) * sizeof(uint32_t), s));
    const int vec = (cols % 4 == 0) && aligned16(w) && aligned16(g) && aligned16(out);
    const int64_t strips = ceil_div(cols, 512);
    const int64_t groups = std::max<int64_t>(1, std::min<int64_t>(ceil_div(rows, 32),
                                                                  ceil_div((int64_t)sm_count() * 4, strips)));
    const unsigned grid = (unsigned)std::min<int64_t>(strips * groups, (int64_t)sm_count() * 8);
    lines_max_kernel<true, true, true><<<grid, 256, 0, s>>>(w, rows, cols, vec, groups, lines, lines + rows,
                                                            lines + rows + cols, g, scale, lr, out);
    J4C_LAUNCH_CHECK("lines_max_kernel (sgd)");
    return J4C_OK;
}

// Any of the splits of X [rows, cols] in one pass over it:
//   r: the stored layout with row lines (read K-major),
//   c: the stored layout with column lines (read MN-major),
//   t: X^T with its rows (X's columns) as lines (read K-major),
// r alone, c alone, t alone, r + c or r + t.  lines_in (may be NULL):
// X's line maxima computed already, rows then columns, as a GEMM epilogue's
// out_lines leaves them (rows, then columns, then the NaN/Inf flag word);
// otherwise a max pass over X computes those needed.
int split_any(const float *src, int64_t rows, int64_t cols, float *hr, float *lr, float *hc, float *lc, float *ht,
              float *lt, const uint32_t *lines_in, cudaStream_t s) {
    if (rows == 0 || cols == 0) return J4C_OK;
    J4C_REQUIRE(!hr == !lr && !hc == !lc && !ht == !lt, "split: hi and lo come in pairs");
    J4C_REQUIRE(hr || hc || ht, "split: no output");
    J4C_REQUIRE(!(hc && ht), "split: the column-line and the transposed split are alternatives, not one pass");
    for (const float *p : {hr, lr, hc, lc, ht, lt})
        J4C_REQUIRE(!p || aligned16(p), "split: hi/lo must be 16-byte aligned");
    J4C_REQUIRE(rows < (1ll << 31) && cols < (1ll << 31), "split: extent too large");
    const bool f16 = split_fp16();
    SplitHeader *hdr_r = hr ? split_header(hr, rows, cols) : nullptr;
    SplitHeader *hdr_c = hc ? split_header(hc, rows, cols) : nullptr;
    SplitHeader *hdr_t = ht ? split_header(ht, cols, rows) : nullptr;
    uint32_t *own_r = hdr_r ? reinterpret_cast<uint32_t *>(hdr_r + 1) : nullptr;
    uint32_t *own_c = hdr_c ? reinterpret_cast<uint32_t *>(hdr_c + 1)
                            : (hdr_t ? reinterpret_cast<uint32_t *>(hdr_t + 1) : nullptr);
    const uint32_t *rmax = nullptr, *cmax = nullptr, *nf = nullptr;
    uint32_t *copy_r = nullptr, *copy_c = nullptr;
    if (lines_in) {
        // the maxima and the NaN/Inf flag came with the call: the kernels
        // copy them into the outputs and write whole headers, nothing to zero
        rmax = lines_in;
        cmax = lines_in + rows;
        nf = lines_in + rows + cols;
        copy_r = own_r;
        copy_c = own_c;
    } else {
        // headers and line words start at zero; the max pass fills the line
        // words and the split kernel ORs the flag into the headers
        if (hdr_r) J4C_CUDA(cudaMemsetAsync(hdr_r, 0, sizeof(SplitHeader) + 4 * rows, s));
        if (hdr_c) J4C_CUDA(cudaMemsetAsync(hdr_c, 0, sizeof(SplitHeader) + 4 * cols, s));
        if (hdr_t) J4C_CUDA(cudaMemsetAsync(hdr_t, 0, sizeof(SplitHeader) + 4 * cols, s));
        int rc = lines_max(src, rows, cols, own_r, own_c, nullptr, s);
        if (rc) return rc;
        rmax = own_r;
        cmax = own_c;
    }
    (void)f16;
    if (ht) {
        const int64_t pitch = split_pitch(rows);
        const int64_t tiles_c = ceil_div(cols, 64), tiles_r = ceil_div(pitch, 64);
        J4C_REQUIRE(tiles_c * tiles_r < (1ll << 31), "split: array too large");
        const int vec_in = (cols % 4 == 0) && aligned16(src);
        if (f16) {
            split16_t_kernel<<<(unsigned)(tiles_c * tiles_r), 256, 0, s>>>(
                src, rows, cols, pitch, tiles_c, vec_in, rmax, cmax, reinterpret_cast<__half *>(ht),
                reinterpret_cast<__half *>(lt), reinterpret_cast<__half *>(hr), reinterpret_cast<__half *>(lr),
                split_pitch(cols), hdr_t, hdr_r, copy_c, copy_r, nf);
            J4C_LAUNCH_CHECK("split16_t_kernel");
        } else {
            split_t_kernel<<<(unsigned)(tiles_c * tiles_r), 256, 0, s>>>(src, rows, cols, pitch, tiles_c, vec_in, rmax,
                                                                         cmax, ht, lt, hr, lr, split_pitch(cols), hdr_t,
                                                                         hdr_r, copy_c, copy_r, nf);
            J4C_LAUNCH_CHECK("split_t_kernel");
        }
        return J4C_OK;
    }
    const int64_t pitch = split_pitch(cols);
    const int vec = (cols % 4 == 0) && aligned16(src);
    if (f16) {
        split16_kernel<<<grid_for(rows * (pitch / 8), 256), 256, 0, s>>>(
            src, rows, cols, pitch, vec, rmax, cmax, reinterpret_cast<__half *>(hr), reinterpret_cast<__half *>(lr),
            reinterpret_cast<__half *>(hc), reinterpret_cast<__half *>(lc), hdr_r, hdr_c, copy_r, copy_c, nf);
        J4C_LAUNCH_CHECK("split16_kernel");
        return J4C_OK;
    }
    split_kernel<<<grid_for(rows * (pitch / 4), 256), 256, 0, s>>>(src, rows, cols, pitch, vec, rmax, cmax, hr, lr, hc,
                                                                   lc, hdr_r, hdr_c, copy_r, copy_c, nf);
    J4C_LAUNCH_CHECK("split_kernel");
    return J4C_OK;
}

}  // namespace tc

bool tc_gemm_supported(int64_t M, int64_t K, int64_t N) {
    // int32 coordinates and extents in the kernel and the tensor maps
    return M >= 1 && N >= 1 && K >= 1 && M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31);
}

// Bytes of one hi or lo array of a split whose data is [rows, cols], 256-byte aligned.
static int64_t split_buf(int64_t rows, int64_t cols) { return ceil_div(tc::split_bytes(rows, cols), 256) * 256; }

// Floats of one hi or lo array of a split whose data is [rows, cols] (either
// line axis): what a caller allocates for each of the two.
int64_t tc_split_floats(int64_t rows, int64_t cols) { return tc::split_bytes(rows, cols) / 4; }

// Elements per row of a split's data with `cols` columns.
int64_t tc_split_pitch(int64_t cols) { return tc::split_pitch(cols); }

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

int tc_split_any(const float *x, int64_t rows, int64_t cols, float *hr, float *lr, float *hc, float *lc, float *ht,
                 float *lt, const uint32_t *lines_in, cudaStream_t s) {
    return tc::split_any(x, rows, cols, hr, lr, hc, lc, ht, lt, lines_in, s);
}

// lines [rows + cols + 1]: X's row maxima, then its column maxima (bits of
// the largest finite |x| of each line), then the NaN/Inf flag, as a GEMM
// epilogue's out_lines.
int tc_sgd_update_lines(const float *w, const float *g, int64_t rows, int64_t cols, float scale, float lr, float *out,
                        uint32_t *lines, cudaStream_t s) {
    return tc::sgd_update_lines(w, g, rows, cols, scale, lr, out, lines, s);
}

int tc_split_lines(const float *x, int64_t rows, int64_t cols, uint32_t *lines, cudaStream_t s) {
    J4C_CUDA(cudaMemsetAsync(lines, 0, (size_t)(rows + cols + 1) * sizeof(uint32_t), s));
    if (rows == 0 || cols == 0) return J4C_OK;
    return tc::lines_max(x, rows, cols, lines, lines + rows, lines + rows + cols, s);
}

// tail_ws: scratch of at least tc::tail_scratch_bound bytes, or NULL to take it
// from the library's pool when the product splits its last wave.
static int gemm_presplit_ws(const float *ah, const float *al, const float *bh, const float *bl, float *c, int64_t M,
                            int64_t K, int64_t N, int trans_a, int trans_b, const float *bias, const float *mask,
                            float *act, int64_t batch, int a_batched, int b_batched, void *tail_ws,
                            cudaStream_t s, uint32_t *out_lines = nullptr, const uint32_t *mask_bits = nullptr,
                            uint32_t *act_bits = nullptr) {
    J4C_REQUIRE(aligned16(ah) && aligned16(al) && aligned16(bh) && aligned16(bl),
                "dot: split operands must be 16-byte aligned");
    J4C_REQUIRE(!out_lines || batch == 1, "dot: line maxima of a batched product");
    // op(A) = A [M,K] is read K-major; A^T (A stored [K,M]) MN-major.
    // op(B) = B [K,N] is read MN-major; B^T (B stored [N,K]) K-major.
    const bool a_mn = trans_a != 0, b_mn = trans_b == 0;
    static const int variant = [] {
        const char *v = getenv("J4C_GEMM_VARIANT");
        return v ? atoi(v) : 1;
    }();
    // bits need C stored untransposed: not the K-major A . MN-major B form,
    // which runs as C^T = op(B)^T . op(A)^T
    J4C_REQUIRE(!(mask_bits || act_bits) || trans_a || trans_b,
                "dot: mask bits need B given as its transposed split (trans_b = 1) or A^T");
    J4C_REQUIRE(!act_bits || act, "dot: relu bits need the relu output");
    J4C_REQUIRE(!(mask_bits || act_bits) || batch == 1, "dot: mask bits of a batched product");
    const tc::Epilogue ep{bias,      mask,     act, out_lines, (int)M, out_lines ? out_lines + M + N : nullptr,
                          mask_bits, act_bits, (int)ceil_div(N, 32)};
    const bool ab = a_batched != 0, bb = b_batched != 0;
    // CTA pairs (256-row tiles, cta_group::2) for 3xFP16 products whose
    // stored rows (the kernel's M: N when C is stored transposed) fill them
    static const bool pair = [] {
        const char *v = getenv("J4C_GEMM_PAIR");
        return !(v && v[0] == '0');
    }();
    const int64_t kernel_m = (!a_mn && b_mn) ? N : M;
    if (tc::split_fp16() && pair && kernel_m >= 2 * tc::BM)
        return tc::launch_gemm_any<256, 6, 16, true, true>(ah, al, bh, bl, c, M, N, K, a_mn, b_mn, ep, batch, ab, bb,
                                                           tail_ws, s);
    if (tc::split_fp16())
        return tc::launch_gemm_any<256, 4, 16, true>(ah, al, bh, bl, c, M, N, K, a_mn, b_mn, ep, batch, ab, bb, tail_ws, s);
    if (variant == 0)
        return tc::launch_gemm_any<256, 2, 32, false>(ah, al, bh, bl, c, M, N, K, a_mn, b_mn, ep, batch, ab, bb, tail_ws, s);
    return tc::launch_gemm_any<256, 4, 16, false>(ah, al, bh, bl, c, M, N, K, a_mn, b_mn, ep, batch, ab, bb, tail_ws, s);
}

int tc_gemm_presplit(const float *ah, const float *al, const float *bh, const float *bl, float *c, int64_t M,
                     int64_t K, int64_t N, int trans_a, int trans_b, const float *bias, const float *mask,
                     float *act, int64_t batch, int a_batched, int b_batched, cudaStream_t s,
                     uint32_t *out_lines, const uint32_t *mask_bits, uint32_t *act_bits) {
    return gemm_presplit_ws(ah, al, bh, bl, c, M, K, N, trans_a, trans_b, bias, mask, act, batch, a_batched,
                            b_batched, nullptr, s, out_lines, mask_bits, act_bits);
}

int tc_gemm_f32(const float *a, const float *b, float *c, int64_t M, int64_t K, int64_t N,
                int trans_a, int trans_b, void *ws, size_t ws_bytes, cudaStream_t s) {
    J4C_REQUIRE(aligned16(ws), "dot: workspace must be 16-byte aligned");
    const int64_t ar = trans_a ? K : M, ac = trans_a ? M : K;  // A as stored
    const int64_t br = trans_b ? N : K, bc = trans_b ? K : N;  // B as stored
    // B stored [K, N] is split as B^T ([bc, pitch(br)], read K-major): both
    // operands K-major is the fastest form
    const bool b_transposed = !trans_b;
    char *w = static_cast<char *>(ws);
    float *ah = reinterpret_cast<float *>(w);
    float *al = reinterpret_cast<float *>(w + split_buf(ar, ac));
    float *bh = reinterpret_cast<float *>(w + 2 * split_buf(ar, ac));
    float *bl = reinterpret_cast<float *>(w + 2 * split_buf(ar, ac) +
                                          (b_transposed ? split_buf(bc, br) : split_buf(br, bc)));
    // the tail-split scratch follows the largest layout of both splits
    void *tail_ws = w + 2 * std::max(split_buf(M, K), split_buf(K, M)) + 2 * std::max(split_buf(K, N), split_buf(N, K));
    int rc;
    // A read K-major (trans_a = 0) takes row lines, MN-major column lines
    if ((rc = trans_a ? tc::split_any(a, ar, ac, nullptr, nullptr, ah, al, nullptr, nullptr, nullptr, s)
                      : tc::split_any(a, ar, ac, ah, al, nullptr, nullptr, nullptr, nullptr, nullptr, s)))
        return rc;
    if (b_transposed) {
        if ((rc = tc::split_any(b, br, bc, nullptr, nullptr, nullptr, nullptr, bh, bl, nullptr, s))) return rc;
        return gemm_presplit_ws(ah, al, bh, bl, c, M, K, N, trans_a, 1, nullptr, nullptr, nullptr, 1, 0, 0, tail_ws, s);
    }
    // B stored [N, K] is read K-major with row lines
    if ((rc = tc::split_any(b, br, bc, bh, bl, nullptr, nullptr, nullptr, nullptr, nullptr, s))) return rc;
    return gemm_presplit_ws(ah, al, bh, bl, c, M, K, N, trans_a, trans_b, nullptr, nullptr, nullptr, 1, 0, 0, tail_ws,
                            s);
}

}  // namespace j4c
