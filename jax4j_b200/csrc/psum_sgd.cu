// psum_sgd.cu -- the gradient all-reduce fused with the SGD update, over
// peer memory (one process per GPU, NVLink / NVSwitch).
//
// The reference's data-parallel step sums every shard's gradients with
// SharedCollective.psum (api/SharedCollective.java:44-54; the PSUM VJP is
// another psum, api/Grad.java:429-434) and then updates each parameter with
// elementwise ops (w - g * (1/D) * lr).  Here one bucket of packed gradients
// goes through, on each rank r of D, on one stream:
//
//   1. entry: a one-CTA kernel tells every peer "my gradients are packed"
//      (st.release.sys into the peer's flag block) and waits until every peer
//      has said the same for this call;
//   2. the NVLink traffic of the reduce-scatter: D - 1 copies (the copy
//      engines, no SM) of the peers' gradients of slice r into a local
//      staging buffer;
//   3. reduce + update (SMs, HBM only): the D contributions of slice r are
//      summed in rank order 0..D-1, w - ((g * scale) * lr) is applied to this
//      rank's parameters of the slice, and the result goes to this rank's
//      exchange buffer U and to its own output; the kernel's last CTA tells
//      every peer "slice r is in U";
//   4. gather wait: a one-CTA kernel waits for every peer's "slice p is in U";
//   5. the NVLink traffic of the all-gather: D - 1 copies of the peers'
//      slices out of their U into this rank's output.
//
// Every rank ends with the same bits.  No rank writes another rank's memory
// except the flag words, so nothing a peer is still reading is changed
// remotely, and the bytes that cross NVLink (2 (D-1)/D of the bucket each
// way, a ring all-reduce's) move on copy engines while the SMs keep running
// the backward's GEMMs.  The update needs no separate pass over HBM.
// Buffer reuse: a rank packs the next call's gradients only after its
// gather wait, which proves every peer finished its reduce (and so its
// copies of this rank's gradients); a rank's next reduce overwrites U only
// after its next entry wait, which proves every peer finished this call's
// copies out of U.
// Every wait is bounded (j4c_set_wait_limit_ns, 2 s unless set): on expiry
// the waiting kernel records status 0x7C05 and marks the group failed (no
// further "slice done" signals), so a rank that never arrives produces an
// error on the others, not a hang.  No cluster multicast and no multimem is
// used; no library kernel is given a peer's memory.
#include <algorithm>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace j4c {
namespace psum_sgd {

constexpr int kMaxRanks = 8;
constexpr int kFlagWords = 64;  // per rank: entry[8], slice_done[8], epoch, done, failed
constexpr int kEntry = 0, kSliceDone = 8, kEpoch = 16, kDone = 17, kFailed = 18;
constexpr int kMaxSegs = 16;
constexpr int kThreads = 256;
constexpr int kStatusTimeout = 0x7C05;

// This rank's parameters of the bucket, leaf by leaf: segment i holds the
// bucket's vectors [end4[i-1], end4[i]) at params[i] (end4[-1] = 0).
struct Segs {
    int n;
    int64_t end4[kMaxSegs];
    const float *params[kMaxSegs];
};

struct Flags {
    uint32_t *peer[kMaxRanks];  // rank p's flag block, mapped here (this rank's own at index r)
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Waits until *flag has reached epoch (wrapping compare); false on expiry.
__device__ __forceinline__ bool wait_epoch(const uint32_t *flag, uint32_t epoch, uint64_t limit_ns) {
    if ((int32_t)(ld_acquire_sys(flag) - epoch) >= 0) return true;
    const uint64_t t0 = now_ns();
    while ((int32_t)(ld_acquire_sys(flag) - epoch) < 0) {
        if (now_ns() - t0 > limit_ns) return false;
        __nanosleep(128);
    }
    return true;
}

__device__ __forceinline__ uint32_t call_epoch(const uint32_t *mine) {
    return *(volatile const uint32_t *)(mine + kEpoch) + 1u;
}

// Thread t < D: signals peer t (when `signal`) and waits for peer t's word
// `slot` of this rank's block to reach this call's epoch.
__global__ void __launch_bounds__(32) barrier_kernel(Flags F, int D, int r, int slot, int signal, int close,
                                                     int *status, uint64_t limit_ns) {
    uint32_t *mine = F.peer[r];
    const uint32_t epoch = call_epoch(mine);
    const int t = threadIdx.x;
    bool ok = true;
    if (t < D) {
        if (signal) {
            __threadfence_system();  // this rank's packed gradients before the word that announces them
            st_release_sys(F.peer[t] + slot + r, epoch);
        }
        ok = wait_epoch(mine + slot + t, epoch, limit_ns);
        if (!ok) {
            atomicCAS(status, 0, kStatusTimeout);
            atomicExch(mine + kFailed, 1u);
        }
    }
    __syncwarp();
    if (close && t == 0) atomicExch(mine + kEpoch, epoch);  // the call is over on this rank
}

// out[lo..hi) and U[lo..hi) = w - ((sum_p g_p) * scale) * lr over this
// rank's slice (float4 vectors [lo4, hi4) of the bucket), the contributions
// in rank order: this rank's own packed gradients at `own`, every peer's in
// `stage` (peer p < r at slot p, p > r at slot p - 1, each hi4 - lo4 vectors).
template <int NR>
__global__ void __launch_bounds__(kThreads) reduce_update_kernel(Flags F, Segs S, int D, int r, int64_t lo4,
                                                                 int64_t hi4, const float *__restrict__ own,
                                                                 const float *__restrict__ stage, float scale,
                                                                 float lr, float *__restrict__ upd,
                                                                 float *__restrict__ out) {
    uint32_t *mine = F.peer[r];
    const int64_t len4 = hi4 - lo4;
    const float4 *own4 = reinterpret_cast<const float4 *>(own);
    const float4 *st4 = reinterpret_cast<const float4 *>(stage);
    float4 *u4 = reinterpret_cast<float4 *>(upd);
    float4 *o4 = reinterpret_cast<float4 *>(out);
    int seg = 0;  // a thread's vectors increase, so its segment only moves forward
    for (int64_t v = lo4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < hi4;
         v += (int64_t)gridDim.x * blockDim.x) {
        float4 g[NR];
#pragma unroll
        for (int p = 0; p < NR; p++)
            if (p < D) g[p] = p == r ? own4[v] : st4[(int64_t)(p < r ? p : p - 1) * len4 + (v - lo4)];
        float4 sum = g[0];
#pragma unroll
        for (int p = 1; p < NR; p++)
            if (p < D) {
                sum.x = __fadd_rn(sum.x, g[p].x);
                sum.y = __fadd_rn(sum.y, g[p].y);
                sum.z = __fadd_rn(sum.z, g[p].z);
                sum.w = __fadd_rn(sum.w, g[p].w);
            }
        while (seg < S.n - 1 && v >= S.end4[seg]) seg++;
        const int64_t base = seg ? S.end4[seg - 1] : 0;
        const float4 w = reinterpret_cast<const float4 *>(S.params[seg])[v - base];
        float4 o;
        o.x = __fsub_rn(w.x, __fmul_rn(__fmul_rn(sum.x, scale), lr));
        o.y = __fsub_rn(w.y, __fmul_rn(__fmul_rn(sum.y, scale), lr));
        o.z = __fsub_rn(w.z, __fmul_rn(__fmul_rn(sum.z, scale), lr));
        o.w = __fsub_rn(w.w, __fmul_rn(__fmul_rn(sum.w, scale), lr));
        u4[v] = o;
        o4[v] = o;
    }
    // every thread's stores of U are visible system-wide before the CTA counts itself done
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint32_t prev = atomicAdd(mine + kDone, 1u);
        if (prev == gridDim.x - 1) {  // the last CTA of this rank: the whole slice is in U
            __threadfence_system();
            const uint32_t epoch = call_epoch(mine);
            // after a failed wait the slice is not announced: peers are left to
            // time out (and report it) rather than read it
            if (atomicAdd(mine + kFailed, 0u) == 0u)
                for (int p = 0; p < D; p++) st_release_sys(F.peer[p] + kSliceDone + r, epoch);
            atomicExch(mine + kDone, 0u);
        }
    }
}

}  // namespace psum_sgd
}  // namespace j4c

using namespace j4c;

int j4c_peer_alloc(size_t bytes, void **ptr, void *handle, size_t handle_len) {
    J4C_REQUIRE(ptr && handle, "j4c_peer_alloc: NULL argument");
    J4C_REQUIRE(handle_len >= sizeof(cudaIpcMemHandle_t), "j4c_peer_alloc: the handle needs %zu bytes",
                sizeof(cudaIpcMemHandle_t));
    J4C_REQUIRE(bytes > 0, "j4c_peer_alloc: empty buffer");
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return set_error(J4C_E_OOM, "j4c_peer_alloc: cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
    J4C_CUDA(cudaMemset(p, 0, bytes));
    cudaIpcMemHandle_t h;
    e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return cuda_status(e, "cudaIpcGetMemHandle");
    }
    memcpy(handle, &h, sizeof(h));
    *ptr = p;
    return J4C_OK;
}

int j4c_peer_open(const void *handle, size_t handle_len, void **ptr) {
    J4C_REQUIRE(ptr && handle, "j4c_peer_open: NULL argument");
    J4C_REQUIRE(handle_len >= sizeof(cudaIpcMemHandle_t), "j4c_peer_open: short handle");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    J4C_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return J4C_OK;
}

int j4c_peer_close(void *ptr) {
    J4C_REQUIRE(ptr, "j4c_peer_close: NULL pointer");
    J4C_CUDA(cudaIpcCloseMemHandle(ptr));
    return J4C_OK;
}

int j4c_peer_free(void *ptr) {
    J4C_REQUIRE(ptr, "j4c_peer_free: NULL pointer");
    J4C_CUDA(cudaFree(ptr));
    return J4C_OK;
}

namespace j4c {
namespace psum_sgd {

// Copies over NVLink are spread over kHelpers side streams, so that several
// copy engines move one bucket at once (one stream's copies run one after
// another): fork from the caller's stream with an event, join back with one
// event per helper.  Under graph capture the fork and join become graph
// edges.  One set of helpers per device, created on first use.
constexpr int kHelpers = 4;
struct Helpers {
    cudaStream_t stream[kHelpers];
    cudaEvent_t fork, join[kHelpers];
};

static int helpers_for_device(Helpers **out) {
    static std::mutex mu;
    static std::vector<Helpers *> per_device;
    int dev = 0;
    J4C_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(mu);
    if ((int)per_device.size() <= dev) per_device.resize(dev + 1, nullptr);
    if (!per_device[dev]) {
        Helpers *h = new Helpers();
        for (int k = 0; k < kHelpers; k++) {
            J4C_CUDA(cudaStreamCreateWithFlags(&h->stream[k], cudaStreamNonBlocking));
            J4C_CUDA(cudaEventCreateWithFlags(&h->join[k], cudaEventDisableTiming));
        }
        J4C_CUDA(cudaEventCreateWithFlags(&h->fork, cudaEventDisableTiming));
        per_device[dev] = h;
    }
    *out = per_device[dev];
    return J4C_OK;
}

struct Copy {
    void *dst;
    const void *src;
    size_t bytes;
};

// Enqueues the copies after everything on s, spread over the helpers in
// pieces of at least kMinPiece bytes (16-byte multiples), and makes s wait
// for all of them.
constexpr size_t kMinPiece = 4u << 20;
static int copies_on_helpers(cudaStream_t s, const std::vector<Copy> &copies) {
    Helpers *h = nullptr;
    int rc = helpers_for_device(&h);
    if (rc != J4C_OK) return rc;
    J4C_CUDA(cudaEventRecord(h->fork, s));
    for (int k = 0; k < kHelpers; k++) J4C_CUDA(cudaStreamWaitEvent(h->stream[k], h->fork, 0));
    int next = 0;
    for (const Copy &c : copies) {
        const size_t pieces = std::max<size_t>(1, std::min<size_t>(kHelpers, c.bytes / kMinPiece));
        const size_t per = (c.bytes / pieces + 15) & ~size_t(15);
        for (size_t off = 0; off < c.bytes; off += per) {
            const size_t b = std::min(per, c.bytes - off);
            J4C_CUDA(cudaMemcpyAsync(static_cast<char *>(c.dst) + off, static_cast<const char *>(c.src) + off, b,
                                     cudaMemcpyDeviceToDevice, h->stream[next]));
            next = (next + 1) % kHelpers;
        }
    }
    for (int k = 0; k < kHelpers; k++) {
        J4C_CUDA(cudaEventRecord(h->join[k], h->stream[k]));
        J4C_CUDA(cudaStreamWaitEvent(s, h->join[k], 0));
    }
    return J4C_OK;
}

}  // namespace psum_sgd
}  // namespace j4c

size_t j4c_psum_sgd_flag_bytes(void) { return psum_sgd::kFlagWords * sizeof(uint32_t); }

int j4c_psum_sgd(const float *const *grads, const float *const *upd, uint32_t *const *flags, int nranks, int rank,
                 int64_t n, int nsegs, const int64_t *seg_len, const float *const *params, float scale, float lr,
                 float *stage, float *out, j4c_stream stream) {
    using namespace psum_sgd;
    J4C_REQUIRE(grads && upd && flags && seg_len && params && out && stage, "j4c_psum_sgd: NULL argument");
    J4C_REQUIRE(nranks >= 1 && nranks <= kMaxRanks, "j4c_psum_sgd: %d ranks (1..%d)", nranks, kMaxRanks);
    J4C_REQUIRE(rank >= 0 && rank < nranks, "j4c_psum_sgd: rank %d of %d", rank, nranks);
    J4C_REQUIRE(n >= 4 * (int64_t)nranks && n % 4 == 0,
                "j4c_psum_sgd: n = %lld must be a multiple of 4 and at least 4 per rank", (long long)n);
    J4C_REQUIRE(nsegs >= 1 && nsegs <= kMaxSegs, "j4c_psum_sgd: %d parameter segments (1..%d)", nsegs, kMaxSegs);
    Flags F;
    memset(&F, 0, sizeof(F));
    for (int p = 0; p < nranks; p++) {
        J4C_REQUIRE(grads[p] && upd[p] && flags[p], "j4c_psum_sgd: rank %d's buffers are NULL", p);
        J4C_REQUIRE(aligned16(grads[p]) && aligned16(upd[p]) && aligned16(flags[p]),
                    "j4c_psum_sgd: rank %d's buffers are not 16-byte aligned", p);
        F.peer[p] = flags[p];
    }
    Segs S;
    memset(&S, 0, sizeof(S));
    S.n = nsegs;
    int64_t end = 0;
    for (int i = 0; i < nsegs; i++) {
        J4C_REQUIRE(seg_len[i] > 0 && seg_len[i] % 4 == 0 && params[i] && aligned16(params[i]),
                    "j4c_psum_sgd: parameter segment %d must be a non-empty multiple of 4 floats, 16-byte aligned", i);
        end += seg_len[i] / 4;
        S.end4[i] = end;
        S.params[i] = params[i];
    }
    J4C_REQUIRE(end * 4 == n, "j4c_psum_sgd: the segments hold %lld floats, the bucket %lld", (long long)(end * 4),
                (long long)n);
    J4C_REQUIRE(aligned16(out) && aligned16(stage), "j4c_psum_sgd: out / stage not 16-byte aligned");
    int *status = device_status_ptr();
    if (!status) return set_error(J4C_E_OOM, "j4c_psum_sgd: no status word");
    const int64_t n4 = n / 4;
    auto lo_of = [&](int p) { return n4 * p / nranks; };
    const int64_t lo4 = lo_of(rank), hi4 = lo_of(rank + 1), len4 = hi4 - lo4;
    const uint64_t limit = wait_limit_ns();
    cudaStream_t s = as_stream(stream);
    const size_t vb = 4 * sizeof(float);
    // 1. entry
    barrier_kernel<<<1, 32, 0, s>>>(F, nranks, rank, kEntry, 1, 0, status, limit);
    count_launch();
    J4C_CUDA(cudaGetLastError());
    // 2. the peers' gradients of this rank's slice, over NVLink by the copy engines
    std::vector<Copy> copies;
    for (int p = 0, k = 0; p < nranks; p++) {
        if (p == rank) continue;
        copies.push_back({stage + (size_t)k * len4 * 4, grads[p] + (size_t)lo4 * 4, (size_t)len4 * vb});
        k++;
    }
    int rc = copies_on_helpers(s, copies);
    if (rc != J4C_OK) return rc;
    // 3. reduce + update of the slice, local
    const unsigned g = (unsigned)std::max<int64_t>(
        1, std::min<int64_t>((len4 + kThreads - 1) / kThreads, 2 * (int64_t)sm_count()));
    float *my_upd = const_cast<float *>(upd[rank]);
    if (nranks <= 2)
        reduce_update_kernel<2><<<g, kThreads, 0, s>>>(F, S, nranks, rank, lo4, hi4, grads[rank], stage, scale, lr,
                                                       my_upd, out);
    else if (nranks <= 4)
        reduce_update_kernel<4><<<g, kThreads, 0, s>>>(F, S, nranks, rank, lo4, hi4, grads[rank], stage, scale, lr,
                                                       my_upd, out);
    else
        reduce_update_kernel<8><<<g, kThreads, 0, s>>>(F, S, nranks, rank, lo4, hi4, grads[rank], stage, scale, lr,
                                                       my_upd, out);
    count_launch();
    J4C_CUDA(cudaGetLastError());
    // 4. every peer's slice is in its U; this call's epoch closes on this rank
    barrier_kernel<<<1, 32, 0, s>>>(F, nranks, rank, kSliceDone, 0, 1, status, limit);
    count_launch();
    J4C_CUDA(cudaGetLastError());
    // 5. the peers' updated slices, over NVLink by the copy engines
    copies.clear();
    for (int p = 0; p < nranks; p++) {
        if (p == rank) continue;
        const int64_t plo = lo_of(p), phi = lo_of(p + 1);
        copies.push_back({out + (size_t)plo * 4, upd[p] + (size_t)plo * 4, (size_t)(phi - plo) * vb});
    }
    return copies_on_helpers(s, copies);
}
