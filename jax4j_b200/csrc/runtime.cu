// runtime.cu -- errors, devices, streams and storage of libjax4j_cuda.so.
//
// Storage replaces the reference's host Storage records
// (core/ConcreteNDArray.java:47-87) and TornadoVM's copy-every-call transfers
// (backend/TornadoVMBackend.java:33-44): buffers stay resident in HBM and
// move only on an explicit j4c_memcpy_*.
#include <atomic>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace j4c {

static thread_local std::string t_last_error;

int set_error(int code, const char *fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return code;
}

void clear_error() { t_last_error.clear(); }

static std::atomic<uint64_t> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int cuda_status(cudaError_t e, const char *what) {
    int code = (e == cudaErrorMemoryAllocation) ? J4C_E_OOM : J4C_E_CUDA;
    return set_error(code, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

int sm_count() {
    static std::mutex mu;
    static std::vector<int> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    std::lock_guard<std::mutex> lock(mu);
    if ((int)cache.size() <= dev) cache.resize(dev + 1, 0);
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

std::atomic<uint64_t> g_wait_limit_ns{2000000000ull};

uint64_t wait_limit_ns() { return g_wait_limit_ns.load(std::memory_order_relaxed); }

int *device_status_ptr() {
    static std::mutex mu;
    static std::vector<int *> words;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if ((int)words.size() <= dev) words.resize(dev + 1, nullptr);
    if (!words[dev]) {
        int *p = nullptr;
        if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
        if (cudaMemset(p, 0, sizeof(int)) != cudaSuccess) return nullptr;
        words[dev] = p;
    }
    return words[dev];
}

// The pool keeps freed blocks for reuse, so stream-ordered scratch costs no
// cudaMalloc after warm-up.
static void configure_pool_once(int dev) {
    static std::mutex mu;
    static std::vector<char> done;
    std::lock_guard<std::mutex> lock(mu);
    if ((int)done.size() <= dev) done.resize(dev + 1, 0);
    if (done[dev]) return;
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
        uint64_t threshold = UINT64_MAX;
        cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold);
    }
    done[dev] = 1;
}

int scratch_alloc(size_t bytes, void **out, cudaStream_t s) {
    int dev = 0;
    J4C_CUDA(cudaGetDevice(&dev));
    configure_pool_once(dev);
    if (bytes == 0) bytes = 16;
    J4C_CUDA(cudaMallocAsync(out, bytes, s));
    return J4C_OK;
}

int scratch_free(void *p, cudaStream_t s) {
    if (p) J4C_CUDA(cudaFreeAsync(p, s));
    return J4C_OK;
}

int64_t shape_numel(const int64_t *d, int r) {
    int64_t n = 1;
    for (int i = 0; i < r; i++) n *= d[i];
    return n;
}

bool broadcast_shape(const int64_t *a, int ar, const int64_t *b, int br, int64_t *out, int *orank) {
    int rank = ar > br ? ar : br;
    if (rank > kMaxDims) return false;
    for (int i = 0; i < rank; i++) {
        int64_t da = i < rank - ar ? 1 : a[i - (rank - ar)];
        int64_t db = i < rank - br ? 1 : b[i - (rank - br)];
        if (da != db && da != 1 && db != 1) return false;
        out[i] = da > db ? da : db;
    }
    *orank = rank;
    return true;
}

bool make_indexer(Indexer &ix, const int64_t *out_dims, int out_rank, int nops,
                  const int64_t *const *op_dims, const int *op_ranks) {
    if (out_rank > kMaxDims || nops > 3) return false;
    // Right-align each operand, derive its row-major strides, zero them on
    // broadcast dims, then drop size-1 output dims and merge contiguous runs.
    int64_t st[3][kMaxDims] = {};
    for (int k = 0; k < nops; k++) {
        int r = op_ranks[k];
        if (r > out_rank) return false;
        int64_t s = 1;
        for (int i = out_rank - 1; i >= 0; i--) {
            int j = i - (out_rank - r);
            int64_t d = j >= 0 ? op_dims[k][j] : 1;
            if (d != out_dims[i] && d != 1) return false;
            st[k][i] = (d == 1) ? 0 : s;
            s *= d;
        }
    }
    ix.nops = nops;
    ix.rank = 0;
    for (int i = 0; i < out_rank; i++) {
        if (out_dims[i] == 1) continue;
        if (ix.rank > 0) {
            int p = ix.rank - 1;
            bool merge = true;
            for (int k = 0; k < nops; k++)
                if (ix.stride[k][p] != st[k][i] * out_dims[i]) merge = false;
            if (merge) {
                ix.size[p] *= out_dims[i];
                for (int k = 0; k < nops; k++) ix.stride[k][p] = st[k][i];
                continue;
            }
        }
        ix.size[ix.rank] = out_dims[i];
        for (int k = 0; k < 3; k++) ix.stride[k][ix.rank] = k < nops ? st[k][i] : 0;
        ix.rank++;
    }
    if (ix.rank == 0) {  // a single element
        ix.rank = 1;
        ix.size[0] = 1;
        for (int k = 0; k < 3; k++) ix.stride[k][0] = 0;
    }
    return true;
}

}  // namespace j4c

using namespace j4c;

extern "C" {

int j4c_abi_version(void) { return J4C_ABI_VERSION; }

int j4c_kernel_launches(uint64_t *out) {
    J4C_REQUIRE(out, "j4c_kernel_launches: out is NULL");
    *out = g_launches.load(std::memory_order_relaxed);
    return J4C_OK;
}

const char *j4c_last_error(void) { return t_last_error.c_str(); }

int j4c_device_count(int *out) {
    J4C_REQUIRE(out, "j4c_device_count: out is NULL");
    int n = 0;
    J4C_CUDA(cudaGetDeviceCount(&n));
    *out = n;
    return J4C_OK;
}

int j4c_set_device(int device) {
    J4C_CUDA(cudaSetDevice(device));
    return J4C_OK;
}

int j4c_get_device(int *out) {
    J4C_REQUIRE(out, "j4c_get_device: out is NULL");
    J4C_CUDA(cudaGetDevice(out));
    return J4C_OK;
}

int j4c_enable_peer_access(int device, int peer) {
    if (device == peer) return J4C_OK;
    int can = 0;
    J4C_CUDA(cudaDeviceCanAccessPeer(&can, device, peer));
    if (!can) return set_error(J4C_E_UNSUPPORTED, "device %d cannot access peer %d", device, peer);
    int cur = 0;
    J4C_CUDA(cudaGetDevice(&cur));
    J4C_CUDA(cudaSetDevice(device));
    cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError();
        e = cudaSuccess;
    }
    cudaSetDevice(cur);
    if (e != cudaSuccess) return cuda_status(e, "cudaDeviceEnablePeerAccess");
    return J4C_OK;
}

int j4c_set_wait_limit_ns(uint64_t ns, uint64_t *previous) {
    J4C_REQUIRE(ns > 0, "j4c_set_wait_limit_ns: the limit must be positive");
    const uint64_t old = j4c::g_wait_limit_ns.exchange(ns);
    if (previous) *previous = old;
    return J4C_OK;
}

int j4c_device_status(int *out_code) {
    J4C_REQUIRE(out_code, "j4c_device_status: out is NULL");
    int *w = device_status_ptr();
    if (!w) return set_error(J4C_E_OOM, "j4c_device_status: no status word");
    int v = 0;
    J4C_CUDA(cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost));
    J4C_CUDA(cudaMemset(w, 0, sizeof(int)));
    *out_code = v;
    return J4C_OK;
}

int j4c_stream_synchronize(j4c_stream stream) {
    J4C_CUDA(cudaStreamSynchronize(as_stream(stream)));
    int *w = device_status_ptr();
    if (!w) return set_error(J4C_E_OOM, "j4c_stream_synchronize: no status word");
    int v = 0;
    J4C_CUDA(cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost));
    if (v != 0) return set_error(J4C_E_DEVICE, "a kernel reported device status %d", v);
    return J4C_OK;
}

int j4c_stream_create(j4c_stream *out) {
    J4C_REQUIRE(out, "j4c_stream_create: out is NULL");
    cudaStream_t s;
    J4C_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    *out = reinterpret_cast<j4c_stream>(s);
    return J4C_OK;
}

int j4c_stream_destroy(j4c_stream stream) {
    J4C_CUDA(cudaStreamDestroy(as_stream(stream)));
    return J4C_OK;
}

int j4c_malloc(size_t bytes, void **out, j4c_stream stream) {
    J4C_REQUIRE(out, "j4c_malloc: out is NULL");
    return scratch_alloc(bytes, out, as_stream(stream));
}

int j4c_free(void *ptr, j4c_stream stream) { return scratch_free(ptr, as_stream(stream)); }

int j4c_memcpy_h2d(void *dst, const void *src, size_t bytes, j4c_stream stream) {
    if (bytes == 0) return J4C_OK;
    J4C_REQUIRE(dst && src, "j4c_memcpy_h2d: NULL pointer");
    J4C_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, as_stream(stream)));
    return J4C_OK;
}

int j4c_memcpy_d2h(void *dst, const void *src, size_t bytes, j4c_stream stream) {
    if (bytes == 0) return J4C_OK;
    J4C_REQUIRE(dst && src, "j4c_memcpy_d2h: NULL pointer");
    J4C_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, as_stream(stream)));
    return J4C_OK;
}

int j4c_memcpy_d2d(void *dst, const void *src, size_t bytes, j4c_stream stream) {
    if (bytes == 0) return J4C_OK;
    J4C_REQUIRE(dst && src, "j4c_memcpy_d2d: NULL pointer");
    J4C_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, as_stream(stream)));
    return J4C_OK;
}

}  // extern "C"
