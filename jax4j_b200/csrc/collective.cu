// collective.cu -- NCCL-backed replacement of SharedCollective
// (api/SharedCollective.java:23-86).
//
// The reference deposits every shard's array in a slot, waits at a
// CyclicBarrier with no timeout, and has every thread re-sum all D slots.
// Here each pmap shard is an NCCL rank bound to its own B200; psum is one
// ncclAllReduce over NVLink/NVSwitch (NVLS in-switch reduction when NCCL
// selects it) and allGather one ncclAllGather.  Communicators are created
// non-blocking and every wait has a deadline: on expiry the communicator is
// aborted and the caller gets J4C_E_TIMEOUT, so a shard that died before
// reaching a collective cannot hang the others forever.
#include <nccl.h>

#include <chrono>
#include <thread>

#include "common.cuh"

struct j4c_comm_s {
    ncclComm_t nccl = nullptr;
    int rank = 0, nranks = 1, device = 0;
    int64_t timeout_ms = 600000;
    bool aborted = false;
};

namespace j4c {

static int nccl_status(ncclResult_t r, const char *what) {
    return set_error(J4C_E_NCCL, "%s: %s", what, ncclGetErrorString(r));
}

using Clock = std::chrono::steady_clock;

// Polls the communicator until no operation is in progress or the deadline
// passes (then aborts it).  A collective on a non-blocking communicator
// usually finishes enqueueing within microseconds, so the first 2 ms are a
// busy poll; only a longer wait (communicator setup, a slow peer) sleeps
// between polls.
static int wait_comm_ready(j4c_comm c, const char *what) {
    const auto start = Clock::now();
    const auto spin_until = start + std::chrono::milliseconds(2);
    auto deadline = start + std::chrono::milliseconds(c->timeout_ms);
    while (true) {
        ncclResult_t st = ncclSuccess;
        ncclResult_t r = ncclCommGetAsyncError(c->nccl, &st);
        if (r != ncclSuccess) return nccl_status(r, what);
        if (st == ncclSuccess) return J4C_OK;
        if (st != ncclInProgress) return nccl_status(st, what);
        if (Clock::now() > deadline) {
            ncclCommAbort(c->nccl);
            c->aborted = true;
            return set_error(J4C_E_TIMEOUT, "%s: timed out after %lld ms; communicator aborted", what,
                             (long long)c->timeout_ms);
        }
        if (Clock::now() < spin_until) std::this_thread::yield();
        else std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

static ncclDataType_t nccl_type(int dtype) {
    return dtype == J4C_FLOAT64 ? ncclFloat64 : ncclFloat32;
}

}  // namespace j4c

using namespace j4c;

extern "C" {

int j4c_comm_unique_id(void *out, size_t len) {
    J4C_REQUIRE(out && len >= sizeof(ncclUniqueId), "j4c_comm_unique_id: need %d bytes",
                (int)sizeof(ncclUniqueId));
    ncclUniqueId id;
    ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) return nccl_status(r, "ncclGetUniqueId");
    memcpy(out, &id, sizeof(id));
    return J4C_OK;
}

int j4c_comm_init_rank(const void *id, size_t len, int nranks, int rank, int device,
                       int64_t timeout_ms, j4c_comm *out) {
    J4C_REQUIRE(id && out && len >= sizeof(ncclUniqueId), "j4c_comm_init_rank: bad id");
    J4C_REQUIRE(nranks >= 1 && rank >= 0 && rank < nranks, "j4c_comm_init_rank: rank %d of %d",
                rank, nranks);
    J4C_CUDA(cudaSetDevice(device));
    j4c_comm c = new j4c_comm_s();
    c->rank = rank;
    c->nranks = nranks;
    c->device = device;
    c->timeout_ms = timeout_ms > 0 ? timeout_ms : 600000;
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
    config.blocking = 0;
    ncclResult_t r = ncclCommInitRankConfig(&c->nccl, nranks, uid, rank, &config);
    if (r != ncclSuccess && r != ncclInProgress) {
        delete c;
        return nccl_status(r, "ncclCommInitRankConfig");
    }
    int rc = wait_comm_ready(c, "ncclCommInitRankConfig");
    if (rc != J4C_OK) {
        if (!c->aborted) ncclCommAbort(c->nccl);
        delete c;
        return rc;
    }
    *out = c;
    return J4C_OK;
}

int j4c_comm_init_all(const int *devices, int ndev, int64_t timeout_ms, j4c_comm *out) {
    J4C_REQUIRE(devices && out && ndev >= 1 && ndev <= 64, "j4c_comm_init_all: bad arguments");
    ncclComm_t comms[64];
    ncclResult_t r = ncclCommInitAll(comms, ndev, devices);
    if (r != ncclSuccess) return nccl_status(r, "ncclCommInitAll");
    for (int i = 0; i < ndev; i++) {
        j4c_comm c = new j4c_comm_s();
        c->nccl = comms[i];
        c->rank = i;
        c->nranks = ndev;
        c->device = devices[i];
        c->timeout_ms = timeout_ms > 0 ? timeout_ms : 600000;
        out[i] = c;
    }
    return J4C_OK;
}

int j4c_comm_rank(j4c_comm comm, int *rank, int *nranks) {
    J4C_REQUIRE(comm, "j4c_comm_rank: NULL communicator");
    if (rank) *rank = comm->rank;
    if (nranks) *nranks = comm->nranks;
    return J4C_OK;
}

int j4c_comm_destroy(j4c_comm comm) {
    if (!comm) return J4C_OK;
    if (!comm->aborted && comm->nccl) {
        ncclResult_t r = ncclCommFinalize(comm->nccl);
        if (r == ncclSuccess || r == ncclInProgress) wait_comm_ready(comm, "ncclCommFinalize");
        if (!comm->aborted) ncclCommDestroy(comm->nccl);
    }
    delete comm;
    return J4C_OK;
}

int j4c_comm_abort(j4c_comm comm) {
    if (!comm) return J4C_OK;
    if (!comm->aborted && comm->nccl) ncclCommAbort(comm->nccl);
    comm->aborted = true;
    return J4C_OK;
}

int j4c_psum(j4c_comm comm, int dtype, const void *in, void *out, int64_t n, j4c_stream stream) {
    J4C_REQUIRE(comm && !comm->aborted, "j4c_psum: communicator is NULL or aborted");
    J4C_REQUIRE(dtype == J4C_FLOAT32 || dtype == J4C_FLOAT64, "j4c_psum: dtype %s",
                dtype_name(dtype));
    if (n == 0) return J4C_OK;
    J4C_REQUIRE(in && out, "j4c_psum: NULL pointer");
    ncclResult_t r = ncclAllReduce(in, out, (size_t)n, nccl_type(dtype), ncclSum, comm->nccl,
                                   as_stream(stream));
    if (r != ncclSuccess && r != ncclInProgress) return nccl_status(r, "ncclAllReduce");
    if (r == ncclInProgress) return wait_comm_ready(comm, "ncclAllReduce");
    return J4C_OK;
}

int j4c_all_gather(j4c_comm comm, int dtype, const void *in, void *out, int64_t n,
                   j4c_stream stream) {
    J4C_REQUIRE(comm && !comm->aborted, "j4c_all_gather: communicator is NULL or aborted");
    J4C_REQUIRE(dtype == J4C_FLOAT32 || dtype == J4C_FLOAT64, "j4c_all_gather: dtype %s",
                dtype_name(dtype));
    if (n == 0) return J4C_OK;
    J4C_REQUIRE(in && out, "j4c_all_gather: NULL pointer");
    ncclResult_t r = ncclAllGather(in, out, (size_t)n, nccl_type(dtype), comm->nccl, as_stream(stream));
    if (r != ncclSuccess && r != ncclInProgress) return nccl_status(r, "ncclAllGather");
    if (r == ncclInProgress) return wait_comm_ready(comm, "ncclAllGather");
    return J4C_OK;
}

int j4c_reduce_scatter(j4c_comm comm, int dtype, const void *in, void *out, int64_t n, j4c_stream stream) {
    J4C_REQUIRE(comm && !comm->aborted, "j4c_reduce_scatter: communicator is NULL or aborted");
    J4C_REQUIRE(dtype == J4C_FLOAT32 || dtype == J4C_FLOAT64, "j4c_reduce_scatter: dtype %s",
                dtype_name(dtype));
    if (n == 0) return J4C_OK;
    J4C_REQUIRE(in && out, "j4c_reduce_scatter: NULL pointer");
    ncclResult_t r = ncclReduceScatter(in, out, (size_t)n, nccl_type(dtype), ncclSum, comm->nccl,
                                       as_stream(stream));
    if (r != ncclSuccess && r != ncclInProgress) return nccl_status(r, "ncclReduceScatter");
    if (r == ncclInProgress) return wait_comm_ready(comm, "ncclReduceScatter");
    return J4C_OK;
}

// Waits (bounded by the communicator's timeout) until all work enqueued on
// `stream` has finished, checking the communicator for asynchronous errors.
int j4c_comm_wait(j4c_comm comm, j4c_stream stream) {
    J4C_REQUIRE(comm, "j4c_comm_wait: NULL communicator");
    if (comm->aborted) return set_error(J4C_E_NCCL, "j4c_comm_wait: communicator was aborted");
    auto deadline = Clock::now() + std::chrono::milliseconds(comm->timeout_ms);
    cudaStream_t s = as_stream(stream);
    while (true) {
        cudaError_t e = cudaStreamQuery(s);
        if (e == cudaSuccess) return J4C_OK;
        if (e != cudaErrorNotReady) return cuda_status(e, "cudaStreamQuery");
        ncclResult_t st = ncclSuccess;
        ncclCommGetAsyncError(comm->nccl, &st);
        if (st != ncclSuccess && st != ncclInProgress) return nccl_status(st, "collective");
        if (Clock::now() > deadline) {
            ncclCommAbort(comm->nccl);
            comm->aborted = true;
            return set_error(J4C_E_TIMEOUT, "collective did not complete within %lld ms; aborted",
                             (long long)comm->timeout_ms);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

}  // extern "C"
