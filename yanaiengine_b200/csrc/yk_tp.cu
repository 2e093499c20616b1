// yk_tp.cu -- tensor parallelism for the 70B-shape target: an NCCL group per
// engine and the all-reduce after o_proj / down_proj.  NCCL is loaded at run
// time (dlopen of libnccl.so.2), so libyk.so itself has no NCCL dependency and
// single-GPU use never touches it.
//
// Failure handling: the communicator is created non-blocking and polled with a
// host deadline, so a peer that never joins ends set-up with YK_ERR_TIMEOUT
// (the half-built communicator is aborted) instead of blocking forever; a wait
// for the engine stream is bounded the same way, and a stream whose collectives
// do not finish in time (a peer stopped taking part) has its communicator
// aborted, which ends the stuck collectives.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>

#include "yk_internal.h"

namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
    bool ok = false;
};

const NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        // prefer an NCCL already in the process (e.g. the one torch.distributed loaded)
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
        api.comm_init_rank_config =
            reinterpret_cast<decltype(api.comm_init_rank_config)>(dlsym(h, "ncclCommInitRankConfig"));
        api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
        api.get_async_error = reinterpret_cast<decltype(api.get_async_error)>(dlsym(h, "ncclCommGetAsyncError"));
        api.comm_abort = reinterpret_cast<decltype(api.comm_abort)>(dlsym(h, "ncclCommAbort"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
        api.ok = api.get_unique_id && api.comm_init_rank_config && api.all_reduce && api.all_gather &&
                 api.get_async_error &&
                 api.comm_abort && api.comm_destroy && api.error_string;
    });
    return api;
}

yk_status nccl_fail(const char* what, ncclResult_t r) {
    const NcclApi& n = nccl();
    yk_set_error(std::string(what) + ": " + (n.error_string ? n.error_string(r) : "NCCL error"));
    return YK_ERR_NCCL;
}

using Clock = std::chrono::steady_clock;

// Polls the communicator's asynchronous state until it leaves ncclInProgress or
// the deadline passes (then *timed_out).
ncclResult_t poll_comm(ncclComm_t comm, Clock::time_point deadline, bool* timed_out) {
    *timed_out = false;
    ncclResult_t st = ncclInProgress;
    while (true) {
        const ncclResult_t r = nccl().get_async_error(comm, &st);
        if (r != ncclSuccess) return r;
        if (st != ncclInProgress) return st;
        if (Clock::now() > deadline) {
            *timed_out = true;
            return ncclInProgress;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
}

}  // namespace

extern "C" yk_status yk_tp_unique_id(uint8_t id_out[128]) {
    YK_ARG(id_out, "null argument");
    const NcclApi& n = nccl();
    if (!n.ok) {
        yk_set_error("libnccl.so.2 could not be loaded");
        return YK_ERR_NCCL;
    }
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
    ncclUniqueId id;
    const ncclResult_t r = n.get_unique_id(&id);
    if (r != ncclSuccess) return nccl_fail("ncclGetUniqueId", r);
    std::memcpy(id_out, &id, sizeof(id));
    return YK_OK;
}

extern "C" yk_status yk_tp_init_timeout(yk_engine* e, const uint8_t id[128], int32_t rank, int32_t world,
                                        int64_t timeout_ms) {
    YK_ARG(e && id, "null argument");
    YK_ARG(world >= 1 && rank >= 0 && rank < world, "rank / world");
    YK_ARG(timeout_ms > 0, "timeout");
    YK_ARG(e->nccl_comm == nullptr, "engine already joined a tensor-parallel group");
    const NcclApi& n = nccl();
    if (!n.ok) {
        yk_set_error("libnccl.so.2 could not be loaded");
        return YK_ERR_NCCL;
    }
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
    config.blocking = 0;
    ncclComm_t comm = nullptr;
    const Clock::time_point deadline = Clock::now() + std::chrono::milliseconds(timeout_ms);
    ncclResult_t r = n.comm_init_rank_config(&comm, world, uid, rank, &config);
    if (r != ncclSuccess && r != ncclInProgress) {
        if (comm) n.comm_abort(comm);
        return nccl_fail("ncclCommInitRankConfig", r);
    }
    bool timed_out = false;
    r = poll_comm(comm, deadline, &timed_out);
    if (timed_out) {
        n.comm_abort(comm);
        yk_set_error("tensor-parallel group set-up: not every rank joined within " + std::to_string(timeout_ms) +
                     " ms (rank " + std::to_string(rank) + " of " + std::to_string(world) + "; communicator aborted)");
        return YK_ERR_TIMEOUT;
    }
    if (r != ncclSuccess) {
        n.comm_abort(comm);
        return nccl_fail("ncclCommInitRankConfig (asynchronous)", r);
    }
    e->nccl_comm = comm;
    e->tp_rank = rank;
    e->tp_world = world;
    e->tp_timeout_ms = timeout_ms;
    return YK_OK;
}

extern "C" yk_status yk_tp_init(yk_engine* e, const uint8_t id[128], int32_t rank, int32_t world) {
    return yk_tp_init_timeout(e, id, rank, world, 300000);
}

namespace yk {

yk_status tp_allreduce(yk_engine* e, void* buf, size_t count, bool bf16) {
    YK_ARG(e->nccl_comm, "engine has not joined a tensor-parallel group");
    ncclComm_t comm = static_cast<ncclComm_t>(e->nccl_comm);
    // bytes each rank moves over NVLink in a ring all-reduce: 2 (w - 1) / w of the payload
    const double payload = (double)count * (bf16 ? 2 : 4);
    ProfScope prof(e, YK_PROF_OTHER, 2.0 * (e->tp_world - 1) / e->tp_world * payload, 0.0);
    ncclResult_t r = nccl().all_reduce(buf, buf, count, bf16 ? ncclBfloat16 : ncclFloat32, ncclSum, comm, e->stream);
    if (r == ncclInProgress) {  // non-blocking communicator: the enqueue completes asynchronously
        bool timed_out = false;
        r = poll_comm(comm, Clock::now() + std::chrono::milliseconds(e->tp_timeout_ms), &timed_out);
        if (timed_out) {
            nccl().comm_abort(comm);
            e->nccl_comm = nullptr;
            yk_set_error("ncclAllReduce could not be enqueued in time (communicator aborted)");
            return YK_ERR_TIMEOUT;
        }
    }
    if (r != ncclSuccess) return nccl_fail("ncclAllReduce", r);
    return YK_OK;
}

yk_status engine_sync_bounded(yk_engine* e) {
    if (!e->nccl_comm) {
        YK_CHECK_CUDA(cudaStreamSynchronize(e->stream));
        return YK_OK;
    }
    const Clock::time_point deadline = Clock::now() + std::chrono::milliseconds(e->tp_timeout_ms);
    while (true) {
        const cudaError_t q = cudaStreamQuery(e->stream);
        if (q == cudaSuccess) return YK_OK;
        if (q != cudaErrorNotReady) YK_CHECK_CUDA(q);
        ncclResult_t st = ncclSuccess;
        if (nccl().get_async_error(static_cast<ncclComm_t>(e->nccl_comm), &st) == ncclSuccess && st != ncclSuccess &&
            st != ncclInProgress) {
            nccl().comm_abort(static_cast<ncclComm_t>(e->nccl_comm));
            e->nccl_comm = nullptr;
            return nccl_fail("tensor-parallel group failed", st);
        }
        if (Clock::now() > deadline) {
            nccl().comm_abort(static_cast<ncclComm_t>(e->nccl_comm));
            e->nccl_comm = nullptr;
            yk_set_error("the engine stream did not finish within " + std::to_string(e->tp_timeout_ms) +
                         " ms (a tensor-parallel peer stopped taking part?); communicator aborted");
            return YK_ERR_TIMEOUT;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

}  // namespace yk

extern "C" yk_status yk_tp_allgather_u32(yk_engine* e, const uint32_t* send, int32_t count, uint32_t* recv) {
    YK_ARG(e && send && recv && count > 0, "arguments");
    YK_ARG(e->nccl_comm, "engine has not joined a tensor-parallel group");
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    const size_t need = (size_t)count * (1 + e->tp_world);
    if (need > e->tp_gather_elems) {
        YK_TRY(yk::engine_sync_bounded(e));
        if (e->tp_gather) cudaFree(e->tp_gather);
        e->tp_gather = nullptr;
        e->tp_gather_elems = 0;
        YK_CHECK_CUDA(cudaMalloc(&e->tp_gather, need * 4));
        e->tp_gather_elems = need;
    }
    uint32_t* dsend = e->tp_gather;
    uint32_t* drecv = e->tp_gather + count;
    YK_CHECK_CUDA(cudaMemcpyAsync(dsend, send, (size_t)count * 4, cudaMemcpyHostToDevice, e->stream));
    ncclComm_t comm = static_cast<ncclComm_t>(e->nccl_comm);
    ncclResult_t r = nccl().all_gather(dsend, drecv, (size_t)count, ncclUint32, comm, e->stream);
    if (r == ncclInProgress) {
        bool timed_out = false;
        r = poll_comm(comm, Clock::now() + std::chrono::milliseconds(e->tp_timeout_ms), &timed_out);
        if (timed_out) {
            nccl().comm_abort(comm);
            e->nccl_comm = nullptr;
            yk_set_error("ncclAllGather could not be enqueued in time (communicator aborted)");
            return YK_ERR_TIMEOUT;
        }
    }
    if (r != ncclSuccess) return nccl_fail("ncclAllGather", r);
    YK_CHECK_CUDA(cudaMemcpyAsync(recv, drecv, (size_t)count * e->tp_world * 4, cudaMemcpyDeviceToHost, e->stream));
    return yk::engine_sync_bounded(e);
}

namespace yk {

void tp_destroy(yk_engine* e) {
    if (e->nccl_comm && nccl().ok) nccl().comm_destroy(static_cast<ncclComm_t>(e->nccl_comm));
    e->nccl_comm = nullptr;
    if (e->tp_gather) cudaFree(e->tp_gather);
    e->tp_gather = nullptr;
    e->tp_gather_elems = 0;
}

}  // namespace yk
