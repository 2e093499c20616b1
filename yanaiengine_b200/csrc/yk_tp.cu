// yk_tp.cu -- tensor parallelism for the 70B-shape target: an NCCL group per
// engine and the all-reduce after o_proj / down_proj.  NCCL is loaded at run
// time (dlopen of libnccl.so.2), so libyk.so itself has no NCCL dependency and
// single-GPU use never touches it.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "yk_internal.h"

namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
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
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
        api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
        api.ok = api.get_unique_id && api.comm_init_rank && api.all_reduce && api.comm_destroy && api.error_string;
    });
    return api;
}

yk_status nccl_fail(const char* what, ncclResult_t r) {
    const NcclApi& n = nccl();
    yk_set_error(std::string(what) + ": " + (n.error_string ? n.error_string(r) : "NCCL error"));
    return YK_ERR_NCCL;
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

extern "C" yk_status yk_tp_init(yk_engine* e, const uint8_t id[128], int32_t rank, int32_t world) {
    YK_ARG(e && id, "null argument");
    YK_ARG(world >= 1 && rank >= 0 && rank < world, "rank / world");
    YK_ARG(e->nccl_comm == nullptr, "engine already joined a tensor-parallel group");
    const NcclApi& n = nccl();
    if (!n.ok) {
        yk_set_error("libnccl.so.2 could not be loaded");
        return YK_ERR_NCCL;
    }
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    ncclComm_t comm = nullptr;
    const ncclResult_t r = n.comm_init_rank(&comm, world, uid, rank);
    if (r != ncclSuccess) return nccl_fail("ncclCommInitRank", r);
    e->nccl_comm = comm;
    e->tp_rank = rank;
    e->tp_world = world;
    return YK_OK;
}

namespace yk {

// Sum of `count` fp32 values across the group, in place, on the engine stream.
yk_status tp_allreduce_f32(yk_engine* e, float* buf, size_t count) {
    YK_ARG(e->nccl_comm, "engine has not joined a tensor-parallel group");
    const ncclResult_t r = nccl().all_reduce(buf, buf, count, ncclFloat32, ncclSum,
                                             static_cast<ncclComm_t>(e->nccl_comm), e->stream);
    if (r != ncclSuccess) return nccl_fail("ncclAllReduce", r);
    return YK_OK;
}

void tp_destroy(yk_engine* e) {
    if (e->nccl_comm && nccl().ok) nccl().comm_destroy(static_cast<ncclComm_t>(e->nccl_comm));
    e->nccl_comm = nullptr;
}

}  // namespace yk
