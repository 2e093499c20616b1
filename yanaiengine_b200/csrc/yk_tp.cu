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
    // An enqueue completes within microseconds: spin (yielding) for the first
    // millisecond, so that back-to-back collectives are not paced by the sleep;
    // longer operations (group set-up) are polled every 200 us.
    const Clock::time_point spin_until = Clock::now() + std::chrono::milliseconds(1);
    while (true) {
        const ncclResult_t r = nccl().get_async_error(comm, &st);
        if (r != ncclSuccess) return r;
        if (st != ncclInProgress) return st;
        const Clock::time_point now = Clock::now();
        if (now > deadline) {
            *timed_out = true;
            return ncclInProgress;
        }
        if (now < spin_until)
            std::this_thread::yield();
        else
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

// ---------------------------------------------------------------------------
// The group's own all-reduce over NVLink peer memory.  Every rank's buffer (CUDA
// IPC, mapped by every other rank): a flag area, two partial slots and two
// reduced slots (alternating by call, so a rank that runs ahead never overwrites
// what a slower peer still reads).  Per call, on every rank (two-shot):
//   A. after the GEMM wrote its bf16 partial into this rank's partial slot, raise
//      "partial ready" in every rank's flag area (system-scope release);
//   B. once every rank's partial is ready: sum this rank's 1/w of the elements
//      over all ranks' partials in rank order 0..w-1 (peer loads, fp32 sums,
//      one bf16 rounding) into this rank's reduced slot; the last CTA to finish
//      raises "reduced ready" everywhere;
//   C. once every rank's share is reduced: copy every rank's reduced share
//      (peer loads) into `out`.
// One shot at w = 2, where both forms read the same bytes from the peer: after
// A, every rank sums every element over all ranks' partials in rank order
// straight into `out`; no B/C hand-off, no second flag exchange.  (At larger w
// it reads (w - 1) x the payload from the peers; two-shot is kept there.)  A partial slot is rewritten two calls later,
// after the writer has seen every peer's "partial ready" of the call between,
// which each peer raises only once its reads of this call are done.
// Every rank thus holds the same bytes.  Each wait is bounded (the device error
// word gets the timeout bit and the kernel returns).  Plain loads and stores
// only: no TMA, no multicast.  All CTAs of the grid are resident together (one
// per SM at most), so the CTAs waiting in B / C never block one still to run.
// ---------------------------------------------------------------------------
constexpr int AR_THREADS = 512;
constexpr size_t AR_FLAGS = 4096;   // flag area (u32 words): A flags [0, 64), C flags [64, 128); the CTA
                                    // counter (u64) at byte 1024

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Thread 0: waits until flags[q] == epoch for every rank q (this rank's flag area).
__device__ __forceinline__ bool ar_wait_all(const uint32_t* flags, int w, uint32_t epoch, uint32_t* err) {
    const uint64_t t0 = globaltimer_ns();
    for (int q = 0; q < w; ++q) {
        for (uint32_t it = 0;; ++it) {
            if (ld_acquire_sys(flags + q) == epoch) break;
            if ((it & 63u) == 63u && globaltimer_ns() - t0 > YK_WAIT_BUDGET_NS) {
                raise_err(err, YK_DEV_ERR_TIMEOUT);
                return false;
            }
        }
    }
    return true;
}

// Phases for a group of W ranks.  A thread takes U = 8 / W indices i at a time
// and issues all U x W of their 16-byte peer loads before it uses any, so each
// thread keeps that many NVLink round trips in flight (one load at a time left
// the 8-rank all-reduce of 10.5 MB latency-bound).
//   AR_SHARE (two-shot B): red(rank)[v0 + i] = bf16(sum over q = 0..W-1 in order
//     of part(q)[v0 + i]), i over this rank's share;
//   AR_GATHER (two-shot C): out[q * share + i] = red(q)[q * share + i] for every q;
//   AR_ALL (one shot): out[i] = bf16(sum over q in order of part(q)[i]), every i.
enum ArMode { AR_SHARE = 0, AR_GATHER = 1, AR_ALL = 2 };
template <int W>
__device__ __forceinline__ void ar_phase(int mode, uint8_t* const* bufs, int rank, int slot, size_t cap,
                                         size_t nv, size_t share, uint4* o4) {
    constexpr int U = 8 / W;
    const bool reduce = mode != AR_GATHER;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    const size_t v0 = mode == AR_SHARE ? (size_t)rank * share : 0;
    const size_t n_b = v0 >= nv ? 0 : (v0 + share < nv ? share : nv - v0);  // this rank's share in B
    const size_t n_i = mode == AR_SHARE ? n_b : (mode == AR_GATHER ? share : nv);
    const uint4* src[W];
#pragma unroll
    for (int q = 0; q < W; ++q)
        src[q] = reinterpret_cast<const uint4*>(bufs[q] + AR_FLAGS + (size_t)(reduce ? slot : 2 + slot) * cap);
    for (size_t i0 = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < n_i; i0 += U * stride) {
        uint4 x[U][W];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const size_t i = i0 + (size_t)u * stride;
#pragma unroll
            for (int q = 0; q < W; ++q) {
                const size_t v = reduce ? v0 + i : (size_t)q * share + i;
                if (i < n_i && v < nv) x[u][q] = src[q][v];
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const size_t i = i0 + (size_t)u * stride;
            if (i >= n_i) continue;
            if (reduce) {
                float acc[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll
                for (int q = 0; q < W; ++q) {
                    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&x[u][q]);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        acc[2 * e] += __low2float(h[e]);
                        acc[2 * e + 1] += __high2float(h[e]);
                    }
                }
                uint4 y;
                __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(&y);
#pragma unroll
                for (int e = 0; e < 4; ++e) o[e] = __floats2bfloat162_rn(acc[2 * e], acc[2 * e + 1]);
                if (mode == AR_ALL) o4[i] = y;
                else reinterpret_cast<uint4*>(bufs[rank] + AR_FLAGS + (size_t)(2 + slot) * cap)[v0 + i] = y;
            } else {
#pragma unroll
                for (int q = 0; q < W; ++q) {
                    const size_t v = (size_t)q * share + i;
                    if (v < nv) o4[v] = x[u][q];
                }
            }
        }
    }
}

// Generic group size (not 2, 4 or 8): one vector at a time, same sums.
__device__ __noinline__ void ar_phase_any(int mode, uint8_t* const* bufs, int rank, int w, int slot, size_t cap,
                                          size_t nv, size_t share, uint4* o4) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    const size_t v0 = mode == AR_SHARE ? (size_t)rank * share : 0;
    const size_t v1 = mode == AR_SHARE ? (v0 + share < nv ? v0 + share : nv) : nv;
    for (size_t v = v0 + (size_t)blockIdx.x * blockDim.x + threadIdx.x; v < v1; v += stride) {
        if (mode == AR_GATHER) {
            o4[v] = reinterpret_cast<const uint4*>(bufs[(int)(v / share)] + AR_FLAGS + (size_t)(2 + slot) * cap)[v];
            continue;
        }
        float acc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = 0.f;
        for (int q = 0; q < w; ++q) {
            const uint4 x = reinterpret_cast<const uint4*>(bufs[q] + AR_FLAGS + (size_t)slot * cap)[v];
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&x);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                acc[2 * i] += __low2float(h[i]);
                acc[2 * i + 1] += __high2float(h[i]);
            }
        }
        uint4 y;
        __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(&y);
#pragma unroll
        for (int i = 0; i < 4; ++i) o[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
        if (mode == AR_ALL) o4[v] = y;
        else reinterpret_cast<uint4*>(bufs[rank] + AR_FLAGS + (size_t)(2 + slot) * cap)[v] = y;
    }
}

__device__ __forceinline__ void ar_run_phase(int mode, uint8_t* const* bufs, int rank, int w, int slot, size_t cap,
                                             size_t nv, size_t share, uint4* o4) {
    switch (w) {
        case 2: ar_phase<2>(mode, bufs, rank, slot, cap, nv, share, o4); break;
        case 4: ar_phase<4>(mode, bufs, rank, slot, cap, nv, share, o4); break;
        case 8: ar_phase<8>(mode, bufs, rank, slot, cap, nv, share, o4); break;
        default: ar_phase_any(mode, bufs, rank, w, slot, cap, nv, share, o4);
    }
}

__global__ void __launch_bounds__(AR_THREADS) ar_peer_kernel(uint8_t* const* bufs, int rank, int w, size_t count,
                                                             size_t cap, uint32_t epoch, int one_shot,
                                                             unsigned long long ctr_target, __nv_bfloat16* out,
                                                             uint32_t* err, unsigned long long* stamps) {
    // stamps (test hook; null otherwise): CTA 0's entry, dependency, "partial ready"
    // seen, share (one shot: everything) reduced, "reduced ready" seen, end; [6] the
    // last CTA's arrival
    const bool st0 = stamps && blockIdx.x == 0 && threadIdx.x == 0;
    if (st0) stamps[0] = globaltimer_ns();
    pdl_trigger();
    pdl_wait();  // the partial (the previous kernel's output) is complete
    if (st0) stamps[1] = globaltimer_ns();
    __shared__ int s_ok;
    const int slot = (int)(epoch & 1u);
    uint8_t* mine = bufs[rank];
    uint32_t* flags = reinterpret_cast<uint32_t*>(mine);
    const size_t nv = count / 8;                 // 16-byte vectors (count is a multiple of 8)
    const size_t share = (nv + w - 1) / w;       // vectors per rank's share
    uint4* o4 = reinterpret_cast<uint4*>(out);
    // A: this rank's partial is ready
    if (blockIdx.x == 0 && threadIdx.x < w) {
        __threadfence_system();
        st_release_sys(reinterpret_cast<uint32_t*>(bufs[threadIdx.x]) + rank, epoch);
    }
    if (threadIdx.x == 0) s_ok = ar_wait_all(flags, w, epoch, err) ? 1 : 0;
    __syncthreads();
    if (!s_ok) return;
    if (st0) stamps[2] = globaltimer_ns();
    if (one_shot) {
        // every element, summed over the ranks in order, straight into out
        ar_run_phase(AR_ALL, bufs, rank, w, slot, cap, nv, share, o4);
        if (stamps && blockIdx.x == 0) {
            __syncthreads();
            if (threadIdx.x == 0) stamps[3] = stamps[5] = globaltimer_ns();
        }
        return;
    }
    // B: this rank's share, summed over the ranks in order
    ar_run_phase(AR_SHARE, bufs, rank, w, slot, cap, nv, share, o4);
    // the last CTA done with B raises "reduced ready" on every rank
    __syncthreads();
    if (st0) stamps[3] = globaltimer_ns();
    if (threadIdx.x == 0) {
        __threadfence();
        unsigned long long* ctr = reinterpret_cast<unsigned long long*>(mine + 1024);
        if (atomicAdd(ctr, 1ULL) == ctr_target) {
            if (stamps) stamps[6] = globaltimer_ns();
            __threadfence_system();
            for (int q = 0; q < w; ++q) st_release_sys(reinterpret_cast<uint32_t*>(bufs[q]) + 64 + rank, epoch);
        }
        s_ok = ar_wait_all(flags + 64, w, epoch, err) ? 1 : 0;
    }
    __syncthreads();
    if (!s_ok) return;
    if (st0) stamps[4] = globaltimer_ns();
    // C: every rank's reduced share into out
    ar_run_phase(AR_GATHER, bufs, rank, w, slot, cap, nv, share, o4);
    if (stamps && blockIdx.x == 0) {
        __syncthreads();
        if (threadIdx.x == 0) stamps[5] = globaltimer_ns();
    }
}

bool tp_ar_enabled(const yk_engine* e) { return e->nccl_comm && e->tp_world > 1 && e->tp_ar_own; }

static void ar_release(yk_engine* e) {
    for (void* p : e->ar_opened)
        if (p) cudaIpcCloseMemHandle(p);
    e->ar_opened.clear();
    if (e->ar_bufs) cudaFree(e->ar_bufs);
    if (e->ar_local) cudaFree(e->ar_local);
    e->ar_bufs = nullptr;
    e->ar_local = nullptr;
    e->ar_cap = 0;
}

yk_status tp_ar_reserve(yk_engine* e, size_t count) {
    const size_t need = ((count * 2 + 255) / 256) * 256;
    if (need <= e->ar_cap) return YK_OK;
    YK_TRY(engine_sync_bounded(e));
    if (e->ar_local) {
        // every rank is past its last use of the old buffers before any is released
        uint32_t one = 1, all[64];
        YK_TRY(yk_tp_allgather_u32(e, &one, 1, all));
        ar_release(e);
    }
    const size_t bytes = AR_FLAGS + 4 * need;
    YK_CHECK_CUDA(cudaMalloc(&e->ar_local, bytes));
    YK_CHECK_CUDA(cudaMemset(e->ar_local, 0, bytes));
    cudaIpcMemHandle_t h;
    YK_CHECK_CUDA(cudaIpcGetMemHandle(&h, e->ar_local));
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle is 64 bytes");
    std::vector<uint32_t> all((size_t)16 * e->tp_world);
    YK_TRY(yk_tp_allgather_u32(e, reinterpret_cast<const uint32_t*>(&h), 16, all.data()));
    std::vector<uint8_t*> ptrs(e->tp_world, nullptr);
    e->ar_opened.assign(e->tp_world, nullptr);
    for (int q = 0; q < e->tp_world; ++q) {
        if (q == e->tp_rank) {
            ptrs[q] = e->ar_local;
            continue;
        }
        cudaIpcMemHandle_t hq;
        std::memcpy(&hq, all.data() + (size_t)16 * q, sizeof(hq));
        void* p = nullptr;
        const cudaError_t r = cudaIpcOpenMemHandle(&p, hq, cudaIpcMemLazyEnablePeerAccess);
        if (r != cudaSuccess) {
            ar_release(e);
            yk_set_error(std::string("cudaIpcOpenMemHandle (all-reduce buffer of rank ") + std::to_string(q) +
                         "): " + cudaGetErrorString(r));
            return YK_ERR_CUDA;
        }
        e->ar_opened[q] = p;
        ptrs[q] = static_cast<uint8_t*>(p);
    }
    YK_CHECK_CUDA(cudaMalloc(&e->ar_bufs, sizeof(uint8_t*) * e->tp_world));
    YK_CHECK_CUDA(cudaMemcpy(e->ar_bufs, ptrs.data(), sizeof(uint8_t*) * e->tp_world, cudaMemcpyHostToDevice));
    e->ar_cap = need;
    e->ar_ctr_base = 0;
    return YK_OK;
}

__nv_bfloat16* tp_ar_slot(yk_engine* e) {
    const uint32_t next = e->ar_epoch + 1 == 0 ? 1 : e->ar_epoch + 1;
    return reinterpret_cast<__nv_bfloat16*>(e->ar_local + AR_FLAGS + (size_t)(next & 1u) * e->ar_cap);
}

yk_status tp_ar_run(yk_engine* e, size_t count, __nv_bfloat16* out, unsigned long long* stamps) {
    YK_ARG(count % 8 == 0 && count * 2 <= e->ar_cap, "all-reduce size");
    e->ar_epoch = e->ar_epoch + 1 == 0 ? 1 : e->ar_epoch + 1;
    const int grid = e->num_sms;
    const double payload = (double)count * 2;
    // (the same choice on every rank: same group size and setting)
    const bool one_shot = e->ar_one_shot && e->tp_world == 2;
    ProfScope prof(e, YK_PROF_OTHER, (one_shot ? 1.0 : 2.0 / e->tp_world) * (e->tp_world - 1) * payload, 0.0);
    YK_CHECK_CUDA(launch_pdl(e, ar_peer_kernel, grid, AR_THREADS, 0, (uint8_t* const*)e->ar_bufs, e->tp_rank,
                             e->tp_world, count, e->ar_cap, e->ar_epoch, one_shot ? 1 : 0,
                             e->ar_ctr_base + (unsigned long long)grid - 1, out, e->d_err, stamps));
    if (!one_shot) e->ar_ctr_base += (unsigned long long)grid;
    e->launches++;
    return YK_OK;
}

void tp_destroy(yk_engine* e) {
    if (e->ar_local) {
        // no rank may still read this rank's buffer when it is released
        if (e->nccl_comm && engine_sync_bounded(e) == YK_OK) {
            uint32_t one = 1, all[64];
            (void)yk_tp_allgather_u32(e, &one, 1, all);
        }
        ar_release(e);
    }
    if (e->nccl_comm && nccl().ok) nccl().comm_destroy(static_cast<ncclComm_t>(e->nccl_comm));
    e->nccl_comm = nullptr;
    if (e->tp_gather) cudaFree(e->tp_gather);
    e->tp_gather = nullptr;
    e->tp_gather_elems = 0;
}

}  // namespace yk

// ---------------------------------------------------------------------------
// Test hook (include/yk_testing.h): the all-reduce alone, back to back.
// ---------------------------------------------------------------------------
#include "../../include/yk_testing.h"

extern "C" yk_status ykt_tp_allreduce_timed(yk_engine* e, int64_t count, int32_t iters, int32_t own,
                                            double* ms_per_call, uint64_t* stamps_out) {
    YK_ARG(e && ms_per_call && count > 0 && count % 8 == 0 && iters > 0, "arguments");
    YK_ARG(e->nccl_comm && e->tp_world > 1, "engine has not joined a tensor-parallel group");
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    if (own) YK_TRY(yk::tp_ar_reserve(e, (size_t)count));
    __nv_bfloat16* buf = nullptr;
    YK_CHECK_CUDA(cudaMalloc(&buf, (size_t)count * 2));
    unsigned long long* dst = nullptr;
    if (cudaMalloc(&dst, 8 * sizeof(unsigned long long)) != cudaSuccess) {
        cudaFree(buf);
        yk_set_error("cudaMalloc (stamps) failed");
        return YK_ERR_CUDA;
    }
    cudaEvent_t t0 = nullptr, t1 = nullptr;
    yk_status st = YK_OK;
    auto call = [&]() -> yk_status {
        return own ? yk::tp_ar_run(e, (size_t)count, buf) : yk::tp_allreduce(e, buf, (size_t)count, true);
    };
    auto run = [&]() -> yk_status {
        YK_CHECK_CUDA(cudaMemsetAsync(buf, 0, (size_t)count * 2, e->stream));
        for (int i = 0; i < 3; ++i) YK_TRY(call());
        YK_TRY(yk::engine_sync_bounded(e));
        YK_CHECK_CUDA(cudaEventCreate(&t0));
        YK_CHECK_CUDA(cudaEventCreate(&t1));
        YK_CHECK_CUDA(cudaEventRecord(t0, e->stream));
        for (int i = 0; i < iters; ++i) YK_TRY(call());
        YK_CHECK_CUDA(cudaEventRecord(t1, e->stream));
        YK_TRY(yk::engine_sync_bounded(e));
        float ms = 0.f;
        YK_CHECK_CUDA(cudaEventElapsedTime(&ms, t0, t1));
        *ms_per_call = (double)ms / iters;
        if (own && stamps_out) {
            // one more call with the kernel's phase stamps
            YK_CHECK_CUDA(cudaMemsetAsync(dst, 0, 8 * sizeof(unsigned long long), e->stream));
            YK_TRY(yk::tp_ar_run(e, (size_t)count, buf, dst));
            YK_TRY(yk::engine_sync_bounded(e));
            YK_CHECK_CUDA(cudaMemcpy(stamps_out, dst, 8 * sizeof(unsigned long long), cudaMemcpyDeviceToHost));
        }
        return YK_OK;
    };
    st = run();
    if (t0) cudaEventDestroy(t0);
    if (t1) cudaEventDestroy(t1);
    if (st == YK_OK) st = yk::engine_sync_bounded(e);
    cudaFree(buf);
    cudaFree(dst);
    return st;
}
