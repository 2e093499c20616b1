// yk_api.cu -- engine / model / KV pool handles and the forward step
// (LlamaModel.forwardStep, S/LlamaModel.swift:134-244; block order of
// LlamaBlock.forwardBatched, S/LlamaBlock.swift:178-276).
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "yk_common.cuh"
#include "yk_internal.h"

static thread_local std::string g_last_error;
void yk_set_error(const std::string& msg) { g_last_error = msg; }

extern "C" int32_t yk_last_error(char* buf, size_t n) {
    if (buf && n) {
        const size_t k = std::min(n - 1, g_last_error.size());
        std::memcpy(buf, g_last_error.data(), k);
        buf[k] = 0;
    }
    return (int32_t)g_last_error.size();
}

yk_status yk_engine::ensure_pinned(size_t bytes) {
    if (bytes <= pinned_bytes) return YK_OK;
    YK_CHECK_CUDA(cudaStreamSynchronize(stream));
    if (pinned) cudaFreeHost(pinned);
    pinned = nullptr;
    pinned_bytes = 0;
    const size_t want = std::max(bytes, (size_t)1 << 20);
    YK_CHECK_CUDA(cudaMallocHost((void**)&pinned, want));
    pinned_bytes = want;
    return YK_OK;
}

yk_status yk_engine::up_acquire(size_t bytes, int* slot, uint8_t** host) {
    const int i = up_next;
    up_next = (up_next + 1) % UP_SLOTS;
    UpSlot& u = up[i];
    if (!u.done) YK_CHECK_CUDA(cudaEventCreateWithFlags(&u.done, cudaEventDisableTiming));
    YK_CHECK_CUDA(cudaEventSynchronize(u.done));  // this slot's previous copy has been read
    if (bytes > u.bytes) {
        if (u.host) cudaFreeHost(u.host);
        u.host = nullptr;
        u.bytes = 0;
        const size_t want = std::max(bytes * 2, (size_t)1 << 20);
        YK_CHECK_CUDA(cudaMallocHost((void**)&u.host, want));
        u.bytes = want;
    }
    *slot = i;
    *host = u.host;
    return YK_OK;
}

yk_status yk_engine::up_submit(int slot, void* dst, size_t bytes) { return up_submit_on(slot, dst, bytes, stream); }

yk_status yk_engine::up_submit_on(int slot, void* dst, size_t bytes, cudaStream_t on) {
    UpSlot& u = up[slot];
    YK_CHECK_CUDA(cudaMemcpyAsync(dst, u.host, bytes, cudaMemcpyHostToDevice, on));
    YK_CHECK_CUDA(cudaEventRecord(u.done, on));
    return YK_OK;
}

// ---------------------------------------------------------------------------
// engine
// ---------------------------------------------------------------------------
extern "C" yk_status yk_engine_create(int32_t device, yk_engine** out) {
    YK_ARG(out != nullptr, "out is null");
    *out = nullptr;
    int ndev = 0;
    YK_CHECK_CUDA(cudaGetDeviceCount(&ndev));
    YK_ARG(device >= 0 && device < ndev, "device index");
    YK_CHECK_CUDA(cudaSetDevice(device));
    int major = 0, minor = 0;
    YK_CHECK_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
    YK_CHECK_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device));
    if (major != 10 || minor != 0) {
        yk_set_error("libyk.so is built for sm_100a (B200); device is sm_" + std::to_string(major * 10 + minor));
        return YK_ERR_UNSUPPORTED;
    }
    auto* e = new yk_engine();
    e->device = device;
    YK_CHECK_CUDA(cudaDeviceGetAttribute(&e->num_sms, cudaDevAttrMultiProcessorCount, device));
    YK_CHECK_CUDA(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));
    YK_CHECK_CUDA(cudaStreamCreateWithFlags(&e->up_stream, cudaStreamNonBlocking));
    YK_CHECK_CUDA(cudaMalloc(&e->d_err, sizeof(uint32_t)));
    YK_CHECK_CUDA(cudaMemset(e->d_err, 0, sizeof(uint32_t)));
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    YK_CHECK_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
    if (!fn || q != cudaDriverEntryPointSuccess) {
        yk_set_error("cuTensorMapEncodeTiled not available from the driver");
        delete e;
        return YK_ERR_CUDA;
    }
    e->encode_tiled = (PFN_tmapEncodeTiled)fn;
    if (const char* v = std::getenv("YK_PDL")) e->pdl = std::strcmp(v, "0") != 0;
    if (const char* v = std::getenv("YK_GEMM_VARIANT")) e->gemm_variant = std::atoi(v);
    if (const char* v = std::getenv("YK_GEMM_PUSH_MIN")) e->gemm_push_min = std::max(0, std::atoi(v));
    if (const char* v = std::getenv("YK_FUSE_NORM")) e->fuse_norm = std::atoi(v) != 0;
    if (const char* v = std::getenv("YK_GEMM_CHAIN")) e->gemm_chain = std::atoi(v) != 0;
    if (const char* v = std::getenv("YK_META_ASYNC")) e->meta_async = std::atoi(v) != 0;
    if (const char* v = std::getenv("YK_ATTN_WAVES")) e->attn_waves = std::max(1, std::atoi(v));
    if (const char* v = std::getenv("YK_ATTN_PLAN")) e->attn_balanced = std::atoi(v) == 1;
    if (const char* v = std::getenv("YK_TP_PAYLOAD")) e->tp_bf16 = std::strcmp(v, "f32") != 0;
    if (const char* v = std::getenv("YK_TP_AR")) {
        e->tp_ar_own = std::strcmp(v, "nccl") != 0;
        if (std::strcmp(v, "twoshot") == 0) e->ar_one_shot = false;
    }
    yk_status s = e->ensure_pinned((size_t)4 << 20);
    if (s != YK_OK) { delete e; return s; }
    *out = e;
    return YK_OK;
}

extern "C" void yk_engine_destroy(yk_engine* e) {
    if (!e) return;
    cudaSetDevice(e->device);
    cudaStreamSynchronize(e->stream);
    if (e->up_stream) cudaStreamSynchronize(e->up_stream);
    if (e->pinned) cudaFreeHost(e->pinned);
    for (auto& u : e->up) {
        if (u.host) cudaFreeHost(u.host);
        if (u.done) cudaEventDestroy(u.done);
    }
    if (e->d_err) cudaFree(e->d_err);
    if (e->trace_rec) cudaFree(e->trace_rec);
    yk::tp_destroy(e);
    if (e->stream) cudaStreamDestroy(e->stream);
    if (e->up_stream) cudaStreamDestroy(e->up_stream);
    delete e;
}

extern "C" yk_status yk_engine_stream(yk_engine* e, void** stream) {
    YK_ARG(e && stream, "null handle");
    *stream = (void*)e->stream;
    return YK_OK;
}

extern "C" yk_status yk_engine_sync(yk_engine* e) {
    YK_ARG(e, "null handle");
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    return yk::engine_sync_bounded(e);
}

extern "C" yk_status yk_engine_device_error(yk_engine* e, uint32_t* code) {
    YK_ARG(e && code, "null handle");
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    YK_CHECK_CUDA(cudaStreamSynchronize(e->stream));
    YK_CHECK_CUDA(cudaMemcpy(code, e->d_err, sizeof(uint32_t), cudaMemcpyDeviceToHost));
    YK_CHECK_CUDA(cudaMemset(e->d_err, 0, sizeof(uint32_t)));
    return YK_OK;
}

extern "C" uint64_t yk_engine_launch_count(yk_engine* e) { return e ? e->launches : 0; }

int yk_engine::prof_begin(int cls, double bytes, double flops) {
    ProfRecord r{cls, nullptr, nullptr, bytes, flops};
    for (cudaEvent_t* ev : {&r.start, &r.stop}) {
        if (!prof_free.empty()) {
            *ev = prof_free.back();
            prof_free.pop_back();
        } else if (cudaEventCreate(ev) != cudaSuccess) {
            *ev = nullptr;
        }
    }
    if (!r.start || !r.stop || cudaEventRecord(r.start, stream) != cudaSuccess) {
        if (r.start) prof_free.push_back(r.start);
        if (r.stop) prof_free.push_back(r.stop);
        return -1;
    }
    prof_pending.push_back(r);
    return (int)prof_pending.size() - 1;
}

void yk_engine::prof_end(int rec) {
    if (rec < 0 || rec >= (int)prof_pending.size()) return;
    // a stop that cannot be recorded leaves the record without a duration: it is left out
    if (cudaEventRecord(prof_pending[(size_t)rec].stop, stream) != cudaSuccess) prof_pending[(size_t)rec].failed = true;
}

void yk_engine::prof_resolve() {
    cudaStreamSynchronize(stream);
    for (auto& r : prof_pending) {
        float ms = 0.f;
        if (!r.failed && cudaEventElapsedTime(&ms, r.start, r.stop) == cudaSuccess) {
            ProfTotals& t = prof[r.cls & 3];
            t.ms += ms;
            t.bytes += r.bytes;
            t.flops += r.flops;
            t.launches++;
        }
        prof_free.push_back(r.start);
        prof_free.push_back(r.stop);
    }
    prof_pending.clear();
}

extern "C" yk_status yk_engine_profile(yk_engine* e, int32_t enable) {
    YK_ARG(e, "null handle");
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    e->prof_resolve();
    for (auto& t : e->prof) t = ProfTotals{};
    e->profiling = enable != 0;
    return YK_OK;
}

extern "C" yk_status yk_engine_profile_read(yk_engine* e, int32_t cls, double* ms, double* bytes, double* flops,
                                            int64_t* launches) {
    YK_ARG(e && cls >= 0 && cls < 4, "arguments");
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    e->prof_resolve();
    if (ms) *ms = e->prof[cls].ms;
    if (bytes) *bytes = e->prof[cls].bytes;
    if (flops) *flops = e->prof[cls].flops;
    if (launches) *launches = e->prof[cls].launches;
    return YK_OK;
}

// ---------------------------------------------------------------------------
// model
// ---------------------------------------------------------------------------
static uint16_t host_bf16(float x) {
    uint32_t u;
    std::memcpy(&u, &x, 4);
    if ((u & 0x7f800000u) == 0x7f800000u) return (uint16_t)((u >> 16) | ((u & 0x7fffffu) ? 0x40u : 0u));
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
static float host_from_bf16(uint16_t b) {
    const uint32_t u = (uint32_t)b << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

static yk_status dalloc(yk_model* m, void** p, size_t bytes) {
    cudaError_t e = cudaMalloc(p, std::max<size_t>(bytes, 256));
    if (e != cudaSuccess) {
        yk_set_error(std::string("cudaMalloc(") + std::to_string(bytes) + "): " + cudaGetErrorString(e));
        return e == cudaErrorMemoryAllocation ? YK_ERR_OOM : YK_ERR_CUDA;
    }
    m->allocations.push_back(*p);
    return YK_OK;
}

static yk_status validate_cfg(const yk_model_config* c) {
    YK_ARG(c, "config is null");
    YK_ARG(c->vocab_size > 0 && c->vocab_size % 4 == 0, "vocab_size must be a positive multiple of 4");
    YK_ARG(c->d_model > 0 && c->d_model % 8 == 0, "d_model must be a positive multiple of 8");
    YK_ARG(c->n_layers > 0 && c->n_heads > 0 && c->n_kv_heads > 0 && c->n_heads % c->n_kv_heads == 0,
           "n_heads must be a positive multiple of n_kv_heads");
    YK_ARG(c->head_dim == 64 || c->head_dim == 128 || c->head_dim == 256, "head_dim must be 64, 128 or 256");
    YK_ARG(c->ffn_dim > 0 && c->ffn_dim % 8 == 0, "ffn_dim must be a positive multiple of 8");
    YK_ARG(c->dtype == YK_DTYPE_F32 || c->dtype == YK_DTYPE_BF16, "dtype");
    YK_ARG(c->act == YK_ACT_SILU || c->act == YK_ACT_GELU_TANH, "act");
    YK_ARG(c->max_tokens > 0 && c->max_seqs > 0, "max_tokens / max_seqs");
    YK_ARG(c->rope_theta > 0.f && c->rms_eps >= 0.f && c->attn_cap >= 0.f && c->final_cap >= 0.f && c->window >= 0,
           "numeric parameters");
    return YK_OK;
}

// A model, or shard tp_rank of tp_world of it (query heads, KV heads and FFN
// columns split; embedding, norms and LM head replicated).
static yk_status create_model(yk_engine* e, const yk_model_config* cfg, int tp_rank, int tp_world, uint64_t seed,
                              float init_std, yk_model** out) {
    YK_ARG(e && out, "null handle");
    *out = nullptr;
    YK_TRY(validate_cfg(cfg));
    YK_ARG(tp_world >= 1 && tp_rank >= 0 && tp_rank < tp_world, "tp_rank / tp_world");
    if (tp_world > 1) {
        YK_ARG(e->nccl_comm && e->tp_world == tp_world && e->tp_rank == tp_rank,
               "the engine must have joined the tensor-parallel group as this rank (yk_tp_init)");
        YK_ARG(cfg->n_kv_heads % tp_world == 0 && cfg->ffn_dim % (8 * tp_world) == 0,
               "n_kv_heads and ffn_dim / 8 must be divisible by tp_world");
        YK_ARG(cfg->ref_compat == 0, "ref_compat (ReLU on projections) needs the full sum: not tensor-parallel");
    }
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    auto* m = new yk_model();
    m->e = e;
    m->cfg = *cfg;
    m->cfg.n_heads /= tp_world;
    m->cfg.n_kv_heads /= tp_world;
    m->cfg.ffn_dim /= tp_world;
    m->tp_rank = tp_rank;
    m->tp_world = tp_world;
    // replicated tensors use `seed` on every rank; each shard its own stream
    const uint64_t shard_seed = tp_world > 1 ? seed ^ (0x9E3779B97F4A7C15ull * (uint64_t)(tp_rank + 1)) : seed;
    const auto& c = m->cfg;
    const size_t es = c.dtype == YK_DTYPE_BF16 ? 2 : 4;
    m->esize = es;
    const size_t d = c.d_model, V = c.vocab_size, F = c.ffn_dim, dh = c.head_dim;
    const size_t qd = (size_t)c.n_heads * dh, kvd = (size_t)c.n_kv_heads * dh;
    const size_t T = c.max_tokens;
    auto fail = [&](yk_status s) { yk_model_destroy(m); return s; };
    yk_status s;
#define ALLOC(ptr, bytes) \
    if ((s = dalloc(m, (void**)&(ptr), (bytes))) != YK_OK) return fail(s)
    ALLOC(m->embed, V * d * es);
    ALLOC(m->lm_head, V * d * es);
    ALLOC(m->final_norm, d * 4);
    m->layers.resize(c.n_layers);
    for (auto& L : m->layers) {
        ALLOC(L.wqkv, (qd + 2 * kvd) * d * es);
        ALLOC(L.wo, d * qd * es);
        ALLOC(L.wgu, 2 * F * d * es);
        ALLOC(L.wdown, d * F * es);
        ALLOC(L.n1, d * 4);
        ALLOC(L.n2, d * 4);
    }
    ALLOC(m->h, T * d * 4);
    ALLOC(m->xn, T * d * es);
    ALLOC(m->q, T * qd * es);
    ALLOC(m->att, T * qd * es);
    ALLOC(m->act, T * F * es);
    ALLOC(m->logits, T * V * 4);
    ALLOC(m->rope_denom, dh / 2 * 4);
    ALLOC(m->rope_tab, T * (dh / 2) * sizeof(float2));
    ALLOC(m->norm_ss, ((d + 31) / 32) * T * 4);
    if (tp_world > 1) ALLOC(m->tp_y, T * d * 4);
    m->gemm_ws_floats = (size_t)2 * e->num_sms * 128 * 256;
    ALLOC(m->gemm_ws, m->gemm_ws_floats * 4);
    m->gemm_counter_cap = 4096;
    if (cudaMalloc(&m->gemm_counters, (size_t)m->gemm_counter_cap * 4) != cudaSuccess) {  // may grow: owned apart
        m->gemm_counters = nullptr;
        yk_set_error("cudaMalloc(gemm counters) failed");
        return fail(YK_ERR_OOM);
    }
#undef ALLOC
    if (cudaMemsetAsync(m->gemm_counters, 0, (size_t)m->gemm_counter_cap * 4, e->stream) != cudaSuccess ||
        cudaMemsetAsync(m->xn, 0, T * d * es, e->stream) != cudaSuccess ||
        cudaMemsetAsync(m->att, 0, T * qd * es, e->stream) != cudaSuccess ||
        cudaMemsetAsync(m->act, 0, T * F * es, e->stream) != cudaSuccess) {
        yk_set_error("cudaMemsetAsync failed");
        return fail(YK_ERR_CUDA);
    }
    // RoPE denominators base^(2p/dh) in fp32 (S/gemm.metal:675).
    std::vector<float> den(dh / 2);
    for (size_t p = 0; p < dh / 2; ++p) den[p] = std::pow(c.rope_theta, (float)(2 * p) / (float)dh);
    if (cudaMemcpy(m->rope_denom, den.data(), den.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
        yk_set_error("rope table upload failed");
        return fail(YK_ERR_CUDA);
    }
    // Random init: matrices N(0, init_std), norms 1.
    uint32_t stream_id = 1;
    auto rnd = [&](void* p, size_t n) { return yk::launch_init(e, p, n, c.dtype, seed, stream_id++, init_std, false); };
    auto rnd_shard = [&](void* p, size_t n) {
        return yk::launch_init(e, p, n, c.dtype, shard_seed, stream_id++, init_std, false);
    };
    auto one = [&](float* p, size_t n) { return yk::launch_init(e, p, n, YK_DTYPE_F32, 0, 0, 1.0f, true); };
    if ((s = rnd(m->embed, V * d)) || (s = rnd(m->lm_head, V * d)) || (s = one(m->final_norm, d))) return fail(s);
    for (auto& L : m->layers) {
        if ((s = rnd_shard(L.wqkv, (qd + 2 * kvd) * d)) || (s = rnd_shard(L.wo, d * qd)) ||
            (s = rnd_shard(L.wgu, 2 * F * d)) || (s = rnd_shard(L.wdown, d * F)) || (s = one(L.n1, d)) ||
            (s = one(L.n2, d)))
            return fail(s);
    }
    if (c.dtype == YK_DTYPE_BF16) {
        for (auto& L : m->layers) {
            if ((s = yk::make_weight_map(e, &L.tm_qkv, L.wqkv, (int)(qd + 2 * kvd), (int)d)) ||
                (s = yk::make_weight_map(e, &L.tm_o, L.wo, (int)d, (int)qd)) ||
                (s = yk::make_weight_map(e, &L.tm_gu, L.wgu, (int)(2 * F), (int)d)) ||
                (s = yk::make_weight_map(e, &L.tm_down, L.wdown, (int)d, (int)F)))
                return fail(s);
        }
        if ((s = yk::make_weight_map(e, &m->tm_lm, m->lm_head, (int)V, (int)d))) return fail(s);
    }
    if (cudaStreamSynchronize(e->stream) != cudaSuccess) {
        yk_set_error("model init failed");
        return fail(YK_ERR_CUDA);
    }
    *out = m;
    return YK_OK;
}

extern "C" yk_status yk_model_create(yk_engine* e, const yk_model_config* cfg, uint64_t seed, float init_std,
                                     yk_model** out) {
    return create_model(e, cfg, 0, 1, seed, init_std, out);
}

extern "C" yk_status yk_model_create_tp(yk_engine* e, const yk_model_config* cfg, int32_t tp_rank, int32_t tp_world,
                                        uint64_t seed, float init_std, yk_model** out) {
    return create_model(e, cfg, tp_rank, tp_world, seed, init_std, out);
}

extern "C" void yk_model_destroy(yk_model* m) {
    if (!m) return;
    cudaSetDevice(m->e->device);
    cudaStreamSynchronize(m->e->stream);
    for (void* p : m->allocations) cudaFree(p);
    if (m->e->up_stream) cudaStreamSynchronize(m->e->up_stream);
    for (int i = 0; i < yk_model::META_SLOTS; ++i) {
        if (m->meta[i]) cudaFree(m->meta[i]);
        if (m->meta_copied[i]) cudaEventDestroy(m->meta_copied[i]);
        if (m->meta_free[i]) cudaEventDestroy(m->meta_free[i]);
    }
    if (m->attn_ws) cudaFree(m->attn_ws);
    if (m->attn_counters) cudaFree(m->attn_counters);
    if (m->attn_stamps) cudaFree(m->attn_stamps);
    if (m->gemm_stamps) cudaFree(m->gemm_stamps);
    if (m->chain_bar) cudaFree(m->chain_bar);
    if (m->gemm_counters) cudaFree(m->gemm_counters);
    delete m;
}

extern "C" yk_status yk_model_get_config(const yk_model* m, yk_model_config* out) {
    YK_ARG(m && out, "null handle");
    *out = m->cfg;
    return YK_OK;
}

yk_status yk::locate_tensor(const yk_model* m, int32_t t, int32_t layer, TensorLoc* L) {
    const auto& c = m->cfg;
    const size_t d = c.d_model, dh = c.head_dim, qd = (size_t)c.n_heads * dh, kvd = (size_t)c.n_kv_heads * dh;
    const size_t es = m->esize;
    const bool per_layer = t >= YK_T_WQ && t <= YK_T_NORM2;
    YK_ARG(t >= 0 && t <= YK_T_LM_HEAD, "tensor id");
    if (per_layer) YK_ARG(layer >= 0 && layer < c.n_layers, "layer index");
    const LayerWeights* W = per_layer ? &m->layers[layer] : nullptr;
    switch (t) {
        case YK_T_EMBED: *L = {(uint8_t*)m->embed, 0, 1, (size_t)c.vocab_size, d, es}; break;
        case YK_T_WQ: *L = {(uint8_t*)W->wqkv, 0, 1, qd, d, es}; break;
        case YK_T_WK: *L = {(uint8_t*)W->wqkv, qd, 1, kvd, d, es}; break;
        case YK_T_WV: *L = {(uint8_t*)W->wqkv, qd + kvd, 1, kvd, d, es}; break;
        case YK_T_WO: *L = {(uint8_t*)W->wo, 0, 1, d, qd, es}; break;
        case YK_T_WGATE: *L = {(uint8_t*)W->wgu, 0, 2, (size_t)c.ffn_dim, d, es}; break;
        case YK_T_WUP: *L = {(uint8_t*)W->wgu, 1, 2, (size_t)c.ffn_dim, d, es}; break;
        case YK_T_WDOWN: *L = {(uint8_t*)W->wdown, 0, 1, d, (size_t)c.ffn_dim, es}; break;
        case YK_T_NORM1: *L = {(uint8_t*)W->n1, 0, 1, 1, d, 4}; break;
        case YK_T_NORM2: *L = {(uint8_t*)W->n2, 0, 1, 1, d, 4}; break;
        case YK_T_FINAL_NORM: *L = {(uint8_t*)m->final_norm, 0, 1, 1, d, 4}; break;
        case YK_T_LM_HEAD: *L = {(uint8_t*)m->lm_head, 0, 1, (size_t)c.vocab_size, d, es}; break;
    }
    return YK_OK;
}

extern "C" yk_status yk_model_tensor_shape(const yk_model* m, int32_t t, int64_t* rows, int64_t* cols) {
    YK_ARG(m && rows && cols, "null handle");
    yk::TensorLoc L;
    YK_TRY(yk::locate_tensor(m, t, 0, &L));
    *rows = (int64_t)L.rows;
    *cols = (int64_t)L.cols;
    return YK_OK;
}

extern "C" yk_status yk_model_set_tensor(yk_model* m, int32_t t, int32_t layer, const float* host, int32_t layout) {
    YK_ARG(m && host, "null handle");
    YK_ARG(layout == YK_LAYOUT_OUT_IN || layout == YK_LAYOUT_IN_OUT, "layout");
    yk::TensorLoc L;
    YK_TRY(yk::locate_tensor(m, t, layer, &L));
    yk_engine* e = m->e;
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    const size_t n = L.rows * L.cols;
    YK_TRY(e->ensure_pinned(n * L.es));
    YK_CHECK_CUDA(cudaStreamSynchronize(e->stream));
    for (size_t r = 0; r < L.rows; ++r)
        for (size_t k = 0; k < L.cols; ++k) {
            const float v = layout == YK_LAYOUT_OUT_IN ? host[r * L.cols + k] : host[k * L.rows + r];
            if (L.es == 2) ((uint16_t*)e->pinned)[r * L.cols + k] = host_bf16(v);
            else ((float*)e->pinned)[r * L.cols + k] = v;
        }
    YK_CHECK_CUDA(cudaMemcpy2DAsync(L.base + L.row0 * L.cols * L.es, L.pitch_rows * L.cols * L.es, e->pinned,
                                    L.cols * L.es, L.cols * L.es, L.rows, cudaMemcpyHostToDevice, e->stream));
    YK_CHECK_CUDA(cudaStreamSynchronize(e->stream));
    return YK_OK;
}

extern "C" yk_status yk_model_get_tensor(yk_model* m, int32_t t, int32_t layer, float* host) {
    YK_ARG(m && host, "null handle");
    yk::TensorLoc L;
    YK_TRY(yk::locate_tensor(m, t, layer, &L));
    yk_engine* e = m->e;
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    const size_t n = L.rows * L.cols;
    YK_TRY(e->ensure_pinned(n * L.es));
    YK_CHECK_CUDA(cudaStreamSynchronize(e->stream));
    YK_CHECK_CUDA(cudaMemcpy2DAsync(e->pinned, L.cols * L.es, L.base + L.row0 * L.cols * L.es,
                                    L.pitch_rows * L.cols * L.es, L.cols * L.es, L.rows, cudaMemcpyDeviceToHost,
                                    e->stream));
    YK_CHECK_CUDA(cudaStreamSynchronize(e->stream));
    for (size_t i = 0; i < n; ++i)
        host[i] = L.es == 2 ? host_from_bf16(((uint16_t*)e->pinned)[i]) : ((float*)e->pinned)[i];
    return YK_OK;
}

// ---------------------------------------------------------------------------
// KV pool
// ---------------------------------------------------------------------------
extern "C" yk_status yk_kv_pool_create_layers(yk_engine* e, const yk_model_config* cfg, int32_t num_blocks,
                                              int32_t layers, yk_kv_pool** out) {
    YK_ARG(e && out, "null handle");
    *out = nullptr;
    YK_TRY(validate_cfg(cfg));
    YK_ARG(num_blocks > 0, "num_blocks");
    YK_ARG(layers >= YK_POOL_ALL_LAYERS && layers <= YK_POOL_WINDOWED_LAYERS, "layers (YK_POOL_*)");
    int n_pool_layers = 0;
    for (int l = 0; l < cfg->n_layers; ++l) n_pool_layers += yk::pool_layer_index(*cfg, layers, l) >= 0 ? 1 : 0;
    YK_ARG(n_pool_layers > 0, "the model has no layer of this kind");
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    auto* p = new yk_kv_pool();
    p->e = e;
    p->cfg = *cfg;
    p->num_blocks = num_blocks;
    p->kind = layers;
    p->n_pool_layers = n_pool_layers;
    p->esize = cfg->dtype == YK_DTYPE_BF16 ? 2 : 4;
    p->layer_elems = (size_t)2 * cfg->n_kv_heads * YK_BLOCK_SIZE * cfg->head_dim;
    p->block_elems = p->layer_elems * n_pool_layers;
    const size_t bytes = p->block_elems * num_blocks * p->esize;
    cudaError_t err = cudaMalloc(&p->data, bytes);
    if (err != cudaSuccess) {
        delete p;
        yk_set_error("KV pool cudaMalloc(" + std::to_string(bytes) + "): " + cudaGetErrorString(err));
        return err == cudaErrorMemoryAllocation ? YK_ERR_OOM : YK_ERR_CUDA;
    }
    err = cudaMemset(p->data, 0, bytes);
    if (err != cudaSuccess) {
        cudaFree(p->data);
        delete p;
        yk_set_error(std::string("KV pool memset: ") + cudaGetErrorString(err));
        return YK_ERR_CUDA;
    }
    if (cfg->dtype == YK_DTYPE_BF16) {
        const yk_status s = yk::make_pool_map(e, p);
        if (s != YK_OK) {
            cudaFree(p->data);
            delete p;
            return s;
        }
    }
    *out = p;
    return YK_OK;
}

extern "C" yk_status yk_kv_pool_create(yk_engine* e, const yk_model_config* cfg, int32_t num_blocks, yk_kv_pool** out) {
    return yk_kv_pool_create_layers(e, cfg, num_blocks, YK_POOL_ALL_LAYERS, out);
}

extern "C" void yk_kv_pool_destroy(yk_kv_pool* p) {
    if (!p) return;
    cudaSetDevice(p->e->device);
    cudaStreamSynchronize(p->e->stream);
    cudaFree(p->data);
    delete p;
}

extern "C" int32_t yk_kv_pool_num_blocks(const yk_kv_pool* p) { return p ? p->num_blocks : 0; }

extern "C" yk_status yk_kv_pool_fill_random(yk_kv_pool* p, uint64_t seed, float std) {
    YK_ARG(p, "null handle");
    YK_CHECK_CUDA(cudaSetDevice(p->e->device));
    YK_TRY(yk::launch_init(p->e, p->data, p->block_elems * p->num_blocks, p->cfg.dtype, seed, 0x4B56u, std, false));
    YK_CHECK_CUDA(cudaStreamSynchronize(p->e->stream));
    return YK_OK;
}

extern "C" yk_status yk_kv_pool_read_page(yk_kv_pool* p, int32_t block, int32_t layer, int32_t kv, float* host) {
    YK_ARG(p && host, "null handle");
    YK_ARG(block >= 0 && block < p->num_blocks && layer >= 0 && layer < p->cfg.n_layers && (kv == 0 || kv == 1),
           "page index");
    const int pl = yk::pool_layer_index(p->cfg, p->kind, layer);
    YK_ARG(pl >= 0, "the pool does not hold this layer");
    yk_engine* e = p->e;
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    const size_t n = (size_t)p->cfg.n_kv_heads * YK_BLOCK_SIZE * p->cfg.head_dim;
    YK_TRY(e->ensure_pinned(n * p->esize));
    YK_CHECK_CUDA(cudaStreamSynchronize(e->stream));
    const uint8_t* src = (const uint8_t*)p->data + ((size_t)block * p->block_elems + (size_t)pl * p->layer_elems +
                                                    (size_t)kv * n) * p->esize;
    YK_CHECK_CUDA(cudaMemcpyAsync(e->pinned, src, n * p->esize, cudaMemcpyDeviceToHost, e->stream));
    YK_CHECK_CUDA(cudaStreamSynchronize(e->stream));
    for (size_t i = 0; i < n; ++i)
        host[i] = p->esize == 2 ? host_from_bf16(((uint16_t*)e->pinned)[i]) : ((float*)e->pinned)[i];
    return YK_OK;
}

// ---------------------------------------------------------------------------
// forward step
// ---------------------------------------------------------------------------
// dt.d: the last dt.nd tokens of every sequence come from device-resident draft
// tokens (tokens[] holds placeholders there); the host never waits for them.
// Split pools (wpool != null): `pool` holds the global layers with block_tables,
// `wpool` the windowed layers with wtables.
struct WindowedPool {
    yk_kv_pool* pool = nullptr;
    const int32_t* tables = nullptr;
    int32_t max_blocks = 0;
};

static yk_status forward_impl(yk_model* m, yk_kv_pool* pool, const uint32_t* tokens, int32_t T,
                              const uint32_t* q_starts, const uint32_t* ctx, int32_t B, const int32_t* block_tables,
                              int32_t max_blocks, int32_t last_n, int32_t* n_rows, const yk::DraftTokens& dt,
                              const WindowedPool& wp = {}) {
    YK_ARG(m && pool && tokens && q_starts && ctx && block_tables, "null argument");
    const auto& c = m->cfg;
    yk_kv_pool* const wpool = wp.pool;
    if (wpool) {
        YK_ARG(wp.tables && wp.max_blocks > 0, "windowed page tables");
        YK_ARG(pool->kind == YK_POOL_GLOBAL_LAYERS && wpool->kind == YK_POOL_WINDOWED_LAYERS,
               "split pools: a YK_POOL_GLOBAL_LAYERS pool and a YK_POOL_WINDOWED_LAYERS pool");
        YK_ARG(wpool->e == m->e && wpool->cfg.n_layers == c.n_layers && wpool->cfg.n_kv_heads == c.n_kv_heads &&
                   wpool->cfg.head_dim == c.head_dim && wpool->cfg.dtype == c.dtype &&
                   wpool->cfg.window == c.window && wpool->cfg.window_layer_parity == c.window_layer_parity &&
                   pool->cfg.window == c.window && pool->cfg.window_layer_parity == c.window_layer_parity,
               "windowed pool does not match the model");
    } else {
        YK_ARG(pool->kind == YK_POOL_ALL_LAYERS, "a pool of one layer kind needs yk_forward_step_split");
    }
    yk_engine* e = m->e;
    YK_ARG(pool->e == e, "pool belongs to another engine");
    YK_ARG(pool->cfg.n_layers == c.n_layers && pool->cfg.n_kv_heads == c.n_kv_heads &&
               pool->cfg.head_dim == c.head_dim && pool->cfg.dtype == c.dtype,
           "pool shape does not match the model");
    YK_ARG(T > 0 && T <= c.max_tokens, "T must be in [1, max_tokens]");
    YK_ARG(B > 0 && B <= c.max_seqs, "B must be in [1, max_seqs]");
    YK_ARG(max_blocks > 0 && last_n >= 0, "max_blocks / last_n");
    YK_ARG(q_starts[0] == 0 && (int32_t)q_starts[B] == T, "q_starts must run from 0 to T");
    // Host-side validation and per-token metadata.
    int R = 0;
    for (int b = 0; b < B; ++b) {
        YK_ARG(q_starts[b + 1] >= q_starts[b], "q_starts must be non-decreasing");
        const uint32_t n = q_starts[b + 1] - q_starts[b];
        YK_ARG(ctx[b] >= n, "context_lens[b] must cover the new tokens");
        YK_ARG((int64_t)(ctx[b] + YK_BLOCK_SIZE - 1) / YK_BLOCK_SIZE <= max_blocks, "page table too short");
        for (uint32_t p = 0; p < (ctx[b] + YK_BLOCK_SIZE - 1) / YK_BLOCK_SIZE; ++p) {
            const int32_t blk = block_tables[(size_t)b * max_blocks + p];
            YK_ARG(blk >= 0 && blk < pool->num_blocks, "block id outside the pool");
        }
        if (wpool) {
            YK_ARG((int64_t)(ctx[b] + YK_BLOCK_SIZE - 1) / YK_BLOCK_SIZE <= wp.max_blocks, "windowed page table too short");
            for (uint32_t p = 0; p < (ctx[b] + YK_BLOCK_SIZE - 1) / YK_BLOCK_SIZE; ++p) {
                const int32_t blk = wp.tables[(size_t)b * wp.max_blocks + p];
                YK_ARG(blk >= 0 && blk < wpool->num_blocks, "block id outside the windowed pool");
            }
        }
        R += last_n > 0 ? std::min<int>(last_n, (int)n) : (int)n;
    }
    for (int b = 0; b < B; ++b) {
        YK_ARG(q_starts[b + 1] - q_starts[b] >= (uint32_t)dt.nd, "fewer new tokens than device draft tokens");
        for (uint32_t t = q_starts[b]; t < q_starts[b + 1] - dt.nd; ++t)
            YK_ARG(tokens[t] < (uint32_t)c.vocab_size, "token id >= vocab_size");
    }
    YK_ARG(R > 0, "no logit rows");
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    // Attention work lists (bf16 tensor-core path): global and windowed layers.
    static thread_local std::vector<int32_t> it_g, cb_g, it_w, cb_w;
    int slots_g = 0, slots_w = 0;
    it_g.clear(); cb_g.clear(); it_w.clear(); cb_w.clear();
    if (c.dtype == YK_DTYPE_BF16) {
        yk::plan_attention(c, e->num_sms, e->attn_waves, e->attn_balanced, q_starts, ctx, B, false, it_g, cb_g,
                           &slots_g);
        if (c.window > 0)
            yk::plan_attention(c, e->num_sms, e->attn_waves, e->attn_balanced, q_starts, ctx, B, true, it_w, cb_w,
                               &slots_w);
        const size_t need = (size_t)std::max(slots_g, slots_w) * yk::attention_ws_floats_per_slot(c.head_dim);
        if (need > m->attn_ws_floats) {
            YK_CHECK_CUDA(cudaStreamSynchronize(e->stream));
            if (m->attn_ws) cudaFree(m->attn_ws);
            m->attn_ws = nullptr;
            m->attn_ws_floats = 0;
            YK_CHECK_CUDA(cudaMalloc(&m->attn_ws, need * 2 * 4));
            m->attn_ws_floats = need * 2;
        }
        const int groups = (int)std::max(cb_g.size(), cb_w.size()) / 5;
        if (groups > m->attn_counter_cap) {
            YK_CHECK_CUDA(cudaStreamSynchronize(e->stream));
            if (m->attn_counters) cudaFree(m->attn_counters);
            m->attn_counters = nullptr;
            m->attn_counter_cap = 0;
            const int cap = std::max(2 * groups, 1024);
            YK_CHECK_CUDA(cudaMalloc(&m->attn_counters, (size_t)cap * 4));
            YK_CHECK_CUDA(cudaMemset(m->attn_counters, 0, (size_t)cap * 4));
            m->attn_counter_cap = cap;
        }
    }
    const size_t nattn = it_g.size() + cb_g.size() + it_w.size() + cb_w.size();
    const size_t nsplit = wpool ? (size_t)T + (size_t)B * wp.max_blocks : 0;  // windowed slots + page tables
    const size_t nmeta = (size_t)4 * T + (B + 1) + B + (size_t)B * max_blocks + R + nattn + nsplit;
    // Metadata slot of this call.  Async: the upload runs on the engine's upload
    // stream as soon as the slot's previous forward (META_SLOTS calls ago) and the
    // work enqueued after it are done, so it overlaps the kernels still running;
    // the compute stream waits only for the copy's event.
    const bool async = e->meta_async;
    const int ms = async ? (int)(m->meta_calls % yk_model::META_SLOTS) : 0;
    if (async) {
        for (int i = 0; i < yk_model::META_SLOTS; ++i) {
            if (!m->meta_copied[i]) YK_CHECK_CUDA(cudaEventCreateWithFlags(&m->meta_copied[i], cudaEventDisableTiming));
            if (!m->meta_free[i]) YK_CHECK_CUDA(cudaEventCreateWithFlags(&m->meta_free[i], cudaEventDisableTiming));
        }
        // everything enqueued so far (the previous call's forward and whatever read
        // its metadata after it) releases the previous call's slot
        if (m->meta_calls > 0) {
            const int prev = (int)((m->meta_calls - 1) % yk_model::META_SLOTS);
            YK_CHECK_CUDA(cudaEventRecord(m->meta_free[prev], e->stream));
        }
        YK_CHECK_CUDA(cudaStreamWaitEvent(e->up_stream, m->meta_free[ms], 0));
    }
    // (a device buffer still read by earlier launches is freed only after cudaFree's implicit synchronisation)
    if (nmeta > m->meta_cap[ms]) {
        if (m->meta[ms]) cudaFree(m->meta[ms]);
        m->meta[ms] = nullptr;
        m->meta_cap[ms] = 0;
        YK_CHECK_CUDA(cudaMalloc(&m->meta[ms], std::max<size_t>(nmeta * 2, 4096) * 4));
        m->meta_cap[ms] = std::max<size_t>(nmeta * 2, 4096);
    }
    int32_t* const meta = m->meta[ms];
    int up_slot = 0;
    uint8_t* up_host = nullptr;
    YK_TRY(e->up_acquire(nmeta * 4, &up_slot, &up_host));  // no wait for the device: a ring of staging slots
    int32_t* hm = (int32_t*)up_host;
    int32_t* h_tok = hm;
    int32_t* h_pos = h_tok + T;
    int32_t* h_slot = h_pos + T;
    int32_t* h_seq = h_slot + T;
    int32_t* h_qs = h_seq + T;
    int32_t* h_ctx = h_qs + (B + 1);
    int32_t* h_bt = h_ctx + B;
    int32_t* h_rows = h_bt + (size_t)B * max_blocks;
    int r = 0;
    for (int b = 0; b <= B; ++b) h_qs[b] = (int32_t)q_starts[b];
    for (int b = 0; b < B; ++b) {
        const int n = (int)(q_starts[b + 1] - q_starts[b]);
        h_ctx[b] = (int32_t)ctx[b];
        for (int i = 0; i < n; ++i) {
            const int t = (int)q_starts[b] + i;
            const int pos = (int)ctx[b] - n + i;
            h_tok[t] = (int32_t)tokens[t];
            h_pos[t] = pos;
            h_seq[t] = b;
            h_slot[t] = block_tables[(size_t)b * max_blocks + pos / YK_BLOCK_SIZE] * YK_BLOCK_SIZE + pos % YK_BLOCK_SIZE;
        }
        const int take = last_n > 0 ? std::min(last_n, n) : n;
        for (int i = n - take; i < n; ++i) h_rows[r++] = (int)q_starts[b] + i;
    }
    std::memcpy(h_bt, block_tables, (size_t)B * max_blocks * 4);
    int32_t* h_attn = h_rows + R;
    const size_t attn_off = (size_t)(h_attn - hm);
    {
        int32_t* w = h_attn;
        for (auto* v : {&it_g, &cb_g, &it_w, &cb_w}) {
            if (!v->empty()) std::memcpy(w, v->data(), v->size() * 4);
            w += v->size();
        }
    }
    int32_t* const h_wslot = h_attn + nattn;  // split pools only
    int32_t* const h_wbt = h_wslot + T;
    if (wpool) {
        for (int b = 0; b < B; ++b) {
            const int n = (int)(q_starts[b + 1] - q_starts[b]);
            for (int i = 0; i < n; ++i) {
                const int pos = (int)ctx[b] - n + i;
                h_wslot[(int)q_starts[b] + i] =
                    wp.tables[(size_t)b * wp.max_blocks + pos / YK_BLOCK_SIZE] * YK_BLOCK_SIZE + pos % YK_BLOCK_SIZE;
            }
        }
        std::memcpy(h_wbt, wp.tables, (size_t)B * wp.max_blocks * 4);
    }
    if (async) {
        YK_TRY(e->up_submit_on(up_slot, meta, nmeta * 4, e->up_stream));
        YK_CHECK_CUDA(cudaEventRecord(m->meta_copied[ms], e->up_stream));
        YK_CHECK_CUDA(cudaStreamWaitEvent(e->stream, m->meta_copied[ms], 0));
        m->meta_calls++;
    } else {
        YK_TRY(e->up_submit(up_slot, meta, nmeta * 4));
    }
    {
        const int32_t* a = meta + attn_off;
        m->cur.attn_items[0] = a;
        m->cur.n_items[0] = (int)(it_g.size() / 7);
        a += it_g.size();
        m->cur.attn_comb[0] = a;
        m->cur.n_comb[0] = (int)(cb_g.size() / 5);
        a += cb_g.size();
        m->cur.attn_items[1] = a;
        m->cur.n_items[1] = (int)(it_w.size() / 7);
        a += it_w.size();
        m->cur.attn_comb[1] = a;
        m->cur.n_comb[1] = (int)(cb_w.size() / 5);
    }
    const int32_t* dm = meta;
    m->cur.wslot = wpool ? meta + (h_wslot - hm) : nullptr;
    m->cur.wbt = wpool ? meta + (h_wbt - hm) : nullptr;
    m->cur.wmax_blocks = wpool ? wp.max_blocks : 0;
    m->cur.tokens = dm;
    m->cur.pos = dm + T;
    m->cur.slot = dm + 2 * T;
    m->cur.seq = dm + 3 * T;
    m->cur.q_starts = dm + 4 * T;
    m->cur.ctx = m->cur.q_starts + (B + 1);
    m->cur.bt = m->cur.ctx + B;
    m->cur.rows = m->cur.bt + (size_t)B * max_blocks;

    using namespace yk;
    const int d = c.d_model, dh = c.head_dim, qd = c.n_heads * dh, kvd = c.n_kv_heads * dh, F = c.ffn_dim;
    // Algorithmic KV bytes one attention launch must read: every cached key/value
    // of each sequence once (windowed layers: at most window + new tokens).
    double kv_full = 0, kv_win = 0;
    for (int b = 0; b < B; ++b) {
        const double n = (double)(q_starts[b + 1] - q_starts[b]);
        kv_full += (double)ctx[b];
        kv_win += c.window > 0 ? std::min((double)ctx[b], (double)c.window + n - 1) : (double)ctx[b];
    }
    const double kv_tok_bytes = 2.0 * kvd * (double)m->esize;
    // Tensor parallel: o_proj / down_proj write partials (bf16, or fp32 with
    // YK_TP_PAYLOAD=f32) that are summed across the group; the sum is added to the
    // residual stream by the next RMSNorm.
    const bool tp = m->tp_world > 1;
    const void* pend = nullptr;  // all-reduced partial not yet added to h
    EpiParams es;
    es.kind = EPI_STORE;
    es.out = m->tp_y;
    es.store_bf16 = e->tp_bf16 ? 1 : 0;
    // the group's own all-reduce over NVLink peer memory (bf16 payload): the GEMM
    // writes its partial into this rank's shared slot, the all-reduce kernel sums
    // every rank's slot into tp_y
    const bool own_ar = tp && e->tp_bf16 && tp_ar_enabled(e);
    if (own_ar) YK_TRY(tp_ar_reserve(e, (size_t)T * d));
    auto tp_reduce = [&]() -> yk_status {
        if (own_ar) return tp_ar_run(e, (size_t)T * d, reinterpret_cast<__nv_bfloat16*>(m->tp_y));
        return tp_allreduce(e, m->tp_y, (size_t)T * d, e->tp_bf16);
    };
    // RMSNorm folded into the GEMMs (bf16, one GPU): the residual epilogue (and the
    // embedding) writes x = bf16(h * gain) and 32-row sums of squares; the next
    // GEMM scales each token's accumulator by its 1/rms.  The final norm stays a
    // kernel (it gathers the logit rows).
    const bool fused = c.dtype == YK_DTYPE_BF16 && !tp && !c.ref_compat && T <= 256 && d % 32 == 0 && e->fuse_norm;
    auto norm_in = [&](EpiParams& p) {
        if (!fused) return;
        p.in_ss = m->norm_ss;
        p.in_groups = d / 32;
        p.ss_ld = T;
        p.in_d = (float)d;
        p.in_eps = c.rms_eps;
    };
    auto norm_out = [&](EpiParams& p, const float* g) {
        if (!fused || !g) return;
        p.nx_g = g;
        p.nx_out = m->xn;
        p.nx_ss = m->norm_ss;
        p.ss_ld = T;
    };
    YK_TRY(launch_embed(m, m->cur.tokens, m->cur.pos, T, dt, fused ? m->layers[0].n1 : nullptr));
    for (int l = 0; l < c.n_layers; ++l) {
        LayerWeights& L = m->layers[l];
        if (!fused) YK_TRY(launch_rmsnorm(m, L.n1, T, nullptr, pend, e->tp_bf16));
        pend = nullptr;
        EpiParams eq;
        eq.kind = EPI_QKV;
        eq.ref_compat = c.ref_compat;
        eq.out = m->q;
        eq.q_dim = qd;
        eq.kv_dim = kvd;
        eq.head_dim = dh;
        eq.n_kv = c.n_kv_heads;
        const bool windowed = layer_windowed(c, l);
        // split pools: the windowed layers' K/V live in wpool under their own page tables
        const bool in_w = wpool && windowed;
        yk_kv_pool* const lpool = in_w ? wpool : pool;
        const int pl = pool_layer_index(c, lpool->kind, l);
        eq.pos = m->cur.pos;
        eq.slot = in_w ? m->cur.wslot : m->cur.slot;
        eq.rope_denom = m->rope_denom;
        eq.rope_tab = m->rope_tab;
        eq.pool = lpool->data;
        eq.block_elems = (long long)lpool->block_elems;
        eq.layer_off = (long long)pl * (long long)lpool->layer_elems;
        eq.pool_blocks = lpool->num_blocks;
        norm_in(eq);
        YK_TRY(gemm_run(m, L.wqkv, &L.tm_qkv, m->xn, qd + 2 * kvd, d, T, eq));
        YK_TRY(attention_run(m, lpool, l, pl, in_w ? m->cur.wbt : m->cur.bt, T, B, in_w ? wp.max_blocks : max_blocks,
                             (windowed ? kv_win : kv_full) * kv_tok_bytes));
        EpiParams er;
        er.kind = EPI_RESID;
        er.ref_compat = c.ref_compat;
        er.h = m->h;
        er.ld = d;
        if (tp) {
            if (own_ar) es.out = tp_ar_slot(e);
            YK_TRY(gemm_run(m, L.wo, &L.tm_o, m->att, d, qd, T, es));
            YK_TRY(tp_reduce());
            pend = m->tp_y;
        } else {
            EpiParams eo = er;
            norm_out(eo, L.n2);
            YK_TRY(gemm_run(m, L.wo, &L.tm_o, m->att, d, qd, T, eo));
        }
        if (!fused) YK_TRY(launch_rmsnorm(m, L.n2, T, nullptr, pend, e->tp_bf16));
        pend = nullptr;
        EpiParams eg;
        eg.kind = EPI_GLU;
        eg.ref_compat = c.ref_compat;
        eg.out = m->act;
        eg.act = c.act;
        norm_in(eg);
        if (!tp && e->gemm_chain && c.dtype == YK_DTYPE_BF16 && T <= 256) {
            // gate/up and down_proj in one launch
            EpiParams ed = er;
            norm_out(ed, l + 1 < c.n_layers ? m->layers[l + 1].n1 : nullptr);
            YK_TRY(gemm_chain_glu_down(m, L.wgu, &L.tm_gu, m->xn, 2 * F, d, L.wdown, &L.tm_down, m->act, d, F, T, eg,
                                       ed));
            continue;
        }
        YK_TRY(gemm_run(m, L.wgu, &L.tm_gu, m->xn, 2 * F, d, T, eg));
        if (tp) {
            if (own_ar) es.out = tp_ar_slot(e);
            YK_TRY(gemm_run(m, L.wdown, &L.tm_down, m->act, d, F, T, es));
            YK_TRY(tp_reduce());
            pend = m->tp_y;
        } else {
            EpiParams ed = er;
            norm_out(ed, l + 1 < c.n_layers ? m->layers[l + 1].n1 : nullptr);
            YK_TRY(gemm_run(m, L.wdown, &L.tm_down, m->act, d, F, T, ed));
        }
    }
    YK_TRY(launch_rmsnorm(m, m->final_norm, R, m->cur.rows, pend, e->tp_bf16));
    EpiParams el;
    el.kind = EPI_LOGITS;
    el.ref_compat = c.ref_compat;
    el.out = m->logits;
    el.cap = c.ref_compat ? 30.0f : c.final_cap;
    YK_TRY(gemm_run(m, m->lm_head, &m->tm_lm, m->xn, c.vocab_size, d, R, el));
    m->last_rows = R;
    if (n_rows) *n_rows = R;
    return YK_OK;
}


extern "C" yk_status yk_forward_step(yk_model* m, yk_kv_pool* pool, const uint32_t* tokens, int32_t T,
                                     const uint32_t* q_starts, const uint32_t* ctx, int32_t B,
                                     const int32_t* block_tables, int32_t max_blocks, int32_t last_n,
                                     int32_t* n_rows) {
    return forward_impl(m, pool, tokens, T, q_starts, ctx, B, block_tables, max_blocks, last_n, n_rows, {});
}

extern "C" yk_status yk_forward_step_drafts(yk_model* m, yk_kv_pool* pool, const uint32_t* tokens, int32_t T,
                                            const uint32_t* q_starts, const uint32_t* ctx, int32_t B,
                                            const int32_t* block_tables, int32_t max_blocks, int32_t last_n,
                                            yk_sampler* s, int32_t j0, int32_t nd, int32_t* n_rows) {
    YK_ARG(s && nd > 0, "sampler / nd");
    yk::DraftTokens dt;
    dt.d = yk::sampler_device_drafts(s, B, &dt.k);
    YK_ARG(dt.d != nullptr, "batch larger than the sampler's");
    YK_ARG(j0 >= 0 && j0 + nd <= dt.k, "draft token range outside 0..k-1");
    dt.j0 = j0;
    dt.nd = nd;
    return forward_impl(m, pool, tokens, T, q_starts, ctx, B, block_tables, max_blocks, last_n, n_rows, dt);
}

extern "C" yk_status yk_forward_step_split(yk_model* m, yk_kv_pool* pool, yk_kv_pool* wpool, const uint32_t* tokens,
                                           int32_t T, const uint32_t* q_starts, const uint32_t* ctx, int32_t B,
                                           const int32_t* block_tables, int32_t max_blocks,
                                           const int32_t* wblock_tables, int32_t wmax_blocks, int32_t last_n,
                                           yk_sampler* s, int32_t j0, int32_t nd, int32_t* n_rows) {
    YK_ARG(wpool != nullptr, "null windowed pool");
    yk::DraftTokens dt;
    if (s && nd > 0) {
        dt.d = yk::sampler_device_drafts(s, B, &dt.k);
        YK_ARG(dt.d != nullptr, "batch larger than the sampler's");
        YK_ARG(j0 >= 0 && j0 + nd <= dt.k, "draft token range outside 0..k-1");
        dt.j0 = j0;
        dt.nd = nd;
    }
    WindowedPool wp;
    wp.pool = wpool;
    wp.tables = wblock_tables;
    wp.max_blocks = wmax_blocks;
    return forward_impl(m, pool, tokens, T, q_starts, ctx, B, block_tables, max_blocks, last_n, n_rows, dt, wp);
}

extern "C" yk_status yk_logits_copy_to_host(yk_model* m, int32_t row0, int32_t rows, float* host) {
    YK_ARG(m && host, "null handle");
    YK_ARG(row0 >= 0 && rows >= 0 && row0 + rows <= m->last_rows, "rows outside the last step's logits");
    yk_engine* e = m->e;
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    const size_t bytes = (size_t)rows * m->cfg.vocab_size * 4;
    YK_CHECK_CUDA(cudaMemcpyAsync(host, m->logits + (size_t)row0 * m->cfg.vocab_size, bytes, cudaMemcpyDeviceToHost,
                                  e->stream));
    YK_CHECK_CUDA(cudaStreamSynchronize(e->stream));
    uint32_t err = 0;
    YK_CHECK_CUDA(cudaMemcpy(&err, e->d_err, 4, cudaMemcpyDeviceToHost));
    if (err) {
        yk_set_error("device check fired (code " + std::to_string(err) + ")");
        cudaMemset(e->d_err, 0, 4);
        return (err & YK_DEV_ERR_TIMEOUT) ? YK_ERR_TIMEOUT : YK_ERR_DEVICE_CHECK;
    }
    return YK_OK;
}

// ---------------------------------------------------------------------------
// Launch trace test hooks (include/yk_testing.h).
// ---------------------------------------------------------------------------
#include "../../include/yk_testing.h"

extern "C" yk_status ykt_trace_enable(yk_engine* e, int32_t cap) {
    YK_ARG(e && cap >= 0, "arguments");
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    YK_CHECK_CUDA(cudaStreamSynchronize(e->stream));
    if (e->trace_rec) cudaFree(e->trace_rec);
    e->trace_rec = nullptr;
    e->trace_cap = 0;
    if (cap == 0) return YK_OK;
    std::vector<yk::TraceRec> init((size_t)cap);
    for (auto& r : init) {
        r.entry = ~0ull;
        r.start = ~0ull;
        r.end = 0;
        r.kind = 0;
    }
    YK_CHECK_CUDA(cudaMalloc(&e->trace_rec, (size_t)cap * sizeof(yk::TraceRec)));
    YK_CHECK_CUDA(cudaMemcpy(e->trace_rec, init.data(), (size_t)cap * sizeof(yk::TraceRec), cudaMemcpyHostToDevice));
    e->trace_cap = (uint32_t)cap;
    return YK_OK;
}

extern "C" yk_status ykt_trace_read(yk_engine* e, uint64_t* host, int32_t cap, uint64_t* launches) {
    YK_ARG(e && host && launches, "arguments");
    YK_ARG(e->trace_rec && (uint32_t)cap == e->trace_cap, "trace not enabled with this capacity");
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    YK_CHECK_CUDA(cudaStreamSynchronize(e->stream));
    YK_CHECK_CUDA(cudaMemcpy(host, e->trace_rec, (size_t)cap * sizeof(yk::TraceRec), cudaMemcpyDeviceToHost));
    *launches = e->launches;
    return YK_OK;
}
