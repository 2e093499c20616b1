// yk_internal.h -- host-side structures behind the opaque handles of yk.h.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <string>
#include <utility>
#include <vector>

#include "../../include/yk.h"
#include "yk_common.cuh"

// ---- error plumbing --------------------------------------------------------
void yk_set_error(const std::string& msg);
#define YK_CHECK_CUDA(call)                                                              \
    do {                                                                                 \
        cudaError_t e_ = (call);                                                         \
        if (e_ != cudaSuccess) {                                                         \
            yk_set_error(std::string(#call) + ": " + cudaGetErrorString(e_));            \
            return e_ == cudaErrorMemoryAllocation ? YK_ERR_OOM : YK_ERR_CUDA;           \
        }                                                                                \
    } while (0)
#define YK_ARG(cond, msg)                                                                \
    do {                                                                                 \
        if (!(cond)) {                                                                   \
            yk_set_error(std::string("invalid argument: ") + (msg));                     \
            return YK_ERR_ARG;                                                           \
        }                                                                                \
    } while (0)
#define YK_TRY(call)                                                                     \
    do {                                                                                 \
        yk_status s_ = (call);                                                           \
        if (s_ != YK_OK) return s_;                                                      \
    } while (0)

typedef CUresult (*PFN_tmapEncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                        const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                        CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                        CUtensorMapFloatOOBfill);

// Per-kernel-class timing with CUDA events on the engine stream (yk_engine_profile).
struct ProfRecord {
    int cls;
    cudaEvent_t start, stop;
    double bytes, flops;
    bool failed = false;  // its stop event could not be recorded: left out of the totals
};
struct ProfTotals {
    double ms = 0, bytes = 0, flops = 0;
    int64_t launches = 0;
};

struct yk_engine {
    int device = 0;
    int num_sms = 148;
    cudaStream_t stream = nullptr;
    cudaStream_t up_stream = nullptr;    // forward metadata uploads, ahead of `stream` (event-ordered)
    bool meta_async = true;              // env YK_META_ASYNC=0: upload on `stream`, in line
    uint32_t* d_err = nullptr;           // device error word
    uint8_t* pinned = nullptr;           // host staging (downloads, and uploads that synchronise anyway)
    size_t pinned_bytes = 0;
    // Ring of pinned upload slots: a per-step upload (forward metadata, sampler
    // sequence ids) fills the next slot while earlier work still runs; a slot is
    // reused once the event recorded after its copy has fired.
    static constexpr int UP_SLOTS = 4;
    struct UpSlot {
        uint8_t* host = nullptr;
        size_t bytes = 0;
        cudaEvent_t done = nullptr;
    };
    UpSlot up[UP_SLOTS];
    int up_next = 0;
    uint64_t launches = 0;
    PFN_tmapEncodeTiled encode_tiled = nullptr;
    bool pdl = true;                     // programmatic dependent launch (env YK_PDL=0 turns it off)
    int gemm_variant = 0;                // GEMM schedule tuning knob (env YK_GEMM_VARIANT): bit 0 = pure
                                         // stream-K instead of whole tiles + stream-K remainder; bit 2 =
                                         // cluster scheduling policy "spread"; bit 3 = cluster split-K
                                         // reduction always by distributed-shared-memory loads; bit 5 =
                                         // no cluster split-K (whole tiles / stream-K for every shape)
    int gemm_push_min = 16384;           // cluster split-K: column shares of at least this many bytes are
                                         // exchanged by copy engine (env YK_GEMM_PUSH_MIN)
    int attn_waves = 1;                  // attention items per resident CTA slot (env YK_ATTN_WAVES)
    bool attn_balanced = false;          // attention pieces <= average slot load (env YK_ATTN_PLAN=1)
    bool fuse_norm = true;               // RMSNorm folded into the GEMMs around it (env YK_FUSE_NORM=0: off)
    bool gemm_chain = false;             // gate/up + down_proj as one persistent launch (env YK_GEMM_CHAIN=1)
    bool profiling = false;
    void* nccl_comm = nullptr;           // tensor-parallel group (yk_tp_init), else null
    int tp_rank = 0, tp_world = 1;
    bool tp_bf16 = true;                 // all-reduce payload bf16 (env YK_TP_PAYLOAD=f32: fp32)
    int64_t tp_timeout_ms = 300000;      // deadline of group set-up and of a wait on the group's work
    uint32_t* tp_gather = nullptr;       // device staging of yk_tp_allgather_u32 (send, then recv)
    size_t tp_gather_elems = 0;
    // The group's own all-reduce over NVLink peer memory (env YK_TP_AR=nccl: NCCL's):
    // each rank's buffer [flags 4 KB | 2 partial slots | 2 reduced slots] of ar_cap bytes
    // per slot, shared with the other ranks through CUDA IPC.
    bool tp_ar_own = true;
    // own all-reduce at two ranks: one shot (each rank sums both whole partials)
    // instead of two-shot; YK_TP_AR=twoshot turns it off
    bool ar_one_shot = true;
    size_t ar_cap = 0;
    uint8_t* ar_local = nullptr;
    std::vector<void*> ar_opened;        // the peers' buffers as mapped here (null for this rank)
    uint8_t** ar_bufs = nullptr;         // device array: every rank's buffer, as mapped here
    uint32_t ar_epoch = 0;
    unsigned long long ar_ctr_base = 0;  // value of this rank's CTA counter before the next all-reduce
    void* trace_rec = nullptr;           // launch trace records (test hook), else null
    uint32_t trace_cap = 0;
    std::vector<ProfRecord> prof_pending;
    std::vector<cudaEvent_t> prof_free;
    ProfTotals prof[4];
    yk_status ensure_pinned(size_t bytes);
    // Next upload slot of at least `bytes` (waits for that slot's previous copy);
    // up_submit copies it to `dst` on the engine stream.
    yk_status up_acquire(size_t bytes, int* slot, uint8_t** host);
    yk_status up_submit(int slot, void* dst, size_t bytes);
    // the same copy on stream `on` (its done event recorded there)
    yk_status up_submit_on(int slot, void* dst, size_t bytes, cudaStream_t on);
    // Opens a timed record; returns its index, or -1 when its events could not
    // be created or recorded (that launch then goes untimed).
    int prof_begin(int cls, double bytes, double flops);
    void prof_end(int rec);
    void prof_resolve();
};

// RAII bracket for one profiled launch.
struct ProfScope {
    yk_engine* e;
    int rec = -1;
    ProfScope(yk_engine* e_, int cls, double bytes, double flops) : e(e_) {
        if (e->profiling) rec = e->prof_begin(cls, bytes, flops);
    }
    ~ProfScope() {
        if (rec >= 0) e->prof_end(rec);
    }
};

// Element counts of the device workspaces.
struct LayerWeights {
    void* wqkv = nullptr;   // [(H + 2Hkv)*dh x d]: Q rows, then K rows, then V rows
    void* wo = nullptr;     // [d x H*dh]
    void* wgu = nullptr;    // [2F x d]: row 2j = gate j, row 2j+1 = up j
    void* wdown = nullptr;  // [d x F]
    float* n1 = nullptr;    // [d]
    float* n2 = nullptr;    // [d]
    CUtensorMap tm_qkv, tm_o, tm_gu, tm_down;
};

struct yk_model {
    yk_engine* e = nullptr;
    yk_model_config cfg{};
    size_t esize = 4;  // bytes per weight / activation element
    // weights
    void* embed = nullptr;     // [V x d]
    void* lm_head = nullptr;   // [V x d]
    float* final_norm = nullptr;
    std::vector<LayerWeights> layers;
    int tp_rank = 0, tp_world = 1;  // tensor-parallel shard (cfg holds the shard's heads / FFN)
    float* tp_y = nullptr;          // [T x d] fp32 partial of o_proj / down_proj, all-reduced
    CUtensorMap tm_lm;
    // activations
    float* h = nullptr;        // [T x d] fp32 residual stream
    void* xn = nullptr;        // [T x d] normed input of the next GEMM
    void* q = nullptr;         // [T x H*dh]
    void* att = nullptr;       // [T x H*dh]
    void* act = nullptr;       // [T x F]
    float* logits = nullptr;   // [T x V]
    float* rope_denom = nullptr;  // [dh/2]
    float2* rope_tab = nullptr;   // [max_tokens x dh/2] (cos, sin) of this step's token positions
    float* norm_ss = nullptr;     // [d/32 x max_tokens] fused RMSNorm: 32-element group sums of squares
    // step metadata (device), packed as int32: a ring of buffers, one per forward
    // call, so that the next call's upload (on the engine's upload stream) runs
    // while this call's kernels still read theirs
    static constexpr int META_SLOTS = 4;
    int32_t* meta[META_SLOTS] = {};
    size_t meta_cap[META_SLOTS] = {};          // int32 elements
    cudaEvent_t meta_copied[META_SLOTS] = {};  // the slot's upload has landed (upload stream)
    cudaEvent_t meta_free[META_SLOTS] = {};    // every reader of the slot's last forward is done (compute stream)
    uint64_t meta_calls = 0;
    int32_t last_rows = 0;
    struct {
        const int32_t *tokens, *pos, *slot, *seq, *q_starts, *ctx, *bt, *rows;
        const int32_t *wslot, *wbt;  // split pools: the windowed layers' slots and page tables (else null)
        int wmax_blocks;
        const int32_t* attn_items[2];  // [0] global layers, [1] windowed layers
        const int32_t* attn_comb[2];
        int n_items[2], n_comb[2];
    } cur{};
    // split-K partials + per-tile arrival counters
    float* gemm_ws = nullptr;
    size_t gemm_ws_floats = 0;
    uint32_t* gemm_counters = nullptr;  // owned apart from `allocations`: may grow
    int gemm_counter_cap = 0;
    // GEMM phase timestamps (test hook only; null otherwise) and the last grid used
    unsigned long long* gemm_stamps = nullptr;
    int gemm_last_grid = 0;
    uint32_t* chain_bar = nullptr;  // grid barrier counter of the chained gate/up + down launch
    uint32_t chain_epoch = 0;       // its value after the last launch's barrier
    uint32_t gemm_stamp_kind = 0;  // test hook: only launches of this trace kind write gemm_stamps
    int gemm_stamp_cap = 0, gemm_stamp_grid = 0;
    // attention split-KV partials and per combine group arrival counters
    float* attn_ws = nullptr;
    size_t attn_ws_floats = 0;
    int32_t* attn_counters = nullptr;
    int attn_counter_cap = 0;
    unsigned long long* attn_stamps = nullptr;  // test hook: per-CTA phase stamps, else null
    int attn_stamps_cap = 0, attn_last_items = 0;
    // TMA maps of activation buffers, keyed by (buffer, token-box rows)
    std::map<std::pair<const void*, int>, CUtensorMap> xmaps;
    std::vector<void*> allocations;
};

struct yk_kv_pool {
    yk_engine* e = nullptr;
    yk_model_config cfg{};
    int32_t num_blocks = 0;
    size_t esize = 4;
    void* data = nullptr;      // [block][layer][2][Hkv][16][dh]
    size_t block_elems = 0;    // elements per block (all layers)
    size_t layer_elems = 0;    // elements per layer within a block
    CUtensorMap tm{};          // bf16 pools: 3-D TMA map (head dim, row in block, block)
    bool has_tm = false;
    int32_t kind = 0;          // YK_POOL_*: the layers a block holds
    int32_t n_pool_layers = 0; // layers per block
};
namespace yk {
// Whether layer l of cfg is windowed, and its index within a pool of `kind`
// (-1: the pool does not hold it).
inline bool layer_windowed(const yk_model_config& c, int l) {
    return c.window > 0 && (c.window_layer_parity < 0 || (l % 2) == c.window_layer_parity);
}
inline int pool_layer_index(const yk_model_config& c, int kind, int l) {
    if (kind == YK_POOL_ALL_LAYERS) return l;
    const bool want_w = kind == YK_POOL_WINDOWED_LAYERS;
    if (layer_windowed(c, l) != want_w) return -1;
    int idx = 0;
    for (int i = 0; i < l; ++i) idx += layer_windowed(c, i) == want_w ? 1 : 0;
    return idx;
}
}  // namespace yk

struct yk_sampler {
    yk_engine* e = nullptr;
    int32_t max_seqs = 0, k = 0, vocab = 0;
    float* probs = nullptr;     // [max_seqs x k x V] draft probabilities
    float* q = nullptr;         // [max_seqs x (k+1) x V] target probs (probs entry) or logits
    float* dlogits = nullptr;   // [max_seqs x k x V] draft logits (yk_spec_sample_logits)
    float* stats = nullptr;     // [max_seqs x (2k+1) x 4] (max, sum, argmax, -)
    float4* part = nullptr;     // [max_seqs x (k+1) x chunks] per-chunk row statistics (draft, then target)
    uint32_t* io = nullptr;     // small device io area
    unsigned long long* stamps = nullptr;  // test hook: per-CTA phase stamps of draft sampling / verify
    int stamps_cap = 0;
    std::vector<uint32_t> dev_seq;  // the sequence ids last uploaded to io[0..B) (re-uploaded only on change)
    int32_t logits_B = 0;           // batch whose logits yk_spec_sample_logits last uploaded (dlogits, q)
};

// ---- internal launchers ----------------------------------------------------
namespace yk {

// Trace handle for the launch about to be made (kinds: see TraceKind).
enum TraceKind : uint32_t {
    TK_EMBED = 1, TK_RMSNORM = 2, TK_GEMM = 3, TK_ATTN = 4, TK_DRAFT_SAMPLE = 5, TK_ROW_STATS = 6, TK_VERIFY = 7
};
inline Trace trace_next(yk_engine* e, uint32_t kind) {
    Trace t;
    t.rec = reinterpret_cast<TraceRec*>(e->trace_rec);
    t.id = e->trace_cap ? (uint32_t)(e->launches % e->trace_cap) : 0u;
    t.kind = kind;
    return t;
}

// Launch on the engine stream with programmatic dependent launch (the kernel
// must call pdl_wait before touching what earlier kernels wrote).  Off while
// profiling: the per-launch events sit between kernels anyway.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(yk_engine* e, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = e->stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = (e->pdl && !e->profiling) ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

enum EpiKind : int { EPI_STORE = 0, EPI_QKV = 1, EPI_RESID = 2, EPI_GLU = 3, EPI_LOGITS = 4 };

// Everything a GEMM epilogue needs.  Row n = output feature, column j = token.
struct EpiParams {
    int kind = EPI_STORE;
    int n_out = 0;          // valid output rows
    int m_tok = 0;          // valid tokens
    int ref_compat = 0;
    // EPI_STORE: out[j * n_out + n], fp32 (bf16 when store_bf16)
    void* out = nullptr;
    int store_bf16 = 0;
    // EPI_QKV
    int q_dim = 0, kv_dim = 0, head_dim = 0, n_kv = 0;
    const int32_t* pos = nullptr;    // [m_tok] token positions
    const int32_t* slot = nullptr;   // [m_tok] pool slot = block*16 + offset
    const float* rope_denom = nullptr;
    const float2* rope_tab = nullptr;  // [m_tok x head_dim/2] (cos, sin); null: computed per element
    void* pool = nullptr;
    long long block_elems = 0, layer_off = 0;
    int pool_blocks = 0;
    // EPI_RESID: h[j * ld + n] += v
    float* h = nullptr;
    int ld = 0;
    // EPI_GLU: out[j * (n_out/2) + n/2] = act(gate) * up
    int act = 0;
    // EPI_LOGITS: logits[j * n_out + n]
    float cap = 0.f;
    // RMSNorm folded into the GEMMs around it (bf16 models).  EPI_RESID with
    // nx_out: also writes the next GEMM's input nx_out[j * ld + n] =
    // bf16(h_new * nx_g[n]) (the norm's gain; its 1/rms follows) and the sums of
    // squares of h_new over each 32-row group: nx_ss[(n / 32) * ss_ld + j].
    // in_ss: this GEMM's input is such an x; the accumulator of token j is scaled
    // by 1 / sqrt(sum_g in_ss[g * ss_ld + j] / in_d + in_eps) first.
    const float* nx_g = nullptr;
    void* nx_out = nullptr;
    float* nx_ss = nullptr;
    const float* in_ss = nullptr;
    int in_groups = 0, ss_ld = 0;  // in_groups: 32-row groups of the input dimension (d / 32)
    float in_d = 0.f, in_eps = 0.f;
    uint32_t* err = nullptr;
};

yk_status gemm_run(yk_model* m, const void* W, const CUtensorMap* tmW, const void* X, int n_out, int K, int m_tok,
                   const EpiParams& ep, int force_grid = 0);
// gate/up (GLU epilogue) then down_proj (residual epilogue) in one persistent
// launch (one CTA per SM, a grid barrier between them); m_tok <= 256.
// Where a logical tensor (YK_T_*) lives: base pointer, first row, row pitch (in
// rows), rows, cols, element size (gate / up rows interleave: pitch 2).
struct TensorLoc {
    uint8_t* base;
    size_t row0, pitch_rows, rows, cols, es;
};
yk_status locate_tensor(const yk_model* m, int32_t t, int32_t layer, TensorLoc* L);
yk_status gemm_chain_glu_down(yk_model* m, const void* Wgu, const CUtensorMap* tmWgu, const void* X0, int n_gu, int K0,
                              const void* Wd, const CUtensorMap* tmWd, const void* X1, int n_d, int K1, int m_tok,
                              const EpiParams& eg, const EpiParams& ed);
yk_status make_weight_map(yk_engine* e, CUtensorMap* map, const void* W, int rows, int K);
yk_status attention_run(yk_model* m, yk_kv_pool* pool, int layer, int pool_layer, const int32_t* bt, int T, int B,
                        int max_blocks,
                        double kv_bytes);
void plan_attention(const yk_model_config& c, int num_sms, int waves, bool balanced, const uint32_t* q_starts,
                    const uint32_t* ctx, int B, bool windowed, std::vector<int32_t>& items, std::vector<int32_t>& comb,
                    int* n_slots);
size_t attention_ws_floats_per_slot(int head_dim);
yk_status make_pool_map(yk_engine* e, yk_kv_pool* pool);
// The last nd input tokens of every sequence taken from device-resident draft
// tokens d[b * k + j0 + i] (the sampler's), instead of the uploaded ids.
struct DraftTokens {
    const uint32_t* d = nullptr;
    int k = 0, j0 = 0, nd = 0;
};
// norm_g: fused RMSNorm of the first layer (bf16): also x = bf16(h * norm_g) and
// the 32-element group sums of squares (m->norm_ss, token stride T).
yk_status launch_embed(yk_model* m, const int32_t* tokens, const int32_t* pos, int T, const DraftTokens& dt = {},
                       const float* norm_g = nullptr);
// Device array [B x k] of the draft tokens yk_draft_sample kept on the device
// for a batch of B sequences.
const uint32_t* sampler_device_drafts(const yk_sampler* s, int B, int* k);
// add: a pending residual [rows of h x d] added to h first (fp32, or bf16 when add_bf16)
yk_status launch_rmsnorm(yk_model* m, const float* g, int rows, const int32_t* row_idx, const void* add = nullptr,
                         int add_bf16 = 0);
// In-place sum over the tensor-parallel group of `count` fp32 (or bf16) values on the engine stream.
yk_status tp_allreduce(yk_engine* e, void* buf, size_t count, bool bf16);
// The group's own bf16 all-reduce: `count` values this rank wrote into tp_ar_slot
// (the partial slot of the next call) are summed over the ranks, in rank order
// (every rank gets the same values), into `out`.
bool tp_ar_enabled(const yk_engine* e);
yk_status tp_ar_reserve(yk_engine* e, size_t count);  // collective: every rank, same count
__nv_bfloat16* tp_ar_slot(yk_engine* e);
yk_status tp_ar_run(yk_engine* e, size_t count, __nv_bfloat16* out, unsigned long long* stamps = nullptr);
// Waits for the engine stream; with a tensor-parallel group, bounded by the
// group's deadline (the communicator is aborted and YK_ERR_TIMEOUT returned when
// it runs out: a peer that stopped taking part leaves its collectives unfinished).
yk_status engine_sync_bounded(yk_engine* e);
void tp_destroy(yk_engine* e);
yk_status launch_init(yk_engine* e, void* p, size_t n, int dtype, uint64_t seed, uint32_t stream, float std,
                      bool constant);

}  // namespace yk
