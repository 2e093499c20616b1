// yk_stub.cpp -- TEST INFRASTRUCTURE ONLY.  A CPU stand-in for the six libyk.so
// entry points that libyk_host.so's scheduler calls (yk_model_get_config,
// yk_kv_pool_num_blocks, yk_forward_step[_drafts], yk_draft_sample,
// yk_spec_verify), compiled together with host/yk_host.cpp into one test
// library, so that the scheduling logic -- admission, page tables, rollback,
// window reclamation, streaming -- runs without a GPU.
//
// The forward checks the page tables it is given: every page a query of the
// call may read (all of the context; from first_query - window + 1 on when
// every layer is windowed) must hold a block id inside the pool, and no block
// may be read by two sequences of one call.  Draft tokens and verification are
// deterministic functions of (sequence id, step, draft index).
#include <cstdint>
#include <cstring>
#include <map>
#include <vector>

#include "../../include/yk.h"

struct yk_model {
    yk_model_config cfg;
};
struct yk_kv_pool {
    int num_blocks;
};
struct yk_sampler {
    int k, V;
    std::vector<uint32_t> drafts;  // [B x k] device-resident drafts
};

namespace {
int64_t g_violations = 0, g_forwards = 0, g_pages_checked = 0;

// windowed_pool: the tables of a pool that holds only windowed layers.
void check_tables(const yk_model* m, const yk_kv_pool* pool, const uint32_t* q_starts, const uint32_t* ctx, int B,
                  const int32_t* tables, int max_blocks, bool windowed_pool = false) {
    const bool windowed = windowed_pool || (m->cfg.window > 0 && m->cfg.window_layer_parity < 0);
    std::map<int, int> owner;
    for (int b = 0; b < B; ++b) {
        const int n = (int)(q_starts[b + 1] - q_starts[b]);
        const int c = (int)ctx[b];
        const int first_q = c - n;
        int lo = 0;
        if (windowed) lo = first_q - m->cfg.window + 1 > 0 ? (first_q - m->cfg.window + 1) / YK_BLOCK_SIZE : 0;
        const int hi = (c + YK_BLOCK_SIZE - 1) / YK_BLOCK_SIZE;
        if (hi > max_blocks) ++g_violations;
        for (int p = lo; p < hi && p < max_blocks; ++p) {
            const int blk = tables[(size_t)b * max_blocks + p];
            ++g_pages_checked;
            if (blk < 0 || blk >= pool->num_blocks) {
                ++g_violations;
                continue;
            }
            auto it = owner.find(blk);
            if (it != owner.end() && it->second != b) ++g_violations;
            owner[blk] = b;
        }
    }
}
}  // namespace

extern "C" {

yk_model* stub_model(int n_layers, int window, int parity, int vocab) {
    auto* m = new yk_model();
    std::memset(&m->cfg, 0, sizeof(m->cfg));
    m->cfg.n_layers = n_layers;
    m->cfg.window = window;
    m->cfg.window_layer_parity = parity;
    m->cfg.vocab_size = vocab;
    m->cfg.max_seqs = 64;
    m->cfg.max_tokens = 1 << 20;
    return m;
}
void stub_model_free(yk_model* m) { delete m; }
yk_kv_pool* stub_pool(int num_blocks) { return new yk_kv_pool{num_blocks}; }
void stub_pool_free(yk_kv_pool* p) { delete p; }
yk_sampler* stub_sampler(int k, int V) { return new yk_sampler{k, V, {}}; }
void stub_sampler_free(yk_sampler* s) { delete s; }
void stub_stats(int64_t* violations, int64_t* forwards, int64_t* pages) {
    *violations = g_violations;
    *forwards = g_forwards;
    *pages = g_pages_checked;
}
void stub_reset() { g_violations = g_forwards = g_pages_checked = 0; }

yk_status yk_model_get_config(const yk_model* m, yk_model_config* out) {
    if (!m || !out) return YK_ERR_ARG;
    *out = m->cfg;
    return YK_OK;
}
int32_t yk_kv_pool_num_blocks(const yk_kv_pool* p) { return p ? p->num_blocks : 0; }

yk_status yk_forward_step(yk_model* m, yk_kv_pool* pool, const uint32_t* tokens, int32_t T, const uint32_t* q_starts,
                          const uint32_t* context_lens, int32_t B, const int32_t* block_tables, int32_t max_blocks,
                          int32_t last_n, int32_t* n_rows) {
    (void)tokens;
    if (q_starts[0] != 0 || (int)q_starts[B] != T) ++g_violations;
    check_tables(m, pool, q_starts, context_lens, B, block_tables, max_blocks);
    ++g_forwards;
    int rows = 0;
    for (int b = 0; b < B; ++b) {
        const int n = (int)(q_starts[b + 1] - q_starts[b]);
        rows += last_n > 0 ? (n < last_n ? n : last_n) : n;
    }
    if (n_rows) *n_rows = rows;
    return YK_OK;
}

yk_status yk_forward_step_drafts(yk_model* m, yk_kv_pool* pool, const uint32_t* tokens, int32_t T,
                                 const uint32_t* q_starts, const uint32_t* context_lens, int32_t B,
                                 const int32_t* block_tables, int32_t max_blocks, int32_t last_n, yk_sampler* s,
                                 int32_t j0, int32_t nd, int32_t* n_rows) {
    if (!s || j0 < 0 || nd < 0 || j0 + nd > s->k) ++g_violations;
    return yk_forward_step(m, pool, tokens, T, q_starts, context_lens, B, block_tables, max_blocks, last_n, n_rows);
}

yk_status yk_forward_step_split(yk_model* m, yk_kv_pool* pool, yk_kv_pool* wpool, const uint32_t* tokens, int32_t T,
                                const uint32_t* q_starts, const uint32_t* context_lens, int32_t B,
                                const int32_t* block_tables, int32_t max_blocks, const int32_t* wblock_tables,
                                int32_t wmax_blocks, int32_t last_n, yk_sampler* s, int32_t j0, int32_t nd,
                                int32_t* n_rows) {
    if (!wpool || m->cfg.window <= 0) ++g_violations;
    if (s && (j0 < 0 || nd < 0 || j0 + nd > s->k)) ++g_violations;
    check_tables(m, wpool, q_starts, context_lens, B, wblock_tables, wmax_blocks, true);
    return yk_forward_step(m, pool, tokens, T, q_starts, context_lens, B, block_tables, max_blocks, last_n, n_rows);
}

yk_status yk_draft_sample(yk_sampler* s, yk_model* draft, int32_t B, int32_t j, float temperature, uint64_t seed,
                          uint32_t step, const uint32_t* seq_ids, uint32_t* out_tokens) {
    (void)draft;
    (void)temperature;
    (void)seed;
    if ((int)s->drafts.size() < B * s->k) s->drafts.resize((size_t)B * s->k);
    for (int b = 0; b < B; ++b) {
        const uint32_t t = (seq_ids[b] * 31u + step * 7u + (uint32_t)j) % (uint32_t)s->V;
        s->drafts[(size_t)b * s->k + j] = t;
        if (out_tokens) out_tokens[b] = t;
    }
    return YK_OK;
}

yk_status yk_spec_verify(yk_sampler* s, yk_model* target, int32_t B, float temperature, uint64_t seed, uint32_t step,
                         const uint32_t* seq_ids, const uint32_t* draft_tokens, uint32_t* out_tokens,
                         int32_t* out_counts) {
    (void)target;
    (void)temperature;
    (void)seed;
    const int k = s->k;
    for (int b = 0; b < B; ++b) {
        const int a = (int)((seq_ids[b] + step) % (uint32_t)(k + 1));  // accepted drafts
        for (int i = 0; i < a; ++i)
            out_tokens[(size_t)b * (k + 1) + i] = draft_tokens ? draft_tokens[(size_t)b * k + i] : s->drafts[(size_t)b * k + i];
        out_tokens[(size_t)b * (k + 1) + a] = (seq_ids[b] + step * 13u + 5u) % (uint32_t)s->V;  // target's token
        out_counts[b] = a + 1;
    }
    return YK_OK;
}

}  // extern "C"
