// yk_stub.cpp -- TEST INFRASTRUCTURE ONLY.  A CPU stand-in for the libyk.so
// entry points that libyk_host.so's scheduler calls (yk_model_get_config,
// yk_kv_pool_num_blocks, yk_forward_step[_drafts|_split], yk_draft_sample,
// yk_spec_verify[_range], yk_sampler_read_drafts, yk_tp_allgather_u32),
// compiled together with host/yk_host.cpp into one test library, so that the
// scheduling logic -- admission, page tables, rollback, window reclamation,
// streaming, sequence-sharded drafting across emulated ranks -- runs without a GPU.
//
// The forward checks the page tables it is given: every page a query of the
// call may read (all of the context; from first_query - window + 1 on when
// every layer is windowed) must hold a block id inside the pool, and no block
// may be read by two sequences of one call.  Draft tokens and verification are
// deterministic functions of (sequence id, step, draft index).
#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <map>
#include <mutex>
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
// A tensor-parallel group emulated in one process: each rank's scheduler runs on
// its own thread, and the all-gather is a rendezvous of those threads.
struct StubGroup {
    std::mutex mu;
    std::condition_variable cv;
    int world = 1, arrived = 0, count = 0;
    uint64_t gen = 0;
    std::vector<uint32_t> slots[2];  // by generation parity: a slot is rewritten only after every rank read it
};
struct yk_engine {
    StubGroup* group;
    int rank;
};

namespace {
std::atomic<int64_t> g_violations{0}, g_forwards{0}, g_pages_checked{0};

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
StubGroup* stub_group(int world) {
    auto* g = new StubGroup();
    g->world = world;
    return g;
}
void stub_group_free(StubGroup* g) { delete g; }
yk_engine* stub_engine(StubGroup* g, int rank) { return new yk_engine{g, rank}; }
void stub_engine_free(yk_engine* e) { delete e; }

yk_status yk_tp_allgather_u32(yk_engine* e, const uint32_t* send, int32_t count, uint32_t* recv) {
    if (!e || !send || !recv || count <= 0) return YK_ERR_ARG;
    StubGroup& g = *e->group;
    std::unique_lock<std::mutex> lk(g.mu);
    const uint64_t my = g.gen;
    std::vector<uint32_t>& buf = g.slots[my & 1];
    if (g.arrived == 0) {
        buf.assign((size_t)count * g.world, 0u);
        g.count = count;
    }
    if (g.count != count) {
        ++g_violations;
        return YK_ERR_ARG;
    }
    std::memcpy(buf.data() + (size_t)e->rank * count, send, (size_t)count * 4);
    if (++g.arrived == g.world) {
        g.arrived = 0;
        ++g.gen;
        g.cv.notify_all();
    } else {
        g.cv.wait(lk, [&] { return g.gen != my; });
    }
    std::memcpy(recv, buf.data(), (size_t)count * g.world * 4);
    return YK_OK;
}

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

yk_status yk_sampler_read_drafts(yk_sampler* s, int32_t B, uint32_t* out) {
    if (!s || !out || B <= 0 || (int)s->drafts.size() < B * s->k) return YK_ERR_ARG;
    std::memcpy(out, s->drafts.data(), (size_t)B * s->k * 4);
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

yk_status yk_spec_verify_range(yk_sampler* s, yk_model* target, int32_t seq0, int32_t B, float temperature,
                               uint64_t seed, uint32_t step, const uint32_t* seq_ids, const uint32_t* draft_tokens,
                               uint32_t* out_tokens, int32_t* out_counts) {
    if (seq0 < 0 || !draft_tokens) ++g_violations;
    return yk_spec_verify(s, target, B, temperature, seed, step, seq_ids, draft_tokens, out_tokens, out_counts);
}

}  // extern "C"
