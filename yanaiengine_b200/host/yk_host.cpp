// yk_host.cpp -- host-side Scheduler / SequenceRequest / PagedKVCache /
// BlockAllocator (see include/yk_host.h), driving libyk.so through yk.h only.
#include "../../include/yk_host.h"

#include <algorithm>
#include <cstring>
#include <deque>
#include <memory>
#include <optional>
#include <set>
#include <string>
#include <vector>

#define YK_TRY(call)                   \
    do {                               \
        yk_status s_ = (call);         \
        if (s_ != YK_OK) return s_;    \
    } while (0)

namespace {

// BlockAllocator (S/BlockAllocator.swift:6-65): LIFO free list, block 0 first.
class BlockAllocator {
  public:
    explicit BlockAllocator(int num_blocks) : num_blocks_(num_blocks) { reset(); }
    std::optional<int> allocate() {
        if (free_.empty()) return std::nullopt;
        const int b = free_.back();
        free_.pop_back();
        allocated_.insert(b);
        return b;
    }
    void deallocate(int b) {
        if (allocated_.erase(b)) free_.push_back(b);
    }
    float usage() const { return (float)allocated_.size() / (float)num_blocks_; }
    void reset() {
        free_.clear();
        for (int i = num_blocks_ - 1; i >= 0; --i) free_.push_back(i);
        allocated_.clear();
    }
    int num_blocks() const { return num_blocks_; }

  private:
    int num_blocks_;
    std::vector<int> free_;
    std::set<int> allocated_;
};

// PagedKVCache (S/PagedKVCache.swift:6-90).  One page table per sequence and
// model covers every layer (the pool is [block][layer][K|V]...).
class PagedKVCache {
  public:
    explicit PagedKVCache(BlockAllocator* a) : alloc_(a) {}
    ~PagedKVCache() { reset(); }
    // Pages for positions < n (appendFromFull allocates at pos % 16 == 0, :29-35).
    // A cache whose first n tokens are already held (a cached prompt) under window
    // reclamation with width w: the pages wholly before the window of the next
    // query (position n) are never read, so they get no block (-1) at all.
    bool reserve_cached_window(int n, int w) {
        const int first_live = n - w + 1;
        const int need = (n + YK_BLOCK_SIZE - 1) / YK_BLOCK_SIZE;
        const int dead = first_live > 0 ? std::min(first_live / YK_BLOCK_SIZE, need) : 0;
        while ((int)page_table.size() < dead) page_table.push_back(-1);
        dead_pages = std::max(dead_pages, dead);
        return reserve(n);
    }
    bool reserve(int n) {
        const int need = (n + YK_BLOCK_SIZE - 1) / YK_BLOCK_SIZE;
        while ((int)page_table.size() < need) {
            auto b = alloc_->allocate();
            if (!b) return false;
            page_table.push_back(*b);
        }
        return true;
    }
    // rollback(to:) :65-76.
    void rollback(int position) {
        if (position > current_position) return;
        const int need = (position + YK_BLOCK_SIZE - 1) / YK_BLOCK_SIZE;
        while ((int)page_table.size() > need) {
            if (page_table.back() >= 0) alloc_->deallocate(page_table.back());
            page_table.pop_back();
        }
        dead_pages = std::min(dead_pages, (int)page_table.size());
        current_position = position;
    }
    void reset() {
        for (int b : page_table)
            if (b >= 0) alloc_->deallocate(b);
        page_table.clear();
        current_position = 0;
        dead_pages = 0;
    }
    // Sliding-window reclamation (every layer windowed, width w): a query at
    // position p >= current_position reads keys from p - w + 1 on, so the pages
    // wholly before current_position - w + 1 are never read again; they go back to
    // the allocator and their table entries become -1 (sent as block 0: the
    // attention's key range starts past them).  The reference never frees them
    // (S/PagedKVCache.swift:65-85).
    void reclaim_window(int w) {
        const int first_live = current_position - w + 1;
        const int dead = first_live > 0 ? std::min<int>(first_live / YK_BLOCK_SIZE, (int)page_table.size()) : 0;
        for (; dead_pages < dead; ++dead_pages) {
            if (page_table[dead_pages] >= 0) alloc_->deallocate(page_table[dead_pages]);
            page_table[dead_pages] = -1;
        }
    }
    int dead_pages = 0;
    std::vector<int> page_table;
    int current_position = 0;

  private:
    BlockAllocator* alloc_;
};

// SequenceRequest (S/Scheduler.swift:5-80).
struct SequenceRequest {
    uint32_t id = 0;
    std::vector<uint32_t> prompt, generated;
    std::unique_ptr<PagedKVCache> cache, draft_cache;
    // split pools: the windowed layers' page tables (same positions as cache /
    // draft_cache), else null
    std::unique_ptr<PagedKVCache> wcache, draft_wcache;
    int max_tokens = 0;
    int64_t stop_token = -1;
    // a cached prompt under sharded drafting: the draft cache of whichever rank
    // drafts this sequence first takes these tokens as held (its pages reserved then)
    int draft_cached = 0;
    bool finished = false;
    // streaming (the server's onTokenGenerated / onCompletion), optional
    ykh_on_tokens on_tokens = nullptr;
    ykh_on_done on_done = nullptr;
    void* user = nullptr;
    int total() const { return (int)(prompt.size() + generated.size()); }
    uint32_t at(int i) const { return i < (int)prompt.size() ? prompt[i] : generated[i - prompt.size()]; }
};

}  // namespace

struct ykh_scheduler {
    yk_model* target = nullptr;
    yk_model* draft = nullptr;
    yk_kv_pool* tpool = nullptr;
    yk_kv_pool* dpool = nullptr;
    yk_sampler* sampler = nullptr;
    int k = 4;
    float temperature = 1.0f;
    uint64_t seed = 0;
    uint32_t step_no = 0;
    std::unique_ptr<BlockAllocator> talloc, dalloc;
    // split pools (ykh_scheduler_create_split): windowed-layer pools and allocators
    yk_kv_pool* twpool = nullptr;
    yk_kv_pool* dwpool = nullptr;
    std::unique_ptr<BlockAllocator> twalloc, dwalloc;
    int tw_width = 0, dw_width = 0;  // their window widths
    std::deque<std::unique_ptr<SequenceRequest>> waiting;
    std::vector<std::unique_ptr<SequenceRequest>> running, done;
    int64_t n_steps = 0, n_emitted = 0, n_accepted = 0;
    // sliding-window reclamation: window width of a model whose every layer is
    // windowed (0: some layer is global, nothing can be freed)
    int t_window = 0, d_window = 0;
    bool reclaim = true;
    // sequence-sharded drafting (ykh_set_draft_shard): this rank drafts and
    // verifies running sequences [B*shard_rank/shard_world, B*(shard_rank+1)/shard_world)
    yk_engine* shard_engine = nullptr;
    int shard_rank = 0, shard_world = 1;
    std::vector<uint32_t> gather_send, gather_recv;
    // per-step scratch
    std::vector<uint32_t> tokens, qstarts, ctx, seq_ids, drafts, out_tokens;
    std::vector<int32_t> tables, wtables, counts;
};

extern "C" yk_status ykh_scheduler_create(yk_model* target, yk_kv_pool* tpool, yk_model* draft, yk_kv_pool* dpool,
                                          yk_sampler* sampler, int32_t k, float temperature, uint64_t seed,
                                          ykh_scheduler** out) {
    if (!target || !tpool || !draft || !dpool || !sampler || !out || k <= 0) return YK_ERR_ARG;
    auto* s = new ykh_scheduler();
    s->target = target;
    s->draft = draft;
    s->tpool = tpool;
    s->dpool = dpool;
    s->sampler = sampler;
    s->k = k;
    s->temperature = temperature;
    s->seed = seed;
    s->talloc = std::make_unique<BlockAllocator>(yk_kv_pool_num_blocks(tpool));
    s->dalloc = std::make_unique<BlockAllocator>(yk_kv_pool_num_blocks(dpool));
    yk_model_config tc{}, dc{};
    if (yk_model_get_config(target, &tc) != YK_OK || yk_model_get_config(draft, &dc) != YK_OK) {
        delete s;
        return YK_ERR_ARG;
    }
    s->t_window = tc.window > 0 && tc.window_layer_parity < 0 ? tc.window : 0;
    s->d_window = dc.window > 0 && dc.window_layer_parity < 0 ? dc.window : 0;
    *out = s;
    return YK_OK;
}

extern "C" yk_status ykh_scheduler_create_split(yk_model* target, yk_kv_pool* target_pool, yk_kv_pool* target_wpool,
                                                yk_model* draft, yk_kv_pool* draft_pool, yk_kv_pool* draft_wpool,
                                                yk_sampler* sampler, int32_t k, float temperature, uint64_t seed,
                                                ykh_scheduler** out) {
    if (!target_wpool || !draft_wpool || !out) return YK_ERR_ARG;
    YK_TRY(ykh_scheduler_create(target, target_pool, draft, draft_pool, sampler, k, temperature, seed, out));
    ykh_scheduler* s = *out;
    yk_model_config tc{}, dc{};
    if (yk_model_get_config(target, &tc) != YK_OK || yk_model_get_config(draft, &dc) != YK_OK || tc.window <= 0 ||
        dc.window <= 0) {
        ykh_scheduler_destroy(s);
        *out = nullptr;
        return YK_ERR_ARG;
    }
    s->twpool = target_wpool;
    s->dwpool = draft_wpool;
    s->twalloc = std::make_unique<BlockAllocator>(yk_kv_pool_num_blocks(target_wpool));
    s->dwalloc = std::make_unique<BlockAllocator>(yk_kv_pool_num_blocks(draft_wpool));
    s->tw_width = tc.window;
    s->dw_width = dc.window;
    return YK_OK;
}

extern "C" void ykh_scheduler_destroy(ykh_scheduler* s) {
    if (!s) return;
    s->waiting.clear();
    s->running.clear();
    s->done.clear();
    delete s;
}

static yk_status submit(ykh_scheduler* s, const uint32_t* prompt, int32_t n, int32_t max_tokens, int64_t stop,
                        uint32_t seq_id, bool cached, ykh_on_tokens on_tokens = nullptr,
                        ykh_on_done on_done = nullptr, void* user = nullptr) {
    if (!s || !prompt || n <= 0) return YK_ERR_ARG;
    auto r = std::make_unique<SequenceRequest>();
    r->id = seq_id;
    r->on_tokens = on_tokens;
    r->on_done = on_done;
    r->user = user;
    r->prompt.assign(prompt, prompt + n);
    r->max_tokens = max_tokens;
    r->stop_token = stop;
    r->cache = std::make_unique<PagedKVCache>(s->talloc.get());
    r->draft_cache = std::make_unique<PagedKVCache>(s->dalloc.get());
    if (s->twpool) {
        r->wcache = std::make_unique<PagedKVCache>(s->twalloc.get());
        r->draft_wcache = std::make_unique<PagedKVCache>(s->dwalloc.get());
    }
    if (cached && s->shard_world > 1) {
        // sharded drafting: the draft side is reserved by the rank whose slice the
        // sequence lands in, at its first step (the draft pools hold one slice each)
        if (!r->cache->reserve(n - 1)) return YK_ERR_OOM;
        r->cache->current_position = n - 1;
        r->draft_cached = n - 1;
        if (r->wcache) {
            if (!(s->reclaim ? r->wcache->reserve_cached_window(n - 1, s->tw_width) : r->wcache->reserve(n - 1)))
                return YK_ERR_OOM;
            r->wcache->current_position = n - 1;
        }
        s->running.push_back(std::move(r));
    } else if (cached) {
        if (!r->cache->reserve(n - 1) || !r->draft_cache->reserve(n - 1)) return YK_ERR_OOM;
        r->cache->current_position = n - 1;
        r->draft_cache->current_position = n - 1;
        if (r->wcache) {
            // the windowed pools hold only the pages inside the window (with reclamation on)
            const bool rw = s->reclaim;
            if (!(rw ? r->wcache->reserve_cached_window(n - 1, s->tw_width) : r->wcache->reserve(n - 1)) ||
                !(rw ? r->draft_wcache->reserve_cached_window(n - 1, s->dw_width) : r->draft_wcache->reserve(n - 1)))
                return YK_ERR_OOM;
            r->wcache->current_position = n - 1;
            r->draft_wcache->current_position = n - 1;
        }
        s->running.push_back(std::move(r));
    } else {
        s->waiting.push_back(std::move(r));
    }
    return YK_OK;
}

extern "C" yk_status ykh_submit(ykh_scheduler* s, const uint32_t* prompt, int32_t n, int32_t max_tokens,
                                int64_t stop_token, uint32_t seq_id) {
    return submit(s, prompt, n, max_tokens, stop_token, seq_id, false);
}
extern "C" yk_status ykh_submit_stream(ykh_scheduler* s, const uint32_t* prompt, int32_t n, int32_t max_tokens,
                                       int64_t stop_token, uint32_t seq_id, ykh_on_tokens on_tokens,
                                       ykh_on_done on_done, void* user) {
    return submit(s, prompt, n, max_tokens, stop_token, seq_id, false, on_tokens, on_done, user);
}
extern "C" yk_status ykh_submit_cached(ykh_scheduler* s, const uint32_t* prompt, int32_t n, int32_t max_tokens,
                                       int64_t stop_token, uint32_t seq_id) {
    return submit(s, prompt, n, max_tokens, stop_token, seq_id, true);
}

// Builds the ragged batch for one forward over the running sequences `idx`
// (all of them when empty): for each the token list `inputs[i]`, starting at
// cache position `start`; reserves pages.  nd > 0: the last nd inputs of every
// sequence are placeholders for the draft tokens j0.. that the sampler keeps on
// the device (no host round trip).
static yk_status forward(ykh_scheduler* s, bool is_draft, const std::vector<std::vector<uint32_t>>& inputs,
                         int last_n, int j0 = 0, int nd = 0, const std::vector<int>& idx = {}) {
    const int B = idx.empty() ? (int)s->running.size() : (int)idx.size();
    auto req = [&](int b) { return s->running[idx.empty() ? b : idx[b]].get(); };
    s->tokens.clear();
    s->qstarts.assign(1, 0);
    s->ctx.clear();
    size_t max_pages = 1;
    const bool split = s->twpool != nullptr;
    size_t wmax_pages = 1;
    for (int b = 0; b < B; ++b) {
        PagedKVCache* c = is_draft ? req(b)->draft_cache.get() : req(b)->cache.get();
        const int n = (int)inputs[b].size();
        if (!c->reserve(c->current_position + n)) return YK_ERR_OOM;  // S/PagedKVCache.swift:31-33
        if (split) {
            PagedKVCache* wc = is_draft ? req(b)->draft_wcache.get() : req(b)->wcache.get();
            if (!wc->reserve(wc->current_position + n)) return YK_ERR_OOM;
            wmax_pages = std::max(wmax_pages, wc->page_table.size());
        }
        s->tokens.insert(s->tokens.end(), inputs[b].begin(), inputs[b].end());
        s->qstarts.push_back((uint32_t)s->tokens.size());
        s->ctx.push_back((uint32_t)(c->current_position + n));
        max_pages = std::max(max_pages, c->page_table.size());
    }
    s->tables.assign((size_t)B * max_pages, 0);
    for (int b = 0; b < B; ++b) {
        PagedKVCache* c = is_draft ? req(b)->draft_cache.get() : req(b)->cache.get();
        int32_t* row = s->tables.data() + (size_t)b * max_pages;
        for (size_t i = 0; i < c->page_table.size(); ++i) row[i] = c->page_table[i] >= 0 ? c->page_table[i] : 0;
    }
    int32_t rows = 0;
    yk_model* m = is_draft ? s->draft : s->target;
    yk_kv_pool* pool = is_draft ? s->dpool : s->tpool;
    if (split) {
        s->wtables.assign((size_t)B * wmax_pages, 0);
        for (int b = 0; b < B; ++b) {
            PagedKVCache* wc = is_draft ? req(b)->draft_wcache.get() : req(b)->wcache.get();
            int32_t* row = s->wtables.data() + (size_t)b * wmax_pages;
            for (size_t i = 0; i < wc->page_table.size(); ++i) row[i] = wc->page_table[i] >= 0 ? wc->page_table[i] : 0;
        }
        YK_TRY(yk_forward_step_split(m, pool, is_draft ? s->dwpool : s->twpool, s->tokens.data(),
                                     (int32_t)s->tokens.size(), s->qstarts.data(), s->ctx.data(), B, s->tables.data(),
                                     (int32_t)max_pages, s->wtables.data(), (int32_t)wmax_pages, last_n,
                                     nd > 0 ? s->sampler : nullptr, j0, nd, &rows));
        for (int b = 0; b < B; ++b) {
            SequenceRequest* r = req(b);
            (is_draft ? r->draft_cache : r->cache)->current_position += (int)inputs[b].size();
            (is_draft ? r->draft_wcache : r->wcache)->current_position += (int)inputs[b].size();
        }
        return YK_OK;
    }
    yk_status st = nd > 0 ? yk_forward_step_drafts(m, pool, s->tokens.data(), (int32_t)s->tokens.size(),
                                                   s->qstarts.data(), s->ctx.data(), B, s->tables.data(),
                                                   (int32_t)max_pages, last_n, s->sampler, j0, nd, &rows)
                          : yk_forward_step(m, pool, s->tokens.data(), (int32_t)s->tokens.size(), s->qstarts.data(),
                                            s->ctx.data(), B, s->tables.data(), (int32_t)max_pages, last_n, &rows);
    if (st != YK_OK) return st;
    for (int b = 0; b < B; ++b) {
        PagedKVCache* c = is_draft ? req(b)->draft_cache.get() : req(b)->cache.get();
        c->current_position += (int)inputs[b].size();
    }
    return YK_OK;
}

// Scheduler.step, speculative branch (S/Scheduler.swift:161-267).
extern "C" yk_status ykh_step(ykh_scheduler* s, int32_t* emitted_out) {
    if (!s) return YK_ERR_ARG;
    if (emitted_out) *emitted_out = 0;
    // Admission (runLoop :122-129): move waiting requests while usage < 0.9.
    yk_model_config tc{}, dc{};
    YK_TRY(yk_model_get_config(s->target, &tc));
    YK_TRY(yk_model_get_config(s->draft, &dc));
    const int max_batch = std::min(tc.max_seqs, dc.max_seqs);
    // (sharded drafting: the draft pools hold different slices on different ranks,
    // so admission looks at the target pools only, which every rank fills alike)
    const bool dfull = s->shard_world == 1 && (s->dalloc->usage() >= 0.9f || (s->dwalloc && s->dwalloc->usage() >= 0.9f));
    while (!s->waiting.empty() && s->talloc->usage() < 0.9f && !dfull &&
           (!s->twalloc || s->twalloc->usage() < 0.9f) && (int)s->running.size() < max_batch) {
        s->running.push_back(std::move(s->waiting.front()));
        s->waiting.pop_front();
    }
    if (s->running.empty()) return YK_OK;
    const int B = (int)s->running.size();
    const int k = s->k;
    s->seq_ids.resize(B);
    std::vector<int> N(B);
    for (int b = 0; b < B; ++b) {
        s->seq_ids[b] = s->running[b]->id;
        N[b] = s->running[b]->total();
    }
    const bool sharded = s->shard_world > 1;
    // this rank's slice of the batch (all of it unless drafting is sharded)
    const int lo = sharded ? (int)((int64_t)B * s->shard_rank / s->shard_world) : 0;
    const int hi = sharded ? (int)((int64_t)B * (s->shard_rank + 1) / s->shard_world) : B;
    const int Bs = hi - lo;
    std::vector<int> own;
    if (sharded) {
        for (int b = lo; b < hi; ++b) own.push_back(b);
        // a sequence outside this rank's slice keeps no draft pages here (slices
        // move when sequences finish; a sequence that moves in is re-fed to the draft)
        for (int b = 0; b < B; ++b)
            if (b < lo || b >= hi) {
                s->running[b]->draft_cache->reset();
                if (s->running[b]->draft_wcache) s->running[b]->draft_wcache->reset();
            }
    }
    std::vector<uint32_t> own_ids(s->seq_ids.begin() + lo, s->seq_ids.begin() + hi);
    if (sharded)
        for (int b = lo; b < hi; ++b) {  // cached prompts reach this rank's draft cache at their first step
            SequenceRequest* r = s->running[b].get();
            if (r->draft_cached > 0 && r->generated.empty() && r->draft_cache->current_position == 0) {
                const int n = r->draft_cached;
                if (!r->draft_cache->reserve(n)) return YK_ERR_OOM;
                r->draft_cache->current_position = n;
                if (r->draft_wcache) {
                    if (!(s->reclaim ? r->draft_wcache->reserve_cached_window(n, s->dw_width)
                                     : r->draft_wcache->reserve(n)))
                        return YK_ERR_OOM;
                    r->draft_wcache->current_position = n;
                }
            }
            r->draft_cached = 0;
        }
    // 1. DRAFT PHASE (:171-190): k draft forwards, sampling after each.  The drafted
    // tokens stay on the device (the sampler keeps them; the next draft forward and
    // the target forward read them there), so the whole phase is queued without
    // waiting for the device.
    std::vector<std::vector<uint32_t>> inputs(Bs);
    for (int j = 0; j < k && Bs > 0; ++j) {
        for (int i = 0; i < Bs; ++i) {
            SequenceRequest* r = s->running[lo + i].get();
            inputs[i].clear();
            if (j == 0) {
                // every token the draft cache has not seen (the prompt on the first step)
                for (int t = r->draft_cache->current_position; t < N[lo + i]; ++t) inputs[i].push_back(r->at(t));
            } else {
                inputs[i].push_back(0u);  // draft j-1 of this sequence, on the device
            }
        }
        if (j == 0) YK_TRY(forward(s, true, inputs, 1, 0, 0, own));
        else YK_TRY(forward(s, true, inputs, 1, j - 1, 1, own));
        YK_TRY(yk_draft_sample(s->sampler, s->draft, Bs, j, s->temperature, s->seed, s->step_no, own_ids.data(),
                               nullptr));
    }
    // Sharded: every rank's drafts, for the target forward over the whole batch.
    std::vector<uint32_t> all_drafts;
    const int Bm = sharded ? (B + s->shard_world - 1) / s->shard_world : 0;  // largest slice
    auto owner_of = [&](int b) {  // rank whose slice holds running sequence b, and b's row there
        int q = (int)(((int64_t)b * s->shard_world) / B);
        while ((int64_t)B * (q + 1) / s->shard_world <= b) ++q;
        while ((int64_t)B * q / s->shard_world > b) --q;
        return q;
    };
    if (sharded) {
        s->gather_send.assign((size_t)Bm * k, 0u);
        if (Bs > 0) YK_TRY(yk_sampler_read_drafts(s->sampler, Bs, s->gather_send.data()));
        s->gather_recv.assign((size_t)Bm * k * s->shard_world, 0u);
        YK_TRY(yk_tp_allgather_u32(s->shard_engine, s->gather_send.data(), Bm * k, s->gather_recv.data()));
        all_drafts.resize((size_t)B * k);
        for (int b = 0; b < B; ++b) {
            const int q = owner_of(b);
            const int row = b - (int)((int64_t)B * q / s->shard_world);
            for (int j = 0; j < k; ++j)
                all_drafts[(size_t)b * k + j] = s->gather_recv[((size_t)q * Bm + row) * k + j];
        }
    }
    // 2-3. VERIFICATION SETUP + TARGET FORWARD (:192-210): unseen tokens + drafts.
    std::vector<std::vector<uint32_t>> tinputs(B);
    for (int b = 0; b < B; ++b) {
        SequenceRequest* r = s->running[b].get();
        for (int i = r->cache->current_position; i < N[b]; ++i) tinputs[b].push_back(r->at(i));
        for (int j = 0; j < k; ++j)  // the k drafts: on the device, or (sharded) gathered on the host
            tinputs[b].push_back(sharded ? all_drafts[(size_t)b * k + j] : 0u);
    }
    if (sharded) YK_TRY(forward(s, false, tinputs, k + 1));
    else YK_TRY(forward(s, false, tinputs, k + 1, 0, k));
    // 4. VERIFICATION & ROLLBACK (:212-267).
    s->out_tokens.assign((size_t)B * (k + 1), 0);
    s->counts.assign(B, 0);
    if (!sharded) {
        YK_TRY(yk_spec_verify(s->sampler, s->target, B, s->temperature, s->seed, s->step_no, s->seq_ids.data(),
                              nullptr, s->out_tokens.data(), s->counts.data()));
    } else {
        // verify this rank's slice, then every rank's results to every rank
        const int W = k + 2;  // per sequence: k+1 tokens, then the count
        s->gather_send.assign((size_t)Bm * W, 0u);
        if (Bs > 0) {
            std::vector<uint32_t> out((size_t)Bs * (k + 1));
            std::vector<int32_t> cnt(Bs);
            YK_TRY(yk_spec_verify_range(s->sampler, s->target, lo, Bs, s->temperature, s->seed, s->step_no,
                                        own_ids.data(), all_drafts.data() + (size_t)lo * k, out.data(), cnt.data()));
            for (int i = 0; i < Bs; ++i) {
                std::memcpy(&s->gather_send[(size_t)i * W], &out[(size_t)i * (k + 1)], (size_t)(k + 1) * 4);
                s->gather_send[(size_t)i * W + k + 1] = (uint32_t)cnt[i];
            }
        }
        s->gather_recv.assign((size_t)Bm * W * s->shard_world, 0u);
        YK_TRY(yk_tp_allgather_u32(s->shard_engine, s->gather_send.data(), Bm * W, s->gather_recv.data()));
        for (int b = 0; b < B; ++b) {
            const int q = owner_of(b);
            const int row = b - (int)((int64_t)B * q / s->shard_world);
            const uint32_t* src = &s->gather_recv[((size_t)q * Bm + row) * W];
            std::memcpy(&s->out_tokens[(size_t)b * (k + 1)], src, (size_t)(k + 1) * 4);
            s->counts[b] = (int32_t)src[k + 1];
            if (s->counts[b] < 1 || s->counts[b] > k + 1) return YK_ERR_DEVICE_CHECK;
        }
    }
    int emitted = 0;
    for (int b = 0; b < B; ++b) {
        SequenceRequest* r = s->running[b].get();
        const int cnt = s->counts[b];
        const int a = cnt - 1;  // accepted drafts
        const bool drafted_here = b >= lo && b < hi;  // (its draft cache lives on this rank)
        r->cache->rollback(N[b] + a);
        if (drafted_here) r->draft_cache->rollback(std::min(r->draft_cache->current_position, N[b] + a));
        if (r->wcache) {
            r->wcache->rollback(N[b] + a);
            if (drafted_here) r->draft_wcache->rollback(std::min(r->draft_wcache->current_position, N[b] + a));
            if (s->reclaim) {  // every layer of these pools is windowed
                r->wcache->reclaim_window(s->tw_width);
                if (drafted_here) r->draft_wcache->reclaim_window(s->dw_width);
            }
        }
        for (int i = 0; i < cnt; ++i) r->generated.push_back(s->out_tokens[(size_t)b * (k + 1) + i]);
        for (int i = 0; i < cnt; ++i)
            if (r->stop_token >= 0 && s->out_tokens[(size_t)b * (k + 1) + i] == (uint32_t)r->stop_token) {
                r->finished = true;
                break;
            }
        if ((int)r->generated.size() >= r->max_tokens) r->finished = true;
        if (s->reclaim && s->t_window > 0) r->cache->reclaim_window(s->t_window);
        if (s->reclaim && s->d_window > 0 && drafted_here) r->draft_cache->reclaim_window(s->d_window);
        if (r->on_tokens && cnt > 0) r->on_tokens(r->user, r->id, r->generated.data() + r->generated.size() - cnt, cnt);
        emitted += cnt;
        s->n_accepted += a;
    }
    s->n_emitted += emitted;
    s->n_steps++;
    s->step_no++;
    // Cleanup (:141-148): finished requests release their pages.
    for (auto it = s->running.begin(); it != s->running.end();) {
        if ((*it)->finished) {
            (*it)->cache->reset();
            (*it)->draft_cache->reset();
            if ((*it)->wcache) {
                (*it)->wcache->reset();
                (*it)->draft_wcache->reset();
            }
            if ((*it)->on_done) (*it)->on_done((*it)->user, (*it)->id, (int32_t)(*it)->generated.size());
            s->done.push_back(std::move(*it));
            it = s->running.erase(it);
        } else {
            ++it;
        }
    }
    if (emitted_out) *emitted_out = emitted;
    return YK_OK;
}

extern "C" yk_status ykh_set_draft_shard(ykh_scheduler* s, yk_engine* e, int32_t rank, int32_t world) {
    if (!s || world < 1 || rank < 0 || rank >= world || (world > 1 && !e)) return YK_ERR_ARG;
    s->shard_engine = world > 1 ? e : nullptr;
    s->shard_rank = world > 1 ? rank : 0;
    s->shard_world = world;
    return YK_OK;
}

extern "C" yk_status ykh_set_window_reclaim(ykh_scheduler* s, int32_t on) {
    if (!s) return YK_ERR_ARG;
    s->reclaim = on != 0;
    return YK_OK;
}

extern "C" int32_t ykh_num_running(const ykh_scheduler* s) { return s ? (int32_t)s->running.size() : 0; }
extern "C" int32_t ykh_num_waiting(const ykh_scheduler* s) { return s ? (int32_t)s->waiting.size() : 0; }

extern "C" yk_status ykh_generated(const ykh_scheduler* s, uint32_t seq_id, uint32_t* out, int32_t cap, int32_t* n) {
    if (!s || !n) return YK_ERR_ARG;
    auto find = [&](const std::vector<std::unique_ptr<SequenceRequest>>& v) -> const SequenceRequest* {
        for (auto& r : v)
            if (r->id == seq_id) return r.get();
        return nullptr;
    };
    const SequenceRequest* r = find(s->running);
    if (!r) r = find(s->done);
    if (!r)
        for (auto& w : s->waiting)
            if (w->id == seq_id) r = w.get();
    if (!r) return YK_ERR_ARG;
    *n = (int32_t)r->generated.size();
    if (out) std::memcpy(out, r->generated.data(), sizeof(uint32_t) * std::min<size_t>(cap, r->generated.size()));
    return YK_OK;
}

extern "C" yk_status ykh_counters(const ykh_scheduler* s, int64_t* steps, int64_t* emitted, int64_t* accepted) {
    if (!s) return YK_ERR_ARG;
    if (steps) *steps = s->n_steps;
    if (emitted) *emitted = s->n_emitted;
    if (accepted) *accepted = s->n_accepted;
    return YK_OK;
}

extern "C" float ykh_usage_windowed(const ykh_scheduler* s, int32_t draft) {
    if (!s || !s->twalloc) return 0.f;
    return draft ? s->dwalloc->usage() : s->twalloc->usage();
}

extern "C" float ykh_usage(const ykh_scheduler* s, int32_t draft) {
    if (!s) return 0.f;
    return draft ? s->dalloc->usage() : s->talloc->usage();
}
