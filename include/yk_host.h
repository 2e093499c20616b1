/*
 * yk_host.h -- C++ restatement of the reference's host side of the path, the
 * caller of yk.h: Scheduler's speculative step (S/Scheduler.swift:155-268),
 * SequenceRequest (S/Scheduler.swift:5-80), PagedKVCache page tables
 * (S/PagedKVCache.swift) and the 16-token BlockAllocator free list
 * (S/BlockAllocator.swift).  In a Swift deployment those classes stay Swift
 * and call yk.h directly; this library exists because no Swift toolchain is
 * available to build them here, and it is what the tests and the benchmark
 * drive end to end (libyk_host.so).
 *
 * Cache-position accounting follows the standard speculative invariant (each
 * cache holds every token of the sequence except the last emitted one) rather
 * than the reference's context-length and rollback arithmetic
 * (S/LlamaModel.swift:149, S/Scheduler.swift:242), which double-count the
 * prompt on the first step and drop one cached token per step.
 */
#pragma once
#include <stdint.h>

#include "yk.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ykh_scheduler ykh_scheduler;

/* One scheduler per GPU: a target and a draft model, each with its own KV pool
 * and BlockAllocator (S/Scheduler.swift:96-102; draft allocator from
 * S/Scheduler.swift:172).  k = draft tokens per step (gamma, :162). */
yk_status ykh_scheduler_create(yk_model* target, yk_kv_pool* target_pool, yk_model* draft, yk_kv_pool* draft_pool,
                               yk_sampler* sampler, int32_t k, float temperature, uint64_t seed,
                               ykh_scheduler** out);
/* The same over split pools (a model with windowed and global layers, e.g.
 * Gemma's alternating schedule): target_pool / draft_pool hold the global layers
 * (YK_POOL_GLOBAL_LAYERS), target_wpool / draft_wpool the windowed ones
 * (YK_POOL_WINDOWED_LAYERS), each with its own BlockAllocator and page tables;
 * with window reclamation on, each step frees the windowed pools' pages wholly
 * before the window.  Both models must have windowed layers. */
yk_status ykh_scheduler_create_split(yk_model* target, yk_kv_pool* target_pool, yk_kv_pool* target_wpool,
                                     yk_model* draft, yk_kv_pool* draft_pool, yk_kv_pool* draft_wpool,
                                     yk_sampler* sampler, int32_t k, float temperature, uint64_t seed,
                                     ykh_scheduler** out);
void ykh_scheduler_destroy(ykh_scheduler* s);

/* Scheduler.submit (S/Scheduler.swift:105).  stop_token < 0: none.  seq_id is
 * the Philox stream id of the request. */
yk_status ykh_submit(ykh_scheduler* s, const uint32_t* prompt, int32_t n, int32_t max_tokens, int64_t stop_token,
                     uint32_t seq_id);
/* Like ykh_submit, but the first n-1 prompt tokens are treated as already in
 * both KV caches (their pages are allocated; the pool holds whatever it holds,
 * e.g. yk_kv_pool_fill_random).  Used for steady-state benchmarks that exclude
 * prefill. */
yk_status ykh_submit_cached(ykh_scheduler* s, const uint32_t* prompt, int32_t n, int32_t max_tokens,
                            int64_t stop_token, uint32_t seq_id);
/* Streaming submission: the InferenceServer's per-request callbacks
 * (onTokenGenerated / onCompletion, S/InferenceServer.swift:118-126,167-176) at
 * the token-id level (detokenisation stays with the server).  on_tokens gets
 * each step's emitted run of the request (accepted drafts + the target's
 * token), in order; on_done is called once, when the request finishes (stop
 * token or max_tokens), with its generated-token count.  Both run inside
 * ykh_step on the calling thread, after the step's verification; either may be
 * null.  The concatenated runs equal ykh_generated's list. */
typedef void (*ykh_on_tokens)(void* user, uint32_t seq_id, const uint32_t* tokens, int32_t n);
typedef void (*ykh_on_done)(void* user, uint32_t seq_id, int32_t n_generated);
yk_status ykh_submit_stream(ykh_scheduler* s, const uint32_t* prompt, int32_t n, int32_t max_tokens,
                            int64_t stop_token, uint32_t seq_id, ykh_on_tokens on_tokens, ykh_on_done on_done,
                            void* user);
/* One speculative step over the running batch (admission as runLoop,
 * S/Scheduler.swift:122-129).  *emitted = tokens appended across the batch. */
yk_status ykh_step(ykh_scheduler* s, int32_t* emitted);
int32_t   ykh_num_running(const ykh_scheduler* s);
int32_t   ykh_num_waiting(const ykh_scheduler* s);
/* Generated tokens of request seq_id (prompt excluded); *n = total count. */
yk_status ykh_generated(const ykh_scheduler* s, uint32_t seq_id, uint32_t* out, int32_t cap, int32_t* n);
/* Counters since creation: steps, emitted tokens, accepted draft tokens. */
yk_status ykh_counters(const ykh_scheduler* s, int64_t* steps, int64_t* emitted, int64_t* accepted);
/* Sliding-window block reclamation (on by default).  For a model whose every
 * layer is windowed (window > 0, window_layer_parity < 0), each step returns
 * the pages wholly before current_position - window + 1 to the allocator: no
 * later query reads them.  The reference never frees them
 * (S/PagedKVCache.swift:65-85).  A model with a global layer frees nothing
 * (one page holds every layer's K/V). */
yk_status ykh_set_window_reclaim(ykh_scheduler* s, int32_t on);
/* Sequence-sharded drafting for a tensor-parallel target (the draft model is
 * replicated on every rank): every rank runs the same scheduler over the whole
 * batch, but drafts only its slice (running sequences [B*rank/world,
 * B*(rank+1)/world)) with its own draft pool and sampler rows, all-gathers the
 * drafted tokens for the target's verify forward (which every rank runs over the
 * whole batch), verifies its slice (yk_spec_verify_range) and all-gathers the
 * results, so every rank updates every sequence identically.  `e` is the
 * engine of the tensor-parallel group (yk_tp_allgather_u32); world = 1 turns it
 * off.  The draft pool only needs room for one slice. */
yk_status ykh_set_draft_shard(ykh_scheduler* s, yk_engine* e, int32_t rank, int32_t world);
/* BlockAllocator.usage of the target / draft pools (S/BlockAllocator.swift:56-58). */
float     ykh_usage(const ykh_scheduler* s, int32_t draft);
/* Usage of the windowed-layer pools of a split scheduler (0 otherwise). */
float     ykh_usage_windowed(const ykh_scheduler* s, int32_t draft);

#ifdef __cplusplus
}
#endif
