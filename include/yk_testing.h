/*
 * yk_testing.h -- test hooks of libyk.so.  Not part of the reference-facing
 * boundary (no reference counterpart): they run one internal kernel in
 * isolation so GPU tests can localise a failure and time a kernel alone.
 */
#pragma once
#include <stdint.h>

#include "yk.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Y[m_tok x n_out] (fp32, host) = X[m_tok x K] * W[n_out x K]^T through the
 * tcgen05 GEMM; W and X are host bf16 bit patterns.  grid: 0 = the production
 * heuristic; > 0 = stream-K over that many persistent CTAs (moves where tiles
 * are cut); < 0 = cluster split-K with -grid CTAs per tile. */
yk_status ykt_gemm_bf16(yk_engine* e, const uint16_t* W, const uint16_t* X, int32_t n_out, int32_t K, int32_t m_tok,
                        int32_t grid, float* Y);
/* Same, then `reps` back-to-back launches timed with CUDA events
 * (*ms_per_rep).  reps < 0: -reps launches, each after a 256 MB write that
 * evicts the weights from L2, timed one by one (mean of the single-launch
 * times: the cold-weight case of a forward step).  stamps (grid x 8, may be
 * null) receives the last launch's
 * per-CTA %globaltimer phase stamps: start, first TMA issued, first stage
 * landed, last MMA issued, last accumulator ready, epilogue done, segments,
 * cluster barrier passed (cluster split-K). */
yk_status ykt_gemm_bf16_timed(yk_engine* e, const uint16_t* W, const uint16_t* X, int32_t n_out, int32_t K,
                              int32_t m_tok, int32_t grid, int32_t reps, float* Y, float* ms_per_rep,
                              uint64_t* stamps, int32_t* grid_used);

/* Same timing with a fused epilogue: epi 0 store, 1 QKV (RoPE, K/V to a pool
 * page per token, head_dim / kv_dim give the split of n_out), 2 residual add,
 * 3 gate/up activation, 4 logits; outputs go to scratch buffers.  reps < 0:
 * one launch per L2 flush as above. */
yk_status ykt_gemm_bf16_epi_timed(yk_engine* e, const uint16_t* W, const uint16_t* X, int32_t n_out, int32_t K,
                                  int32_t m_tok, int32_t grid, int32_t reps, int32_t epi, int32_t head_dim,
                                  int32_t kv_dim, float* ms_per_rep, uint64_t* stamps, int32_t* grid_used);

/* Per-CTA phase stamps of the paged-attention kernel.  After enable (cap CTAs,
 * cap > 0; 0 disables), every bf16 attention launch of `m` overwrites a device
 * record of 8 words per CTA: %globaltimer at start, first page landed (consumer
 * warp 0), consumer loop done, output written; pages of the item; SM id;
 * items in the launch.  read copies the last launch's records (cap x 8). */
yk_status ykt_attention_stamps_enable(yk_model* m, int32_t cap);
yk_status ykt_attention_stamps_read(yk_model* m, uint64_t* host, int32_t cap, int32_t* n_ctas);

/* Per-CTA phase stamps of the bf16 GEMM launches of one trace kind (as in
 * ykt_trace_enable: 3 | epilogue << 4 | 128-row tiles << 8 | tokens/16 << 24;
 * 0 disables) inside normal forward steps.  Each matching launch overwrites 8
 * words per CTA (%globaltimer ns): start (before the grid dependency wait),
 * first activation copy issued (after it), first k-block landed, last MMA
 * issued, accumulator ready, epilogue done, segments, cluster barrier passed.
 * read copies the last matching launch's records. */
yk_status ykt_gemm_stamps_enable(yk_model* m, uint32_t kind);
yk_status ykt_gemm_stamps_read(yk_model* m, uint64_t* host, int32_t cap, int32_t* n_ctas);

/* Launch trace of the kernels on the engine stream.  enable(cap) (cap > 0)
 * resets cap records; launch i (the i-th launch counted by
 * yk_engine_launches) writes record i % cap: first CTA entry, first CTA past
 * its grid dependency wait, last CTA exit (%globaltimer ns) and kind (1 embed,
 * 2 rmsnorm, 3 GEMM, 4 attention, 5 draft sample, 6 row statistics, 7 verify
 * in the low 4 bits; GEMM adds epilogue << 4, 128-row tiles << 8 and
 * tokens/16 << 24, attention adds head dim << 8).
 * cap == 0 turns tracing off.  read copies cap x 4 words (entry, start, end,
 * kind) and the number of launches so far. */
yk_status ykt_trace_enable(yk_engine* e, int32_t cap);
yk_status ykt_trace_read(yk_engine* e, uint64_t* host, int32_t cap, uint64_t* launches);

/* Sampler phase stamps: after enable (cap CTAs; 0 disables) the draft
 * sampling kernel writes 8 words per CTA at [cta] and the verify kernel at
 * [cap + cta]: %globaltimer at start, row statistics done, probabilities
 * written, end; chain rounds, chain rounds ended by a special step,
 * sequential segments (low 32 bits) and rounding ties resolved in rounds
 * (high 32 bits); the sampled token (draft).  read copies 2 x cap x 8. */
yk_status ykt_sampler_stamps_enable(yk_sampler* s, int32_t cap);
yk_status ykt_sampler_stamps_read(yk_sampler* s, uint64_t* host, int32_t cap);

/* The failure path of the bounded device waits: one kernel waits on a
 * shared-memory barrier that nothing arrives at, with the wait every kernel
 * uses but a budget of budget_ms (<= 2000); when it gives up the kernel records
 * the timeout in the engine's error word and returns, and this call reports
 * YK_ERR_TIMEOUT (clearing the word) with *waited_ms the kernel's wait.  The
 * engine stays usable. */
yk_status ykt_wait_timeout(yk_engine* e, int32_t budget_ms, double* waited_ms);

/* The tensor-parallel all-reduce alone: 3 untimed calls, then `iters` calls
 * back to back on the engine stream over `count` bf16 elements (a multiple of
 * 8), timed with CUDA events; *ms_per_call = the average.  own != 0: the
 * group's own kernel over NVLink peer memory; 0: ncclAllReduce.  With own
 * and stamps_out (8 words, may be NULL), one more call records the kernel's
 * global-timer stamps (ns): CTA 0's entry, dependency resolved, every
 * partial ready, its share reduced, every share reduced, end; [6] the last
 * CTA's arrival; [7] unused.  Every rank of the group calls it with the same
 * arguments (it is a collective). */
yk_status ykt_tp_allreduce_timed(yk_engine* e, int64_t count, int32_t iters, int32_t own, double* ms_per_call,
                                 uint64_t* stamps_out);

/* The target probabilities q[B x (k+1) x V] exactly as the last verification
 * of yk_spec_sample_logits formed them from its logits (same chunk statistics,
 * same per-element expression), temperature > 0: lets a test hold the
 * logits-mode verification to bit-exact decisions against the oracle run on
 * these rows. */
yk_status ykt_sampler_target_probs(yk_sampler* s, int32_t B, float temperature, float* host);

#ifdef __cplusplus
}
#endif
