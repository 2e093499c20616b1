/*
 * oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of YanAIEngine's speculative draft->verify hot path, used as
 * the reference the CUDA module is tested against (tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py).  Nothing in yanaiengine_b200/ links, loads or
 * calls this library; the product path fails loudly without its CUDA module.
 *
 * Parity status: the reference ships no tests, golden vectors or fixtures for
 * this path and cannot be built here (Swift + Metal, no toolchain), so parity
 * is UNPINNED BY THE REFERENCE.  The oracle is pinned instead by:
 *   - Philox4x32-10 known-answer vectors of Salmon et al. (SC'11, Random123);
 *   - hand-derived known answers read off the reference source
 *     (tests/golden/sampler_kat.json, made by tests/golden/make_golden.py);
 *   - the one known answer the reference states: 20 appended tokens occupy
 *     2 pages of 16 (Sources/yanaiengine/PagedAttentionVerification.swift:27-36);
 *   - for orc_forward_step, an independent float64 numpy restatement that
 *     recomputes every sequence from its whole history without pages
 *     (tests/test_oracle_forward_numpy.py).
 *
 * Citations are relative to the reference project root; S/ = Sources/yanaiengine/.
 * Compiled with -O2 -ffp-contract=off and no fast-math so every fp32 operation
 * rounds exactly once, in the reference's order.
 */
#pragma once
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- counter-based RNG (Salmon et al., SC'11) -------------------------- */
void orc_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]);
/* Uniform in [0,1): (word0 >> 8) * 2^-24 of Philox(ctr=(step,seq,pos,slot), key=seed). */
float orc_uniform(uint64_t seed, uint32_t step, uint32_t seq, uint32_t pos, uint32_t slot);
enum { ORC_SLOT_DRAFT = 0, ORC_SLOT_ACCEPT = 1, ORC_SLOT_RESAMPLE = 2, ORC_SLOT_BONUS = 3 };

/* ---- SpeculativeSampler (S/SpeculativeSampler.swift) -------------------- */
/* softmax(logits) :76-91 ; logits are divided by T first when T != 1 (the
 * S/Sampler.swift:19-23 temperature convention). */
void orc_softmax(const float* logits, int64_t V, float temperature, float* probs);
/* sampleFromProbs :63-73 with the uniform r injected. */
uint32_t orc_sample_from_probs(const float* probs, int64_t V, float r);
/* verifyToken :20-60.  Returns 1 on accept; on reject writes the resampled
 * token (drawn with r_resample) to *new_token and returns 0. */
int orc_verify_token(uint32_t drafted, const float* p_draft, const float* q_target, int64_t V,
                     float r_accept, float r_resample, uint32_t* new_token);
/* verifySequence :95-129 on probabilities: p = k draft rows, q = k+1 target
 * rows (already softmaxed).  Uniforms come from orc_uniform(seed, step, seq,
 * i, slot).  Writes <= k+1 tokens to out, returns the count. */
int orc_verify_sequence_probs(const uint32_t* drafts, int k, const float* p, const float* q,
                              int64_t V, uint64_t seed, uint32_t step, uint32_t seq, uint32_t* out);
/* verifySequence on target logits (softmax inside, :107,:124).  T == 0 is
 * greedy: accept iff argmax(target row) == draft, emit the argmax otherwise. */
int orc_verify_sequence_logits(const uint32_t* drafts, int k, const float* p, const float* target_logits,
                               int64_t V, float temperature, uint64_t seed, uint32_t step, uint32_t seq,
                               uint32_t* out);
/* Scheduler draft sampling (S/Scheduler.swift:177-187): p = softmax(logits),
 * token = sampleFromProbs(p) with orc_uniform(seed, step, seq, j, DRAFT).
 * T == 0: argmax, p one-hot. Writes p (V floats) and returns the token. */
uint32_t orc_draft_sample(const float* logits, int64_t V, float temperature, uint64_t seed,
                          uint32_t step, uint32_t seq, uint32_t j, float* p_out);
/* Greedy argmax, first maximum wins (strict >) -- S/Sampler.swift:81-91. */
uint32_t orc_argmax(const float* x, int64_t V);

/* ---- sampler batch helpers (bench cpu_baseline, tests) ------------------- */
/* Whole verify phase for B sequences on probabilities, nthreads host threads
 * (one sequence per thread at a time).  out: B*(k+1), counts: B. */
void orc_verify_batch_probs(int B, int k, int64_t V, const uint32_t* drafts, const float* p, const float* q,
                            uint64_t seed, uint32_t step, const uint32_t* seq_ids, int nthreads,
                            uint32_t* out, int32_t* counts);
/* Whole C1-style sampler step on logits: draft sampling of k tokens from the
 * draft logits (B*k*V) then verification against target logits (B*(k+1)*V). */
void orc_spec_sample_batch(int B, int k, int64_t V, const float* draft_logits, const float* target_logits,
                           float temperature, uint64_t seed, uint32_t step, const uint32_t* seq_ids,
                           int nthreads, uint32_t* drafts_out, uint32_t* out, int32_t* counts);

/* ---- verify forward (S/LlamaModel.swift:134-244, S/LlamaBlock.swift:178-276,
 *      S/gemm.metal kernels, Gemma variants from S/GemmaBlock.swift) ----------- */
typedef struct {
    int32_t vocab_size, d_model, n_layers, n_heads, n_kv_heads, head_dim, ffn_dim;
    float rope_theta, rms_eps, attn_cap, final_cap;
    int32_t window;              /* 0 = global attention */
    int32_t window_layer_parity; /* window on layers with l%2==parity; -1 = all layers */
    int32_t act;                 /* 0 = SiLU (SwiGLU), 1 = tanh-GELU (GeGLU) */
    int32_t ref_compat;          /* 1 = bias 0.1 + ReLU on every projection, LM-head cap 30 */
    int32_t emulate_bf16;        /* 1 = round to bf16 where the bf16 CUDA path stores bf16 */
    int32_t block_size;          /* tokens per KV page (16) */
} orc_cfg;

/* Weights, all fp32 row-major [out x in] (the CUDA module's logical layout).
 * Per layer: wq [H*dh x d], wk/wv [Hkv*dh x d], wo [d x H*dh], wg/wu [ffn x d],
 * wd [d x ffn], n1/n2 [d].  Arrays of per-layer pointers. */
typedef struct {
    const float* embed;   /* [V x d] */
    const float* const* wq; const float* const* wk; const float* const* wv; const float* const* wo;
    const float* const* wg; const float* const* wu; const float* const* wd;
    const float* const* n1; const float* const* n2;
    const float* final_norm; /* [d] */
    const float* lm_head;    /* [V x d] */
} orc_weights;

/* Paged KV pool: [num_blocks][n_layers][2][n_kv][block_size][head_dim] fp32. */
size_t orc_pool_floats(const orc_cfg* c, int32_t num_blocks);

/* One ragged forward step.  tokens[T]; q_starts[B+1]; context_lens[B] (length
 * after this step); block_tables[B x max_blocks].  The new tokens of sequence
 * b sit at positions context_lens[b]-n_b ... context_lens[b]-1.  Their K/V are
 * written into the pool first, then attention reads it.  Logits for every
 * token are written to logits[T x V] (or only the last `last_n` of each
 * sequence when last_n > 0, in sequence order).  nthreads host threads. */
int orc_forward_step(const orc_cfg* c, const orc_weights* w, float* pool, int32_t num_blocks,
                     const uint32_t* tokens, int32_t T, const uint32_t* q_starts,
                     const uint32_t* context_lens, int32_t B, const int32_t* block_tables,
                     int32_t max_blocks, int32_t last_n, int nthreads, float* logits);

/* bf16 round-to-nearest-even, returned as fp32. */
float orc_bf16_round(float x);

/* IEEE half -> fp32, the reference's bit-level conversion of F16 checkpoint
 * tensors (S/ModelLoader.swift:75-100: signed zero, subnormals normalised by
 * shifting the mantissa, inf / nan kept); n values. */
void orc_f16_to_f32(const uint16_t* h, size_t n, float* out);

#ifdef __cplusplus
}
#endif
