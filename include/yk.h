/*
 * yk.h -- C-ABI of the B200 speculative draft->verify module (libyk.so).
 *
 * This is the boundary the reference's Swift host would bind (through a
 * module map and a thin Swift shim).  Everything above it -- Scheduler's
 * draft/verify loop, SequenceRequest, PagedKVCache page tables and the
 * BlockAllocator free list -- stays on the host; everything below it runs as
 * hand-written sm_100a kernels on one CUDA stream per engine.
 *
 * Conventions
 *   - Plain C types only; every call returns a yk_status (YK_OK == 0) and never
 *     aborts.  yk_last_error() returns the calling thread's last message.
 *   - Host arrays passed in are borrowed for the duration of the call.
 *     Results written to host arrays are complete when the call returns
 *     (the call synchronises its stream, like the reference's
 *     commit(); waitUntilCompleted()).
 *   - Device memory (weights, KV pool, logits, draft probabilities) is owned by
 *     the handles and freed by the matching *_destroy.
 *   - A handle is not re-entrant: one host thread (the Scheduler actor) drives
 *     it.  One engine per GPU; sequences shard across engines/processes.
 *
 * Reference citations are relative to the reference project root,
 * S/ = Sources/yanaiengine/.
 */
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t yk_status;
#define YK_OK               0
#define YK_ERR_ARG          1  /* bad shape, token >= vocab, block id outside the pool ... */
#define YK_ERR_OOM          2  /* device allocation failed                               */
#define YK_ERR_CUDA         3  /* CUDA runtime/driver error                              */
#define YK_ERR_NCCL         4  /* NCCL error (tensor-parallel target only)               */
#define YK_ERR_TIMEOUT      5  /* a bounded device-side wait gave up                     */
#define YK_ERR_DEVICE_CHECK 6  /* an in-kernel bounds check fired                        */
#define YK_ERR_UNSUPPORTED  7  /* shape/dtype combination this module does not run       */

#define YK_DTYPE_F32  0
#define YK_DTYPE_BF16 1
#define YK_DTYPE_F16  2  /* checkpoint sources only (yk_model_load_tensor)       */

#define YK_ACT_SILU      0 /* SwiGLU, silu_kernel S/gemm.metal:405-413           */
#define YK_ACT_GELU_TANH 1 /* GeGLU, gelu_kernel S/gemm.metal:231-241 (Gemma-2)  */

#define YK_BLOCK_SIZE 16   /* tokens per KV page, S/LlamaModel.swift:47         */

typedef struct yk_engine  yk_engine;
typedef struct yk_model   yk_model;
typedef struct yk_kv_pool yk_kv_pool;
typedef struct yk_sampler yk_sampler;

/*
 * Model shape and numerics.  Replaces LlamaConfig (S/LlamaModel.swift:301-362)
 * and GemmaConfig (S/GemmaModel.swift:98-118) with explicit head_dim / ffn_dim
 * (the reference derives them: S/LlamaBlock.swift:69-72) and the constants the
 * reference hard-codes (RoPE base, eps, caps, window schedule).
 */
typedef struct yk_model_config {
    int32_t vocab_size;
    int32_t d_model;
    int32_t n_layers;
    int32_t n_heads;
    int32_t n_kv_heads;
    int32_t head_dim;            /* 64, 128 or 256                                   */
    int32_t ffn_dim;
    float   rope_theta;          /* 1e4 (S/gemm.metal:675) or 5e5 (Llama-3)           */
    float   rms_eps;             /* 1e-5 Llama (S/LlamaModel.swift:283), 1e-6 Gemma   */
    float   attn_cap;            /* 0 = off; 50 Gemma-2 (S/GemmaModel.swift:44)       */
    float   final_cap;           /* 0 = off; 30 (S/LMHead.swift:34)                   */
    int32_t window;              /* 0 = global; sliding window (S/gemm.metal:572)     */
    int32_t window_layer_parity; /* window on layers l%2==parity (0: even, as
                                    S/GemmaModel.swift:39-43); -1 = every layer      */
    int32_t act;                 /* YK_ACT_*                                          */
    int32_t ref_compat;          /* 1 = reproduce LinearLayer's bias 0.1 + ReLU on
                                    every projection and the unconditional LM-head
                                    cap 30 (S/LinearLayer.swift:29,61; S/LMHead.swift:20-35) */
    int32_t dtype;               /* YK_DTYPE_*: weights, activations and KV pool      */
    int32_t max_tokens;          /* largest T of one forward step (sizes workspaces)  */
    int32_t max_seqs;            /* largest batch B of one forward step               */
} yk_model_config;

/* Logical tensors of a model, all [out x in] row-major unless noted. */
#define YK_T_EMBED      0  /* [vocab x d]          EmbeddingLayer.weights        */
#define YK_T_WQ         1  /* [H*dh x d]           queryProj                     */
#define YK_T_WK         2  /* [Hkv*dh x d]         keyProj                       */
#define YK_T_WV         3  /* [Hkv*dh x d]         valueProj                     */
#define YK_T_WO         4  /* [d x H*dh]           outputProj                    */
#define YK_T_WGATE      5  /* [ffn x d]            gateProj                      */
#define YK_T_WUP        6  /* [ffn x d]            upProj                        */
#define YK_T_WDOWN      7  /* [d x ffn]            downProj                      */
#define YK_T_NORM1      8  /* [d]                  rmsGamma1                     */
#define YK_T_NORM2      9  /* [d]                  rmsGamma2                     */
#define YK_T_FINAL_NORM 10 /* [d]                  finalNormGamma                */
#define YK_T_LM_HEAD    11 /* [vocab x d]          LMHead.projection             */

#define YK_LAYOUT_OUT_IN 0 /* [out x in], this module's layout                     */
#define YK_LAYOUT_IN_OUT 1 /* [in x out], the reference's LinearLayer layout
                              (S/LinearLayer.swift:33-38); transposed on upload    */

/* ---- errors -------------------------------------------------------------- */
/* Copies the calling thread's last error message (NUL-terminated); returns its length. */
int32_t yk_last_error(char* buf, size_t buf_len);

/* ---- engine: one GPU, one stream.  Replaces MetalEngine (S/MetalEngine.swift:6-25). */
yk_status yk_engine_create(int32_t device, yk_engine** out);
void      yk_engine_destroy(yk_engine* e);
/* The engine's cudaStream_t, for callers that time work with CUDA events. */
yk_status yk_engine_stream(yk_engine* e, void** stream);
yk_status yk_engine_sync(yk_engine* e);
/* Reads and clears the device error word set by in-kernel checks and bounded waits. */
yk_status yk_engine_device_error(yk_engine* e, uint32_t* code);
/* Number of kernels this engine has launched (all of this module's kernels). */
uint64_t  yk_engine_launch_count(yk_engine* e);
/* Kernel timing: while enabled, every launch of the classes below is bracketed
 * by CUDA events on the engine stream and its algorithmic bytes / flops are
 * accumulated.  Class 0 = tcgen05/SIMT GEMM, 1 = paged attention, 2 = sampler,
 * 3 = other (the tensor-parallel all-reduce; bytes = what one rank moves over
 * NVLink in a ring all-reduce).  Reading resolves pending events (syncs). */
#define YK_PROF_GEMM    0
#define YK_PROF_ATTN    1
#define YK_PROF_SAMPLER 2
#define YK_PROF_OTHER   3
yk_status yk_engine_profile(yk_engine* e, int32_t enable);
yk_status yk_engine_profile_read(yk_engine* e, int32_t kernel_class, double* total_ms, double* total_bytes,
                                 double* total_flops, int64_t* launches);

/* ---- model: LlamaModel / GemmaModel weights + forward workspaces. -------- */
/* Random init on the device: matrices N(0, init_std) from Philox(seed), norms 1
 * (the reference fills U(-1,1): S/Tensor.swift:47-52 -- the benchmark workloads use N(0,0.02)). */
yk_status yk_model_create(yk_engine* e, const yk_model_config* cfg, uint64_t seed, float init_std,
                          yk_model** out);
void      yk_model_destroy(yk_model* m);
yk_status yk_model_get_config(const yk_model* m, yk_model_config* out);
yk_status yk_model_tensor_shape(const yk_model* m, int32_t tensor, int64_t* rows, int64_t* cols);
/* Upload one logical tensor from fp32 host memory (converted to the model dtype). */
yk_status yk_model_set_tensor(yk_model* m, int32_t tensor, int32_t layer, const float* host,
                              int32_t layout);
/* Download one logical tensor as fp32 [out x in]. */
yk_status yk_model_get_tensor(yk_model* m, int32_t tensor, int32_t layer, float* host);

/* ---- checkpoints.  Replaces SafetensorsReader (S/SafetensorsReader.swift:18-128)
 * and ModelLoader.loadLinearLayer (S/ModelLoader.swift:9-72). --------------- */
typedef struct yk_safetensors yk_safetensors;
typedef struct yk_tensor_info {
    int32_t     dtype;          /* YK_DTYPE_F32 / BF16 / F16, or -1 (another dtype)   */
    char        dtype_name[12]; /* as in the header: "F32", "BF16", "I8", ...          */
    int32_t     ndim;
    int64_t     shape[8];
    const void* data;           /* the mapped bytes, valid until yk_safetensors_close */
    uint64_t    nbytes;
} yk_tensor_info;
/* mmap a .safetensors file and parse its header (SafetensorsReader.open).  A
 * header that does not parse, or whose entries' offsets leave the data block or
 * disagree with dtype x shape, is YK_ERR_ARG (the reference trusts the file). */
yk_status yk_safetensors_open(const char* path, yk_safetensors** out);
void      yk_safetensors_close(yk_safetensors* st);
int32_t   yk_safetensors_count(const yk_safetensors* st);
/* Name of tensor i, 0 <= i < count, in name order (pointer valid until close). */
yk_status yk_safetensors_name(const yk_safetensors* st, int32_t i, const char** name);
/* tensorInfo + tensorData; YK_ERR_ARG if the name is absent. */
yk_status yk_safetensors_info(const yk_safetensors* st, const char* name, yk_tensor_info* out);

/* loadLinearLayer: upload one logical tensor from host memory in a checkpoint
 * dtype (F32, BF16 or F16; converted on the device, round-to-nearest-even into
 * bf16).  rows x cols is the stored shape of the FULL tensor: [out x in] for
 * YK_LAYOUT_OUT_IN (PyTorch / safetensors), [in x out] for YK_LAYOUT_IN_OUT (the
 * reference's LinearLayer); norms are [1 x d].  A tensor-parallel shard takes
 * its window (its heads' / FFN rows of column-parallel weights, its columns of
 * o_proj and down_proj). */
yk_status yk_model_load_tensor(yk_model* m, int32_t tensor, int32_t layer, const void* host, int32_t src_dtype,
                               int64_t rows, int64_t cols, int32_t layout);
/* Q / K rows stored in rotate-half order (Hugging Face Llama checkpoints): row
 * 2i + j of a head is read from stored row j * head_dim / 2 + i, so that RoPE's
 * interleaved pairs (S/gemm.metal:674-682) rotate the same dimensions. */
#define YK_LOAD_ROPE_HALF 1
/* Every weight of the model from the files of a (sharded) checkpoint under the
 * Hugging Face Llama / Gemma names (model.embed_tokens.weight,
 * model.layers.N.self_attn.{q,k,v,o}_proj.weight, mlp.{gate,up,down}_proj.weight,
 * input_layernorm.weight, post_attention_layernorm.weight, model.norm.weight,
 * lm_head.weight -- absent: tied to the embedding).  norm_offset is added to
 * every norm gain (1 for checkpoints that store gain - 1).  A missing tensor, a
 * shape mismatch or a tensor in two files is YK_ERR_ARG; an unknown tensor of a
 * decoder layer (a layer kind this module lacks) is YK_ERR_UNSUPPORTED. */
yk_status yk_model_load_safetensors(yk_model* m, yk_safetensors* const* files, int32_t n_files, float norm_offset,
                                    int32_t flags, int32_t* n_loaded);
/* The logical tensor (YK_T_*) and layer of a Hugging Face Llama / Gemma
 * checkpoint name, as yk_model_load_safetensors maps it (for callers that walk a
 * checkpoint themselves, e.g. a Swift ModelLoader calling yk_model_load_tensor);
 * YK_ERR_ARG for any other name or a layer >= n_layers.  No device needed. */
yk_status yk_hf_tensor_id(const char* name, int32_t n_layers, int32_t* tensor, int32_t* layer);

/* ---- paged KV pool.  Replaces BlockAllocator's MTLBuffers
 * (S/BlockAllocator.swift:13-36).  Block ids, the free list and the page
 * tables stay with the caller (BlockAllocator / PagedKVCache); a block id
 * covers every layer: pool layout [block][layer][K|V][kv_head][16][head_dim]. */
yk_status yk_kv_pool_create(yk_engine* e, const yk_model_config* cfg, int32_t num_blocks,
                            yk_kv_pool** out);
/* A pool for one kind of layer only: YK_POOL_GLOBAL_LAYERS holds the layers
 * without a window, YK_POOL_WINDOWED_LAYERS the windowed ones (cfg.window,
 * cfg.window_layer_parity), each block [its layers][K|V][kv head][16][dh].  With
 * one pool of each kind (yk_forward_step_split) the windowed layers get their
 * own page tables, so the pages before their window can be freed while the
 * global layers keep every page (Gemma's alternating schedule; the reference
 * never frees them, S/PagedKVCache.swift:65-85).  YK_POOL_ALL_LAYERS is
 * yk_kv_pool_create. */
#define YK_POOL_ALL_LAYERS      0
#define YK_POOL_GLOBAL_LAYERS   1
#define YK_POOL_WINDOWED_LAYERS 2
yk_status yk_kv_pool_create_layers(yk_engine* e, const yk_model_config* cfg, int32_t num_blocks, int32_t layers,
                                   yk_kv_pool** out);
void      yk_kv_pool_destroy(yk_kv_pool* p);
int32_t   yk_kv_pool_num_blocks(const yk_kv_pool* p);
/* Fills every slot with N(0, std) values (synthetic context for benchmarks). */
yk_status yk_kv_pool_fill_random(yk_kv_pool* p, uint64_t seed, float std);
/* Copies one page [n_kv_heads x 16 x head_dim] of layer `layer`, kv 0=K 1=V, as fp32. */
yk_status yk_kv_pool_read_page(yk_kv_pool* p, int32_t block, int32_t layer, int32_t kv, float* host);

/* ---- forward.  Replaces LlamaModel.forwardStep(batch:allocator:isDraft:)
 * (S/LlamaModel.swift:134-244).  tokens[T] concatenated per sequence;
 * q_starts[B+1] (:137,147); context_lens[B] = length of each sequence after
 * this step (:149-150); block_tables[B x max_blocks] int32 page tables
 * (:154-162).  Token i of sequence b sits at position
 * context_lens[b] - n_b + i (S/gemm.metal:656-659); its K (rotated) and V are
 * written to its page before attention reads the pool.  Every page covering
 * positions < context_lens[b] must be in the table.
 * Logits stay on the device ([rows x vocab] fp32): all T rows when
 * last_n == 0, else the last min(last_n, n_b) rows of each sequence in
 * sequence order (the rows Scheduler.step reads, S/Scheduler.swift:177,225).
 * *n_rows receives the row count. */
yk_status yk_forward_step(yk_model* m, yk_kv_pool* pool, const uint32_t* tokens, int32_t T,
                          const uint32_t* q_starts, const uint32_t* context_lens, int32_t B,
                          const int32_t* block_tables, int32_t max_blocks, int32_t last_n,
                          int32_t* n_rows);
/* yk_forward_step whose last nd input tokens of every sequence are the draft
 * tokens j0..j0+nd-1 that yk_draft_sample kept on the device for this batch
 * (tokens[] holds placeholders there).  The speculative loop's draft inputs
 * (S/Scheduler.swift:180-188) and the verify batch's drafts (:196-201) without
 * a device-to-host round trip: the host can queue the whole draft phase. */
yk_status yk_forward_step_drafts(yk_model* m, yk_kv_pool* pool, const uint32_t* tokens, int32_t T,
                                 const uint32_t* q_starts, const uint32_t* context_lens, int32_t B,
                                 const int32_t* block_tables, int32_t max_blocks, int32_t last_n,
                                 yk_sampler* s, int32_t j0, int32_t nd, int32_t* n_rows);
/* yk_forward_step over split pools: `pool` (YK_POOL_GLOBAL_LAYERS) with
 * block_tables for the global layers, `wpool` (YK_POOL_WINDOWED_LAYERS) with
 * wblock_tables for the windowed ones; both tables cover every position of each
 * sequence (pages wholly before a windowed layer's window may hold any valid
 * block id: they are not read).  s != NULL and nd > 0: the device-resident draft
 * tokens of yk_forward_step_drafts. */
yk_status yk_forward_step_split(yk_model* m, yk_kv_pool* pool, yk_kv_pool* wpool, const uint32_t* tokens, int32_t T,
                                const uint32_t* q_starts, const uint32_t* context_lens, int32_t B,
                                const int32_t* block_tables, int32_t max_blocks, const int32_t* wblock_tables,
                                int32_t wmax_blocks, int32_t last_n, yk_sampler* s, int32_t j0, int32_t nd,
                                int32_t* n_rows);
/* Copies logits rows [row0, row0+rows) of the last forward step to host (tests). */
yk_status yk_logits_copy_to_host(yk_model* m, int32_t row0, int32_t rows, float* host);

/* ---- sampler.  Replaces SpeculativeSampler (S/SpeculativeSampler.swift) and
 * the Scheduler's draft sampling (S/Scheduler.swift:171-189).  Uniform draws
 * are Philox4x32-10 keyed by seed, counter (step, seq_id, position, slot) with
 * slot 0 draft / 1 accept / 2 resample / 3 bonus; u = (x0 >> 8) * 2^-24.
 * temperature T > 0 scales logits by 1/T (S/Sampler.swift:19-23); T == 0 is
 * greedy (argmax, first maximum wins). */
yk_status yk_sampler_create(yk_engine* e, int32_t max_seqs, int32_t k, int32_t vocab, yk_sampler** out);
void      yk_sampler_destroy(yk_sampler* s);
/* Draft iteration j: p = softmax(draft logits row b / T) kept on the device for
 * verification, token = sampleFromProbs(p) (S/SpeculativeSampler.swift:63-91).
 * Reads rows 0..B-1 of `draft`'s logits (forward with last_n = 1).  The tokens
 * are also kept on the device (draft column j of the batch); out_tokens NULL:
 * returns without waiting for the device (errors surface at verification). */
yk_status yk_draft_sample(yk_sampler* s, yk_model* draft, int32_t B, int32_t j, float temperature,
                          uint64_t seed, uint32_t step, const uint32_t* seq_ids, uint32_t* out_tokens);
/* verifySequence (S/SpeculativeSampler.swift:95-129) for B sequences against
 * `target`'s logits rows b*(k+1)+i (forward with last_n = k+1) and the draft
 * probabilities kept by yk_draft_sample.  out_tokens[B x (k+1)], out_counts[B].
 * draft_tokens NULL: the drafts yk_draft_sample kept on the device. */
yk_status yk_spec_verify(yk_sampler* s, yk_model* target, int32_t B, float temperature, uint64_t seed,
                         uint32_t step, const uint32_t* seq_ids, const uint32_t* draft_tokens,
                         uint32_t* out_tokens, int32_t* out_counts);
/* Bit-exact parity entry: verifySequence on probability tensors.
 * p[B x k x V] draft probs, q[B x (k+1) x V] target probs, host fp32. */
yk_status yk_spec_verify_probs(yk_sampler* s, int32_t B, const float* p, const float* q,
                               const uint32_t* draft_tokens, uint64_t seed, uint32_t step,
                               const uint32_t* seq_ids, uint32_t* out_tokens, int32_t* out_counts);
/* Whole sampler phase of one step from host logits (draft sampling of k tokens
 * per sequence, then verification): draft_logits[B x k x V],
 * target_logits[B x (k+1) x V].  Both NULL: the logits the previous call
 * uploaded for this B are still on the device and are sampled again (with this
 * call's seed / step), so the device phase can be run without the upload. */
yk_status yk_spec_sample_logits(yk_sampler* s, int32_t B, const float* draft_logits,
                                const float* target_logits, float temperature, uint64_t seed,
                                uint32_t step, const uint32_t* seq_ids, uint32_t* draft_tokens_out,
                                uint32_t* out_tokens, int32_t* out_counts);
/* verifySequence for sequences seq0 .. seq0+B-1 of `target`'s logits (rows
 * (seq0+b)*(k+1)+i) against draft probabilities rows 0..B-1 of this sampler:
 * a rank that drafted only its own slice of the batch verifies that slice
 * (sequence-sharded drafting under tensor parallelism). */
yk_status yk_spec_verify_range(yk_sampler* s, yk_model* target, int32_t seq0, int32_t B, float temperature,
                               uint64_t seed, uint32_t step, const uint32_t* seq_ids, const uint32_t* draft_tokens,
                               uint32_t* out_tokens, int32_t* out_counts);
/* The [B x k] draft tokens yk_draft_sample kept on the device for batch size B
 * (waits for the device; reports device checks raised during the draft phase). */
yk_status yk_sampler_read_drafts(yk_sampler* s, int32_t B, uint32_t* out);
/* Copies draft probabilities p[b][j][0..V) kept by yk_draft_sample (tests). */
yk_status yk_sampler_read_probs(yk_sampler* s, int32_t b, int32_t j, float* host);

/* Verification that allocates no device memory.  No counterpart in the
 * reference: it exists for hosts that own all device memory themselves (a
 * serving loop that carves every free byte of HBM into its own arenas at
 * start-up cannot let a call allocate -- cudaMalloc may fail once the arenas
 * own the memory, and it can synchronise the device mid-step).
 * Same kernels and the same result, bit for bit, as yk_spec_verify:
 * verifySequence over target logits [B x (k+1) x V] and draft probabilities
 * [B x k x V] (as yk_draft_sample keeps them), draft tokens [B x k], Philox
 * stream ids [B]; outputs tokens [B x (k+1)] and counts [B].  Every pointer is
 * DEVICE memory of `device`; the work is queued on `stream` (a cudaStream_t)
 * and is complete when that stream is.  A draft token >= V is never used as an
 * index: that sequence's count is -1 and its tokens are not written.
 * Its only scratch is a fixed 256 KB static device array (held by every GPU
 * that loads libyk.so until exit), so B*(k+1) is limited to 2048 rows; larger
 * calls fail with YK_ERR_ARG before anything is launched.  The first call on a
 * device looks the array's device address up (cudaGetSymbolAddress) and caches
 * it per context, so that first call should come before any stream capture.
 * All calls on a device share the array: calls that overlap on the GPU race.
 * A CUDA error left pending by earlier work on the calling thread is returned
 * as YK_ERR_CUDA (its message says so) and nothing is launched. */
yk_status yk_spec_verify_logits_noalloc(int32_t device, void* stream, const float* target_logits,
                                        const float* draft_probs, const uint32_t* draft_tokens,
                                        const uint32_t* seq_ids, int32_t B, int32_t k, int32_t V,
                                        float temperature, uint64_t seed, uint32_t step, uint32_t* out_tokens,
                                        int32_t* out_counts);

/* ---- tensor parallelism: the 70B-shape target (Llama-3-70B, TP over the 8
 * GPUs of a box).  Replaces nothing in the reference (its models run on one
 * Metal device); the layer math is LlamaBlock.forwardBatched with o_proj and
 * down_proj split by input columns and summed by an NCCL all-reduce over
 * NVLink.  NCCL is loaded at run time (libnccl.so.2). */
/* A new NCCL unique id (128 bytes) for rank 0 to hand to every rank. */
yk_status yk_tp_unique_id(uint8_t id_out[128]);
/* Joins the group: one engine per rank, all with the same id and world.  The
 * set-up runs non-blocking and is abandoned (communicator aborted,
 * YK_ERR_TIMEOUT) if the group is not complete within timeout_ms; the same
 * deadline then bounds every wait on the engine's work (yk_engine_sync and the
 * sampler's result reads): a stream whose collectives do not finish in time (a
 * peer stopped taking part) ends with YK_ERR_TIMEOUT and the communicator
 * aborted.  yk_tp_init uses 300 s.  The all-reduce payload is bf16 (env
 * YK_TP_PAYLOAD=f32 at engine creation: fp32, through NCCL).  The bf16
 * all-reduce is the module's own kernel over NVLink peer memory (one shot at
 * two ranks, two-shot above); env YK_TP_AR=nccl uses ncclAllReduce, and
 * YK_TP_AR=twoshot the two-shot form at two ranks too. */
yk_status yk_tp_init(yk_engine* e, const uint8_t id[128], int32_t rank, int32_t world);
yk_status yk_tp_init_timeout(yk_engine* e, const uint8_t id[128], int32_t rank, int32_t world, int64_t timeout_ms);
/* Shard tp_rank of tp_world of the model `cfg`: query heads, KV heads and FFN
 * columns split evenly (n_kv_heads and ffn_dim divisible by tp_world); the
 * embedding, the norms and the LM head are replicated (same seed on every
 * rank).  yk_model_get_config and the tensor shapes report the shard, which is
 * also the config its KV pool is created with.  The engine must have joined a
 * group of tp_world ranks; yk_forward_step then all-reduces after o_proj and
 * down_proj, so every rank must run the same steps. */
yk_status yk_model_create_tp(yk_engine* e, const yk_model_config* cfg, int32_t tp_rank, int32_t tp_world,
                             uint64_t seed, float init_std, yk_model** out);
/* All-gather of `count` uint32 per rank over the group (host buffers; recv holds
 * world x count values in rank order).  Waits for the engine stream, bounded by
 * the group's deadline.  Used by the host scheduler to exchange drafted and
 * verified tokens when each rank drafts its own slice of the batch. */
yk_status yk_tp_allgather_u32(yk_engine* e, const uint32_t* send, int32_t count, uint32_t* recv);

#ifdef __cplusplus
}
#endif
