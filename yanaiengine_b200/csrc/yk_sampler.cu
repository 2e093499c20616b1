// yk_sampler.cu -- fused speculative sampling on the device.  Replaces the
// CPU SpeculativeSampler (S/SpeculativeSampler.swift:4-130) and the
// Scheduler's per-sequence draft sampling (S/Scheduler.swift:171-189).
//
// Bit-exact contract: given identical probability tensors and uniforms, every
// acceptance decision and emitted token equals the reference's, because every
// value the reference derives from the probabilities is derived here with the
// same single IEEE fp32 operation (__fdiv_rn, __fsub_rn, __fadd_rn; no FMA
// contraction) in the same order:
//   ratio = q[d] / p[d]; accept iff r < ratio                    (:25-34)
//   residual = max(0, q - p) summed sequentially, divided by the sum (:37-55)
//   cdf += prob[i] sequentially; first i with r <= cdf, else V-1  (:63-73)
// The two sequential sums are "chains": one thread adds in index order while
// the rest of the CTA stages the next chunk of summands in shared memory.
#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>

#include "yk_chain.cuh"
#include "yk_common.cuh"
#include "yk_internal.h"

namespace yk {

constexpr int SMP_THREADS = CHAIN_THREADS;  // block_chain needs the whole block

// Swift's max(0, y): y if y >= 0 else 0 (max(0, NaN) = 0, max(0, -0.0) = -0.0).
__device__ __forceinline__ float swift_max0(float y) { return (y >= 0.0f) ? y : 0.0f; }

// softmax element from logits with row stats (max m and sum s of exp(x - m)):
// exp(x/T - m) / s  (S/SpeculativeSampler.swift:80-88, temperature per
// S/Sampler.swift:19-23).
__device__ __forceinline__ float scale_t(float l, float T) { return (T == 1.0f) ? l : __fdiv_rn(l, T); }
__device__ __forceinline__ float q_from_logit(float l, float T, float m, float s) {
    return __fdiv_rn(expf(__fsub_rn(scale_t(l, T), m)), s);
}

// Block-wide (max, sum-exp, first argmax) of x_i = l_i / T over one row.
// Each accumulator visits its indices in increasing order and merges keep the
// smallest index among equal maxima (first maximum wins); float4 loads when the
// row is 16-byte aligned.
__device__ __forceinline__ void stats_update(float raw, int idx, float T, float& m, float& s, float& best, int& arg) {
    const float x = scale_t(raw, T);
    if (raw > best) { best = raw; arg = idx; }
    if (x > m) {
        s = s * expf(m - x) + 1.0f;
        m = x;
    } else {
        s += expf(x - m);
    }
}

struct RowStats4 {
    float m, s, best;
    int arg;
};
// (max, sum-exp, best raw value, first argmax) over row[0, V) whose first element
// has index idx0 in its full row.
__device__ RowStats4 block_stats4(const float* __restrict__ row, int64_t V, int idx0, float T) {
    float m = -INFINITY, s = 0.f, best = -INFINITY;
    int arg = 0x7fffffff;
    if ((V & 3) == 0 && ((uintptr_t)row & 15) == 0) {
        // eight float4 loads per thread in flight before any use; the four lanes
        // of a float4 feed four independent (max, sum, argmax) accumulators, so the
        // exp/rescale chains run side by side, merged at the end
        const float4* r4 = reinterpret_cast<const float4*>(row);
        const int64_t n4 = V >> 2;
        constexpr int U = 8;
        float am[4], as[4], ab[4];
        int aa[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) { am[q] = -INFINITY; as[q] = 0.f; ab[q] = -INFINITY; aa[q] = 0x7fffffff; }
        for (int64_t i0 = threadIdx.x; i0 < n4; i0 += (int64_t)U * blockDim.x) {
            float4 v[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int64_t i = i0 + (int64_t)u * blockDim.x;
                if (i < n4) v[u] = __ldg(r4 + i);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int64_t i = i0 + (int64_t)u * blockDim.x;
                if (i < n4) {
                    const int ia = idx0 + (int)(i * 4);
                    stats_update(v[u].x, ia, T, am[0], as[0], ab[0], aa[0]);
                    stats_update(v[u].y, ia + 1, T, am[1], as[1], ab[1], aa[1]);
                    stats_update(v[u].z, ia + 2, T, am[2], as[2], ab[2], aa[2]);
                    stats_update(v[u].w, ia + 3, T, am[3], as[3], ab[3], aa[3]);
                }
            }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float M = fmaxf(m, am[q]);
            if (M != -INFINITY) s = s * expf(m - M) + as[q] * expf(am[q] - M);
            m = M;
            if (ab[q] > best || (ab[q] == best && aa[q] < arg)) { best = ab[q]; arg = aa[q]; }
        }
    } else {
        for (int64_t i = threadIdx.x; i < V; i += blockDim.x) stats_update(row[i], idx0 + (int)i, T, m, s, best, arg);
    }
    __shared__ float sm_m[32], sm_s[32], sm_b[32];
    __shared__ int sm_a[32];
    // warp reduce
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
        const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
        const float b2 = __shfl_xor_sync(0xffffffffu, best, o);
        const int a2 = __shfl_xor_sync(0xffffffffu, arg, o);
        const float M = fmaxf(m, m2);
        if (M != -INFINITY) s = s * expf(m - M) + s2 * expf(m2 - M);
        m = M;
        if (b2 > best || (b2 == best && a2 < arg)) { best = b2; arg = a2; }
    }
    const int w = threadIdx.x >> 5, ln = threadIdx.x & 31;
    if (ln == 0) { sm_m[w] = m; sm_s[w] = s; sm_b[w] = best; sm_a[w] = arg; }
    __syncthreads();
    if (w == 0) {
        const int nw = blockDim.x >> 5;
        m = ln < nw ? sm_m[ln] : -INFINITY;
        s = ln < nw ? sm_s[ln] : 0.f;
        best = ln < nw ? sm_b[ln] : -INFINITY;
        arg = ln < nw ? sm_a[ln] : 0x7fffffff;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
            const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
            const float b2 = __shfl_xor_sync(0xffffffffu, best, o);
            const int a2 = __shfl_xor_sync(0xffffffffu, arg, o);
            const float M = fmaxf(m, m2);
            if (M != -INFINITY) s = s * expf(m - M) + s2 * expf(m2 - M);
            m = M;
            if (b2 > best || (b2 == best && a2 < arg)) { best = b2; arg = a2; }
        }
        if (ln == 0) { sm_m[0] = m; sm_s[0] = s; sm_b[0] = best; sm_a[0] = arg; }
    }
    __syncthreads();
    RowStats4 r{sm_m[0], sm_s[0], sm_b[0], sm_a[0]};
    __syncthreads();
    return r;
}

// Merge of per-chunk statistics in chunk order (deterministic); first maximum wins.
constexpr int SMP_CHUNKS = 8;  // CTAs per row for the draft statistics and probability passes
__device__ __forceinline__ RowStats4 merge_chunks(const float4* __restrict__ part) {
    RowStats4 r{-INFINITY, 0.f, -INFINITY, 0x7fffffff};
#pragma unroll
    for (int c = 0; c < SMP_CHUNKS; ++c) {
        const float4 q = part[c];
        const float M = fmaxf(r.m, q.x);
        if (M != -INFINITY) r.s = r.s * expf(r.m - M) + q.y * expf(q.x - M);
        r.m = M;
        const int qa = __float_as_int(q.w);
        if (q.z > r.best || (q.z == r.best && qa < r.arg)) { r.best = q.z; r.arg = qa; }
    }
    if (r.arg == 0x7fffffff) r.arg = 0;
    return r;
}

// ---------------------------------------------------------------------------
// Draft sampling: one CTA per (sequence b, draft iteration j).
// p row -> probs[(b*k + j) * V]; token -> tokens[b*k + j] (or tokens[b]).
// ---------------------------------------------------------------------------
struct DraftArgs {
    const float* logits;   // row for CTA x: logits + row(x) * V
    int logit_row_stride;  // rows between consecutive sequences
    int logit_row_j_mul;   // rows between consecutive draft iterations
    int64_t V;
    int k, j_fixed;        // j_fixed >= 0: single iteration j for all CTAs
    float T;
    uint64_t seed;
    uint32_t step;
    const uint32_t* seq_ids;
    float* probs;
    uint32_t* tokens_out;
    uint32_t* tokens_keep = nullptr;  // also [b * k + j] of the device-resident draft matrix, if set
    float4* part = nullptr;  // [rows x SMP_CHUNKS] per-chunk (max, sum, best, argmax bits)
    unsigned long long* stamps = nullptr;  // test hook: 8 words per CTA
    Trace tr;
};

__device__ __forceinline__ void draft_row(const DraftArgs& a, int x, int& b, int& j) {
    b = a.j_fixed >= 0 ? x : x / a.k;
    j = a.j_fixed >= 0 ? a.j_fixed : x % a.k;
}
__device__ __forceinline__ int64_t draft_chunk(int64_t V) { return ((V + SMP_CHUNKS - 1) / SMP_CHUNKS + 3) & ~int64_t(3); }

// Draft rows, pass 1: statistics of chunk blockIdx.y of row blockIdx.x.
__global__ void __launch_bounds__(SMP_THREADS) draft_partial_kernel(DraftArgs a) {
    if (threadIdx.x == 0) trace_mark(a.tr, TR_ENTRY);
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x == 0) trace_mark(a.tr, TR_START);
    int b, j;
    draft_row(a, blockIdx.x, b, j);
    const float* row = a.logits + ((size_t)b * a.logit_row_stride + (size_t)j * a.logit_row_j_mul) * a.V;
    const int64_t ch = draft_chunk(a.V), c0 = (int64_t)blockIdx.y * ch, c1 = min(a.V, c0 + ch);
    const RowStats4 st = block_stats4(row + c0, max((int64_t)0, c1 - c0), (int)c0, a.T > 0.f ? a.T : 1.0f);
    if (threadIdx.x == 0) {
        a.part[(size_t)blockIdx.x * SMP_CHUNKS + blockIdx.y] = make_float4(st.m, st.s, st.best, __int_as_float(st.arg));
        trace_mark(a.tr, TR_END);
    }
}

// Draft rows, pass 2: p = softmax(row / T) for chunk blockIdx.y (one-hot argmax when T <= 0).
__global__ void __launch_bounds__(SMP_THREADS) draft_prob_kernel(DraftArgs a) {
    if (threadIdx.x == 0) trace_mark(a.tr, TR_ENTRY);
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x == 0) trace_mark(a.tr, TR_START);
    int b, j;
    draft_row(a, blockIdx.x, b, j);
    const float* row = a.logits + ((size_t)b * a.logit_row_stride + (size_t)j * a.logit_row_j_mul) * a.V;
    float* p = a.probs + ((size_t)b * a.k + j) * a.V;
    const RowStats4 st = merge_chunks(a.part + (size_t)blockIdx.x * SMP_CHUNKS);
    const int64_t ch = draft_chunk(a.V), c0 = (int64_t)blockIdx.y * ch, c1 = min(a.V, c0 + ch);
    if (a.T <= 0.f) {
        for (int64_t i = c0 + threadIdx.x; i < c1; i += blockDim.x) p[i] = (i == st.arg) ? 1.0f : 0.0f;
    } else {
        const float T = a.T, m = st.m, s = st.s;
        if (((uintptr_t)(row + c0) & 15) == 0 && ((uintptr_t)(p + c0) & 15) == 0 && ((c1 - c0) & 3) == 0) {
            const float4* r4 = reinterpret_cast<const float4*>(row + c0);
            float4* p4 = reinterpret_cast<float4*>(p + c0);
            const int64_t n4 = (c1 - c0) >> 2;
            constexpr int U = 4;
            for (int64_t i0 = threadIdx.x; i0 < n4; i0 += (int64_t)U * blockDim.x) {
                float4 l[U];
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int64_t i = i0 + (int64_t)u * blockDim.x;
                    if (i < n4) l[u] = __ldg(r4 + i);
                }
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int64_t i = i0 + (int64_t)u * blockDim.x;
                    if (i < n4)
                        p4[i] = make_float4(q_from_logit(l[u].x, T, m, s), q_from_logit(l[u].y, T, m, s),
                                            q_from_logit(l[u].z, T, m, s), q_from_logit(l[u].w, T, m, s));
                }
            }
        } else {
            for (int64_t i = c0 + threadIdx.x; i < c1; i += blockDim.x) p[i] = q_from_logit(row[i], T, m, s);
        }
    }
    if (threadIdx.x == 0) trace_mark(a.tr, TR_END);
}

// Draft rows, pass 3: the token, sampleFromProbs over p (first maximum when T <= 0).
__global__ void __launch_bounds__(SMP_THREADS) draft_sample_kernel(DraftArgs a) {
    __shared__ ChainSmem cs;
    if (threadIdx.x == 0) trace_mark(a.tr, TR_ENTRY);
    pdl_trigger();
    pdl_wait();
    unsigned long long* stp = a.stamps ? a.stamps + (size_t)blockIdx.x * 8 : nullptr;
    if (threadIdx.x == 0) {
        trace_mark(a.tr, TR_START);
        cs.n_rounds = cs.n_special = cs.n_seq = cs.n_ties = 0;
        if (stp) stp[0] = globaltimer_ns();
    }
    int b, j;
    draft_row(a, blockIdx.x, b, j);
    const float* p = a.probs + ((size_t)b * a.k + j) * a.V;
    const int64_t V = a.V;
    if (stp && threadIdx.x == 0) stp[1] = stp[2] = globaltimer_ns();
    uint32_t tok;
    if (a.T <= 0.f) {  // greedy: the merged first maximum
        tok = (uint32_t)merge_chunks(a.part + (size_t)blockIdx.x * SMP_CHUNKS).arg;
    } else {
        const float r = uniform_at(a.seed, a.step, a.seq_ids[b], (uint32_t)j, SLOT_DRAFT);
        tok = (uint32_t)block_chain(cs, [&](int64_t i) { return p[i]; }, V, true, r, nullptr,
                                    [&](long long i) { prefetch_l2(p + i); });
    }
    if (threadIdx.x == 0) {
        if (a.j_fixed >= 0) a.tokens_out[b] = tok;
        else a.tokens_out[(size_t)b * a.k + j] = tok;
        if (a.tokens_keep) a.tokens_keep[(size_t)b * a.k + j] = tok;
        trace_mark(a.tr, TR_END);
        if (stp) {
            stp[3] = globaltimer_ns();
            stp[4] = (unsigned long long)cs.n_rounds;
            stp[5] = (unsigned long long)cs.n_special;
            stp[6] = (unsigned long long)cs.n_seq | ((unsigned long long)cs.n_ties << 32);
            stp[7] = tok;
        }
    }
}

// ---------------------------------------------------------------------------
// verifySequence: one CTA per sequence.
// ---------------------------------------------------------------------------
struct VerifyArgs {
    const float* q;         // probs mode: q rows; logits mode: target logits rows
    const float* stats;     // logits mode: per target row (max, sum, argmax)
    const float* p;         // draft probs [B x k x V]
    const uint32_t* drafts; // [B x k]
    int64_t V;
    int k;
    int from_logits;
    float T;
    uint64_t seed;
    uint32_t step;
    const uint32_t* seq_ids;
    uint32_t* out;          // [B x (k+1)]
    int32_t* counts;        // [B]
    const float4* qpart = nullptr;  // logits mode: per-chunk target row statistics (else `stats`)
    uint32_t* err = nullptr;        // device error word (YK_DEV_ERR_BOUNDS on a draft token >= V), if any
    unsigned long long* stamps = nullptr;  // test hook: 8 words per CTA
    Trace tr;
};

// A draft token >= V (device-resident drafts are not checked by the host) is
// never used as an index: the sequence gets count -1, no token, and the error
// word (if given) the bounds bit.
__global__ void __launch_bounds__(SMP_THREADS) verify_kernel(VerifyArgs a) {
    __shared__ ChainSmem cs;
    if (threadIdx.x == 0) trace_mark(a.tr, TR_ENTRY);
    pdl_trigger();
    pdl_wait();
    unsigned long long* stp = a.stamps ? a.stamps + (size_t)blockIdx.x * 8 : nullptr;
    if (threadIdx.x == 0) {
        trace_mark(a.tr, TR_START);
        cs.n_rounds = cs.n_special = cs.n_seq = cs.n_ties = 0;
        if (stp) stp[0] = globaltimer_ns();
    }
    const int b = blockIdx.x;
    const int k = a.k;
    const int64_t V = a.V;
    const uint32_t seq = a.seq_ids[b];
    const bool greedy = a.from_logits && a.T <= 0.f;
    const float T = a.T > 0.f ? a.T : 1.0f;
    auto qrow = [&](int i) { return a.q + ((size_t)b * (k + 1) + i) * V; };
    __shared__ float s_stats[17 * 4];  // k + 1 <= 17 target rows: merged (max, sum, argmax bits, -)
    if (a.qpart) {
        if (threadIdx.x <= k) {
            const RowStats4 r = merge_chunks(a.qpart + ((size_t)b * (k + 1) + threadIdx.x) * SMP_CHUNKS);
            s_stats[threadIdx.x * 4 + 0] = r.m;
            s_stats[threadIdx.x * 4 + 1] = r.s;
            s_stats[threadIdx.x * 4 + 2] = __int_as_float(r.arg);
        }
        __syncthreads();
    }
    auto st = [&](int i) -> const float* {
        return a.qpart ? s_stats + i * 4 : a.stats + ((size_t)b * (k + 1) + i) * 4;
    };
    auto qval = [&](int i, int64_t x) -> float {
        if (!a.from_logits) return qrow(i)[x];
        return q_from_logit(qrow(i)[x], T, st(i)[0], st(i)[1]);
    };
    __shared__ int s_rej, s_bad;
    if (threadIdx.x == 0) {
        int rej = k, bad = 0;
        for (int i = 0; i < k; ++i) bad |= (int64_t)a.drafts[(size_t)b * k + i] >= V;
        for (int i = 0; i < k && !bad; ++i) {
            const uint32_t d = a.drafts[(size_t)b * k + i];
            bool acc;
            if (greedy) {
                acc = (uint32_t)__float_as_int(st(i)[2]) == d;
            } else {
                const float px = a.p[((size_t)b * k + i) * V + d];
                const float qx = qval(i, d);
                const float ratio = __fdiv_rn(qx, px);
                const float r = uniform_at(a.seed, a.step, seq, (uint32_t)i, SLOT_ACCEPT);
                acc = r < ratio;
            }
            if (!acc) { rej = i; break; }
        }
        s_rej = rej;
        s_bad = bad;
    }
    __syncthreads();
    if (s_bad) {
        if (threadIdx.x == 0) {
            a.counts[b] = -1;
            raise_err(a.err, YK_DEV_ERR_BOUNDS);
            trace_mark(a.tr, TR_END);
        }
        return;
    }
    const int rej = s_rej;
    uint32_t tok;
    if (greedy) {
        tok = (uint32_t)__float_as_int(st(rej)[2]);
    } else if (rej < k) {
        const float* pr = a.p + ((size_t)b * k + rej) * V;
        float S = 0.f;
        auto diff = [&](int64_t x) { return swift_max0(__fsub_rn(qval(rej, x), pr[x])); };
        auto pf_diff = [&](long long x) {
            prefetch_l2(qrow(rej) + x);
            prefetch_l2(pr + x);
        };
        block_chain(cs, diff, V, false, 0.f, &S, pf_diff);
        const float r = uniform_at(a.seed, a.step, seq, (uint32_t)rej, SLOT_RESAMPLE);
        if (S > 0.0f)
            tok = (uint32_t)block_chain(cs, [&](int64_t x) { return __fdiv_rn(diff(x), S); }, V, true, r, nullptr,
                                        pf_diff);
        else
            tok = (uint32_t)block_chain(cs, [&](int64_t x) { return qval(rej, x); }, V, true, r, nullptr,
                                        [&](long long x) { prefetch_l2(qrow(rej) + x); });
    } else {
        const float r = uniform_at(a.seed, a.step, seq, (uint32_t)k, SLOT_BONUS);
        tok = (uint32_t)block_chain(cs, [&](int64_t x) { return qval(k, x); }, V, true, r, nullptr,
                                    [&](long long x) { prefetch_l2(qrow(k) + x); });
    }
    if (threadIdx.x == 0) {
        uint32_t* o = a.out + (size_t)b * (k + 1);
        for (int i = 0; i < rej; ++i) o[i] = a.drafts[(size_t)b * k + i];
        o[rej] = tok;
        a.counts[b] = rej + 1;
    }
    if (stp && threadIdx.x == 0) {
        stp[3] = globaltimer_ns();
        stp[4] = (unsigned long long)cs.n_rounds;
        stp[5] = (unsigned long long)cs.n_special;
        stp[6] = (unsigned long long)cs.n_seq | ((unsigned long long)cs.n_ties << 32);
    }
    if (threadIdx.x == 0) trace_mark(a.tr, TR_END);
}

}  // namespace yk

// ---------------------------------------------------------------------------
// C-ABI
// ---------------------------------------------------------------------------
using namespace yk;

extern "C" yk_status yk_sampler_create(yk_engine* e, int32_t max_seqs, int32_t k, int32_t vocab, yk_sampler** out) {
    YK_ARG(e && out, "null handle");
    YK_ARG(max_seqs > 0 && k > 0 && k <= 16 && vocab > 0, "sampler shape");
    *out = nullptr;
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    auto* s = new yk_sampler();
    s->e = e;
    s->max_seqs = max_seqs;
    s->k = k;
    s->vocab = vocab;
    const size_t V = vocab;
    cudaError_t err = cudaSuccess;
    if ((err = cudaMalloc(&s->probs, (size_t)max_seqs * k * V * 4)) != cudaSuccess ||
        (err = cudaMalloc(&s->q, (size_t)max_seqs * (k + 1) * V * 4)) != cudaSuccess ||
        (err = cudaMalloc(&s->stats, (size_t)max_seqs * (2 * k + 1) * 4 * 4)) != cudaSuccess ||
        (err = cudaMalloc(&s->part, (size_t)max_seqs * (k + 1) * SMP_CHUNKS * sizeof(float4))) != cudaSuccess ||
        (err = cudaMalloc(&s->io, (size_t)max_seqs * (3 * k + 8) * 4 + 4096)) != cudaSuccess) {
        yk_sampler_destroy(s);
        yk_set_error(std::string("sampler cudaMalloc: ") + cudaGetErrorString(err));
        return err == cudaErrorMemoryAllocation ? YK_ERR_OOM : YK_ERR_CUDA;
    }
    *out = s;
    return YK_OK;
}

extern "C" void yk_sampler_destroy(yk_sampler* s) {
    if (!s) return;
    cudaSetDevice(s->e->device);
    cudaStreamSynchronize(s->e->stream);
    if (s->probs) cudaFree(s->probs);
    if (s->q) cudaFree(s->q);
    if (s->dlogits) cudaFree(s->dlogits);
    if (s->stats) cudaFree(s->stats);
    if (s->part) cudaFree(s->part);
    if (s->io) cudaFree(s->io);
    if (s->stamps) cudaFree(s->stamps);
    delete s;
}

// io area layout (uint32): [0, B) seq ids | [B, B + B*k) drafts | then out B*(k+1) | counts B | err 1
struct IoLayout {
    uint32_t *seq, *drafts, *out;
    int32_t* counts;
};
static IoLayout io_layout(yk_sampler* s, int B) {
    IoLayout L;
    L.seq = s->io;
    L.drafts = L.seq + B;
    L.out = L.drafts + (size_t)B * s->k;
    L.counts = (int32_t*)(L.out + (size_t)B * (s->k + 1));
    return L;
}

static yk_status finish_verify(yk_sampler* s, int B, const IoLayout& L, uint32_t* out_tokens, int32_t* out_counts) {
    yk_engine* e = s->e;
    const int k = s->k;
    const size_t nout = (size_t)B * (k + 1) + B;
    YK_CHECK_CUDA(cudaMemcpyAsync(e->pinned, L.out, nout * 4, cudaMemcpyDeviceToHost, e->stream));
    YK_CHECK_CUDA(cudaMemcpyAsync(e->pinned + nout * 4, e->d_err, 4, cudaMemcpyDeviceToHost, e->stream));
    YK_TRY(engine_sync_bounded(e));
    uint32_t err;
    std::memcpy(&err, e->pinned + nout * 4, 4);
    if (err) {
        cudaMemset(e->d_err, 0, 4);
        yk_set_error("device check fired during the step (code " + std::to_string(err) + ")");
        return (err & YK_DEV_ERR_TIMEOUT) ? YK_ERR_TIMEOUT : YK_ERR_DEVICE_CHECK;
    }
    std::memcpy(out_tokens, e->pinned, (size_t)B * (k + 1) * 4);
    std::memcpy(out_counts, e->pinned + (size_t)B * (k + 1) * 4, (size_t)B * 4);
    return YK_OK;
}

// Sequence ids (and host draft tokens, if given) to the device, through the
// engine's upload ring: the host does not wait for earlier work.
static yk_status upload_small(yk_sampler* s, int B, const uint32_t* seq_ids, const uint32_t* drafts,
                              const IoLayout& L) {
    yk_engine* e = s->e;
    // the ids of every draft step of a batch are the same: upload them once
    if (!drafts && s->dev_seq.size() == (size_t)B && std::memcmp(s->dev_seq.data(), seq_ids, (size_t)B * 4) == 0)
        return YK_OK;
    s->dev_seq.assign(seq_ids, seq_ids + B);
    const size_t n = (size_t)B + (drafts ? (size_t)B * s->k : 0);
    int slot = 0;
    uint8_t* host = nullptr;
    YK_TRY(e->up_acquire(n * 4, &slot, &host));
    std::memcpy(host, seq_ids, (size_t)B * 4);
    if (drafts) std::memcpy(host + (size_t)B * 4, drafts, (size_t)B * s->k * 4);
    return e->up_submit(slot, L.seq, n * 4);
}

// The draft tokens yk_draft_sample keeps on the device: [B x k] (column j is
// written by the sample of draft step j), valid for this B until the next
// call with another batch size.
const uint32_t* yk::sampler_device_drafts(const yk_sampler* s, int B, int* k) {
    if (B <= 0 || B > s->max_seqs) return nullptr;
    *k = s->k;
    return io_layout(const_cast<yk_sampler*>(s), B).drafts;
}

// Draft sampling of `rows` rows: chunked statistics, chunked probabilities, token.
static yk_status launch_draft(yk_sampler* s, DraftArgs a, int rows) {
    yk_engine* e = s->e;
    const double row_bytes = (double)rows * a.V * 4;  // algorithmic bytes: logits read, probabilities written
    {
        ProfScope prof(e, YK_PROF_SAMPLER, row_bytes, 0.0);
        a.tr = trace_next(e, TK_ROW_STATS);
        YK_CHECK_CUDA(launch_pdl(e, draft_partial_kernel, dim3(rows, SMP_CHUNKS), SMP_THREADS, 0, a));
        e->launches++;
    }
    {
        ProfScope prof(e, YK_PROF_SAMPLER, 2.0 * row_bytes, 0.0);
        a.tr = trace_next(e, TK_DRAFT_SAMPLE);
        YK_CHECK_CUDA(launch_pdl(e, draft_prob_kernel, dim3(rows, SMP_CHUNKS), SMP_THREADS, 0, a));
        e->launches++;
    }
    {
        ProfScope prof(e, YK_PROF_SAMPLER, 0.0, 0.0);  // reads p up to the sampled index
        a.tr = trace_next(e, TK_DRAFT_SAMPLE);
        a.stamps = (s->stamps && rows <= s->stamps_cap) ? s->stamps : nullptr;
        YK_CHECK_CUDA(launch_pdl(e, draft_sample_kernel, rows, SMP_THREADS, 0, a));
        e->launches++;
    }
    return YK_OK;
}

extern "C" yk_status yk_draft_sample(yk_sampler* s, yk_model* draft, int32_t B, int32_t j, float temperature,
                                     uint64_t seed, uint32_t step, const uint32_t* seq_ids, uint32_t* out_tokens) {
    YK_ARG(s && draft && seq_ids, "null argument");
    YK_ARG(B > 0 && B <= s->max_seqs && j >= 0 && j < s->k, "B / j");
    YK_ARG(draft->cfg.vocab_size == s->vocab, "vocab mismatch");
    YK_ARG(draft->last_rows >= B, "draft logits hold fewer rows than B (forward with last_n = 1)");
    yk_engine* e = s->e;
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    IoLayout L = io_layout(s, B);
    YK_TRY(upload_small(s, B, seq_ids, nullptr, L));
    DraftArgs a;
    a.logits = draft->logits;
    a.logit_row_stride = 1;
    a.logit_row_j_mul = 0;
    a.V = s->vocab;
    a.k = s->k;
    a.j_fixed = j;
    a.T = temperature;
    a.seed = seed;
    a.step = step;
    a.seq_ids = L.seq;
    a.probs = s->probs;
    a.tokens_out = L.out;
    // the tokens also stay on the device as draft column j ([B x k]) for the next
    // draft forward (yk_forward_step_drafts) and the verification
    a.tokens_keep = L.drafts;
    a.part = s->part;
    YK_TRY(launch_draft(s, a, B));
    if (!out_tokens) return YK_OK;  // asynchronous: device checks are reported by the verification
    YK_CHECK_CUDA(cudaMemcpyAsync(e->pinned, L.out, (size_t)B * 4, cudaMemcpyDeviceToHost, e->stream));
    YK_CHECK_CUDA(cudaMemcpyAsync(e->pinned + (size_t)B * 4, e->d_err, 4, cudaMemcpyDeviceToHost, e->stream));
    YK_TRY(engine_sync_bounded(e));
    uint32_t err;
    std::memcpy(&err, e->pinned + (size_t)B * 4, 4);
    if (err) {
        cudaMemset(e->d_err, 0, 4);
        yk_set_error("device check fired during the draft step (code " + std::to_string(err) + ")");
        return (err & YK_DEV_ERR_TIMEOUT) ? YK_ERR_TIMEOUT : YK_ERR_DEVICE_CHECK;
    }
    std::memcpy(out_tokens, e->pinned, (size_t)B * 4);
    return YK_OK;
}

static yk_status run_verify(yk_sampler* s, int B, const float* qsrc, int from_logits, float T, uint64_t seed,
                            uint32_t step, const IoLayout& L) {
    yk_engine* e = s->e;
    const int k = s->k;
    if (from_logits) {  // chunked statistics of the k + 1 target rows of each sequence
        DraftArgs d;
        d.logits = qsrc;
        d.logit_row_stride = k + 1;
        d.logit_row_j_mul = 1;
        d.V = s->vocab;
        d.k = k + 1;
        d.j_fixed = -1;
        d.T = T;
        d.part = s->part;
        d.tr = trace_next(e, TK_ROW_STATS);
        ProfScope prof(e, YK_PROF_SAMPLER, (double)B * (k + 1) * s->vocab * 4, 0.0);
        YK_CHECK_CUDA(launch_pdl(e, draft_partial_kernel, dim3(B * (k + 1), SMP_CHUNKS), SMP_THREADS, 0, d));
        e->launches++;
    }
    VerifyArgs a;
    a.q = qsrc;
    a.stats = s->stats;
    a.qpart = from_logits ? s->part : nullptr;
    a.p = s->probs;
    a.drafts = L.drafts;
    a.V = s->vocab;
    a.k = k;
    a.from_logits = from_logits;
    a.T = T;
    a.seed = seed;
    a.step = step;
    a.seq_ids = L.seq;
    a.out = L.out;
    a.counts = L.counts;
    a.err = e->d_err;
    a.tr = trace_next(e, TK_VERIFY);
    a.stamps = (s->stamps && B <= s->stamps_cap) ? s->stamps + (size_t)s->stamps_cap * 8 : nullptr;
    ProfScope prof(e, YK_PROF_SAMPLER, 0.0, 0.0);  // reads q, p at the drafts and a residual row up to the hit
    YK_CHECK_CUDA(launch_pdl(e, verify_kernel, B, SMP_THREADS, 0, a));
    e->launches++;
    return YK_OK;
}

extern "C" yk_status yk_spec_verify(yk_sampler* s, yk_model* target, int32_t B, float temperature, uint64_t seed,
                                    uint32_t step, const uint32_t* seq_ids, const uint32_t* draft_tokens,
                                    uint32_t* out_tokens, int32_t* out_counts) {
    YK_ARG(s && target && seq_ids && out_tokens && out_counts, "null argument");
    YK_ARG(B > 0 && B <= s->max_seqs, "B");
    YK_ARG(target->cfg.vocab_size == s->vocab, "vocab mismatch");
    YK_ARG(target->last_rows == B * (s->k + 1), "target logits must hold k+1 rows per sequence (last_n = k+1)");
    if (draft_tokens)  // else: the device-resident drafts of this batch's yk_draft_sample calls
        for (int i = 0; i < B * s->k; ++i) YK_ARG(draft_tokens[i] < (uint32_t)s->vocab, "draft token >= vocab");
    yk_engine* e = s->e;
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    IoLayout L = io_layout(s, B);
    YK_TRY(upload_small(s, B, seq_ids, draft_tokens, L));
    YK_TRY(run_verify(s, B, target->logits, 1, temperature, seed, step, L));
    return finish_verify(s, B, L, out_tokens, out_counts);
}

extern "C" yk_status yk_spec_verify_range(yk_sampler* s, yk_model* target, int32_t seq0, int32_t B, float temperature,
                                          uint64_t seed, uint32_t step, const uint32_t* seq_ids,
                                          const uint32_t* draft_tokens, uint32_t* out_tokens, int32_t* out_counts) {
    YK_ARG(s && target && seq_ids && out_tokens && out_counts, "null argument");
    YK_ARG(B > 0 && B <= s->max_seqs && seq0 >= 0, "B / seq0");
    YK_ARG(target->cfg.vocab_size == s->vocab, "vocab mismatch");
    YK_ARG(target->last_rows >= (seq0 + B) * (s->k + 1),
           "target logits must hold k+1 rows for each of sequences seq0 .. seq0+B-1 (last_n = k+1)");
    if (draft_tokens)
        for (int i = 0; i < B * s->k; ++i) YK_ARG(draft_tokens[i] < (uint32_t)s->vocab, "draft token >= vocab");
    yk_engine* e = s->e;
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    IoLayout L = io_layout(s, B);
    YK_TRY(upload_small(s, B, seq_ids, draft_tokens, L));
    const float* rows = target->logits + (size_t)seq0 * (s->k + 1) * s->vocab;
    YK_TRY(run_verify(s, B, rows, 1, temperature, seed, step, L));
    return finish_verify(s, B, L, out_tokens, out_counts);
}

extern "C" yk_status yk_sampler_read_drafts(yk_sampler* s, int32_t B, uint32_t* out) {
    YK_ARG(s && out, "null argument");
    YK_ARG(B > 0 && B <= s->max_seqs, "B");
    yk_engine* e = s->e;
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    IoLayout L = io_layout(s, B);
    const size_t n = (size_t)B * s->k;
    YK_CHECK_CUDA(cudaMemcpyAsync(e->pinned, L.drafts, n * 4, cudaMemcpyDeviceToHost, e->stream));
    YK_CHECK_CUDA(cudaMemcpyAsync(e->pinned + n * 4, e->d_err, 4, cudaMemcpyDeviceToHost, e->stream));
    YK_TRY(engine_sync_bounded(e));
    uint32_t err;
    std::memcpy(&err, e->pinned + n * 4, 4);
    if (err) {
        cudaMemset(e->d_err, 0, 4);
        yk_set_error("device check fired during the draft phase (code " + std::to_string(err) + ")");
        return (err & YK_DEV_ERR_TIMEOUT) ? YK_ERR_TIMEOUT : YK_ERR_DEVICE_CHECK;
    }
    std::memcpy(out, e->pinned, n * 4);
    return YK_OK;
}

extern "C" yk_status yk_spec_verify_probs(yk_sampler* s, int32_t B, const float* p, const float* q,
                                          const uint32_t* draft_tokens, uint64_t seed, uint32_t step,
                                          const uint32_t* seq_ids, uint32_t* out_tokens, int32_t* out_counts) {
    YK_ARG(s && p && q && draft_tokens && seq_ids && out_tokens && out_counts, "null argument");
    YK_ARG(B > 0 && B <= s->max_seqs, "B");
    for (int i = 0; i < B * s->k; ++i) YK_ARG(draft_tokens[i] < (uint32_t)s->vocab, "draft token >= vocab");
    yk_engine* e = s->e;
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    const size_t V = s->vocab;
    IoLayout L = io_layout(s, B);
    YK_TRY(upload_small(s, B, seq_ids, draft_tokens, L));
    YK_CHECK_CUDA(cudaMemcpyAsync(s->probs, p, (size_t)B * s->k * V * 4, cudaMemcpyHostToDevice, e->stream));
    s->logits_B = 0;  // s->q now holds probabilities, not logits
    YK_CHECK_CUDA(cudaMemcpyAsync(s->q, q, (size_t)B * (s->k + 1) * V * 4, cudaMemcpyHostToDevice, e->stream));
    YK_TRY(run_verify(s, B, s->q, 0, 1.0f, seed, step, L));
    return finish_verify(s, B, L, out_tokens, out_counts);
}

extern "C" yk_status yk_spec_sample_logits(yk_sampler* s, int32_t B, const float* draft_logits,
                                           const float* target_logits, float temperature, uint64_t seed,
                                           uint32_t step, const uint32_t* seq_ids, uint32_t* draft_tokens_out,
                                           uint32_t* out_tokens, int32_t* out_counts) {
    YK_ARG(s && seq_ids && draft_tokens_out && out_tokens && out_counts, "null argument");
    YK_ARG((draft_logits == nullptr) == (target_logits == nullptr), "draft and target logits: both or neither");
    YK_ARG(B > 0 && B <= s->max_seqs, "B");
    const bool resident = draft_logits == nullptr;
    YK_ARG(!resident || s->logits_B == B, "no logits of this batch size are resident (pass host logits first)");
    yk_engine* e = s->e;
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    const size_t V = s->vocab;
    const int k = s->k;
    if (!s->dlogits) YK_CHECK_CUDA(cudaMalloc(&s->dlogits, (size_t)s->max_seqs * k * V * 4));
    IoLayout L = io_layout(s, B);
    YK_TRY(upload_small(s, B, seq_ids, nullptr, L));
    if (!resident) {
        s->logits_B = 0;
        YK_CHECK_CUDA(cudaMemcpyAsync(s->dlogits, draft_logits, (size_t)B * k * V * 4, cudaMemcpyHostToDevice,
                                      e->stream));
        YK_CHECK_CUDA(cudaMemcpyAsync(s->q, target_logits, (size_t)B * (k + 1) * V * 4, cudaMemcpyHostToDevice,
                                      e->stream));
        s->logits_B = B;
    }
    DraftArgs a;
    a.logits = s->dlogits;
    a.logit_row_stride = k;
    a.logit_row_j_mul = 1;
    a.V = V;
    a.k = k;
    a.j_fixed = -1;
    a.T = temperature;
    a.seed = seed;
    a.step = step;
    a.seq_ids = L.seq;
    a.probs = s->probs;
    a.tokens_out = L.drafts;
    a.part = s->part;
    YK_TRY(launch_draft(s, a, B * k));
    YK_TRY(run_verify(s, B, s->q, 1, temperature, seed, step, L));
    YK_CHECK_CUDA(cudaMemcpyAsync(draft_tokens_out, L.drafts, (size_t)B * k * 4, cudaMemcpyDeviceToHost, e->stream));
    return finish_verify(s, B, L, out_tokens, out_counts);
}

extern "C" yk_status yk_sampler_read_probs(yk_sampler* s, int32_t b, int32_t j, float* host) {
    YK_ARG(s && host, "null argument");
    YK_ARG(b >= 0 && b < s->max_seqs && j >= 0 && j < s->k, "index");
    YK_CHECK_CUDA(cudaSetDevice(s->e->device));
    YK_CHECK_CUDA(cudaStreamSynchronize(s->e->stream));
    YK_CHECK_CUDA(cudaMemcpy(host, s->probs + ((size_t)b * s->k + j) * s->vocab, (size_t)s->vocab * 4,
                             cudaMemcpyDeviceToHost));
    return YK_OK;
}

// ---------------------------------------------------------------------------
// Verification that allocates nothing (yk_spec_verify_logits_noalloc in yk.h).
//
// For callers that cannot allocate device memory at this point: a serving host
// that has handed all free HBM to its own arenas (weights, KV pages, its own
// logit and probability buffers) at start-up.  For such a host a per-call
// cudaMalloc is not an option: it can fail once the arenas own the memory, and
// it may synchronise the whole device in the middle of a step.  This entry point
// runs the same two kernels as yk_spec_verify (chunked target-row statistics,
// then verification) on buffers the caller already owns and keeps its only
// scratch -- the per-chunk softmax statistics -- in the fixed array below, so
// its results equal yk_spec_verify's bit for bit.
// ---------------------------------------------------------------------------
// Largest B * (k+1) (target logit rows) one call may verify.
constexpr int YK_NOALLOC_MAX_ROWS = 2048;

// Per-chunk (max, sum, best, argmax bits) of every target row: 256 KB that every
// GPU loading libyk.so holds until the process exits.  Every call on a device
// shares it; each call rewrites every entry it reads before reading it (the
// statistics kernel runs first on the same stream), so nothing has to start at
// zero.  Calls that overlap on the GPU race on it.
static __device__ __align__(256) float4 g_noalloc_row_part[YK_NOALLOC_MAX_ROWS * SMP_CHUNKS];

// Device address of g_noalloc_row_part per device.  In host code the array's
// name is only a host-side stand-in, so the address is looked up with the device
// current, on the first call there (and again if the device's context was
// replaced since, e.g. after cudaDeviceReset: the cache is keyed by the
// context's unique id).
struct NoallocScratch {
    unsigned long long ctx_id = 0;
    float4* part = nullptr;
};
static NoallocScratch g_noalloc_scratch[64];
static std::mutex g_noalloc_mu;

typedef CUresult (*PFN_ctxGetCurrent)(CUcontext*);
typedef CUresult (*PFN_ctxGetId)(CUcontext, unsigned long long*);

// Unique id of the calling thread's current context, 0 if it cannot be read.
static unsigned long long current_ctx_id() {
    static PFN_ctxGetCurrent get_cur = nullptr;
    static PFN_ctxGetId get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_cur = (PFN_ctxGetCurrent)f;
        f = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = (PFN_ctxGetId)f;
    });
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (!get_cur || !get_id || get_cur(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS) return 0;
    return id;
}

static yk_status noalloc_part_address(int device, float4** out) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    YK_ARG(device >= 0 && device < 64, "device index");
    NoallocScratch& sc = g_noalloc_scratch[device];
    const unsigned long long id = current_ctx_id();
    if (!sc.part || id == 0 || id != sc.ctx_id) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_row_part);
        if (e != cudaSuccess || !p) {
            yk_set_error(std::string("cudaGetSymbolAddress(row statistics scratch): ") + cudaGetErrorString(e));
            return YK_ERR_CUDA;
        }
        sc.part = static_cast<float4*>(p);
        sc.ctx_id = id;
    }
    *out = sc.part;
    return YK_OK;
}

extern "C" yk_status yk_spec_verify_logits_noalloc(int32_t device, void* stream, const float* target_logits,
                                                   const float* draft_probs, const uint32_t* draft_tokens,
                                                   const uint32_t* seq_ids, int32_t B, int32_t k, int32_t V,
                                                   float temperature, uint64_t seed, uint32_t step,
                                                   uint32_t* out_tokens, int32_t* out_counts) {
    YK_ARG(target_logits && draft_probs && draft_tokens && seq_ids && out_tokens && out_counts, "null argument");
    YK_ARG(B > 0 && k > 0 && k <= 16 && V > 0, "B, k or V out of range");
    if ((int64_t)B * (k + 1) > YK_NOALLOC_MAX_ROWS) {
        yk_set_error("yk_spec_verify_logits_noalloc: B*(k+1) = " + std::to_string((int64_t)B * (k + 1)) +
                     " target rows exceed the fixed limit of " + std::to_string(YK_NOALLOC_MAX_ROWS));
        return YK_ERR_ARG;
    }
    // An error left pending by earlier work on this thread is reported as such,
    // before anything is launched, so it is not mistaken for this call's.
    const cudaError_t pending = cudaGetLastError();
    if (pending != cudaSuccess) {
        yk_set_error(std::string("yk_spec_verify_logits_noalloc: a CUDA error from earlier work was pending "
                                 "before this call (nothing launched): ") + cudaGetErrorString(pending));
        return YK_ERR_CUDA;
    }
    int prev = 0;
    YK_CHECK_CUDA(cudaGetDevice(&prev));
    YK_CHECK_CUDA(cudaSetDevice(device));
    float4* part = nullptr;
    yk_status s = noalloc_part_address(device, &part);
    if (s == YK_OK) {
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        DraftArgs d;  // chunked statistics of the k + 1 target rows of each sequence, as run_verify
        d.logits = target_logits;
        d.logit_row_stride = k + 1;
        d.logit_row_j_mul = 1;
        d.V = V;
        d.k = k + 1;
        d.j_fixed = -1;
        d.T = temperature;
        d.part = part;
        draft_partial_kernel<<<dim3(B * (k + 1), SMP_CHUNKS), SMP_THREADS, 0, st>>>(d);
        VerifyArgs a;
        a.q = target_logits;
        a.stats = nullptr;
        a.qpart = part;
        a.p = draft_probs;
        a.drafts = draft_tokens;
        a.V = V;
        a.k = k;
        a.from_logits = 1;
        a.T = temperature;
        a.seed = seed;
        a.step = step;
        a.seq_ids = seq_ids;
        a.out = out_tokens;
        a.counts = out_counts;
        verify_kernel<<<B, SMP_THREADS, 0, st>>>(a);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) {
            yk_set_error(std::string("yk_spec_verify_logits_noalloc launch: ") + cudaGetErrorString(e));
            s = YK_ERR_CUDA;
        }
    }
    cudaSetDevice(prev);
    return s;
}

// ---------------------------------------------------------------------------
// Test hooks (include/yk_testing.h).
// ---------------------------------------------------------------------------
#include "../../include/yk_testing.h"

extern "C" yk_status ykt_sampler_stamps_enable(yk_sampler* s, int32_t cap) {
    YK_ARG(s && cap >= 0, "arguments");
    YK_CHECK_CUDA(cudaSetDevice(s->e->device));
    YK_CHECK_CUDA(cudaStreamSynchronize(s->e->stream));
    if (s->stamps) cudaFree(s->stamps);
    s->stamps = nullptr;
    s->stamps_cap = 0;
    if (cap > 0) {
        YK_CHECK_CUDA(cudaMalloc(&s->stamps, (size_t)cap * 2 * 8 * 8));
        YK_CHECK_CUDA(cudaMemset(s->stamps, 0, (size_t)cap * 2 * 8 * 8));
        s->stamps_cap = cap;
    }
    return YK_OK;
}

extern "C" yk_status ykt_sampler_stamps_read(yk_sampler* s, uint64_t* host, int32_t cap) {
    YK_ARG(s && host && cap == s->stamps_cap && s->stamps, "stamps not enabled with this capacity");
    YK_CHECK_CUDA(cudaSetDevice(s->e->device));
    YK_CHECK_CUDA(cudaStreamSynchronize(s->e->stream));
    YK_CHECK_CUDA(cudaMemcpy(host, s->stamps, (size_t)cap * 2 * 8 * 8, cudaMemcpyDeviceToHost));
    return YK_OK;
}

// Target probabilities exactly as the last verification formed them: the
// probability pass of draft sampling over the target logits uploaded by
// yk_spec_sample_logits with the chunk statistics that verification merged (the
// same merge and the same q_from_logit per element), into a scratch buffer.
extern "C" yk_status ykt_sampler_target_probs(yk_sampler* s, int32_t B, float temperature, float* host) {
    YK_ARG(s && host && s->q, "arguments");
    YK_ARG(B > 0 && B <= s->max_seqs && temperature > 0.f, "B / temperature");
    yk_engine* e = s->e;
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    const size_t n = (size_t)B * (s->k + 1) * s->vocab;
    float* tmp = nullptr;
    YK_CHECK_CUDA(cudaMalloc(&tmp, n * 4));
    DraftArgs d;
    d.logits = s->q;
    d.logit_row_stride = s->k + 1;
    d.logit_row_j_mul = 1;
    d.V = s->vocab;
    d.k = s->k + 1;
    d.j_fixed = -1;
    d.T = temperature;
    d.probs = tmp;
    d.part = s->part;
    draft_prob_kernel<<<dim3(B * (s->k + 1), SMP_CHUNKS), SMP_THREADS, 0, e->stream>>>(d);
    cudaError_t err = cudaGetLastError();
    if (err == cudaSuccess) err = cudaMemcpyAsync(host, tmp, n * 4, cudaMemcpyDeviceToHost, e->stream);
    if (err == cudaSuccess) err = cudaStreamSynchronize(e->stream);
    cudaFree(tmp);
    YK_CHECK_CUDA(err);
    return YK_OK;
}
