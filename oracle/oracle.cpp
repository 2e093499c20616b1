// oracle.cpp -- TEST INFRASTRUCTURE ONLY (see oracle.h).  CPU restatement of
// the reference speculative draft->verify path; the CUDA module is checked
// against it and never calls it.  S/ = Sources/yanaiengine/ in the reference.
#include "oracle.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

// ---------------------------------------------------------------------------
// Philox4x32-10, written from Salmon, Moraes, Dror, Shaw, "Parallel random
// numbers: as easy as 1, 2, 3" (SC'11): 10 rounds of two 32x32->64 multiplies
// with the published multipliers and Weyl key increments.
// ---------------------------------------------------------------------------
static inline void philox_round(uint32_t c[4], const uint32_t k[2]) {
    const uint64_t p0 = (uint64_t)0xD2511F53u * c[0];
    const uint64_t p1 = (uint64_t)0xCD9E8D57u * c[2];
    const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    const uint32_t n0 = hi1 ^ c[1] ^ k[0];
    const uint32_t n2 = hi0 ^ c[3] ^ k[1];
    c[0] = n0; c[1] = lo1; c[2] = n2; c[3] = lo0;
}

extern "C" void orc_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]) {
    uint32_t c[4] = {ctr[0], ctr[1], ctr[2], ctr[3]};
    uint32_t k[2] = {key[0], key[1]};
    for (int r = 0; r < 10; ++r) {
        philox_round(c, k);
        k[0] += 0x9E3779B9u;
        k[1] += 0xBB67AE85u;
    }
    std::memcpy(out, c, sizeof c);
}

extern "C" float orc_uniform(uint64_t seed, uint32_t step, uint32_t seq, uint32_t pos, uint32_t slot) {
    const uint32_t ctr[4] = {step, seq, pos, slot};
    const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
    uint32_t o[4];
    orc_philox4x32_10(ctr, key, o);
    return (float)(o[0] >> 8) * (1.0f / 16777216.0f);
}

extern "C" float orc_bf16_round(float x) {
    uint32_t u;
    std::memcpy(&u, &x, 4);
    if ((u & 0x7f800000u) == 0x7f800000u) {  // inf / nan: keep (quiet nan)
        if (u & 0x007fffffu) u |= 0x00400000u;
        u &= 0xffff0000u;
    } else {
        u += 0x7fffu + ((u >> 16) & 1u);
        u &= 0xffff0000u;
    }
    float r;
    std::memcpy(&r, &u, 4);
    return r;
}

// S/ModelLoader.swift:75-100, one value at a time.
extern "C" void orc_f16_to_f32(const uint16_t* h, size_t n, float* out) {
    for (size_t i = 0; i < n; ++i) {
        const uint32_t sign = (h[i] >> 15) & 1u, exponent = (h[i] >> 10) & 0x1fu, mantissa = h[i] & 0x3ffu;
        uint32_t bits;
        if (exponent == 0) {
            if (mantissa == 0) {
                bits = sign << 31;
            } else {
                // subnormal: shift the mantissa up to its implicit bit, lowering the exponent
                int32_t e = 0;
                uint32_t m = mantissa;
                while ((m & 0x400u) == 0) {
                    m <<= 1;
                    e -= 1;
                }
                e += 1;
                m &= ~0x400u;
                bits = (sign << 31) | ((uint32_t)(e + 112) << 23) | (m << 13);
            }
        } else if (exponent == 31) {
            bits = (sign << 31) | 0x7f800000u | (mantissa << 13);
        } else {
            bits = (sign << 31) | ((exponent + 112) << 23) | (mantissa << 13);
        }
        std::memcpy(&out[i], &bits, 4);
    }
}

// ---------------------------------------------------------------------------
// SpeculativeSampler -- S/SpeculativeSampler.swift
// ---------------------------------------------------------------------------

// Swift's max(x, y) returns y when y >= x, else x (so max(0, NaN) == 0 and
// max(0, -0.0) == -0.0); :42 is max(0, q - p).
static inline float swift_max0(float y) { return (y >= 0.0f) ? y : 0.0f; }

// softmax(logits:) :76-91.  max, exp(l - max), sequential fp32 sum, divide.
extern "C" void orc_softmax(const float* logits, int64_t V, float T, float* probs) {
    std::vector<float> scaled;
    const float* l = logits;
    if (T > 0.0f && T != 1.0f) {  // S/Sampler.swift:19-23 convention
        scaled.resize(V);
        for (int64_t i = 0; i < V; ++i) scaled[i] = logits[i] / T;
        l = scaled.data();
    }
    if (V <= 0) return;
    float mx = l[0];
    for (int64_t i = 1; i < V; ++i) if (l[i] > mx) mx = l[i];
    float sum = 0.0f;
    for (int64_t i = 0; i < V; ++i) {
        const float e = std::exp(l[i] - mx);
        probs[i] = e;
        sum += e;
    }
    if (sum > 0.0f)
        for (int64_t i = 0; i < V; ++i) probs[i] /= sum;
}

// sampleFromProbs :63-73.
extern "C" uint32_t orc_sample_from_probs(const float* probs, int64_t V, float r) {
    float cdf = 0.0f;
    for (int64_t i = 0; i < V; ++i) {
        cdf += probs[i];
        if (r <= cdf) return (uint32_t)i;
    }
    return (uint32_t)(V - 1);  // :72 fallback
}

// verifyToken :20-60.
extern "C" int orc_verify_token(uint32_t drafted, const float* p, const float* q, int64_t V,
                                float r_accept, float r_resample, uint32_t* new_token) {
    const float p_x = p[drafted];
    const float q_x = q[drafted];
    const float ratio = q_x / p_x;
    if (r_accept < ratio) return 1;                       // :32
    std::vector<float> adjusted(V);
    float sum = 0.0f;
    for (int64_t i = 0; i < V; ++i) {                     // :40-45
        const float diff = swift_max0(q[i] - p[i]);
        adjusted[i] = diff;
        sum += diff;
    }
    if (sum > 0.0f) {                                     // :48-55
        for (int64_t i = 0; i < V; ++i) adjusted[i] /= sum;
    } else {
        std::memcpy(adjusted.data(), q, sizeof(float) * V);
    }
    *new_token = orc_sample_from_probs(adjusted.data(), V, r_resample);  // :58
    return 0;
}

extern "C" uint32_t orc_argmax(const float* x, int64_t V) {
    float best = -INFINITY;
    uint32_t idx = 0;
    for (int64_t i = 0; i < V; ++i)
        if (x[i] > best) { best = x[i]; idx = (uint32_t)i; }
    return idx;
}

// verifySequence :95-129 on probability rows.
extern "C" int orc_verify_sequence_probs(const uint32_t* drafts, int k, const float* p, const float* q,
                                         int64_t V, uint64_t seed, uint32_t step, uint32_t seq,
                                         uint32_t* out) {
    int n = 0;
    for (int i = 0; i < k; ++i) {
        uint32_t nt = 0;
        const float ra = orc_uniform(seed, step, seq, (uint32_t)i, ORC_SLOT_ACCEPT);
        const float rr = orc_uniform(seed, step, seq, (uint32_t)i, ORC_SLOT_RESAMPLE);
        if (orc_verify_token(drafts[i], p + (size_t)i * V, q + (size_t)i * V, V, ra, rr, &nt)) {
            out[n++] = drafts[i];
        } else {
            out[n++] = nt;
            return n;                                     // :114-117
        }
    }
    const float rb = orc_uniform(seed, step, seq, (uint32_t)k, ORC_SLOT_BONUS);
    out[n++] = orc_sample_from_probs(q + (size_t)k * V, V, rb);   // :123-126
    return n;
}

extern "C" int orc_verify_sequence_logits(const uint32_t* drafts, int k, const float* p,
                                          const float* target_logits, int64_t V, float T,
                                          uint64_t seed, uint32_t step, uint32_t seq, uint32_t* out) {
    if (T <= 0.0f) {  // greedy: one-hot p and q
        int n = 0;
        for (int i = 0; i < k; ++i) {
            const uint32_t a = orc_argmax(target_logits + (size_t)i * V, V);
            if (a == drafts[i]) { out[n++] = a; continue; }
            out[n++] = a;
            return n;
        }
        out[n++] = orc_argmax(target_logits + (size_t)k * V, V);
        return n;
    }
    std::vector<float> q((size_t)(k + 1) * V);
    for (int i = 0; i <= k; ++i) orc_softmax(target_logits + (size_t)i * V, V, T, q.data() + (size_t)i * V);
    return orc_verify_sequence_probs(drafts, k, p, q.data(), V, seed, step, seq, out);
}

extern "C" uint32_t orc_draft_sample(const float* logits, int64_t V, float T, uint64_t seed,
                                     uint32_t step, uint32_t seq, uint32_t j, float* p_out) {
    if (T <= 0.0f) {
        const uint32_t a = orc_argmax(logits, V);
        if (p_out) { std::fill(p_out, p_out + V, 0.0f); p_out[a] = 1.0f; }
        return a;
    }
    std::vector<float> tmp;
    float* p = p_out;
    if (!p) { tmp.resize(V); p = tmp.data(); }
    orc_softmax(logits, V, T, p);
    return orc_sample_from_probs(p, V, orc_uniform(seed, step, seq, j, ORC_SLOT_DRAFT));
}

template <class F>
static void parallel_for(int n, int nthreads, F&& f) {
    if (nthreads <= 1 || n <= 1) { for (int i = 0; i < n; ++i) f(i); return; }
    std::vector<std::thread> th;
    const int nt = std::min(nthreads, n);
    for (int t = 0; t < nt; ++t)
        th.emplace_back([&, t] { for (int i = t; i < n; i += nt) f(i); });
    for (auto& x : th) x.join();
}

extern "C" void orc_verify_batch_probs(int B, int k, int64_t V, const uint32_t* drafts, const float* p,
                                       const float* q, uint64_t seed, uint32_t step, const uint32_t* seq_ids,
                                       int nthreads, uint32_t* out, int32_t* counts) {
    parallel_for(B, nthreads, [&](int b) {
        counts[b] = orc_verify_sequence_probs(drafts + (size_t)b * k, k, p + (size_t)b * k * V,
                                              q + (size_t)b * (k + 1) * V, V, seed, step, seq_ids[b],
                                              out + (size_t)b * (k + 1));
    });
}

extern "C" void orc_spec_sample_batch(int B, int k, int64_t V, const float* draft_logits,
                                      const float* target_logits, float T, uint64_t seed, uint32_t step,
                                      const uint32_t* seq_ids, int nthreads, uint32_t* drafts_out,
                                      uint32_t* out, int32_t* counts) {
    parallel_for(B, nthreads, [&](int b) {
        std::vector<float> p((size_t)k * V);
        for (int j = 0; j < k; ++j)
            drafts_out[(size_t)b * k + j] =
                orc_draft_sample(draft_logits + ((size_t)b * k + j) * V, V, T, seed, step, seq_ids[b],
                                 (uint32_t)j, p.data() + (size_t)j * V);
        counts[b] = orc_verify_sequence_logits(drafts_out + (size_t)b * k, k, p.data(),
                                               target_logits + (size_t)b * (k + 1) * V, V, T, seed, step,
                                               seq_ids[b], out + (size_t)b * (k + 1));
    });
}

// ---------------------------------------------------------------------------
// Verify forward.
// ---------------------------------------------------------------------------
extern "C" size_t orc_pool_floats(const orc_cfg* c, int32_t nb) {
    return (size_t)nb * c->n_layers * 2 * c->n_kv_heads * c->block_size * c->head_dim;
}

namespace {

struct Ctx {
    const orc_cfg* c;
    int nthreads;
    float rd(float x) const { return c->emulate_bf16 ? orc_bf16_round(x) : x; }
};

// y[t][o] = sum_k W[o][k] * x[t][k], sequential in k (S/gemm.metal:6-34 order).
void linear(const Ctx& cx, const float* W, int out_dim, int in_dim, const float* x, int T, float* y,
            bool compat_relu, bool compat_bias_only) {
    auto store = [&](int t, int o, float s) {
        if (compat_relu) { s = s + 0.1f; s = s > 0.0f ? s : 0.0f; }   // S/LinearLayer.swift:61,99-121
        else if (compat_bias_only) s = s + 0.1f;                        // LMHead: bias, no ReLU
        y[(size_t)t * out_dim + o] = s;
    };
    // Eight tokens' dot products side by side: each is still one sequential chain
    // in k with a separate multiply and add (the same result as one at a time),
    // but the eight chains overlap in time.  x is regrouped as [T/8][in_dim][8] so
    // the eight tokens' k-th inputs are adjacent.
    constexpr int U = 8;
    const int G = T / U;
    std::vector<float> xg((size_t)G * in_dim * U);
    for (int g = 0; g < G; ++g)
        for (int u = 0; u < U; ++u) {
            const float* xr = x + (size_t)(g * U + u) * in_dim;
            float* dst = xg.data() + (size_t)g * in_dim * U + u;
            for (int k = 0; k < in_dim; ++k) dst[(size_t)k * U] = xr[k];
        }
    parallel_for(out_dim, cx.nthreads, [&](int o) {
        const float* wr = W + (size_t)o * in_dim;
        for (int g = 0; g < G; ++g) {
            const float* xk = xg.data() + (size_t)g * in_dim * U;
            float s[U] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            for (int k = 0; k < in_dim; ++k) {
                const float wk = wr[k];
                for (int u = 0; u < U; ++u) s[u] += xk[(size_t)k * U + u] * wk;
            }
            for (int u = 0; u < U; ++u) store(g * U + u, o, s[u]);
        }
        for (int t = G * U; t < T; ++t) {
            const float* xr = x + (size_t)t * in_dim;
            float s = 0.0f;
            for (int k = 0; k < in_dim; ++k) s += xr[k] * wr[k];
            store(t, o, s);
        }
    });
}

// rmsnorm_kernel, S/gemm.metal:377-401: x * rsqrt(mean(x^2) + eps) * gamma.
void rmsnorm(const Ctx& cx, const float* x, const float* g, int T, int d, float eps, float* y) {
    for (int t = 0; t < T; ++t) {
        const float* xr = x + (size_t)t * d;
        float ss = 0.0f;
        for (int i = 0; i < d; ++i) ss += xr[i] * xr[i];
        const float rms = 1.0f / std::sqrt(ss / (float)d + eps);
        for (int i = 0; i < d; ++i) y[(size_t)t * d + i] = cx.rd(xr[i] * rms * g[i]);
    }
}

}  // namespace

extern "C" int orc_forward_step(const orc_cfg* c, const orc_weights* w, float* pool, int32_t num_blocks,
                                const uint32_t* tokens, int32_t T, const uint32_t* q_starts,
                                const uint32_t* ctx_lens, int32_t B, const int32_t* block_tables,
                                int32_t max_blocks, int32_t last_n, int nthreads, float* logits) {
    const Ctx cx{c, nthreads};
    const int d = c->d_model, H = c->n_heads, Hkv = c->n_kv_heads, dh = c->head_dim, F = c->ffn_dim;
    const int V = c->vocab_size, bs = c->block_size, L = c->n_layers;
    if (T <= 0 || B <= 0 || (int)q_starts[B] != T || H % Hkv) return 1;
    // Per-token sequence, position and pool slot (S/LlamaModel.swift:143-162; position
    // formula of batched_paged_attention_kernel, S/gemm.metal:656-659).
    std::vector<int> seq_of(T), pos_of(T), blk_of(T);
    for (int b = 0; b < B; ++b) {
        const int n = (int)(q_starts[b + 1] - q_starts[b]);
        if (n < 0 || (int)ctx_lens[b] < n) return 1;
        for (int i = 0; i < n; ++i) {
            const int t = (int)q_starts[b] + i;
            const int pos = (int)ctx_lens[b] - n + i;
            if (pos / bs >= max_blocks) return 1;
            const int blk = block_tables[(size_t)b * max_blocks + pos / bs];
            if (blk < 0 || blk >= num_blocks) return 1;
            seq_of[t] = b; pos_of[t] = pos; blk_of[t] = blk;
        }
        for (int p = 0; p < (int)ctx_lens[b]; ++p) {
            const int blk = block_tables[(size_t)b * max_blocks + p / bs];
            if (p / bs >= max_blocks || blk < 0 || blk >= num_blocks) return 1;
        }
    }
    const size_t layer_stride = (size_t)2 * Hkv * bs * dh;
    const size_t block_stride = (size_t)L * layer_stride;
    auto kv_ptr = [&](int blk, int layer, int kv, int h, int off) {
        return pool + (size_t)blk * block_stride + (size_t)layer * layer_stride +
               ((size_t)kv * Hkv + h) * bs * dh + (size_t)off * dh;
    };
    // RoPE denominators base^(2p/dh), in fp32 as S/gemm.metal:675 computes them.
    std::vector<float> denom(dh / 2);
    for (int p = 0; p < dh / 2; ++p) denom[p] = std::pow(c->rope_theta, (float)(2 * p) / (float)dh);
    const float scale = 1.0f / std::sqrt((float)dh);

    std::vector<float> h((size_t)T * d), xn((size_t)T * d);
    std::vector<float> q((size_t)T * H * dh), k((size_t)T * Hkv * dh), v((size_t)T * Hkv * dh);
    std::vector<float> att((size_t)T * H * dh), o((size_t)T * d);
    std::vector<float> g((size_t)T * F), u((size_t)T * F), a((size_t)T * F);
    for (int t = 0; t < T; ++t) {                         // embedding_lookup_kernel :326-341
        if (tokens[t] >= (uint32_t)V) return 1;
        std::memcpy(&h[(size_t)t * d], w->embed + (size_t)tokens[t] * d, sizeof(float) * d);
    }
    const bool compat = c->ref_compat != 0;
    auto rope = [&](float* x, int pos) {                  // :674-682 interleaved pairs
        for (int p = 0; p < dh / 2; ++p) {
            const float th = (float)pos / denom[p];
            const float cs = std::cos(th), sn = std::sin(th);
            const float x0 = x[2 * p], x1 = x[2 * p + 1];
            x[2 * p] = x0 * cs - x1 * sn;
            x[2 * p + 1] = x0 * sn + x1 * cs;
        }
    };
    for (int l = 0; l < L; ++l) {
        rmsnorm(cx, h.data(), w->n1[l], T, d, c->rms_eps, xn.data());
        linear(cx, w->wq[l], H * dh, d, xn.data(), T, q.data(), compat, false);
        linear(cx, w->wk[l], Hkv * dh, d, xn.data(), T, k.data(), compat, false);
        linear(cx, w->wv[l], Hkv * dh, d, xn.data(), T, v.data(), compat, false);
        for (int t = 0; t < T; ++t) {
            for (int hh = 0; hh < H; ++hh) {
                float* qr = &q[((size_t)t * H + hh) * dh];
                rope(qr, pos_of[t]);
                for (int i = 0; i < dh; ++i) qr[i] = cx.rd(qr[i]);
            }
            for (int hh = 0; hh < Hkv; ++hh) {
                float* kr = &k[((size_t)t * Hkv + hh) * dh];
                const float* vr = &v[((size_t)t * Hkv + hh) * dh];
                rope(kr, pos_of[t]);      // K stored rotated (mathematically the per-read rotation of :704-713)
                float* kd = kv_ptr(blk_of[t], l, 0, hh, pos_of[t] % bs);
                float* vd = kv_ptr(blk_of[t], l, 1, hh, pos_of[t] % bs);
                for (int i = 0; i < dh; ++i) { kd[i] = cx.rd(kr[i]); vd[i] = cx.rd(vr[i]); }
            }
        }
        const bool windowed = c->window > 0 && (c->window_layer_parity < 0 || (l % 2) == c->window_layer_parity);
        const float cap = c->attn_cap;
        // batched_paged_attention_kernel :629-737 + window (:572) and cap (:604-606).
        parallel_for(T * H, nthreads, [&](int th) {
            const int t = th / H, hq = th % H, kvh = hq / (H / Hkv);
            const int b = seq_of[t], pos = pos_of[t];
            const float* qr = &q[((size_t)t * H + hq) * dh];
            std::vector<float> acc(dh, 0.0f);
            float m = -INFINITY, lsum = 0.0f;
            for (int j = 0; j < (int)ctx_lens[b]; ++j) {
                if (j > pos) continue;
                if (windowed && pos - j >= c->window) continue;
                const int blk = block_tables[(size_t)b * max_blocks + j / bs];
                const float* kr = kv_ptr(blk, l, 0, kvh, j % bs);
                const float* vr = kv_ptr(blk, l, 1, kvh, j % bs);
                float s = 0.0f;
                for (int i = 0; i < dh; ++i) s += qr[i] * kr[i];
                s *= scale;
                if (cap > 0.0f) s = cap * std::tanh(s / cap);
                const float mp = m;
                m = std::max(mp, s);
                const float e = std::exp(s - m);
                const float ps = std::exp(mp - m);
                for (int i = 0; i < dh; ++i) acc[i] = acc[i] * ps + e * vr[i];
                lsum = lsum * ps + e;
            }
            float* orow = &att[((size_t)t * H + hq) * dh];
            for (int i = 0; i < dh; ++i) orow[i] = cx.rd(acc[i] / lsum);
        });
        linear(cx, w->wo[l], d, H * dh, att.data(), T, o.data(), compat, false);
        for (size_t i = 0; i < h.size(); ++i) h[i] = h[i] + o[i];        // elementwise_add :282-291
        rmsnorm(cx, h.data(), w->n2[l], T, d, c->rms_eps, xn.data());
        linear(cx, w->wg[l], F, d, xn.data(), T, g.data(), compat, false);
        linear(cx, w->wu[l], F, d, xn.data(), T, u.data(), compat, false);
        for (size_t i = 0; i < g.size(); ++i) {
            const float x = g[i];
            float act;
            if (c->act == 1) {                                            // gelu_kernel :231-241
                const float cdf = 0.5f * (1.0f + std::tanh(0.7978845608f * (x + 0.044715f * x * x * x)));
                act = x * cdf;
            } else {
                act = x / (1.0f + std::exp(-x));                          // silu_kernel :405-413
            }
            a[i] = cx.rd(act * u[i]);                                     // S/LlamaBlock.swift:264-267
        }
        linear(cx, w->wd[l], d, F, a.data(), T, o.data(), compat, false);
        for (size_t i = 0; i < h.size(); ++i) h[i] = h[i] + o[i];
    }
    // Rows that get logits.
    std::vector<int> rows;
    for (int b = 0; b < B; ++b) {
        const int n = (int)(q_starts[b + 1] - q_starts[b]);
        const int take = last_n > 0 ? std::min(last_n, n) : n;
        for (int i = n - take; i < n; ++i) rows.push_back((int)q_starts[b] + i);
    }
    const int R = (int)rows.size();
    std::vector<float> hr((size_t)R * d);
    for (int r = 0; r < R; ++r) std::memcpy(&hr[(size_t)r * d], &h[(size_t)rows[r] * d], sizeof(float) * d);
    rmsnorm(cx, hr.data(), w->final_norm, R, d, c->rms_eps, xn.data());  // S/LlamaModel.swift:225
    linear(cx, w->lm_head, V, d, xn.data(), R, logits, false, compat);    // S/LMHead.swift:20-23
    const float fcap = compat ? 30.0f : c->final_cap;                     // S/LMHead.swift:34
    if (fcap > 0.0f)
        for (size_t i = 0; i < (size_t)R * V; ++i) logits[i] = fcap * std::tanh(logits[i] / fcap);
    return 0;
}
