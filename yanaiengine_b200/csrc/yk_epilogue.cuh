// yk_epilogue.cuh -- fused GEMM epilogues, shared by the tcgen05 and SIMT GEMMs.
// Each call handles an adjacent output-row pair (n, n+1), n even, for token j:
//   EPI_QKV    RoPE on (2p, 2p+1) pairs of Q and K (S/gemm.metal:674-682,704-713);
//              Q -> q buffer, K/V -> their KV-pool page slot (replaces the CPU
//              PagedKVCache.appendFromFull, S/PagedKVCache.swift:24-62).
//   EPI_RESID  residual add into the fp32 stream (elementwise_add_kernel :282-291).
//   EPI_GLU    silu(gate)*up or gelu_tanh(gate)*up (S/LlamaBlock.swift:262-268,
//              S/GemmaBlock.swift:135-146); rows are interleaved gate/up.
//   EPI_LOGITS LM-head logits with optional soft-cap cap*tanh(x/cap) (S/LMHead.swift:20-46).
// ref_compat reproduces LinearLayer's bias 0.1 + ReLU (S/LinearLayer.swift:61,99-121).
#pragma once
#include "yk_common.cuh"
#include "yk_internal.h"

namespace yk {

__device__ __forceinline__ float compat_relu(float v) {
    v = v + 0.1f;
    return v > 0.f ? v : 0.f;
}

__device__ __forceinline__ float act_silu(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float act_gelu_tanh(float x) {
    const float cdf = 0.5f * (1.0f + tanhf(0.7978845608f * (x + 0.044715f * x * x * x)));
    return x * cdf;
}

template <typename AT>
__device__ __forceinline__ void epi_pair(const EpiParams& p, int n, int j, float v0, float v1) {
    if (j >= p.m_tok || n >= p.n_out) return;
    switch (p.kind) {
        case EPI_STORE: {  // plain fp32 result (test hook)
            float* o = reinterpret_cast<float*>(p.out) + (size_t)j * p.n_out + n;
            o[0] = v0;
            if (n + 1 < p.n_out) o[1] = v1;
            break;
        }
        case EPI_QKV: {
            if (p.ref_compat) { v0 = compat_relu(v0); v1 = compat_relu(v1); }
            const int dh = p.head_dim;
            if (n < p.q_dim + p.kv_dim) {  // Q or K: rotate the pair
                const int c = (n < p.q_dim ? n : n - p.q_dim) % dh;
                const float th = __fdiv_rn((float)p.pos[j], p.rope_denom[c >> 1]);
                float sn, cs;
                sincosf(th, &sn, &cs);
                const float r0 = v0 * cs - v1 * sn;
                const float r1 = v0 * sn + v1 * cs;
                v0 = r0;
                v1 = r1;
            }
            if (n < p.q_dim) {
                AT* o = reinterpret_cast<AT*>(p.out) + (size_t)j * p.q_dim + n;
                o[0] = from_f32<AT>(v0);
                o[1] = from_f32<AT>(v1);
            } else {
                const int kv = n < p.q_dim + p.kv_dim ? 0 : 1;
                const int nn = n - p.q_dim - kv * p.kv_dim;
                const int hh = nn / dh, c = nn % dh;
                const int slot = p.slot[j];
                const int blk = slot >> 4, off = slot & 15;
                if (blk < 0 || blk >= p.pool_blocks) {
                    raise_err(p.err, YK_DEV_ERR_BOUNDS);
                    return;
                }
                AT* o = reinterpret_cast<AT*>(p.pool) + (size_t)blk * p.block_elems + p.layer_off +
                        ((size_t)(kv * p.n_kv + hh) * 16 + off) * dh + c;
                o[0] = from_f32<AT>(v0);
                o[1] = from_f32<AT>(v1);
            }
            break;
        }
        case EPI_RESID: {
            if (p.ref_compat) { v0 = compat_relu(v0); v1 = compat_relu(v1); }
            float* o = p.h + (size_t)j * p.ld + n;
            o[0] = o[0] + v0;
            o[1] = o[1] + v1;
            break;
        }
        case EPI_GLU: {
            if (p.ref_compat) { v0 = compat_relu(v0); v1 = compat_relu(v1); }
            const float a = (p.act == 1 ? act_gelu_tanh(v0) : act_silu(v0)) * v1;
            reinterpret_cast<AT*>(p.out)[(size_t)j * (p.n_out >> 1) + (n >> 1)] = from_f32<AT>(a);
            break;
        }
        case EPI_LOGITS: {
            if (p.ref_compat) { v0 = v0 + 0.1f; v1 = v1 + 0.1f; }
            if (p.cap > 0.f) {
                v0 = p.cap * tanhf(v0 / p.cap);
                v1 = p.cap * tanhf(v1 / p.cap);
            }
            float* o = reinterpret_cast<float*>(p.out) + (size_t)j * p.n_out + n;
            o[0] = v0;
            if (n + 1 < p.n_out) o[1] = v1;
            break;
        }
        default: break;
    }
}

// NB consecutive tokens j0.. of one row pair.  The residual epilogue issues all
// its loads of the fp32 stream before any store, so a warp keeps NB
// read-modify-writes in flight instead of one.
template <typename AT, int NB>
__device__ __forceinline__ void epi_batch(const EpiParams& p, int n, int j0, const float (&v0)[NB],
                                          const float (&v1)[NB]) {
    if (p.kind == EPI_RESID) {
        if (n >= p.n_out) return;
        float2 hv[NB];
#pragma unroll
        for (int i = 0; i < NB; ++i)
            if (j0 + i < p.m_tok) hv[i] = *reinterpret_cast<const float2*>(p.h + (size_t)(j0 + i) * p.ld + n);
#pragma unroll
        for (int i = 0; i < NB; ++i) {
            if (j0 + i >= p.m_tok) continue;
            float a = v0[i], b = v1[i];
            if (p.ref_compat) { a = compat_relu(a); b = compat_relu(b); }
            *reinterpret_cast<float2*>(p.h + (size_t)(j0 + i) * p.ld + n) = make_float2(hv[i].x + a, hv[i].y + b);
        }
        return;
    }
#pragma unroll
    for (int i = 0; i < NB; ++i) epi_pair<AT>(p, n, j0 + i, v0[i], v1[i]);
}

}  // namespace yk
