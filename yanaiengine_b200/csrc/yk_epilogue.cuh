// yk_epilogue.cuh -- fused GEMM epilogues, shared by the tcgen05 and SIMT GEMMs.
// Row n = output feature, column j = token:
//   EPI_QKV    RoPE on (2p, 2p+1) pairs of Q and K (S/gemm.metal:674-682,704-713);
//              Q -> q buffer, K/V -> their KV-pool page slot (replaces the CPU
//              PagedKVCache.appendFromFull, S/PagedKVCache.swift:24-62).
//   EPI_RESID  residual add into the fp32 stream (elementwise_add_kernel :282-291).
//   EPI_GLU    silu(gate)*up or gelu_tanh(gate)*up (S/LlamaBlock.swift:262-268,
//              S/GemmaBlock.swift:135-146); rows are interleaved gate/up.
//   EPI_LOGITS LM-head logits with optional soft-cap cap*tanh(x/cap) (S/LMHead.swift:20-46).
//   EPI_STORE  plain fp32 result (test hook).
// ref_compat reproduces LinearLayer's bias 0.1 + ReLU (S/LinearLayer.swift:61,99-121).
// The kind is a template parameter: each GEMM instantiation carries only its own
// epilogue, which keeps the fully unrolled drain loops small and in cache.
#pragma once
#include "yk_common.cuh"
#include "yk_internal.h"

namespace yk {

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float compat_relu(float v) {
    v = v + 0.1f;
    return v > 0.f ? v : 0.f;
}

// x * sigmoid(x) with the fast exponential and division intrinsics: relative
// error ~1e-6, far below the bf16 rounding of the stored activation.
__device__ __forceinline__ float act_silu(float x) { return __fdividef(x, 1.0f + __expf(-x)); }
__device__ __forceinline__ float act_gelu_tanh(float x) {
    const float cdf = 0.5f * (1.0f + tanhf(0.7978845608f * (x + 0.044715f * x * x * x)));
    return x * cdf;
}

// RoPE rotation of the pair (x, y) by (cos, sin): (x cos - y sin, x sin + y cos),
// each product rounded before the sum (no contraction into FMA, so the result
// does not depend on where the compiler inlines it; the reference's fp32
// expression).
__device__ __forceinline__ float2 rope_rot(float x, float y, float cs, float sn) {
    return make_float2(__fsub_rn(__fmul_rn(x, cs), __fmul_rn(y, sn)), __fadd_rn(__fmul_rn(x, sn), __fmul_rn(y, cs)));
}

__device__ __forceinline__ float logit_out(const EpiParams& p, float v) {
    if (p.ref_compat) v = v + 0.1f;
    if (p.cap > 0.f) v = p.cap * tanhf(v / p.cap);
    return v;
}

// RoPE angle of pair (c, c+1) of a head at token j: theta = pos / denom[c/2]
// (fp32 division), cos and sin of theta; from the step's table when present.
__device__ __forceinline__ void rope_cs(const EpiParams& p, int c, int j, float& cs, float& sn) {
    if (p.rope_tab) {
        const float2 t = p.rope_tab[(size_t)j * (p.head_dim >> 1) + (c >> 1)];
        cs = t.x;
        sn = t.y;
        return;
    }
    const float th = __fdiv_rn((float)p.pos[j], p.rope_denom[c >> 1]);
    sincosf(th, &sn, &cs);
}

// KV-pool address of element (kv, head, dim c) of token j; null (and error bit)
// if the slot's page lies outside the pool.
template <typename AT>
__device__ __forceinline__ AT* pool_elem(const EpiParams& p, int kv, int hh, int c, int j) {
    const int slot = p.slot[j];
    const int blk = slot >> 4, off = slot & 15;
    if (blk < 0 || blk >= p.pool_blocks) {
        raise_err(p.err, YK_DEV_ERR_BOUNDS);
        return nullptr;
    }
    return reinterpret_cast<AT*>(p.pool) + (size_t)blk * p.block_elems + p.layer_off +
           ((size_t)(kv * p.n_kv + hh) * 16 + off) * p.head_dim + c;
}

// Row pair (n, n+1), n even, of token j (SIMT GEMM).
template <int KIND, typename AT>
__device__ __forceinline__ void epi_pair(const EpiParams& p, int n, int j, float v0, float v1) {
    if (j >= p.m_tok || n >= p.n_out) return;
    if constexpr (KIND == EPI_STORE || KIND == EPI_LOGITS) {
        if constexpr (KIND == EPI_LOGITS) { v0 = logit_out(p, v0); v1 = logit_out(p, v1); }
        if (KIND == EPI_STORE && p.store_bf16) {
            __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.out) + (size_t)j * p.n_out + n;
            o[0] = __float2bfloat16_rn(v0);
            if (n + 1 < p.n_out) o[1] = __float2bfloat16_rn(v1);
            return;
        }
        float* o = reinterpret_cast<float*>(p.out) + (size_t)j * p.n_out + n;
        o[0] = v0;
        if (n + 1 < p.n_out) o[1] = v1;
    } else if constexpr (KIND == EPI_RESID) {
        if (p.ref_compat) { v0 = compat_relu(v0); v1 = compat_relu(v1); }
        float* o = p.h + (size_t)j * p.ld + n;
        o[0] = o[0] + v0;
        o[1] = o[1] + v1;
    } else if constexpr (KIND == EPI_GLU) {
        if (p.ref_compat) { v0 = compat_relu(v0); v1 = compat_relu(v1); }
        const float a = (p.act == 1 ? act_gelu_tanh(v0) : act_silu(v0)) * v1;
        reinterpret_cast<AT*>(p.out)[(size_t)j * (p.n_out >> 1) + (n >> 1)] = from_f32<AT>(a);
    } else if constexpr (KIND == EPI_QKV) {
        if (p.ref_compat) { v0 = compat_relu(v0); v1 = compat_relu(v1); }
        const int dh = p.head_dim;
        if (n < p.q_dim + p.kv_dim) {
            const int c = (n < p.q_dim ? n : n - p.q_dim) % dh;
            float cs, sn;
            rope_cs(p, c, j, cs, sn);
            const float2 r = rope_rot(v0, v1, cs, sn);
            v0 = r.x;
            v1 = r.y;
        }
        if (n < p.q_dim) {
            AT* o = reinterpret_cast<AT*>(p.out) + (size_t)j * p.q_dim + n;
            o[0] = from_f32<AT>(v0);
            o[1] = from_f32<AT>(v1);
        } else {
            const int kv = n < p.q_dim + p.kv_dim ? 0 : 1;
            const int nn = n - p.q_dim - kv * p.kv_dim;
            AT* o = pool_elem<AT>(p, kv, nn / dh, nn % dh, j);
            if (o) { o[0] = from_f32<AT>(v0); o[1] = from_f32<AT>(v1); }
        }
    }
}

// Two / four consecutive outputs with one store (o aligned to 2 / 4 elements).
__device__ __forceinline__ void store2(float* o, float a, float b) { *reinterpret_cast<float2*>(o) = make_float2(a, b); }
__device__ __forceinline__ void store2(__nv_bfloat16* o, float a, float b) {
    *reinterpret_cast<__nv_bfloat162*>(o) = __floats2bfloat162_rn(a, b);
}
__device__ __forceinline__ void store4(float* o, float a, float b, float c, float d) {
    *reinterpret_cast<float4*>(o) = make_float4(a, b, c, d);
}
__device__ __forceinline__ void store4(__nv_bfloat16* o, float a, float b, float c, float d) {
    const __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
    *reinterpret_cast<uint2*>(o) = make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
}

// Destination of QKV row n (an aligned group of rows within one head) for token
// j: the q buffer, or the token's KV-pool slot (null if its page is outside the pool).
template <typename AT>
__device__ __forceinline__ AT* qkv_dst(const EpiParams& p, int n, int j) {
    if (n < p.q_dim) return reinterpret_cast<AT*>(p.out) + (size_t)j * p.q_dim + n;
    const int kv = n < p.q_dim + p.kv_dim ? 0 : 1;
    const int nn = n - p.q_dim - kv * p.kv_dim;
    const int sh = __ffs(p.head_dim) - 1;  // head_dim is a power of two
    return pool_elem<AT>(p, kv, nn >> sh, nn & (p.head_dim - 1), j);
}

// QKV rows (n, n+1), n even, of token j with the RoPE (cos, sin) of their pair
// given (ignored for V rows): Q to the q buffer, K/V to the token's pool slot.
template <typename AT>
__device__ __forceinline__ void qkv_pair_cs(const EpiParams& p, int n, int j, float v0, float v1, float cs, float sn) {
    if (j >= p.m_tok || n >= p.n_out) return;
    if (p.ref_compat) { v0 = compat_relu(v0); v1 = compat_relu(v1); }
    if (n < p.q_dim + p.kv_dim) {
        const float2 r = rope_rot(v0, v1, cs, sn);
        v0 = r.x;
        v1 = r.y;
    }
    AT* o = qkv_dst<AT>(p, n, j);
    if (o) store2(o, v0, v1);
}
// (cos, sin) of RoPE pair index i (= dim / 2) at token j: the step's table, or computed.
__device__ __forceinline__ float2 rope_pair(const EpiParams& p, int i, int j) {
    if (p.rope_tab) return p.rope_tab[(size_t)j * (p.head_dim >> 1) + i];
    float sn, cs;
    sincosf(__fdiv_rn((float)p.pos[j], p.rope_denom[i]), &sn, &cs);
    return make_float2(cs, sn);
}
// RoPE dimension of row n within its head (Q and K rows; V rows give a value that is not used).
__device__ __forceinline__ int rope_dim(const EpiParams& p, int n) {
    return (n < p.q_dim ? n : n - p.q_dim) & (p.head_dim - 1);
}

// Drains 16 consecutive tokens j0.. of row n: one row per lane, all 32 lanes of
// the warp call it together.  Fully unrolled; the residual epilogue issues its
// 16 loads of the fp32 stream before any store.  FN: the residual epilogue also
// writes the fused norm's x and 32-row sums of squares.
template <int KIND, typename AT, bool FN = false>
__device__ __forceinline__ void drain16(const EpiParams& p, int n, int j0, const float (&v)[16]) {
    if constexpr (KIND == EPI_QKV) {
        // rows (n, n^1) form one RoPE pair: the even lane writes the pair for tokens
        // j0..j0+7, the odd lane for j0+8..j0+15 (both hold all 16 pairs)
        float w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) w[i] = __shfl_xor_sync(0xffffffffu, v[i], 1);
        if (n >= p.n_out) return;
        const bool odd = n & 1;
        const int ci = rope_dim(p, n) >> 1;
        float2 r[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {  // table reads first, all in flight together
            const int j = j0 + (odd ? i + 8 : i);
            r[i] = j < p.m_tok ? rope_pair(p, ci, j) : make_float2(1.f, 0.f);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int j = j0 + (odd ? i + 8 : i);
            const float vl = v[i], vh = v[i + 8], wl = w[i], wh = w[i + 8];
            const float x0 = odd ? wh : vl, x1 = odd ? vh : wl;
            if (j < p.m_tok) qkv_pair_cs<AT>(p, n & ~1, j, x0, x1, r[i].x, r[i].y);
        }
    } else if constexpr (KIND == EPI_GLU) {
        // rows (n, n^1) = (gate, up) of one output column: the even lane writes
        // tokens j0..j0+7, the odd lane j0+8..j0+15 (both hold all 16 pairs)
        float w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) w[i] = __shfl_xor_sync(0xffffffffu, v[i], 1);
        if (n >= p.n_out) return;
        const bool odd = n & 1;
        AT* o = reinterpret_cast<AT*>(p.out) + (n >> 1);
        // (every array index is a compile-time constant and the selects are on
        // values, so v and w stay in registers)
        if (!p.ref_compat && p.act != 1) {  // SiLU, the common case
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int j = j0 + (odd ? i + 8 : i);
                const float vl = v[i], vh = v[i + 8], wl = w[i], wh = w[i + 8];
                const float g = odd ? wh : vl, u = odd ? vh : wl;
                if (j < p.m_tok) o[(size_t)j * (p.n_out >> 1)] = from_f32<AT>(act_silu(g) * u);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int j = j0 + (odd ? i + 8 : i);
                const float vl = v[i], vh = v[i + 8], wl = w[i], wh = w[i + 8];
                float g = odd ? wh : vl, u = odd ? vh : wl;
                if (p.ref_compat) { g = compat_relu(g); u = compat_relu(u); }
                if (j < p.m_tok) o[(size_t)j * (p.n_out >> 1)] = from_f32<AT>((p.act == 1 ? act_gelu_tanh(g) : act_silu(g)) * u);
            }
        }
    } else if constexpr (KIND == EPI_RESID && !FN) {
        if (n >= p.n_out) return;
        float hv[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
            if (j0 + i < p.m_tok) hv[i] = p.h[(size_t)(j0 + i) * p.ld + n];
#pragma unroll
        for (int i = 0; i < 16; ++i)
            if (j0 + i < p.m_tok) p.h[(size_t)(j0 + i) * p.ld + n] = hv[i] + (p.ref_compat ? compat_relu(v[i]) : v[i]);
    } else if constexpr (KIND == EPI_RESID) {
        // (every lane of the warp runs this: the fused norm's group sums shuffle)
        const bool valid = n < p.n_out;
        float hv[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
            if (valid && j0 + i < p.m_tok) hv[i] = p.h[(size_t)(j0 + i) * p.ld + n];
        const float g = valid ? p.nx_g[n] : 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const bool ok = valid && j0 + i < p.m_tok;
            const float hn = ok ? hv[i] + (p.ref_compat ? compat_relu(v[i]) : v[i]) : 0.f;
            if (ok) {
                p.h[(size_t)(j0 + i) * p.ld + n] = hn;
                reinterpret_cast<__nv_bfloat16*>(p.nx_out)[(size_t)(j0 + i) * p.ld + n] = __float2bfloat16_rn(hn * g);
            }
            const float ss = warp_sum_f(hn * hn);  // this warp's 32 rows form one group
            if ((threadIdx.x & 31) == 0 && j0 + i < p.m_tok && (n & ~31) < p.n_out)
                p.nx_ss[(size_t)(n >> 5) * p.ss_ld + j0 + i] = ss;
        }
    } else {  // EPI_STORE, EPI_LOGITS
        if (n >= p.n_out) return;
        float* o = reinterpret_cast<float*>(p.out);
        if (KIND == EPI_STORE && p.store_bf16) {
            __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(p.out);
#pragma unroll
            for (int i = 0; i < 16; ++i)
                if (j0 + i < p.m_tok) ob[(size_t)(j0 + i) * p.n_out + n] = __float2bfloat16_rn(v[i]);
        } else if (KIND == EPI_STORE || (!p.ref_compat && p.cap <= 0.f)) {  // plain store
#pragma unroll
            for (int i = 0; i < 16; ++i)
                if (j0 + i < p.m_tok) o[(size_t)(j0 + i) * p.n_out + n] = v[i];
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i)
                if (j0 + i < p.m_tok) o[(size_t)(j0 + i) * p.n_out + n] = logit_out(p, v[i]);
        }
    }
}

// Residual add of rows n..n+3 of token j whose current values h were loaded by
// the caller.  FN: also the next GEMM's input bf16(h_new * g) (gains g loaded by
// the caller); returns the sum of squares of the four new values.
template <bool FN = false>
__device__ __forceinline__ float epi_quad_resid(const EpiParams& p, int n, int j, float4 v, float4 h,
                                                float4 g = float4{}) {
    if (p.ref_compat) { v.x = compat_relu(v.x); v.y = compat_relu(v.y); v.z = compat_relu(v.z); v.w = compat_relu(v.w); }
    const float4 hn = make_float4(h.x + v.x, h.y + v.y, h.z + v.z, h.w + v.w);
    *reinterpret_cast<float4*>(p.h + (size_t)j * p.ld + n) = hn;
    if constexpr (FN) {
        store4(reinterpret_cast<__nv_bfloat16*>(p.nx_out) + (size_t)j * p.ld + n, hn.x * g.x, hn.y * g.y, hn.z * g.z,
               hn.w * g.w);
        return hn.x * hn.x + hn.y * hn.y + hn.z * hn.z + hn.w * hn.w;
    }
    return 0.f;
}
// Fused norm: lanes 8g..8g+7 hold 4 rows each of the 32-row group starting at
// their first lane's row n; the group's sum of squares for token j goes to
// nx_ss[(n / 32) * ss_ld + j].  Every lane of the warp calls it.
__device__ __forceinline__ void ss_quad_groups(const EpiParams& p, int n, int j, float ss, bool write) {
    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
    ss += __shfl_xor_sync(0xffffffffu, ss, 2);
    ss += __shfl_xor_sync(0xffffffffu, ss, 4);
    if (write && (threadIdx.x & 7) == 0) p.nx_ss[(size_t)(n >> 5) * p.ss_ld + j] = ss;
}

// QKV rows n..n+3 (n % 4 == 0) of token j with the (cos, sin) of their two RoPE
// pairs loaded by the caller; one 4-element store.
template <typename AT>
__device__ __forceinline__ void epi_quad_qkv(const EpiParams& p, int n, int j, float4 v, float4 rope) {
    if (j >= p.m_tok || n >= p.n_out) return;
    if (p.ref_compat) { v.x = compat_relu(v.x); v.y = compat_relu(v.y); v.z = compat_relu(v.z); v.w = compat_relu(v.w); }
    if (n < p.q_dim + p.kv_dim) {
        const float2 r0 = rope_rot(v.x, v.y, rope.x, rope.y), r1 = rope_rot(v.z, v.w, rope.z, rope.w);
        v = make_float4(r0.x, r0.y, r1.x, r1.y);
    }
    AT* o = qkv_dst<AT>(p, n, j);
    if (o) store4(o, v.x, v.y, v.z, v.w);
}

// Rows n..n+3 (n % 4 == 0; n_out is a multiple of 4) of token j with one vector
// store (split-tile reductions).
template <int KIND, typename AT>
__device__ __forceinline__ void epi_quad(const EpiParams& p, int n, int j, float4 v) {
    if (j >= p.m_tok || n >= p.n_out) return;
    if constexpr (KIND == EPI_RESID) {
        (void)epi_quad_resid<false>(p, n, j, v, *reinterpret_cast<const float4*>(p.h + (size_t)j * p.ld + n));
    } else if constexpr (KIND == EPI_STORE || KIND == EPI_LOGITS) {
        if (KIND == EPI_LOGITS && (p.ref_compat || p.cap > 0.f)) {
            v.x = logit_out(p, v.x); v.y = logit_out(p, v.y); v.z = logit_out(p, v.z); v.w = logit_out(p, v.w);
        }
        if (KIND == EPI_STORE && p.store_bf16) {
            store4(reinterpret_cast<__nv_bfloat16*>(p.out) + (size_t)j * p.n_out + n, v.x, v.y, v.z, v.w);
            return;
        }
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + (size_t)j * p.n_out + n) = v;
    } else if constexpr (KIND == EPI_GLU) {
        float g0 = v.x, u0 = v.y, g1 = v.z, u1 = v.w;
        float a0, a1;
        if (!p.ref_compat && p.act != 1) {
            a0 = act_silu(g0) * u0;
            a1 = act_silu(g1) * u1;
        } else {
            if (p.ref_compat) { g0 = compat_relu(g0); u0 = compat_relu(u0); g1 = compat_relu(g1); u1 = compat_relu(u1); }
            a0 = (p.act == 1 ? act_gelu_tanh(g0) : act_silu(g0)) * u0;
            a1 = (p.act == 1 ? act_gelu_tanh(g1) : act_silu(g1)) * u1;
        }
        store2(reinterpret_cast<AT*>(p.out) + (size_t)j * (p.n_out >> 1) + (n >> 1), a0, a1);
    } else if constexpr (KIND == EPI_QKV) {
        const int ci = rope_dim(p, n) >> 1;
        const float2 r0 = rope_pair(p, ci, j), r1 = rope_pair(p, ci + 1, j);
        epi_quad_qkv<AT>(p, n, j, v, make_float4(r0.x, r0.y, r1.x, r1.y));
    }
}

}  // namespace yk
