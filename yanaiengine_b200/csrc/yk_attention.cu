// yk_attention.cu -- paged attention over block tables for the ragged verify
// batch.  Semantics of batched_paged_attention_kernel (S/gemm.metal:629-737):
// query token at position pos attends causally to keys 0..pos of its own
// sequence through that sequence's page table; GQA kv = h / (H/Hkv); score
// (q.k) * d^-1/2, soft-capped cap*tanh(s/cap) when cap > 0 (:604-606,:719-721);
// keys with pos - j >= window skipped on windowed layers
// (paged_fused_attention_kernel :572).  K is stored already rotated.
//
// bf16 path: one CTA per work item (sequence, KV head, 64-row query tile,
// key split).  The rows are the (token, query-head) pairs of one GQA group, so
// the k+1 verify tokens x group heads share every K/V page the CTA streams.
// 16-token pages are staged with cp.async into padded shared memory (double
// buffered), scores and P.V run on tensor cores (mma.sync m16n8k16 bf16,
// fp32 accumulate) with an online softmax in the log2 domain; split-KV
// partials are merged by a log-sum-exp combine kernel.
// fp32 path: a SIMT kernel (one warp per token x head).
#include <algorithm>
#include <vector>

#include "yk_common.cuh"
#include "yk_internal.h"

namespace yk {

struct AttnParams {
    const void* q;        // [T][H][dh]
    void* out;            // [T][H][dh]
    const void* pool;     // [block][layer][2][Hkv][16][dh]
    const int32_t* seq_of;
    const int32_t* pos;
    const int32_t* q_starts;
    const int32_t* ctx;
    const int32_t* block_tables;
    const int32_t* items;  // bf16 path: work items (b, g, qt, kbeg, kend, slot)
    const int32_t* comb;   // bf16 path: combine entries (b, g, qt, first slot, n slots)
    float* ws;             // split partials [slot][64][dh + 2]
    int max_blocks, T, H, Hkv, dh;
    long long block_elems, layer_off;
    int pool_blocks;
    float scale, cap;
    int window;
    uint32_t* err;
};

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---------------------------------------------------------------------------
// SIMT kernel (fp32 models).
// ---------------------------------------------------------------------------
template <typename AT, int DPL>
__global__ void __launch_bounds__(128) attn_simt_kernel(AttnParams p) {
    pdl_trigger();
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gw = blockIdx.x * 4 + warp;
    if (gw >= p.T * p.H) return;
    const int t = gw / p.H, h = gw % p.H;
    const int dh = p.dh;
    const int kvh = h / (p.H / p.Hkv);
    const int b = p.seq_of[t];
    const int pos = p.pos[t];
    const int jend = pos + 1;
    const int jbeg = p.window > 0 ? max(0, pos - p.window + 1) : 0;
    __shared__ float sq[4][256];
    const AT* qr = reinterpret_cast<const AT*>(p.q) + ((size_t)t * p.H + h) * dh;
    for (int i = lane; i < dh; i += 32) sq[warp][i] = to_f32(qr[i]);
    __syncwarp();
    const AT* pool = reinterpret_cast<const AT*>(p.pool);
    const int32_t* bt = p.block_tables + (size_t)b * p.max_blocks;
    float acc[DPL];
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[i] = 0.f;
    float m = -INFINITY, l = 0.f;
    for (int base = jbeg; base < jend; base += 32) {
        const int j = base + lane;
        float s = -INFINITY;
        if (j < jend) {
            const int blk = bt[j >> 4];
            if (blk < 0 || blk >= p.pool_blocks) {
                raise_err(p.err, YK_DEV_ERR_BOUNDS);
            } else {
                const AT* kp = pool + (size_t)blk * p.block_elems + p.layer_off + ((size_t)kvh * 16 + (j & 15)) * dh;
                float dot = 0.f;
                for (int i = 0; i < dh; ++i) dot = fmaf(sq[warp][i], to_f32(kp[i]), dot);
                s = dot * p.scale;
                if (p.cap > 0.f) s = p.cap * tanhf(s / p.cap);
            }
        }
        const float mb = warp_max(s);
        const float mn = fmaxf(m, mb);
        const float corr = expf(m - mn);
        const float pj = (s == -INFINITY) ? 0.f : expf(s - mn);
        l = l * corr + warp_sum(pj);
#pragma unroll
        for (int i = 0; i < DPL; ++i) acc[i] *= corr;
        const int nv = min(32, jend - base);
        for (int jj = 0; jj < nv; ++jj) {
            const float pw = __shfl_sync(0xffffffffu, pj, jj);
            const int jx = base + jj;
            const int blk = bt[jx >> 4];
            if (blk < 0 || blk >= p.pool_blocks) continue;
            const AT* vp = pool + (size_t)blk * p.block_elems + p.layer_off +
                           ((size_t)(p.Hkv + kvh) * 16 + (jx & 15)) * dh;
#pragma unroll
            for (int i = 0; i < DPL; ++i) acc[i] = fmaf(pw, to_f32(vp[lane + 32 * i]), acc[i]);
        }
        m = mn;
    }
    AT* orow = reinterpret_cast<AT*>(p.out) + ((size_t)t * p.H + h) * dh;
    const float inv = 1.0f / l;
#pragma unroll
    for (int i = 0; i < DPL; ++i) orow[lane + 32 * i] = from_f32<AT>(acc[i] * inv);
}

// ---------------------------------------------------------------------------
// Tensor-core kernel (bf16 models).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

constexpr int AT_ROWS = 64;  // query rows per CTA (4 m16 tiles)

template <int DH>
struct AttnCfg {
    static constexpr int KC = DH == 256 ? 32 : 64;  // keys per staged chunk
    static constexpr int LD = DH + 8;               // padded smem row (elements): conflict-free ldmatrix
    static constexpr int Q_ELEMS = AT_ROWS * LD;
    static constexpr int KV_ELEMS = KC * LD;        // one of K or V, one buffer
    static constexpr size_t SMEM = (size_t)(Q_ELEMS + 4 * KV_ELEMS) * 2;
    static constexpr size_t RED = (size_t)4 * 16 * (DH + 2) * 4;  // per-warp partials for the final merge
    static constexpr size_t SMEM_TOTAL = SMEM > RED + (size_t)Q_ELEMS * 2 ? SMEM : RED + (size_t)Q_ELEMS * 2;
};

template <int DH>
__global__ void __launch_bounds__(128) attn_mma_kernel(AttnParams p) {
    using C = AttnCfg<DH>;
    constexpr int KC = C::KC, LD = C::LD;
    constexpr int NT = DH / 8;   // n-tiles of the output
    constexpr int KS = DH / 16;  // k-steps of the score MMA
    extern __shared__ __align__(16) uint8_t smem_raw[];
    __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem_raw);
    __nv_bfloat16* sK = sQ + C::Q_ELEMS;        // [2][KC][LD]
    __nv_bfloat16* sV = sK + 2 * C::KV_ELEMS;   // [2][KC][LD]
    pdl_trigger();
    pdl_wait();

    const int32_t* it = p.items + (size_t)blockIdx.x * 6;
    const int b = it[0], g = it[1], qt = it[2], kbeg = it[3], kend = it[4], slot = it[5];
    const int G = p.H / p.Hkv;
    const int qs0 = p.q_starts[b];
    const int n = p.q_starts[b + 1] - qs0;
    const int ctx = p.ctx[b];
    const int rows = min(AT_ROWS, n * G - qt * AT_ROWS);
    const int MT = (rows + 15) >> 4;
    const int wpm = MT == 1 ? min(4, KC / 16) : (MT == 2 ? min(2, KC / 16) : 1);
    const int KW = KC / wpm;  // keys per warp per chunk
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int my_mt = warp / wpm, my_part = warp % wpm;
    const bool active = my_mt < MT;
    const __nv_bfloat16* q = reinterpret_cast<const __nv_bfloat16*>(p.q);
    const __nv_bfloat16* pool = reinterpret_cast<const __nv_bfloat16*>(p.pool);
    const int32_t* bt = p.block_tables + (size_t)b * p.max_blocks;

    // ---- stage Q (64 rows x DH), zero rows beyond `rows`
    constexpr int CPR = DH / 8;  // 16-byte chunks per row
    for (int i = threadIdx.x; i < AT_ROWS * CPR; i += 128) {
        const int r = i / CPR, c = i % CPR;
        const int rr = qt * AT_ROWS + r;
        const bool ok = r < rows;
        const __nv_bfloat16* src = q;
        if (ok) src = q + ((size_t)(qs0 + rr / G) * p.H + (size_t)g * G + rr % G) * DH + c * 8;
        cp_async16(smem_u32(sQ + r * LD + c * 8), src, ok ? 16u : 0u);
    }
    // ---- K/V chunk loader: pages of 16 keys, rows beyond kend zero-filled
    auto load_chunk = [&](int c0, int buf) {
        __nv_bfloat16* dk = sK + buf * C::KV_ELEMS;
        __nv_bfloat16* dv = sV + buf * C::KV_ELEMS;
        for (int i = threadIdx.x; i < KC * CPR; i += 128) {
            const int r = i / CPR, c = i % CPR;
            const int j = c0 + r;
            bool ok = j < kend;
            const __nv_bfloat16* srck = pool;
            const __nv_bfloat16* srcv = pool;
            if (ok) {
                const int blk = bt[j >> 4];
                if (blk < 0 || blk >= p.pool_blocks) {
                    raise_err(p.err, YK_DEV_ERR_BOUNDS);
                    ok = false;
                } else {
                    const size_t base = (size_t)blk * p.block_elems + p.layer_off + (size_t)(j & 15) * DH + c * 8;
                    srck = pool + base + (size_t)g * 16 * DH;
                    srcv = pool + base + (size_t)(p.Hkv + g) * 16 * DH;
                }
            }
            cp_async16(smem_u32(dk + r * LD + c * 8), srck, ok ? 16u : 0u);
            cp_async16(smem_u32(dv + r * LD + c * 8), srcv, ok ? 16u : 0u);
        }
    };
    const int nchunks = (kend - kbeg + KC - 1) / KC;
    load_chunk(kbeg, 0);
    cp_async_commit();

    // per-lane rows (m-tile rows lane/4 and lane/4+8) and their positions
    const int r0 = my_mt * 16 + (lane >> 2), r1 = r0 + 8;
    const int pos0 = (r0 < rows) ? ctx - n + (qt * AT_ROWS + r0) / G : -1;
    const int pos1 = (r1 < rows) ? ctx - n + (qt * AT_ROWS + r1) / G : -1;
    // last key any row of this warp's m-tile can see (warp-uniform skip test)
    int wmaxpos = max(pos0, pos1);
#pragma unroll
    for (int o2 = 16; o2 > 0; o2 >>= 1) wmaxpos = max(wmaxpos, __shfl_xor_sync(0xffffffffu, wmaxpos, o2));
    const float LOG2E = 1.4426950408889634f;
    float o[NT][4];
#pragma unroll
    for (int t = 0; t < NT; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    uint32_t qf[DH <= 128 ? KS : 1][4];

    for (int c = 0; c < nchunks; ++c) {
        if (c + 1 < nchunks) load_chunk(kbeg + (c + 1) * KC, (c + 1) & 1);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        if (c == 0 && DH <= 128 && active) {
#pragma unroll
            for (int ks = 0; ks < (DH <= 128 ? KS : 1); ++ks) {
                const uint32_t a = smem_u32(sQ + (my_mt * 16 + (lane & 15)) * LD + ks * 16 + (lane >> 4) * 8);
                ldsm_x4(a, qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3]);
            }
        }
        if (active) {
            const __nv_bfloat16* ck = sK + (c & 1) * C::KV_ELEMS;
            const __nv_bfloat16* cv = sV + (c & 1) * C::KV_ELEMS;
            for (int sb = 0; sb < KW; sb += 16) {
                const int kr = my_part * KW + sb;   // key row within the chunk
                const int j0 = kbeg + c * KC + kr;  // first key of this 16-block
                if (j0 >= kend || j0 > wmaxpos) continue;  // whole 16-key block masked for the m-tile
                // S = Q K^T : two n8 tiles (keys j0..j0+7, j0+8..j0+15)
                float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
                for (int ks = 0; ks < KS; ks += 2) {
                    uint32_t a[2][4];
                    if constexpr (DH <= 128) {
#pragma unroll
                        for (int u = 0; u < 4; ++u) { a[0][u] = qf[ks][u]; a[1][u] = qf[ks + 1][u]; }
                    } else {
#pragma unroll
                        for (int h2 = 0; h2 < 2; ++h2) {
                            const uint32_t aa =
                                smem_u32(sQ + (my_mt * 16 + (lane & 15)) * LD + (ks + h2) * 16 + (lane >> 4) * 8);
                            ldsm_x4(aa, a[h2][0], a[h2][1], a[h2][2], a[h2][3]);
                        }
                    }
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt) {
                        uint32_t b0, b1, b2, b3;
                        const uint32_t ba = smem_u32(ck + (kr + nt * 8 + (lane & 7)) * LD + ks * 16 + (lane >> 3) * 8);
                        ldsm_x4(ba, b0, b1, b2, b3);
                        mma_bf16(s[nt], a[0][0], a[0][1], a[0][2], a[0][3], b0, b1);
                        mma_bf16(s[nt], a[1][0], a[1][1], a[1][2], a[1][3], b2, b3);
                    }
                }
                // scale, cap, mask (log2 domain)
                float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int j = j0 + nt * 8 + 2 * (lane & 3) + (e & 1);
                        const int ps = (e < 2) ? pos0 : pos1;
                        float x = s[nt][e] * p.scale;
                        if (p.cap > 0.f) x = p.cap * tanhf(x / p.cap);
                        x *= LOG2E;
                        const bool masked = j >= kend || j > ps || (p.window > 0 && ps - j >= p.window);
                        x = masked ? -INFINITY : x;
                        s[nt][e] = x;
                        if (e < 2) mx0 = fmaxf(mx0, x); else mx1 = fmaxf(mx1, x);
                    }
                }
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
                const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
                const float mu0 = mn0 == -INFINITY ? 0.f : mn0, mu1 = mn1 == -INFINITY ? 0.f : mn1;
                const float c0f = exp2f(m0 - mu0), c1f = exp2f(m1 - mu1);
                float ps[2][4];
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) {
                    ps[nt][0] = exp2f(s[nt][0] - mu0);
                    ps[nt][1] = exp2f(s[nt][1] - mu0);
                    ps[nt][2] = exp2f(s[nt][2] - mu1);
                    ps[nt][3] = exp2f(s[nt][3] - mu1);
                }
                l0 = l0 * c0f + ps[0][0] + ps[0][1] + ps[1][0] + ps[1][1];
                l1 = l1 * c1f + ps[0][2] + ps[0][3] + ps[1][2] + ps[1][3];
                m0 = mn0;
                m1 = mn1;
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    o[t][0] *= c0f; o[t][1] *= c0f;
                    o[t][2] *= c1f; o[t][3] *= c1f;
                }
                const uint32_t pa0 = pack_bf16(ps[0][0], ps[0][1]), pa1 = pack_bf16(ps[0][2], ps[0][3]);
                const uint32_t pa2 = pack_bf16(ps[1][0], ps[1][1]), pa3 = pack_bf16(ps[1][2], ps[1][3]);
                // O += P V : V rows kr..kr+15, output n-tiles in pairs
#pragma unroll
                for (int t = 0; t < NT; t += 2) {
                    uint32_t b0, b1, b2, b3;
                    const uint32_t va = smem_u32(cv + (kr + (lane & 7) + ((lane >> 3) & 1) * 8) * LD + t * 8 + (lane >> 4) * 8);
                    ldsm_x4_t(va, b0, b1, b2, b3);
                    mma_bf16(o[t], pa0, pa1, pa2, pa3, b0, b1);
                    mma_bf16(o[t + 1], pa0, pa1, pa2, pa3, b2, b3);
                }
            }
        }
        __syncthreads();
    }
    cp_async_wait<0>();
    // ---- merge the warps of each m-tile through shared memory, then write
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    float* red = reinterpret_cast<float*>(smem_raw + (size_t)C::Q_ELEMS * 2);  // [4 warps][16][DH + 2]
    __syncthreads();
    if (active) {
        float* rw = red + (size_t)warp * 16 * (DH + 2);
        const int lr = lane >> 2;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const int col = t * 8 + 2 * (lane & 3);
            rw[lr * (DH + 2) + 2 + col] = o[t][0];
            rw[lr * (DH + 2) + 3 + col] = o[t][1];
            rw[(lr + 8) * (DH + 2) + 2 + col] = o[t][2];
            rw[(lr + 8) * (DH + 2) + 3 + col] = o[t][3];
        }
        if ((lane & 3) == 0) {
            rw[lr * (DH + 2)] = m0;
            rw[lr * (DH + 2) + 1] = l0;
            rw[(lr + 8) * (DH + 2)] = m1;
            rw[(lr + 8) * (DH + 2) + 1] = l1;
        }
    }
    __syncthreads();
    __nv_bfloat16* outp = reinterpret_cast<__nv_bfloat16*>(p.out);
    for (int i = threadIdx.x; i < rows * DH; i += 128) {
        const int r = i / DH, col = i % DH;
        const int mt = r >> 4, lr = r & 15;
        float M = -INFINITY;
        for (int w = 0; w < wpm; ++w) M = fmaxf(M, red[((size_t)(mt * wpm + w) * 16 + lr) * (DH + 2)]);
        const float Mu = M == -INFINITY ? 0.f : M;
        float L = 0.f, O = 0.f;
        for (int w = 0; w < wpm; ++w) {
            const float* rw = red + ((size_t)(mt * wpm + w) * 16 + lr) * (DH + 2);
            const float f = exp2f(rw[0] - Mu);
            L += f * rw[1];
            O += f * rw[2 + col];
        }
        const int rr = qt * AT_ROWS + r;
        if (slot < 0) {
            outp[((size_t)(qs0 + rr / G) * p.H + (size_t)g * G + rr % G) * DH + col] =
                __float2bfloat16_rn(L > 0.f ? O / L : 0.f);
        } else {
            float* wsr = p.ws + ((size_t)slot * AT_ROWS + r) * (DH + 2);
            wsr[2 + col] = O;
            if (col == 0) { wsr[0] = M; wsr[1] = L; }
        }
    }
}

// Split-KV merge: one CTA per (sequence, KV head, query tile) with > 1 split.
template <int DH>
__global__ void __launch_bounds__(128) attn_combine_kernel(AttnParams p) {
    pdl_trigger();
    pdl_wait();
    const int32_t* e = p.comb + (size_t)blockIdx.x * 5;
    const int b = e[0], g = e[1], qt = e[2], first = e[3], ns = e[4];
    const int G = p.H / p.Hkv;
    const int qs0 = p.q_starts[b];
    const int n = p.q_starts[b + 1] - qs0;
    const int rows = min(AT_ROWS, n * G - qt * AT_ROWS);
    __nv_bfloat16* outp = reinterpret_cast<__nv_bfloat16*>(p.out);
    for (int i = threadIdx.x; i < rows * DH; i += 128) {
        const int r = i / DH, col = i % DH;
        float M = -INFINITY;
        for (int s = 0; s < ns; ++s) M = fmaxf(M, p.ws[((size_t)(first + s) * AT_ROWS + r) * (DH + 2)]);
        const float Mu = M == -INFINITY ? 0.f : M;
        float L = 0.f, O = 0.f;
        for (int s = 0; s < ns; ++s) {
            const float* w = p.ws + ((size_t)(first + s) * AT_ROWS + r) * (DH + 2);
            const float f = exp2f(w[0] - Mu);
            L += f * w[1];
            O += f * w[2 + col];
        }
        const int rr = qt * AT_ROWS + r;
        outp[((size_t)(qs0 + rr / G) * p.H + (size_t)g * G + rr % G) * DH + col] =
            __float2bfloat16_rn(L > 0.f ? O / L : 0.f);
    }
}

template <typename AT>
static cudaError_t launch_simt(const AttnParams& p, yk_engine* e) {
    const int warps = p.T * p.H;
    const int blocks = (warps + 3) / 4;
    switch (p.dh) {
        case 64: return launch_pdl(e, attn_simt_kernel<AT, 2>, blocks, 128, 0, p);
        case 128: return launch_pdl(e, attn_simt_kernel<AT, 4>, blocks, 128, 0, p);
        default: return launch_pdl(e, attn_simt_kernel<AT, 8>, blocks, 128, 0, p);
    }
}

template <int DH>
static yk_status launch_mma(const AttnParams& p, int n_items, int n_comb, yk_engine* e) {
    const size_t smem = AttnCfg<DH>::SMEM_TOTAL;
    static bool attr = false;
    if (!attr) {
        YK_CHECK_CUDA(cudaFuncSetAttribute(attn_mma_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        attr = true;
    }
    YK_CHECK_CUDA(launch_pdl(e, attn_mma_kernel<DH>, n_items, 128, smem, p));
    e->launches++;
    if (n_comb > 0) {
        YK_CHECK_CUDA(launch_pdl(e, attn_combine_kernel<DH>, n_comb, 128, 0, p));
        e->launches++;
    }
    return YK_OK;
}

// Work list for one forward step and one window setting (see yk_forward_step).
void plan_attention(const yk_model_config& c, int num_sms, const uint32_t* q_starts, const uint32_t* ctx, int B,
                    bool windowed, std::vector<int32_t>& items, std::vector<int32_t>& comb, int* n_slots) {
    const int G = c.n_heads / c.n_kv_heads;
    const int KC = c.head_dim == 256 ? 32 : 64;
    struct Span { int b, qt, kb, ke; };
    std::vector<Span> spans;
    long long total = 0;
    for (int b = 0; b < B; ++b) {
        const int n = (int)(q_starts[b + 1] - q_starts[b]);
        if (n == 0) continue;
        const int rows = n * G;
        for (int qt = 0; qt * AT_ROWS < rows; ++qt) {
            const int i_lo = (qt * AT_ROWS) / G, i_hi = (std::min(rows, qt * AT_ROWS + AT_ROWS) - 1) / G;
            const int pos_lo = (int)ctx[b] - n + i_lo, pos_hi = (int)ctx[b] - n + i_hi;
            int kb = windowed ? std::max(0, pos_lo - c.window + 1) : 0;
            kb = (kb / KC) * KC;
            const int ke = pos_hi + 1;
            spans.push_back({b, qt, kb, ke});
            total += (long long)(ke - kb) * c.n_kv_heads;
        }
    }
    const long long target_items = 3LL * num_sms;
    long long ks = (total + target_items - 1) / std::max(1LL, target_items);
    ks = std::max<long long>(KC, ((ks + KC - 1) / KC) * KC);
    items.clear();
    comb.clear();
    int slot = 0;
    for (const auto& s : spans) {
        const int ns = (int)((s.ke - s.kb + ks - 1) / ks);
        for (int g = 0; g < c.n_kv_heads; ++g) {
            if (ns <= 1) {
                items.insert(items.end(), {s.b, g, s.qt, s.kb, s.ke, -1});
            } else {
                comb.insert(comb.end(), {s.b, g, s.qt, slot, ns});
                for (int i = 0; i < ns; ++i) {
                    const int kb = s.kb + (int)(i * ks), ke = std::min(s.ke, s.kb + (int)((i + 1) * ks));
                    items.insert(items.end(), {s.b, g, s.qt, kb, ke, slot++});
                }
            }
        }
    }
    *n_slots = slot;
}

yk_status attention_run(yk_model* m, yk_kv_pool* pool, int layer, int T, int B, int max_blocks, double kv_bytes) {
    (void)B;
    const auto& c = m->cfg;
    const double es = c.dtype == YK_DTYPE_BF16 ? 2.0 : 4.0;
    ProfScope prof(m->e, YK_PROF_ATTN, kv_bytes + 2.0 * T * c.n_heads * c.head_dim * es, 0.0);
    AttnParams p;
    p.q = m->q;
    p.out = m->att;
    p.pool = pool->data;
    p.seq_of = m->cur.seq;
    p.pos = m->cur.pos;
    p.q_starts = m->cur.q_starts;
    p.ctx = m->cur.ctx;
    p.block_tables = m->cur.bt;
    p.max_blocks = max_blocks;
    p.T = T;
    p.H = c.n_heads;
    p.Hkv = c.n_kv_heads;
    p.dh = c.head_dim;
    p.block_elems = (long long)pool->block_elems;
    p.layer_off = (long long)layer * (long long)pool->layer_elems;
    p.pool_blocks = pool->num_blocks;
    p.scale = 1.0f / sqrtf((float)c.head_dim);
    p.cap = c.attn_cap;
    const bool windowed = c.window > 0 && (c.window_layer_parity < 0 || (layer % 2) == c.window_layer_parity);
    p.window = windowed ? c.window : 0;
    p.err = m->e->d_err;
    p.ws = m->attn_ws;
    if (c.dtype != YK_DTYPE_BF16) {
        YK_CHECK_CUDA(launch_simt<float>(p, m->e));
        m->e->launches++;
        return YK_OK;
    }
    const int w = windowed ? 1 : 0;
    p.items = m->cur.attn_items[w];
    p.comb = m->cur.attn_comb[w];
    const int ni = m->cur.n_items[w], nc = m->cur.n_comb[w];
    switch (c.head_dim) {
        case 64: return launch_mma<64>(p, ni, nc, m->e);
        case 128: return launch_mma<128>(p, ni, nc, m->e);
        default: return launch_mma<256>(p, ni, nc, m->e);
    }
}

size_t attention_ws_floats_per_slot(int head_dim) { return (size_t)AT_ROWS * (head_dim + 2); }

}  // namespace yk
