// yk_attention.cu -- paged attention over block tables for the ragged verify
// batch.  Semantics of batched_paged_attention_kernel (S/gemm.metal:629-737):
// query token at position pos attends causally to keys 0..pos of its own
// sequence through that sequence's page table; GQA kv = h / (H/Hkv); score
// (q.k) * d^-1/2, soft-capped cap*tanh(s/cap) when cap > 0 (:604-606,:719-721);
// keys with pos - j >= window skipped on windowed layers
// (paged_fused_attention_kernel :572).  K is stored already rotated.
#include "yk_common.cuh"
#include "yk_internal.h"

namespace yk {

struct AttnParams {
    const void* q;        // [T][H][dh]
    void* out;            // [T][H][dh]
    const void* pool;     // [block][layer][2][Hkv][16][dh]
    const int32_t* seq_of;
    const int32_t* pos;
    const int32_t* block_tables;
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

// One warp per (token, query head).  Keys are taken 32 at a time: lane l scores
// key base+l, the block of scores updates the running max / sum, and the
// weighted V rows are accumulated with each lane owning dh/32 output dims.
template <typename AT, int DPL>
__global__ void __launch_bounds__(128) attn_simt_kernel(AttnParams p) {
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

template <typename AT>
static void launch_simt(const AttnParams& p, cudaStream_t st) {
    const int warps = p.T * p.H;
    const int blocks = (warps + 3) / 4;
    switch (p.dh) {
        case 64: attn_simt_kernel<AT, 2><<<blocks, 128, 0, st>>>(p); break;
        case 128: attn_simt_kernel<AT, 4><<<blocks, 128, 0, st>>>(p); break;
        default: attn_simt_kernel<AT, 8><<<blocks, 128, 0, st>>>(p); break;
    }
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
    if (c.dtype == YK_DTYPE_BF16) launch_simt<__nv_bfloat16>(p, m->e->stream);
    else launch_simt<float>(p, m->e->stream);
    m->e->launches++;
    YK_CHECK_CUDA(cudaGetLastError());
    return YK_OK;
}

}  // namespace yk
