// yk_attention.cu -- paged attention over block tables for the ragged verify
// batch.  Semantics of batched_paged_attention_kernel (S/gemm.metal:629-737):
// query token at position pos attends causally to keys 0..pos of its own
// sequence through that sequence's page table; GQA kv = h / (H/Hkv); score
// (q.k) * d^-1/2, soft-capped cap*tanh(s/cap) when cap > 0 (:604-606,:719-721);
// keys with pos - j >= window skipped on windowed layers
// (paged_fused_attention_kernel :572).  K is stored already rotated.
//
// bf16 path: one CTA per work item (sequence, KV head, 64-row query tile,
// key range).  The rows are the (token, query-head) pairs of one GQA group, so
// the k+1 verify tokens x group heads share every K/V page the CTA streams.
// A producer warp streams 16-token K and V pages by TMA (a 3-D tensor map over
// the pool, 128-byte swizzle) into an mbarrier ring of pages; consumer warps
// compute scores and P.V on tensor cores (mma.sync m16n8k16 bf16, fp32
// accumulate) with an online softmax in the log2 domain.  Items cut along the
// keys publish (M, L, O) partials and the last CTA of the group to finish
// merges them in split order.
// fp32 path: a SIMT kernel (one warp per token x head).
#include <algorithm>
#include <climits>
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
    const int32_t* items;  // bf16 path: work items (b, g, qt, kbeg, kend, slot, combine group)
    const int32_t* comb;   // bf16 path: combine groups (b, g, qt, first slot, n slots)
    int32_t* counters;     // bf16 path: per combine group arrival counters (zero between launches)
    float* ws;             // split partials [slot][64][dh + 4]: (M, L, -, -, O[dh])
    int layer;
    unsigned long long* stamps;  // test hook: 8 words per CTA, else null
    Trace tr;
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
//
// One CTA per work item (sequence b, KV head g, query tile qt, key range
// [kbeg, kend)): 4 consumer warps + 1 producer warp.  The producer streams the
// item's 16-token pages (K page, then V page) with TMA through a 3-D tensor map
// over the pool (x = head dim, y = row within the block, z = block) into an
// mbarrier ring, 128-byte swizzled so the ldmatrix reads below are conflict
// free.  Pages that precede this step's new tokens were not written by the
// previous kernel and are requested before the grid dependency wait.  Consumer
// warp (m-tile mt, part) takes pages part, part + wpm, ... of the item for its
// 16 query rows: S = Q K^T and O += P V on tensor cores (mma.sync m16n8k16
// bf16, fp32 accumulate), online softmax in the log2 domain.  Items cut along
// the keys publish (M, L, O) partials; the last of them to finish merges all
// partials in split order (deterministic) and writes the output.
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
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int32_t x, int32_t y, int32_t z,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
        "l"((uint64_t)map), "r"(x), "r"(y), "r"(z), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void consumer_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

constexpr int AT_ROWS = 64;       // query rows per item (4 m16 tiles)
constexpr int AT_THREADS = 160;   // warps 0-3 consumers, warp 4 producer
constexpr int AT_ITEM_INTS = 7;   // b, g, qt, kbeg, kend, slot, combine group
constexpr int AT_COMB_INTS = 5;   // b, g, qt, first slot, n slots
constexpr int AT_MAX_SPLITS = 64; // key splits per (sequence, KV head, query tile)

template <int DH>
struct AttnCfg {
    static constexpr int BOXES = DH / 64;                    // 64-column TMA boxes per K (or V) page
    static constexpr uint32_t HALF = 16u * DH * 2u;          // bytes of one K (or V) page
    static constexpr uint32_t STAGE = 2u * HALF;
    // A consumer warp takes chunks of CP pages.  Stages: a multiple of 4*CP (4 =
    // every warps-per-m-tile value), so a consumer that waits only on its own
    // chunks never waits two phases ahead of a stage.
    // Ring depth: a warp's chunk time is mostly page latency, so what sets a
    // CTA's rate is how many pages the ring holds beyond the ones in use.  With
    // one-page chunks only one page per consuming warp is in use (decode-like,
    // head_dim 64: 4 of 12 pages; verify, 2 m-tiles x 2 warps: 2 of 12), the rest
    // stream ahead (two-page chunks: 1.5 % slower per step, target and draft).
    // head_dim 128: 12 pages at 2 CTAs per SM (the Q tile lives in registers, so
    // they fit; 8 pages: verify attention 46.8 -> 47.9 us; 3 CTAs per SM with 8
    // pages: slower).  head_dim 64 (decode-shaped draft): resident slots matter
    // more than depth there (the planner splits long spans over the spare slots):
    // 4 CTAs per SM (96 registers) with 12 pages beat 3 with 16 and 2 with 24.
    // head_dim 256 (Gemma): the consumer warps, not the ring, set the rate (8 or 12
    // pages stream no faster than 4 at one CTA per SM, 34 GB/s per CTA); two CTAs per
    // SM with 4-page rings (168 registers, a few spilled) stream 5.7 TB/s on the
    // 9B-shape verify (657 -> 482 us per layer) and the 2B-shape decode 323 -> 276 us.
    static constexpr int CP = 1;
    static constexpr int S = DH == 256 ? 4 : 12;
    static constexpr int CTAS_PER_SM = DH == 64 ? 4 : 2;  // registers / shared memory
    static constexpr int LDQ = DH + 8;                       // padded Q row (elements)
    // head_dim <= 128: Q goes straight from global memory into the score MMA's A
    // fragments (registers), no shared-memory copy; the room goes to the ring
    static constexpr size_t Q_BYTES = DH <= 128 ? 0 : (size_t)AT_ROWS * LDQ * 2;
    // after the page loop the ring holds the merge: per-warp O and (m, l), per-row
    // weights; or, for the last CTA of a split group, per-row split weights
    static constexpr size_t RED_BYTES = ((size_t)4 * 16 * DH + 4 * 16 * 2 + 64 * 4 + 64 * 2) * 4;
    static constexpr size_t SPLIT_BYTES = ((size_t)64 * 64 + 64) * 4;
    static constexpr size_t RMAX = RED_BYTES > SPLIT_BYTES ? RED_BYTES : SPLIT_BYTES;
    static constexpr size_t RING = (size_t)S * STAGE > RMAX ? (size_t)S * STAGE : RMAX;
    static constexpr size_t SMEM = 1024 + RING + Q_BYTES + (size_t)2 * S * 8 + 16;
};
// Split partial row: (M, L, -, -) then O[DH]; rows 16-byte aligned.
__host__ __device__ constexpr int ws_row(int dh) { return dh + 4; }

// Byte offset of 16-byte chunk c of row r (key within the page) in a K or V page
// written by TMA with 128-byte swizzle: 64-column boxes of 16 rows x 128 B.
__device__ __forceinline__ uint32_t sw_off(int r, int c) {
    return (uint32_t)((c >> 3) * 2048 + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

template <int DH>
__global__ void __launch_bounds__(AT_THREADS, AttnCfg<DH>::CTAS_PER_SM)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmKV, AttnParams p) {
    using C = AttnCfg<DH>;
    constexpr int NT = DH / 8;   // n-tiles of the output
    constexpr int KS = DH / 16;  // k-steps of the score MMA
    constexpr int S = C::S;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(ring + C::RING);
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + C::RING + C::Q_BYTES);
    uint64_t* empty = full + S;
    volatile int* flags = reinterpret_cast<volatile int*>(empty + S);  // [0] last arriver

    const int32_t* it = p.items + (size_t)blockIdx.x * AT_ITEM_INTS;
    const int b = it[0], g = it[1], qt = it[2], kbeg = it[3], kend = it[4], slot = it[5], cg = it[6];
    const int G = p.H / p.Hkv;
    const int qs0 = p.q_starts[b];
    const int n = p.q_starts[b + 1] - qs0;
    const int ctx = p.ctx[b];
    const int rows = min(AT_ROWS, n * G - qt * AT_ROWS);
    const int MT = (rows + 15) >> 4;
    const int wpm = MT == 1 ? 4 : (MT == 2 ? 2 : 1);
    const int pg0 = kbeg >> 4;
    const int npages = (kend - kbeg + 15) >> 4;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        trace_mark(p.tr, TR_ENTRY);
        for (int s = 0; s < S; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), (uint32_t)MT);
        }
        flags[0] = 0;
        mbar_fence_init();
    }
    __syncthreads();
    pdl_trigger();
    unsigned long long* stp = p.stamps ? p.stamps + (size_t)blockIdx.x * 8 : nullptr;
    if (stp && threadIdx.x == 0) {
        uint32_t smid;
        asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
        stp[0] = globaltimer_ns();
        stp[1] = 0;
        stp[4] = (unsigned long long)npages;
        stp[5] = smid;
        stp[6] = gridDim.x;
    }

    if (warp == 4) {
        // ---------------- producer ----------------
        const int32_t* bt = p.block_tables + (size_t)b * p.max_blocks;
        // pages entirely before this step's first new token: untouched by the previous kernel
        const int first_new = ctx - n;
        int pre = 0;
        while (pre < S && pre < npages && (pg0 + pre + 1) * 16 <= first_new) ++pre;
        bool stop = false;
        int issued = 0;
        for (int c0 = 0; c0 < npages; c0 += 32) {
            int bid = 0;
            if (c0 + lane < npages) {
                bid = bt[pg0 + c0 + lane];
                if (bid < 0 || bid >= p.pool_blocks) {
                    raise_err(p.err, YK_DEV_ERR_BOUNDS);
                    bid = 0;
                }
            }
            const int cend = min(npages, c0 + 32);
            for (int i = c0; i < cend; ++i) {
                if (i == pre) pdl_wait();
                const int blk = __shfl_sync(0xffffffffu, bid, i - c0);
                if (lane == 0 && !stop) {
                    const int s = i % S;
                    if (i >= S && !mbar_wait_bounded(smem_u32(&empty[s]), (uint32_t)(((i / S) - 1) & 1))) {
                        raise_err(p.err, YK_DEV_ERR_TIMEOUT);
                        stop = true;
                    } else {
                        const uint32_t fb = smem_u32(&full[s]);
                        const uint32_t dst = smem_u32(ring + (size_t)s * C::STAGE);
                        const int yk = ((p.layer * 2 + 0) * p.Hkv + g) * 16;
                        const int yv = ((p.layer * 2 + 1) * p.Hkv + g) * 16;
                        mbar_arrive_expect_tx(fb, C::STAGE);
#pragma unroll
                        for (int bx = 0; bx < C::BOXES; ++bx) {
                            tma_load_3d(dst + bx * 2048u, &tmKV, bx * 64, yk, blk, fb);
                            tma_load_3d(dst + C::HALF + bx * 2048u, &tmKV, bx * 64, yv, blk, fb);
                        }
                        issued = i + 1;
                    }
                }
                __syncwarp();
            }
        }
        if (pre >= npages) pdl_wait();
        // every issued page must land before the CTA may exit
        if (lane == 0)
            for (int i = max(0, issued - S); i < issued; ++i)
                (void)mbar_wait_bounded(smem_u32(&full[i % S]), (uint32_t)((i / S) & 1));
        return;
    }

    // ---------------- consumers: warps 0..3 ----------------
    pdl_wait();
    if (threadIdx.x == 0) trace_mark(p.tr, TR_START);
    const int my_mt = warp / wpm, my_part = warp % wpm;
    const bool active = my_mt < MT;
    const __nv_bfloat16* q = reinterpret_cast<const __nv_bfloat16*>(p.q);
    if constexpr (DH > 128) {
        // stage Q (64 rows x DH, padded rows), zero rows beyond `rows`
        constexpr int CPR = DH / 8;  // 16-byte chunks per row
        for (int i = threadIdx.x; i < AT_ROWS * CPR; i += 128) {
            const int r = i / CPR, c = i % CPR;
            const int rr = qt * AT_ROWS + r;
            const bool ok = r < rows;
            const __nv_bfloat16* src = q;
            if (ok) src = q + ((size_t)(qs0 + rr / G) * p.H + (size_t)g * G + rr % G) * DH + c * 8;
            cp_async16(smem_u32(sQ + r * C::LDQ + c * 8), src, ok ? 16u : 0u);
        }
        cp_async_commit();
        cp_async_wait<0>();
        consumer_bar();
    }

    const int r0 = my_mt * 16 + (lane >> 2), r1 = r0 + 8;
    const int pos0 = (r0 < rows) ? ctx - n + (qt * AT_ROWS + r0) / G : -1;
    const int pos1 = (r1 < rows) ? ctx - n + (qt * AT_ROWS + r1) / G : -1;
    // last key any row of this warp's m-tile sees, and the first position of its
    // valid rows (rows past `rows` are zero queries whose results are never written)
    int wmaxpos = max(pos0, pos1);
    int wminpos = min(r0 < rows ? pos0 : INT_MAX, r1 < rows ? pos1 : INT_MAX);
#pragma unroll
    for (int o2 = 16; o2 > 0; o2 >>= 1) {
        wmaxpos = max(wmaxpos, __shfl_xor_sync(0xffffffffu, wmaxpos, o2));
        wminpos = min(wminpos, __shfl_xor_sync(0xffffffffu, wminpos, o2));
    }
    const float LOG2E = 1.4426950408889634f;
    const float qk2 = p.scale * LOG2E;  // score -> log2 domain in one multiply (no soft cap)
    float o[NT][4];
#pragma unroll
    for (int t = 0; t < NT; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    uint32_t qf[DH <= 128 ? KS : 1][4];
    if (DH <= 128 && active) {
        // A fragments of the m16k16 tiles: registers {0,1,2,3} hold rows (r, r+8, r,
        // r+8), columns (c, c, c+8, c+8) with r = lane/4, c = 2*(lane%4) -- the
        // ldmatrix.x4 order; rows past `rows` are zero queries
        const uint32_t* qrow[2] = {nullptr, nullptr};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int r = my_mt * 16 + (lane >> 2) + 8 * h;
            const int rr = qt * AT_ROWS + r;
            if (r < rows)
                qrow[h] = reinterpret_cast<const uint32_t*>(
                    q + ((size_t)(qs0 + rr / G) * p.H + (size_t)g * G + rr % G) * DH + 2 * (lane & 3));
        }
#pragma unroll
        for (int ks = 0; ks < (DH <= 128 ? KS : 1); ++ks) {
            // (L2 loads: Q was written by the previous kernel, after PDL overlap)
            qf[ks][0] = qrow[0] ? __ldcg(qrow[0] + ks * 8) : 0u;
            qf[ks][1] = qrow[1] ? __ldcg(qrow[1] + ks * 8) : 0u;
            qf[ks][2] = qrow[0] ? __ldcg(qrow[0] + ks * 8 + 4) : 0u;
            qf[ks][3] = qrow[1] ? __ldcg(qrow[1] + ks * 8 + 4) : 0u;
        }
    }
    constexpr int CP = C::CP;          // pages per chunk
    constexpr int NS = 2 * CP;         // n8 score tiles per chunk
    const int nchunks = (npages + CP - 1) / CP;
    bool ok = true;
    if (active) {
        for (int ch = my_part; ch < nchunks; ch += wpm) {
            const int i0 = ch * CP;
            const int np = min(CP, npages - i0);  // pages in this chunk
#pragma unroll
            for (int u = 0; u < CP; ++u) {
                const int i = i0 + u;
                if (u < np && ok && !mbar_wait_bounded(smem_u32(&full[i % S]), (uint32_t)((i / S) & 1))) {
                    raise_err(p.err, YK_DEV_ERR_TIMEOUT);
                    ok = false;
                }
            }
            if (stp && ch == 0 && lane == 0) stp[1] = globaltimer_ns();
            const int j0 = (pg0 + i0) * 16;
            if (ok && j0 <= wmaxpos) {
                uint32_t kb[CP], vb[CP];
#pragma unroll
                for (int u = 0; u < CP; ++u) {
                    // a missing second page (odd page count) reads the first again; its keys are masked
                    const int i = i0 + (u < np ? u : 0);
                    kb[u] = smem_u32(ring + (size_t)(i % S) * C::STAGE);
                    vb[u] = kb[u] + C::HALF;
                }
                // S = Q K^T : NS n8 tiles, even and odd k-steps in separate accumulators
                float sc[NS][4], sd[NS][4];
#pragma unroll
                for (int nt = 0; nt < NS; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) sc[nt][e] = sd[nt][e] = 0.f;
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
                                smem_u32(sQ + (my_mt * 16 + (lane & 15)) * C::LDQ + (ks + h2) * 16 + (lane >> 4) * 8);
                            ldsm_x4(aa, a[h2][0], a[h2][1], a[h2][2], a[h2][3]);
                        }
                    }
#pragma unroll
                    for (int nt = 0; nt < NS; ++nt) {
                        uint32_t b0, b1, b2, b3;
                        ldsm_x4(kb[nt >> 1] + sw_off((nt & 1) * 8 + (lane & 7), ks * 2 + (lane >> 3)), b0, b1, b2, b3);
                        mma_bf16(sc[nt], a[0][0], a[0][1], a[0][2], a[0][3], b0, b1);
                        mma_bf16(sd[nt], a[1][0], a[1][1], a[1][2], a[1][3], b2, b3);
                    }
                }
                // scale, cap, mask (log2 domain).  Fast path: every key of the chunk is
                // visible to every valid row of the warp and there is no soft cap.
                float mx0 = -INFINITY, mx1 = -INFINITY;
                const bool fast = np == CP && p.cap <= 0.f && j0 >= kbeg && j0 + 16 * CP <= kend &&
                                  j0 + 16 * CP - 1 <= wminpos && (p.window <= 0 || wmaxpos - j0 < p.window);
                if (fast) {
#pragma unroll
                    for (int nt = 0; nt < NS; ++nt) {
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float x = (sc[nt][e] + sd[nt][e]) * qk2;
                            sc[nt][e] = x;
                            if (e < 2) mx0 = fmaxf(mx0, x); else mx1 = fmaxf(mx1, x);
                        }
                    }
                } else {
#pragma unroll
                    for (int nt = 0; nt < NS; ++nt) {
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int j = j0 + nt * 8 + 2 * (lane & 3) + (e & 1);
                            const int ps = (e < 2) ? pos0 : pos1;
                            float x = (sc[nt][e] + sd[nt][e]) * p.scale;
                            if (p.cap > 0.f) x = p.cap * tanhf(x / p.cap);
                            x *= LOG2E;
                            const bool masked = j < kbeg || j >= kend || j > ps || (p.window > 0 && ps - j >= p.window);
                            x = masked ? -INFINITY : x;
                            sc[nt][e] = x;
                            if (e < 2) mx0 = fmaxf(mx0, x); else mx1 = fmaxf(mx1, x);
                        }
                    }
                }
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
                const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
                const float mu0 = mn0 == -INFINITY ? 0.f : mn0, mu1 = mn1 == -INFINITY ? 0.f : mn1;
                const float c0f = exp2f(m0 - mu0), c1f = exp2f(m1 - mu1);
                float ps[NS][4];
                float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
                for (int nt = 0; nt < NS; ++nt) {
                    ps[nt][0] = exp2f(sc[nt][0] - mu0);
                    ps[nt][1] = exp2f(sc[nt][1] - mu0);
                    ps[nt][2] = exp2f(sc[nt][2] - mu1);
                    ps[nt][3] = exp2f(sc[nt][3] - mu1);
                    sum0 += ps[nt][0] + ps[nt][1];
                    sum1 += ps[nt][2] + ps[nt][3];
                }
                l0 = l0 * c0f + sum0;
                l1 = l1 * c1f + sum1;
                m0 = mn0;
                m1 = mn1;
                // rescale O only when some row's running max moved (the common case
                // after the first chunks is c == 1 for every row of the warp)
                if (__any_sync(0xffffffffu, c0f != 1.0f || c1f != 1.0f)) {
#pragma unroll
                    for (int t = 0; t < NT; ++t) {
                        o[t][0] *= c0f; o[t][1] *= c0f;
                        o[t][2] *= c1f; o[t][3] *= c1f;
                    }
                }
                // O += P V : one 16-key k-step per page of the chunk, output n-tiles in pairs
#pragma unroll
                for (int u = 0; u < CP; ++u) {
                    const uint32_t pa0 = pack_bf16(ps[2 * u][0], ps[2 * u][1]), pa1 = pack_bf16(ps[2 * u][2], ps[2 * u][3]);
                    const uint32_t pa2 = pack_bf16(ps[2 * u + 1][0], ps[2 * u + 1][1]);
                    const uint32_t pa3 = pack_bf16(ps[2 * u + 1][2], ps[2 * u + 1][3]);
#pragma unroll
                    for (int t = 0; t < NT; t += 2) {
                        uint32_t b0, b1, b2, b3;
                        ldsm_x4_t(vb[u] + sw_off((lane & 7) + ((lane >> 3) & 1) * 8, t + (lane >> 4)), b0, b1, b2, b3);
                        mma_bf16(o[t], pa0, pa1, pa2, pa3, b0, b1);
                        mma_bf16(o[t + 1], pa0, pa1, pa2, pa3, b2, b3);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) {
#pragma unroll
                for (int u = 0; u < CP; ++u)
                    if (u < np) mbar_arrive(smem_u32(&empty[(i0 + u) % S]));
            }
        }
    }
    if (stp && threadIdx.x == 0) stp[2] = globaltimer_ns();
    // ---- merge the warps of each m-tile through shared memory (the ring is idle now)
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    float* red = reinterpret_cast<float*>(ring);      // [4 warps][16][DH] partial O
    float* ml = red + 4 * 16 * DH;                     // [4 warps][16][2] (m, l)
    float* fw = ml + 4 * 16 * 2;                       // [64][4] per-row weights of the warps
    float* rml = fw + AT_ROWS * 4;                     // [64][2] merged (M, L)
    consumer_bar();
    if (active) {
        float* rw = red + (size_t)warp * 16 * DH;
        const int lr = lane >> 2;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const int col = t * 8 + 2 * (lane & 3);
            *reinterpret_cast<float2*>(rw + lr * DH + col) = make_float2(o[t][0], o[t][1]);
            *reinterpret_cast<float2*>(rw + (lr + 8) * DH + col) = make_float2(o[t][2], o[t][3]);
        }
        if ((lane & 3) == 0) {
            ml[(warp * 16 + lr) * 2] = m0;
            ml[(warp * 16 + lr) * 2 + 1] = l0;
            ml[(warp * 16 + lr + 8) * 2] = m1;
            ml[(warp * 16 + lr + 8) * 2 + 1] = l1;
        }
    }
    consumer_bar();
    if (threadIdx.x < rows) {
        const int r = threadIdx.x, mt = r >> 4, lr = r & 15;
        float M = -INFINITY;
        for (int w = 0; w < wpm; ++w) M = fmaxf(M, ml[((mt * wpm + w) * 16 + lr) * 2]);
        const float Mu = M == -INFINITY ? 0.f : M;
        float f[4] = {0.f, 0.f, 0.f, 0.f};
        float L = 0.f;
        for (int w = 0; w < wpm; ++w) {
            f[w] = exp2f(ml[((mt * wpm + w) * 16 + lr) * 2] - Mu);
            L += f[w] * ml[((mt * wpm + w) * 16 + lr) * 2 + 1];
        }
        // whole item: normalised weights; split item: raw weights and the (M, L) of the partial
        const float sc = slot < 0 ? (L > 0.f ? 1.0f / L : 0.f) : 1.0f;
        for (int w = 0; w < 4; ++w) fw[r * 4 + w] = f[w] * sc;
        rml[r * 2] = M;
        rml[r * 2 + 1] = L;
    }
    consumer_bar();
    __nv_bfloat16* outp = reinterpret_cast<__nv_bfloat16*>(p.out);
    const int WR = ws_row(DH);
    constexpr int D8 = DH / 8;
    for (int i = threadIdx.x; i < rows * D8; i += 128) {
        const int r = i / D8, c8 = (i % D8) * 8;
        const int mt = r >> 4, lr = r & 15;
        float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
        for (int w = 0; w < wpm; ++w) {
            const float f = fw[r * 4 + w];
            const float* src = red + ((size_t)(mt * wpm + w) * 16 + lr) * DH + c8;
            const float4 v0 = *reinterpret_cast<const float4*>(src), v1 = *reinterpret_cast<const float4*>(src + 4);
            a0.x += f * v0.x; a0.y += f * v0.y; a0.z += f * v0.z; a0.w += f * v0.w;
            a1.x += f * v1.x; a1.y += f * v1.y; a1.z += f * v1.z; a1.w += f * v1.w;
        }
        if (slot < 0) {
            const int rr = qt * AT_ROWS + r;
            __nv_bfloat16* dst = outp + ((size_t)(qs0 + rr / G) * p.H + (size_t)g * G + rr % G) * DH + c8;
            *reinterpret_cast<uint4*>(dst) =
                make_uint4(pack_bf16(a0.x, a0.y), pack_bf16(a0.z, a0.w), pack_bf16(a1.x, a1.y), pack_bf16(a1.z, a1.w));
        } else {
            float* wsr = p.ws + ((size_t)slot * AT_ROWS + r) * WR;
            __stcg(reinterpret_cast<float4*>(wsr + 4 + c8), a0);
            __stcg(reinterpret_cast<float4*>(wsr + 4 + c8 + 4), a1);
            if (c8 == 0) __stcg(reinterpret_cast<float4*>(wsr), make_float4(rml[r * 2], rml[r * 2 + 1], 0.f, 0.f));
        }
    }
    if (stp && threadIdx.x == 0) stp[3] = globaltimer_ns();
    if (threadIdx.x == 0) trace_mark(p.tr, TR_END);
    if (slot < 0) return;
    // ---- split item: the last of the group to finish merges all partials in split order
    __threadfence();
    consumer_bar();
    const int32_t* ce = p.comb + (size_t)cg * AT_COMB_INTS;
    const int first = ce[3], ns = ce[4];
    if (threadIdx.x == 0) flags[0] = (atomicAdd(&p.counters[cg], 1) == ns - 1) ? 1 : 0;
    consumer_bar();
    if (!flags[0]) return;
    __threadfence();
    // per-row split weights f = exp2(M_s - max M) and the total L, then O = sum f O_s
    float* sfw = reinterpret_cast<float*>(ring);          // [64][AT_MAX_SPLITS]
    float* lt = sfw + AT_ROWS * AT_MAX_SPLITS;             // [64]
    if (threadIdx.x < rows) {
        const int r = threadIdx.x;
        float M = -INFINITY;
        for (int sp = 0; sp < ns; ++sp) M = fmaxf(M, __ldcg(p.ws + ((size_t)(first + sp) * AT_ROWS + r) * WR));
        const float Mu = M == -INFINITY ? 0.f : M;
        float L = 0.f;
        for (int sp = 0; sp < ns; ++sp) {
            const float* w = p.ws + ((size_t)(first + sp) * AT_ROWS + r) * WR;
            const float f = exp2f(__ldcg(w) - Mu);
            L += f * __ldcg(w + 1);
            sfw[r * AT_MAX_SPLITS + sp] = f;
        }
        lt[r] = L;
    }
    consumer_bar();
    constexpr int D4 = DH / 4;
#pragma unroll 2
    for (int i = threadIdx.x; i < rows * D4; i += 128) {
        const int r = i / D4, c4 = (i % D4) * 4;
        float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int sp = 0; sp < ns; ++sp) {
            const float f = sfw[r * AT_MAX_SPLITS + sp];
            const float4 v =
                __ldcg(reinterpret_cast<const float4*>(p.ws + ((size_t)(first + sp) * AT_ROWS + r) * WR + 4 + c4));
            O.x += f * v.x;
            O.y += f * v.y;
            O.z += f * v.z;
            O.w += f * v.w;
        }
        const float L = lt[r];
        const int rr = qt * AT_ROWS + r;
        __nv_bfloat16* dst = outp + ((size_t)(qs0 + rr / G) * p.H + (size_t)g * G + rr % G) * DH + c4;
        *reinterpret_cast<uint2*>(dst) = make_uint2(pack_bf16(L > 0.f ? O.x / L : 0.f, L > 0.f ? O.y / L : 0.f),
                                                    pack_bf16(L > 0.f ? O.z / L : 0.f, L > 0.f ? O.w / L : 0.f));
    }
    if (threadIdx.x == 0) {
        p.counters[cg] = 0;
        trace_mark(p.tr, TR_END);
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
static yk_status launch_tc(const CUtensorMap& tm, const AttnParams& p, int n_items, yk_engine* e) {
    const size_t smem = AttnCfg<DH>::SMEM;
    static bool attr = false;
    if (!attr) {
        YK_CHECK_CUDA(cudaFuncSetAttribute(attn_tc_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        attr = true;
    }
    YK_CHECK_CUDA(launch_pdl(e, attn_tc_kernel<DH>, n_items, AT_THREADS, smem, tm, p));
    e->launches++;
    return YK_OK;
}

int attention_ctas_per_sm(int head_dim) {
    return head_dim == 64 ? AttnCfg<64>::CTAS_PER_SM : (head_dim == 128 ? AttnCfg<128>::CTAS_PER_SM : AttnCfg<256>::CTAS_PER_SM);
}

// Work list for one forward step and one window setting (see yk_forward_step):
// spans (sequence, query tile) x KV heads, each cut into equal page-aligned
// key ranges so the item count fills about `waves` waves of resident CTAs (or,
// balanced, no piece is longer than the average load of a resident slot);
// items sorted longest first so the block scheduler balances the tail.
void plan_attention(const yk_model_config& c, int num_sms, int waves, bool balanced, const uint32_t* q_starts,
                    const uint32_t* ctx, int B, bool windowed, std::vector<int32_t>& items, std::vector<int32_t>& comb,
                    int* n_slots) {
    const int G = c.n_heads / c.n_kv_heads;
    struct Span { int b, qt, kb, ke; };
    std::vector<Span> spans;
    int max_pages = 1;
    for (int b = 0; b < B; ++b) {
        const int n = (int)(q_starts[b + 1] - q_starts[b]);
        if (n == 0) continue;
        const int rows = n * G;
        for (int qt = 0; qt * AT_ROWS < rows; ++qt) {
            const int i_lo = (qt * AT_ROWS) / G, i_hi = (std::min(rows, qt * AT_ROWS + AT_ROWS) - 1) / G;
            const int pos_lo = (int)ctx[b] - n + i_lo, pos_hi = (int)ctx[b] - n + i_hi;
            int kb = windowed ? std::max(0, pos_lo - c.window + 1) : 0;
            kb = (kb / 16) * 16;
            const int ke = pos_hi + 1;
            spans.push_back({b, qt, kb, ke});
            max_pages = std::max(max_pages, (ke - kb + 15) / 16);
        }
    }
    // Long spans (Gemma-shape contexts of thousands of tokens) go in two waves of
    // half-size pieces: a piece's fixed cost (first page, partial merge: ~5 us) is
    // small against its page loop there, and the longest piece no longer sets the
    // end (9B/2B-shape step 86.4 -> 79.5 ms; 4 waves 81.4).  At the 8B/1B-shape
    // verify and decode spans (tens of pages) one wave is faster.
    long long span_pages = 0;
    for (const auto& s : spans) span_pages += (s.ke - s.kb + 15) / 16;
    const bool long_spans = !spans.empty() && span_pages >= 160LL * (long long)spans.size();
    const long long target =
        (long long)num_sms * attention_ctas_per_sm(c.head_dim) * std::max(1, waves) * (long_spans ? 2 : 1);
    auto splits = [&](const Span& s, int kp) {  // pieces of a span at kp pages per piece
        const int pages = (s.ke - s.kb + 15) / 16;
        return std::min(AT_MAX_SPLITS, (pages + kp - 1) / kp);
    };
    auto count = [&](int kp) {
        long long nitems = 0;
        for (const auto& s : spans) nitems += (long long)splits(s, kp) * c.n_kv_heads;
        return nitems;
    };
    int kp;
    if (balanced) {
        // pieces of at most the average load of a resident slot: the longest item
        // is no longer than that average, the scheduler fills slots longest first
        long long pages = 0;
        for (const auto& s : spans) pages += (long long)((s.ke - s.kb + 15) / 16) * c.n_kv_heads;
        kp = (int)std::max<long long>(1, (pages + target - 1) / target);
    } else {
        int lo = 1, hi = max_pages;  // smallest pages-per-piece whose item count fits the target
        while (lo < hi) {
            const int mid = (lo + hi) / 2;
            if (count(mid) <= target) hi = mid; else lo = mid + 1;
        }
        kp = lo;
    }
    struct Item { int b, g, qt, kb, ke, slot, cg; };
    std::vector<Item> list;
    comb.clear();
    int slot = 0;
    for (const auto& s : spans) {
        const int ns = splits(s, kp);
        const int pages = (s.ke - s.kb + 15) / 16;
        for (int g = 0; g < c.n_kv_heads; ++g) {
            if (ns <= 1) {
                list.push_back({s.b, g, s.qt, s.kb, s.ke, -1, -1});
            } else {
                const int cg = (int)(comb.size() / AT_COMB_INTS);
                comb.insert(comb.end(), {s.b, g, s.qt, slot, ns});
                for (int i = 0; i < ns; ++i) {
                    const int kb = s.kb + 16 * (int)((long long)i * pages / ns);
                    const int ke = std::min(s.ke, s.kb + 16 * (int)((long long)(i + 1) * pages / ns));
                    list.push_back({s.b, g, s.qt, kb, ke, slot++, cg});
                }
            }
        }
    }
    std::stable_sort(list.begin(), list.end(), [](const Item& x, const Item& y) { return x.ke - x.kb > y.ke - y.kb; });
    items.clear();
    items.reserve(list.size() * AT_ITEM_INTS);
    for (const auto& t : list) items.insert(items.end(), {t.b, t.g, t.qt, t.kb, t.ke, t.slot, t.cg});
    *n_slots = slot;
}

// layer: the model's layer (its window); pool_layer: its index within `pool`;
// bt: the page tables of `pool` ([B x max_blocks]).
yk_status attention_run(yk_model* m, yk_kv_pool* pool, int layer, int pool_layer, const int32_t* bt, int T, int B,
                        int max_blocks, double kv_bytes) {
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
    p.block_tables = bt;
    p.max_blocks = max_blocks;
    p.T = T;
    p.H = c.n_heads;
    p.Hkv = c.n_kv_heads;
    p.dh = c.head_dim;
    p.block_elems = (long long)pool->block_elems;
    p.layer_off = (long long)pool_layer * (long long)pool->layer_elems;
    p.layer = pool_layer;
    p.pool_blocks = pool->num_blocks;
    p.scale = 1.0f / sqrtf((float)c.head_dim);
    p.cap = c.attn_cap;
    const bool windowed = c.window > 0 && (c.window_layer_parity < 0 || (layer % 2) == c.window_layer_parity);
    p.window = windowed ? c.window : 0;
    p.err = m->e->d_err;
    p.ws = m->attn_ws;
    p.counters = m->attn_counters;
    p.stamps = nullptr;
    p.tr = trace_next(m->e, TK_ATTN | ((uint32_t)c.head_dim << 8));  // kind | head dim << 8
    if (c.dtype != YK_DTYPE_BF16) {
        YK_CHECK_CUDA(launch_simt<float>(p, m->e));
        m->e->launches++;
        return YK_OK;
    }
    YK_ARG(pool->has_tm, "KV pool has no tensor map");
    const int w = windowed ? 1 : 0;
    p.items = m->cur.attn_items[w];
    p.comb = m->cur.attn_comb[w];
    const int ni = m->cur.n_items[w];
    if (m->attn_stamps && ni <= m->attn_stamps_cap) {
        p.stamps = m->attn_stamps;
        m->attn_last_items = ni;
    }
    switch (c.head_dim) {
        case 64: return launch_tc<64>(pool->tm, p, ni, m->e);
        case 128: return launch_tc<128>(pool->tm, p, ni, m->e);
        default: return launch_tc<256>(pool->tm, p, ni, m->e);
    }
}

size_t attention_ws_floats_per_slot(int head_dim) { return (size_t)AT_ROWS * ws_row(head_dim); }

// Tensor map of a bf16 pool for the attention kernel: x = head dim, y = row
// within a block ([layer][K|V][kv head][16 slots]), z = block; box 64 x 16 x 1.
yk_status make_pool_map(yk_engine* e, yk_kv_pool* pool) {
    const auto& c = pool->cfg;
    const cuuint64_t dims[3] = {(cuuint64_t)c.head_dim, (cuuint64_t)pool->n_pool_layers * 2 * c.n_kv_heads * 16,
                                (cuuint64_t)pool->num_blocks};
    const cuuint64_t strides[2] = {(cuuint64_t)c.head_dim * 2, (cuuint64_t)pool->block_elems * 2};
    const cuuint32_t box[3] = {64, 16, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = e->encode_tiled(&pool->tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, pool->data, dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        yk_set_error("cuTensorMapEncodeTiled(KV pool) failed: " + std::to_string((int)r));
        return YK_ERR_CUDA;
    }
    pool->has_tm = true;
    return YK_OK;
}

}  // namespace yk

// ---------------------------------------------------------------------------
// Test hooks (include/yk_testing.h).
// ---------------------------------------------------------------------------
#include "../../include/yk_testing.h"

extern "C" yk_status ykt_attention_stamps_enable(yk_model* m, int32_t cap) {
    YK_ARG(m && cap >= 0, "arguments");
    YK_CHECK_CUDA(cudaSetDevice(m->e->device));
    YK_CHECK_CUDA(cudaStreamSynchronize(m->e->stream));
    if (m->attn_stamps) cudaFree(m->attn_stamps);
    m->attn_stamps = nullptr;
    m->attn_stamps_cap = 0;
    m->attn_last_items = 0;
    if (cap > 0) {
        YK_CHECK_CUDA(cudaMalloc(&m->attn_stamps, (size_t)cap * 8 * 8));
        YK_CHECK_CUDA(cudaMemset(m->attn_stamps, 0, (size_t)cap * 8 * 8));
        m->attn_stamps_cap = cap;
    }
    return YK_OK;
}

extern "C" yk_status ykt_attention_stamps_read(yk_model* m, uint64_t* host, int32_t cap, int32_t* n_ctas) {
    YK_ARG(m && host && n_ctas, "arguments");
    YK_ARG(m->attn_stamps, "attention stamps are not enabled");
    YK_CHECK_CUDA(cudaSetDevice(m->e->device));
    YK_CHECK_CUDA(cudaStreamSynchronize(m->e->stream));
    const int n = std::min(cap, m->attn_last_items);
    YK_CHECK_CUDA(cudaMemcpy(host, m->attn_stamps, (size_t)n * 8 * 8, cudaMemcpyDeviceToHost));
    *n_ctas = n;
    return YK_OK;
}
