// yk_gemm.cu -- the verify-forward linear layers (replaces LinearLayer.forward /
// gemm_kernel, S/LinearLayer.swift:71-128, S/gemm.metal:6-34).
//
// bf16: persistent, warp-specialised tcgen05 GEMM.
//   D[n][j] = sum_k W[n][k] * X[j][k] ("swap-AB"): a 128-row weight tile is the
//   MMA A operand and the tokens (BN <= 256) are the MMA N dimension, so at
//   verify batch sizes every weight byte crosses HBM once.
//   Warp 0 streams W and X k-blocks with TMA (128-byte swizzle, no multicast)
//   into a shared-memory ring; warp 1 issues tcgen05.mma into one of two TMEM
//   accumulators; warps 2-5 drain the other accumulator through the fused
//   epilogue, so the epilogue of one segment overlaps the next mainloop.
//   Work split, chosen per layer shape:
//   * stream-K (tiles >= SMs/2): the (tile x 64-wide k-block) space is cut into
//     equal contiguous ranges, one per CTA, so every SM streams the same number
//     of weight bytes.  A tile cut across CTAs is finished by the segment that
//     arrives last: it sums the published fp32 partials in k order and runs the
//     epilogue.  No CTA waits for another.
//   * cluster split-K (few tiles): the CS CTAs sharing a tile form a cluster; each
//     parks its partial in shared memory and each rank sums 1/CS of the tile's
//     columns over all ranks, in rank order: through distributed-shared-memory
//     loads, or, for large column shares, after the copy engine has moved every
//     rank's share into that rank's shared memory (all loads then local).
//   Both reductions are deterministic.
//
// fp32: a SIMT kernel with the same epilogues (the fp32 reference-numerics
// config; tensor cores have no fp32 x fp32 mode).
#include <algorithm>
#include <cstring>

#include "yk_common.cuh"
#include "yk_epilogue.cuh"
#include "yk_internal.h"

namespace yk {

constexpr int TC_BM = 128;       // weight rows per tile (MMA M)
constexpr int TC_BK = 64;        // k per stage: one 128-byte swizzle row of bf16
constexpr int TC_THREADS = 192;  // warp 0 TMA, warp 1 MMA, warps 2..5 epilogue
constexpr int TC_SMEM_BUDGET = 200 * 1024;
constexpr int TC_QKV_STAGE_TOK = 256;  // tokens whose QKV epilogue metadata is staged in shared memory
// align slack, barriers, QKV staging, per-token 1/rms of the fused norm
constexpr int TC_SMEM_TAIL = 1024 + 256 + (2 * TC_QKV_STAGE_TOK + 128) * 4 + TC_QKV_STAGE_TOK * 4;

struct TcArgs {
    int n_out, K, m_tok;
    int tiles_m, kb_total;      // k-blocks per tile
    int BN, stages;
    int tiles;                  // tiles_m * tiles_n
    int grid;
    int cluster_s;              // > 0: cluster split-K with cluster_s CTAs per tile
    int sk_tiles, sk_ctas;      // stream-K part: tiles [0, sk_tiles) cut over CTAs [0, sk_ctas)
    uint32_t idesc, tmem_cols;  // columns of one accumulator stage
    float* ws;                  // stream-K partials: slot (2*cta + first/last) x [BN][128]
    uint32_t* counters;         // per-tile arrival counters (zero between launches)
    EpiParams epi;
    unsigned long long* stamps;  // optional per-CTA phase timestamps (test hook), else null
    Trace tr;
    int push;                    // cluster split-K: exchange column shares by copy engine (else DSMEM loads)
    int rope_stage;              // push, QKV: copy the RoPE table rows of a rank's columns into shared memory
};

// Phase timestamps of one CTA (ns, %globaltimer), recorded only when a.stamps != null.
enum : int {
    ST_START = 0, ST_FIRST_TMA, ST_FIRST_FULL, ST_LAST_MMA, ST_LAST_ACC, ST_EPI_DONE, ST_SEGS, ST_CLUSTER, ST_N = 8
};
__device__ __forceinline__ void stamp(const TcArgs& a, int what) {
    if (a.stamps) a.stamps[(size_t)blockIdx.x * ST_N + what] = globaltimer_ns();
}

__device__ __forceinline__ long long unit_begin(int c, long long U, int G) { return ((long long)c * U) / G; }
// CTA whose range contains unit u (inverse of unit_begin).
__device__ __forceinline__ int cta_of_unit(long long u, long long U, int G) {
    return (int)(((u + 1) * G + U - 1) / U) - 1;
}

// This CTA's work, fixed at kernel start:
//  * cluster split-K: one segment, k-blocks [r*KB/CS, (r+1)*KB/CS) of tile c/CS.
//  * otherwise: first this CTA's equal share of the stream-K units of tiles
//    [0, sk_tiles) (nrem segments, the first and last possibly cut with a
//    neighbour), then whole tiles sk_tiles + c + w*grid.  Cut tiles are
//    finished early, while the whole tiles stream, so no fix-up sits at the end.
struct TcSched {
    int nrem, t0, kbf, kbl;  // remainder segments: tiles t0.., first from kbf, last up to kbl
};
__device__ __forceinline__ TcSched tc_sched(const TcArgs& a, int c) {
    TcSched r;
    const int KB = a.kb_total;
    r.nrem = 0;
    r.t0 = 0;
    r.kbf = 0;
    r.kbl = KB;
    if (a.cluster_s > 0) {
        const int q = c % a.cluster_s;
        r.nrem = 1;
        r.t0 = c / a.cluster_s;
        r.kbf = q * KB / a.cluster_s;
        r.kbl = (q + 1) * KB / a.cluster_s;
    } else if (c < a.sk_ctas) {
        const long long RU = (long long)a.sk_tiles * KB;
        const long long u0 = unit_begin(c, RU, a.sk_ctas), u1 = unit_begin(c + 1, RU, a.sk_ctas);
        if (u1 > u0) {
            r.t0 = (int)(u0 / KB);
            r.nrem = (int)((u1 - 1) / KB) - r.t0 + 1;
            r.kbf = (int)(u0 - (long long)r.t0 * KB);
            r.kbl = (int)(u1 - (long long)(r.t0 + r.nrem - 1) * KB);
        }
    }
    return r;
}
// Segment i: tile and k-block range [kb0, kb1); false past the end.
__device__ __forceinline__ bool tc_segment(const TcArgs& a, const TcSched& sc, int c, int i, int& tile, int& kb0,
                                           int& kb1) {
    if (i < sc.nrem) {
        tile = sc.t0 + i;
        kb0 = i == 0 ? sc.kbf : 0;
        kb1 = i == sc.nrem - 1 ? sc.kbl : a.kb_total;
        return true;
    }
    if (a.cluster_s > 0) return false;
    tile = a.sk_tiles + c + (i - sc.nrem) * a.grid;
    kb0 = 0;
    kb1 = a.kb_total;
    return tile < a.tiles;
}
// Partial slot of stream-K CTA cta for cut tile `tile`.
__device__ __forceinline__ int partial_slot(const TcArgs& a, int cta, int tile) {
    const long long RU = (long long)a.sk_tiles * a.kb_total;
    return 2 * cta + ((long long)tile == unit_begin(cta, RU, a.sk_ctas) / a.kb_total ? 0 : 1);
}
__device__ __forceinline__ void epi_bar_sync() {  // named barrier over the 4 epilogue warps
    asm volatile("bar.sync 1, 128;" ::: "memory");
}

// Cluster reduction of columns [c0, c1) of tile (tm, tn) by rank `rank`: sums
// the CS partials ([BN][128] fp32, parked at red_addr in each CTA) in rank
// order.  !LOCAL: loads them from the ranks' shared memory (distributed shared
// memory).  LOCAL: the other ranks' copies of these columns sit in this CTA's
// receive slots at recv_addr (slot s or s - 1 for rank s, slot_cols columns
// each).  QN items per thread and round keep QN*CS loads in flight; with every
// operand local (the QKV RoPE rows of tokens c0.. staged at rope_addr) short
// rounds do, and their small unrolled body runs from a warm instruction cache
// after the first round.
template <int KIND, int CS, bool LOCAL, bool FN>
__device__ __forceinline__ void cluster_reduce(const TcArgs& a, const EpiParams& ep, uint32_t red_addr,
                                               uint32_t recv_addr, uint32_t rope_addr, int rank, int slot_cols, int tm,
                                               int tn, int c0, int c1, bool ok, const float* inv) {
    constexpr int QN = (LOCAL && KIND == EPI_QKV)     ? 2
                       : (KIND == EPI_RESID && FN) ? (CS >= 8 ? 1 : 8 / CS)  // (register budget: gains in flight too)
                                                   : (CS >= 16 ? 1 : 16 / CS);
    const int nitems = (c1 - c0) * 32;  // (column, 4-row group) items
    uint32_t rb[CS];  // address of column c0 of rank s's partial (shared::cta if LOCAL, else shared::cluster)
#pragma unroll
    for (int s = 0; s < CS; ++s) {
        if (LOCAL)
            rb[s] = s == rank ? red_addr + (uint32_t)c0 * (TC_BM * 4)
                              : recv_addr + (uint32_t)((s < rank ? s : s - 1) * slot_cols) * (TC_BM * 4);
        else
            rb[s] = mapa_shared(red_addr + (uint32_t)c0 * (TC_BM * 4), (uint32_t)s);
    }
    for (int base = threadIdx.x; base < nitems; base += TC_THREADS * QN) {
        float4 tv[QN][CS];
        float4 hv[(KIND == EPI_RESID || KIND == EPI_QKV) ? QN : 1];
        float4 gv[(KIND == EPI_RESID && FN) ? QN : 1];
        if constexpr (KIND == EPI_RESID) {
            // the residual stream values (and the fused norm's gains), in flight
            // together with the partials
#pragma unroll
            for (int q = 0; q < QN; ++q) {
                const int it = base + q * TC_THREADS;
                const int n = tm * TC_BM + (it % 32) * 4, j = tn * a.BN + c0 + it / 32;
                if (ok && it < nitems && j < a.epi.m_tok && n < a.epi.n_out) {
                    hv[q] = *reinterpret_cast<const float4*>(a.epi.h + (size_t)j * a.epi.ld + n);
                    if constexpr (FN) gv[q] = *reinterpret_cast<const float4*>(a.epi.nx_g + n);
                }
            }
        } else if constexpr (KIND == EPI_QKV) {
            // the RoPE (cos, sin) of the quad's two pairs, in flight with the partials
#pragma unroll
            for (int q = 0; q < QN; ++q) {
                const int it = base + q * TC_THREADS;
                const int n = tm * TC_BM + (it % 32) * 4, j = tn * a.BN + c0 + it / 32;
                hv[q] = make_float4(1.f, 0.f, 1.f, 0.f);
                if (ok && it < nitems && j < ep.m_tok && n < ep.q_dim + ep.kv_dim) {
                    const int ci = rope_dim(ep, n) >> 1;
                    if (rope_addr) {
                        hv[q] = lds_v4(rope_addr + (uint32_t)(((it / 32) * (ep.head_dim >> 1) + ci) * 8));
                    } else if (ep.rope_tab) {
                        hv[q] = *reinterpret_cast<const float4*>(ep.rope_tab + (size_t)j * (ep.head_dim >> 1) + ci);
                    } else {
                        const float2 r0 = rope_pair(ep, ci, j), r1 = rope_pair(ep, ci + 1, j);
                        hv[q] = make_float4(r0.x, r0.y, r1.x, r1.y);
                    }
                }
            }
        }
#pragma unroll
        for (int q = 0; q < QN; ++q) {
            const int it = base + q * TC_THREADS;
            if (it < nitems) {
                const uint32_t off = (uint32_t)(((it / 32) * TC_BM + (it % 32) * 4) * 4);
#pragma unroll
                for (int s = 0; s < CS; ++s) tv[q][s] = LOCAL ? lds_v4(rb[s] + off) : ld_shared_cluster_v4(rb[s] + off);
            }
        }
#pragma unroll
        for (int q = 0; q < QN; ++q) {
            const int it = base + q * TC_THREADS;
            if (ok && it < nitems) {
                float4 acc = tv[q][0];
#pragma unroll
                for (int s = 1; s < CS; ++s) {
                    acc.x += tv[q][s].x;
                    acc.y += tv[q][s].y;
                    acc.z += tv[q][s].z;
                    acc.w += tv[q][s].w;
                }
                const int n = tm * TC_BM + (it % 32) * 4, j = tn * a.BN + c0 + it / 32;
                if constexpr (FN && KIND != EPI_RESID) {  // this token's 1/rms (the input was bf16(h * g))
                    const float s = inv[j];
                    acc = make_float4(acc.x * s, acc.y * s, acc.z * s, acc.w * s);
                }
                if constexpr (KIND == EPI_RESID && FN) {
                    // (it, hence j, is the same on every lane of the warp: the group sums shuffle)
                    const bool live = j < a.epi.m_tok && n < a.epi.n_out;
                    const float ss = live ? epi_quad_resid<true>(a.epi, n, j, acc, hv[q], gv[q]) : 0.f;
                    ss_quad_groups(a.epi, n, j, ss, j < a.epi.m_tok && (n & ~31) < a.epi.n_out);
                } else if constexpr (KIND == EPI_RESID) {
                    if (j < a.epi.m_tok && n < a.epi.n_out) epi_quad_resid<false>(a.epi, n, j, acc, hv[q]);
                } else if constexpr (KIND == EPI_QKV) {
                    epi_quad_qkv<__nv_bfloat16>(ep, n, j, acc, hv[q]);
                } else {
                    epi_quad<KIND, __nv_bfloat16>(ep, n, j, acc);
                }
            }
        }
    }
}

// Fused norm: 1 / rms of each token of this GEMM's input, from the 32-row group
// sums of squares the previous GEMM wrote (a fixed summation order); the
// epilogue warps run it (thread et of 128) while the mainloop streams.
__device__ __forceinline__ void tc_inv_rms(const EpiParams& e, float* s_inv, int et) {
    const EpiParams& ep = e;
    const int G = ep.in_groups, ld = ep.ss_ld;
    for (int j = et; j < ep.m_tok; j += 128) {
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
        int g = 0;
        for (; g + 8 <= G; g += 8) {
            float v8[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v8[u] = ep.in_ss[(size_t)(g + u) * ld + j];
            s0 += v8[0] + v8[4];
            s1 += v8[1] + v8[5];
            s2 += v8[2] + v8[6];
            s3 += v8[3] + v8[7];
        }
        for (; g < G; ++g) s0 += ep.in_ss[(size_t)g * ld + j];
        const float tot = (s0 + s1) + (s2 + s3);
        s_inv[j] = 1.0f / sqrtf(tot / ep.in_d + ep.in_eps);
    }
}

// Epilogue of a whole tile held in TMEM (this warp's 32 rows at taddr): one row
// per lane, 16 tokens per drain.
template <int KIND, bool FN>
__device__ __forceinline__ void tc_whole_tile(const EpiParams& ep, uint32_t taddr, int n, int j_base, int BN,
                                              const float* inv) {
    for (int cc = 0; cc < BN; cc += 16) {
        uint32_t r[16];
        tmem_ld16(taddr + (uint32_t)cc, r);
        float v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            v[i] = __uint_as_float(r[i]);
            if constexpr (FN && KIND != EPI_RESID) v[i] *= inv[j_base + cc + i];
        }
        drain16<KIND, __nv_bfloat16, FN>(ep, n, j_base + cc, v);
    }
}

// Epilogue of a segment that holds part of a tile cut across CTAs (stream-K):
// publish this CTA's partial; the last arriver sums the partials in k order and
// runs the epilogue.  All 128 epilogue threads call it.
template <int KIND, bool FN, int FIX = 4>
__device__ __forceinline__ void tc_cut_tile(const TcArgs& a, const EpiParams& ep, const float* inv, int c, int t,
                                            uint32_t taddr, int row, int et, volatile int* flags) {
    const int BN = a.BN;
    const int tm = t % a.tiles_m, tn = t / a.tiles_m;
    const int j_base = tn * BN;
    const long long RU = (long long)a.sk_tiles * a.kb_total;
    const int c_lo = cta_of_unit((long long)t * a.kb_total, RU, a.sk_ctas);
    const int c_hi = cta_of_unit((long long)(t + 1) * a.kb_total - 1, RU, a.sk_ctas);
    const int nseg = c_hi - c_lo + 1;
    float* mine = a.ws + (size_t)partial_slot(a, c, t) * TC_BM * BN;
    for (int cc = 0; cc < BN; cc += 16) {
        uint32_t r[16];
        tmem_ld16(taddr + (uint32_t)cc, r);
#pragma unroll
        for (int i = 0; i < 16; ++i) __stcg(mine + (size_t)(cc + i) * TC_BM + row, __uint_as_float(r[i]));
    }
    __threadfence();
    epi_bar_sync();
    if (et == 0) flags[1] = (atomicAdd(&a.counters[t], 1u) == (uint32_t)(nseg - 1)) ? 1 : 0;
    epi_bar_sync();
    if (flags[1]) {
        // Sum the nseg partials in k order (deterministic).  Thread et owns rows
        // 4*(et&31)..+3 of columns (et>>5) + 4i, i < 8: float4 loads, 8 columns x
        // up to FIX segments in flight per round, one vector store per quad.
        __threadfence();
        const int r4 = (et & 31) * 4, cq = et >> 5;
        for (int cc = 0; cc < BN; cc += 32) {
            float4 acc[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int sg0 = 0; sg0 < nseg; sg0 += FIX) {
                float4 tv[FIX][8];
#pragma unroll
                for (int s4 = 0; s4 < FIX; ++s4) {
                    if (sg0 + s4 < nseg) {
                        const float* src =
                            a.ws + (size_t)partial_slot(a, c_lo + sg0 + s4, t) * TC_BM * BN + r4;
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const int col = cc + cq + 4 * i;
                            if (col < BN)
                                tv[s4][i] = __ldcg(reinterpret_cast<const float4*>(src + (size_t)col * TC_BM));
                        }
                    }
                }
#pragma unroll
                for (int s4 = 0; s4 < FIX; ++s4) {
                    if (sg0 + s4 < nseg) {
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            acc[i].x += tv[s4][i].x;
                            acc[i].y += tv[s4][i].y;
                            acc[i].z += tv[s4][i].z;
                            acc[i].w += tv[s4][i].w;
                        }
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int col = cc + cq + 4 * i;  // (the same on every lane of the warp)
                if (col >= BN) continue;
                const int n = tm * TC_BM + r4, j = j_base + col;
                float4 v = acc[i];
                if constexpr (FN && KIND != EPI_RESID) {
                    const float s = inv[j];
                    v = make_float4(v.x * s, v.y * s, v.z * s, v.w * s);
                }
                if constexpr (KIND == EPI_RESID && FN) {
                    const bool live = j < ep.m_tok && n < ep.n_out;
                    const float ss =
                        live ? epi_quad_resid<true>(ep, n, j, v,
                                                    *reinterpret_cast<const float4*>(ep.h + (size_t)j * ep.ld + n),
                                                    *reinterpret_cast<const float4*>(ep.nx_g + n))
                             : 0.f;
                    ss_quad_groups(ep, n, j, ss, j < ep.m_tok && (n & ~31) < ep.n_out);
                } else {
                    epi_quad<KIND, __nv_bfloat16>(ep, n, j, v);
                }
            }
        }
        if (et == 0) a.counters[t] = 0u;
    }
    epi_bar_sync();  // flags[1] is rewritten by the next cut tile
}

// FN: the RMSNorm folded in (EpiParams nx_* for the residual kind, in_ss for the
// kinds that consume its output).
template <int KIND, bool FN>
__global__ void __launch_bounds__(TC_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, const TcArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int BN = a.BN, S = a.stages;
    const uint32_t stage_bytes = 16384u + (uint32_t)BN * 128u;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * stage_bytes);
    uint64_t* empty = full + S;
    uint64_t* acc_full = empty + S;      // [2]
    uint64_t* acc_empty = acc_full + 2;  // [2]
    uint64_t* recv_bar = acc_empty + 2;  // cluster split-K: the other ranks' column copies have landed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv_bar + 1);
    // [0] abort, [1] last arriver of a cut tile, [2..3] epilogue's broadcast of [0] by segment parity
    volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = blockIdx.x, KB = a.kb_total;
    const int CS = a.cluster_s;
    const TcSched sc = tc_sched(a, c);
    // The QKV epilogue's per-token positions / page slots and the RoPE
    // denominators, staged in shared memory (verify-sized token counts).
    EpiParams ep = a.epi;
    constexpr bool kStageQkv = KIND == EPI_QKV;
    int32_t* qkv_smem = reinterpret_cast<int32_t*>(tmem_slot + 8);  // past the slot and the 4 flags
    const bool stage_qkv = kStageQkv && a.epi.m_tok <= TC_QKV_STAGE_TOK;
    // fused norm: per-token 1/rms of this GEMM's input (computed by the epilogue warps)
    float* s_inv = reinterpret_cast<float*>(qkv_smem + 2 * TC_QKV_STAGE_TOK + 128);
    const float* inv = (FN && KIND != EPI_RESID) ? s_inv : nullptr;  // (host: m_tok <= TC_QKV_STAGE_TOK)

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(smem_u32(&acc_full[s]), 1);
            mbar_init(smem_u32(&acc_empty[s]), 128);
        }
        mbar_init(smem_u32(recv_bar), 1);
        flags[0] = flags[1] = flags[2] = flags[3] = 0;
        mbar_fence_init();
    }
    if (threadIdx.x == 0) trace_mark(a.tr, TR_ENTRY);
    if (stage_qkv) {
        // step metadata is uploaded before the step's first kernel: no dependency wait needed
        float* den = reinterpret_cast<float*>(qkv_smem + 2 * TC_QKV_STAGE_TOK);
        for (int i = threadIdx.x; i < a.epi.m_tok; i += TC_THREADS) {
            qkv_smem[i] = a.epi.pos[i];
            qkv_smem[TC_QKV_STAGE_TOK + i] = a.epi.slot[i];
        }
        for (int i = threadIdx.x; i < a.epi.head_dim / 2; i += TC_THREADS) den[i] = a.epi.rope_denom[i];
        ep.pos = qkv_smem;
        ep.slot = qkv_smem + TC_QKV_STAGE_TOK;
        ep.rope_denom = den;
    }
    if (warp == 1) tmem_alloc(smem_u32(tmem_slot), 2 * a.tmem_cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    pdl_trigger();
    const uint32_t tmem = *tmem_slot;
    if (threadIdx.x == 0) stamp(a, ST_START);
    // Everything but the weight prefetch below reads or writes what earlier kernels touch.
    if (threadIdx.x != 0) pdl_wait();
    if (threadIdx.x == 32) trace_mark(a.tr, TR_START);

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            const uint64_t pol_w = policy_evict_first();
            const uint64_t pol_x = policy_evict_last();
            int t, k0, k1;
            // The weights do not depend on the previous kernel: fill the ring with
            // them while that kernel finishes.
            long long pre = 0;
            for (int i = 0; pre < S && tc_segment(a, sc, c, i, t, k0, k1); ++i)
                for (int kb = k0; kb < k1 && pre < S; ++kb, ++pre) {
                    const uint32_t fb = smem_u32(&full[pre]);
                    mbar_arrive_expect_tx(fb, stage_bytes);
                    tma_load_2d(smem_u32(smem + (size_t)pre * stage_bytes), &tmW, kb * TC_BK, (t % a.tiles_m) * TC_BM,
                                fb, pol_w);
                }
            pdl_wait();  // the activations are the previous kernel's output
            long long g = 0;
            bool stop = false;
            for (int i = 0; !stop && tc_segment(a, sc, c, i, t, k0, k1); ++i) {
                const int tm = t % a.tiles_m, tn = t / a.tiles_m;
                for (int kb = k0; kb < k1; ++kb, ++g) {
                    const int s = (int)(g % S);
                    const uint32_t sdst = smem_u32(smem + (size_t)s * stage_bytes);
                    const uint32_t fb = smem_u32(&full[s]);
                    if (g >= pre) {
                        const long long r = g / S;
                        if (flags[0] || (r > 0 && !mbar_wait_bounded(smem_u32(&empty[s]), (uint32_t)((r - 1) & 1)))) {
                            if (!flags[0]) raise_err(a.epi.err, YK_DEV_ERR_TIMEOUT);
                            flags[0] = 1;
                            stop = true;
                            break;
                        }
                        mbar_arrive_expect_tx(fb, stage_bytes);
                        tma_load_2d(sdst, &tmW, kb * TC_BK, tm * TC_BM, fb, pol_w);
                    }
                    tma_load_2d(sdst + 16384u, &tmX, kb * TC_BK, tn * BN, fb, pol_x);
                    if (g == 0) stamp(a, ST_FIRST_TMA);
                }
            }
            // Every issued copy must land before shared memory is reused or released.
            const long long issued = g;
            for (long long j = max(0LL, issued - S); j < issued; ++j)
                (void)mbar_wait_bounded(smem_u32(&full[j % S]), (uint32_t)((j / S) & 1));
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            long long g = 0;
            int seg = 0, t, k0, k1;
            for (; !flags[0] && tc_segment(a, sc, c, seg, t, k0, k1); ++seg) {
                const int st = seg & 1;
                if (seg >= 2 && !mbar_wait_bounded(smem_u32(&acc_empty[st]), (uint32_t)(((seg >> 1) - 1) & 1))) {
                    flags[0] = 1;
                    raise_err(a.epi.err, YK_DEV_ERR_TIMEOUT);
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)st * a.tmem_cols;
                bool ok = true;
                for (int kb = k0; kb < k1; ++kb, ++g) {
                    const int s = (int)(g % S);
                    if (!mbar_wait_bounded(smem_u32(&full[s]), (uint32_t)((g / S) & 1))) {
                        flags[0] = 1;
                        raise_err(a.epi.err, YK_DEV_ERR_TIMEOUT);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (g == 0) stamp(a, ST_FIRST_FULL);
                    const uint32_t wsm = smem_u32(smem + (size_t)s * stage_bytes);
#pragma unroll
                    for (int kk = 0; kk < TC_BK / 16; ++kk)
                        tc_mma_bf16(d, sw128_kmajor_desc(wsm + kk * 32), sw128_kmajor_desc(wsm + 16384u + kk * 32),
                                    a.idesc, (kb > k0 || kk > 0) ? 1u : 0u);
                    tc_commit(smem_u32(&empty[s]));
                }
                tc_commit(smem_u32(&acc_full[st]));
                if (!ok) break;
            }
            stamp(a, ST_LAST_MMA);
            if (a.stamps) a.stamps[(size_t)blockIdx.x * ST_N + ST_SEGS] = (unsigned long long)seg;
        }
    } else {
        // ---------------- epilogue: warps 2..5 ----------------
        const int q = warp & 3;           // TMEM lane quadrant this warp may read
        const int row = q * 32 + lane;    // output row within the tile
        const int et = threadIdx.x - 64;  // 0..127
        if constexpr (FN && KIND != EPI_RESID) tc_inv_rms(a.epi, s_inv, et);  // read after the first barrier below
        int t, kb_b, kb_e;
        for (int seg = 0; tc_segment(a, sc, c, seg, t, kb_b, kb_e); ++seg) {
            const int st = seg & 1;
            // One thread waits (bounded) and broadcasts, so the epilogue warps always
            // take the same path through their named barriers.
            if (et == 0) {
                if (!mbar_wait_bounded(smem_u32(&acc_full[st]), (uint32_t)((seg >> 1) & 1))) {
                    flags[0] = 1;
                    raise_err(a.epi.err, YK_DEV_ERR_TIMEOUT);
                }
                flags[2 + st] = flags[0];  // per-parity slot: rewritten only after the next barrier
            }
            epi_bar_sync();
            if (flags[2 + st]) break;
            tc_fence_after();
            if (et == 0) stamp(a, ST_LAST_ACC);
            const uint32_t taddr = tmem + (uint32_t)st * a.tmem_cols + ((uint32_t)(q * 32) << 16);
            const int tm = t % a.tiles_m, tn = t / a.tiles_m;
            const int n = tm * TC_BM + row;
            const int j_base = tn * BN;
            if (CS > 0) {
                // park the partial in shared memory [BN][128] fp32; the ring is idle
                // (every staged k-block was consumed before acc_full fired)
                float* red = reinterpret_cast<float*>(smem);
                for (int cc = 0; cc < BN; cc += 16) {
                    uint32_t r[16];
                    tmem_ld16(taddr + (uint32_t)cc, r);
#pragma unroll
                    for (int i = 0; i < 16; ++i) red[(cc + i) * TC_BM + row] = __uint_as_float(r[i]);
                }
                fence_proxy_async_smem();  // the copy engine reads the parked partial
            } else if (kb_b == 0 && kb_e == KB) {
                tc_whole_tile<KIND, FN>(ep, taddr, n, j_base, BN, inv);
            } else {
                tc_cut_tile<KIND, FN>(a, ep, inv, c, t, taddr, row, et, flags);
            }
            tc_fence_before();
            mbar_arrive(smem_u32(&acc_empty[st]));
        }
        if (et == 0) stamp(a, ST_EPI_DONE);
    }

    if (CS > 0) {
        // ---------------- cluster reduction ----------------
        // Rank r owns columns [r*BN/CS, (r+1)*BN/CS) of tile t.  After the barrier every
        // CTA's partial is parked and every ring idle.  a.push: each CTA's copy engine
        // sends each other rank its partial's share of that rank's columns (receive
        // slots past the parked partial).  Each rank then sums its columns in rank
        // order and runs their epilogue.
        const int rank = (int)cluster_ctarank();
        const int t = c / CS;
        const int tm = t % a.tiles_m, tn = t / a.tiles_m;
        const int c0 = rank * BN / CS, c1 = (rank + 1) * BN / CS;
        const int slot_cols = (BN + CS - 1) / CS;
        const uint32_t red_addr = smem_u32(smem);
        const uint32_t recv_addr = red_addr + (uint32_t)BN * (TC_BM * 4);
        const uint32_t rbar = smem_u32(recv_bar);
        // QKV rows that take RoPE: this rank's tokens' rows of the RoPE table, copied
        // in past the receive slots
        const bool push = a.push != 0;
        const int rrows = min(c1, a.epi.m_tok - tn * BN) - c0;
        const bool stage_rope =
            KIND == EPI_QKV && push && a.rope_stage && rrows > 0 && tm * TC_BM < ep.q_dim + ep.kv_dim;
        const uint32_t rope_addr = stage_rope ? recv_addr + (uint32_t)((CS - 1) * slot_cols) * (TC_BM * 4) : 0u;
        const uint32_t rope_bytes = stage_rope ? (uint32_t)(rrows * ep.head_dim * 4) : 0u;
        if (push && threadIdx.x == 0)
            mbar_arrive_expect_tx(rbar, (uint32_t)((CS - 1) * (c1 - c0) * TC_BM * 4) + rope_bytes);
        // After the barrier every ring of the cluster is idle: the epilogue warps parked
        // each partial only after the tile's last MMA (the ring's last reader) completed.
        cluster_sync_any();
        if (threadIdx.x == 64) stamp(a, ST_CLUSTER);
        if (push && threadIdx.x == 0) {
            if (stage_rope)
                bulk_load(rope_addr, ep.rope_tab + (size_t)(tn * BN + c0) * (ep.head_dim >> 1), rope_bytes, rbar);
            // sent even after an abort, so that no peer waits for bytes that never come
            for (int r = 0; r < CS; ++r) {
                if (r == rank) continue;
                const int r0 = r * BN / CS, r1 = (r + 1) * BN / CS;
                const int slot = rank < r ? rank : rank - 1;
                bulk_copy_to_peer(mapa_shared(recv_addr + (uint32_t)(slot * slot_cols) * (TC_BM * 4), (uint32_t)r),
                                  red_addr + (uint32_t)r0 * (TC_BM * 4), (uint32_t)((r1 - r0) * TC_BM * 4),
                                  mapa_shared(rbar, (uint32_t)r));
            }
        }
        bool ok = flags[0] == 0;
        if (push) {
            if (!mbar_wait_bounded(rbar, 0u)) {
                raise_err(a.epi.err, YK_DEV_ERR_TIMEOUT);
                ok = false;
            }
            // Every byte sent to this CTA has landed, so every peer's copy to it has
            // read its source: the closing barrier's arrival can go now, and the
            // reduction below (local operands only) overlaps its latency.
            cluster_arrive_any();
        }
#define YK_CLUSTER_REDUCE(N)                                                                                        \
    (push ? cluster_reduce<KIND, N, true, FN>(a, ep, red_addr, recv_addr, rope_addr, rank, slot_cols, tm, tn, c0, c1, \
                                              ok, inv)                                                                \
          : cluster_reduce<KIND, N, false, FN>(a, ep, red_addr, recv_addr, rope_addr, rank, slot_cols, tm, tn, c0, c1, \
                                               ok, inv))
        switch (CS) {
            case 1: YK_CLUSTER_REDUCE(1); break;
            case 2: YK_CLUSTER_REDUCE(2); break;
            case 3: YK_CLUSTER_REDUCE(3); break;
            case 4: YK_CLUSTER_REDUCE(4); break;
            case 5: YK_CLUSTER_REDUCE(5); break;
            case 6: YK_CLUSTER_REDUCE(6); break;
            case 7: YK_CLUSTER_REDUCE(7); break;
            default: YK_CLUSTER_REDUCE(8); break;
        }
#undef YK_CLUSTER_REDUCE
        // no peer still reads (or copies out of) this CTA's shared memory
        if (push) cluster_wait_any(); else cluster_sync_any();
        if (threadIdx.x == 64) stamp(a, ST_EPI_DONE);
    }

    // ---------------- teardown ----------------
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 2 * a.tmem_cols);
    if (threadIdx.x == 0) trace_mark(a.tr, TR_END);
}

// ---------------------------------------------------------------------------
// Two GEMMs chained in one persistent grid (gate/up then down_proj): one CTA
// per SM, both stages with whole tiles / stream-K (no clusters), the ring and
// the TMEM accumulators running on across the stage boundary.  A CTA that has
// finished its stage-0 epilogue arrives on a grid-wide counter; the producer
// streams stage 1's first weight k-blocks into the ring meanwhile and issues
// their activation halves once every CTA has arrived (bounded wait).  The grid's
// dependents are released only then (every CTA is resident by that point, so
// the barrier cannot wait on a CTA that a dependent keeps off its SM).
// ---------------------------------------------------------------------------
struct ChainArgs {
    uint32_t* bar;    // grid barrier counter (monotonic across launches)
    uint32_t target;  // its value once every CTA of this launch finished stage 0
};

template <int K0, bool F0, int K1, bool F1>
__global__ void __launch_bounds__(TC_THREADS, 1)
    gemm_chain_kernel(const __grid_constant__ CUtensorMap tmW0, const __grid_constant__ CUtensorMap tmX0,
                      const __grid_constant__ CUtensorMap tmW1, const __grid_constant__ CUtensorMap tmX1,
                      const TcArgs a0, const TcArgs a1, const ChainArgs ch) {
    static_assert(K1 == EPI_RESID || !F1, "stage 1 consumes no folded norm");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int BN = a0.BN, S = a0.stages;  // (the host makes both stages' tiles and rings equal)
    const uint32_t stage_bytes = 16384u + (uint32_t)BN * 128u;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * stage_bytes);
    uint64_t* empty = full + S;
    uint64_t* acc_full = empty + S;      // [2]
    uint64_t* acc_empty = acc_full + 2;  // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 3);
    volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 1);  // [0] abort, [1] last arriver, [2..3] broadcast
    float* s_inv = reinterpret_cast<float*>(tmem_slot + 8 + 2 * TC_QKV_STAGE_TOK + 128);
    const float* inv = (F0 && K0 != EPI_RESID) ? s_inv : nullptr;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = blockIdx.x;
    const TcSched sc0 = tc_sched(a0, c), sc1 = tc_sched(a1, c);
    int n0 = 0;  // stage-0 segments of this CTA
    {
        int tt, x, y;
        while (tc_segment(a0, sc0, c, n0, tt, x, y)) ++n0;
    }
    // segment i of the chain: stage 0's, then stage 1's
    auto seg_of = [&](int i, int& stage, int& t, int& k0, int& k1) -> bool {
        if (i < n0) {
            stage = 0;
            return tc_segment(a0, sc0, c, i, t, k0, k1);
        }
        stage = 1;
        return tc_segment(a1, sc1, c, i - n0, t, k0, k1);
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(smem_u32(&acc_full[s]), 1);
            mbar_init(smem_u32(&acc_empty[s]), 128);
        }
        flags[0] = flags[1] = flags[2] = flags[3] = 0;
        mbar_fence_init();
        trace_mark(a0.tr, TR_ENTRY);
    }
    if (warp == 1) tmem_alloc(smem_u32(tmem_slot), 2 * a0.tmem_cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (threadIdx.x != 0) pdl_wait();
    if (threadIdx.x == 32) trace_mark(a0.tr, TR_START);

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            const uint64_t pol_w = policy_evict_first();
            const uint64_t pol_x = policy_evict_last();
            long long g = 0;
            bool stop = false;
            // stage 0, with the first ring of weights ahead of the dependency wait
            long long pre = 0;
            {
                int t, k0, k1;
                for (int i = 0; pre < S && tc_segment(a0, sc0, c, i, t, k0, k1); ++i)
                    for (int kb = k0; kb < k1 && pre < S; ++kb, ++pre) {
                        const uint32_t fb = smem_u32(&full[pre]);
                        mbar_arrive_expect_tx(fb, stage_bytes);
                        tma_load_2d(smem_u32(smem + (size_t)pre * stage_bytes), &tmW0, kb * TC_BK,
                                    (t % a0.tiles_m) * TC_BM, fb, pol_w);
                    }
            }
            pdl_wait();
            auto slot_ready = [&](long long gg) -> bool {  // ring slot of k-block gg free again
                const long long r = gg / S;
                if (flags[0] || (r > 0 && !mbar_wait_bounded(smem_u32(&empty[gg % S]), (uint32_t)((r - 1) & 1)))) {
                    if (!flags[0]) raise_err(a0.epi.err, YK_DEV_ERR_TIMEOUT);
                    flags[0] = 1;
                    return false;
                }
                return true;
            };
            {
                int t, k0, k1;
                for (int i = 0; !stop && tc_segment(a0, sc0, c, i, t, k0, k1); ++i) {
                    const int tm = t % a0.tiles_m, tn = t / a0.tiles_m;
                    for (int kb = k0; kb < k1; ++kb, ++g) {
                        const uint32_t sdst = smem_u32(smem + (size_t)(g % S) * stage_bytes);
                        const uint32_t fb = smem_u32(&full[g % S]);
                        if (g >= pre) {
                            if (!slot_ready(g)) { stop = true; break; }
                            mbar_arrive_expect_tx(fb, stage_bytes);
                            tma_load_2d(sdst, &tmW0, kb * TC_BK, tm * TC_BM, fb, pol_w);
                        }
                        tma_load_2d(sdst + 16384u, &tmX0, kb * TC_BK, tn * BN, fb, pol_x);
                    }
                }
            }
            // stage 1: weights of the first ring's worth of k-blocks now ...
            int pend_kb[16], pend_tn[16];
            long long g1 = g;
            int npend = 0;
            {
                int t, k0, k1;
                for (int i = 0; !stop && npend < S && tc_segment(a1, sc1, c, i, t, k0, k1); ++i)
                    for (int kb = k0; kb < k1 && npend < S; ++kb) {
                        if (!slot_ready(g)) { stop = true; break; }
                        const uint32_t fb = smem_u32(&full[g % S]);
                        mbar_arrive_expect_tx(fb, stage_bytes);
                        tma_load_2d(smem_u32(smem + (size_t)(g % S) * stage_bytes), &tmW1, kb * TC_BK,
                                    (t % a1.tiles_m) * TC_BM, fb, pol_w);
                        pend_kb[npend] = kb;
                        pend_tn[npend] = t / a1.tiles_m;
                        ++npend;
                        ++g;
                    }
            }
            // ... their activations once every CTA has written its stage-0 output
            bool passed = false;
            {
                const uint64_t t0 = globaltimer_ns();
                for (uint32_t it = 0;; ++it) {
                    if ((int32_t)(ld_acquire_gpu(ch.bar) - ch.target) >= 0) { passed = true; break; }
                    if ((it & 63u) == 63u && globaltimer_ns() - t0 > YK_WAIT_BUDGET_NS) break;
                }
            }
            if (!passed) {
                raise_err(a0.epi.err, YK_DEV_ERR_TIMEOUT);
                flags[0] = 1;
            }
            pdl_trigger();  // every CTA of the grid is resident and past stage 0
            fence_proxy_async_global();
            // (issued even after a failed wait, so that every armed slot completes)
            for (int u = 0; u < npend; ++u) {
                const long long gg = g1 + u;
                tma_load_2d(smem_u32(smem + (size_t)(gg % S) * stage_bytes) + 16384u, &tmX1, pend_kb[u] * TC_BK,
                            pend_tn[u] * BN, smem_u32(&full[gg % S]), pol_x);
            }
            {
                int t, k0, k1;
                int done = 0;  // k-blocks of stage 1 already issued
                for (int i = 0; !stop && tc_segment(a1, sc1, c, i, t, k0, k1); ++i) {
                    const int tm = t % a1.tiles_m, tn = t / a1.tiles_m;
                    for (int kb = k0; kb < k1; ++kb) {
                        if (done < npend) { ++done; continue; }
                        if (!slot_ready(g)) { stop = true; break; }
                        const uint32_t sdst = smem_u32(smem + (size_t)(g % S) * stage_bytes);
                        const uint32_t fb = smem_u32(&full[g % S]);
                        mbar_arrive_expect_tx(fb, stage_bytes);
                        tma_load_2d(sdst, &tmW1, kb * TC_BK, tm * TC_BM, fb, pol_w);
                        tma_load_2d(sdst + 16384u, &tmX1, kb * TC_BK, tn * BN, fb, pol_x);
                        ++g;
                    }
                }
            }
            // Every issued copy must land before shared memory is reused or released.
            for (long long j = max(0LL, g - S); j < g; ++j)
                (void)mbar_wait_bounded(smem_u32(&full[j % S]), (uint32_t)((j / S) & 1));
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            long long g = 0;
            int stage, t, k0, k1;
            for (int seg = 0; !flags[0] && seg_of(seg, stage, t, k0, k1); ++seg) {
                const int st = seg & 1;
                if (seg >= 2 && !mbar_wait_bounded(smem_u32(&acc_empty[st]), (uint32_t)(((seg >> 1) - 1) & 1))) {
                    flags[0] = 1;
                    raise_err(a0.epi.err, YK_DEV_ERR_TIMEOUT);
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)st * a0.tmem_cols;
                const uint32_t idesc = stage == 0 ? a0.idesc : a1.idesc;
                bool ok = true;
                for (int kb = k0; kb < k1; ++kb, ++g) {
                    const int s = (int)(g % S);
                    if (!mbar_wait_bounded(smem_u32(&full[s]), (uint32_t)((g / S) & 1))) {
                        flags[0] = 1;
                        raise_err(a0.epi.err, YK_DEV_ERR_TIMEOUT);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t wsm = smem_u32(smem + (size_t)s * stage_bytes);
#pragma unroll
                    for (int kk = 0; kk < TC_BK / 16; ++kk)
                        tc_mma_bf16(d, sw128_kmajor_desc(wsm + kk * 32), sw128_kmajor_desc(wsm + 16384u + kk * 32),
                                    idesc, (kb > k0 || kk > 0) ? 1u : 0u);
                    tc_commit(smem_u32(&empty[s]));
                }
                tc_commit(smem_u32(&acc_full[st]));
                if (!ok) break;
            }
        }
    } else {
        // ---------------- epilogue: warps 2..5 ----------------
        const int q = warp & 3;
        const int row = q * 32 + lane;
        const int et = threadIdx.x - 64;
        if constexpr (F0 && K0 != EPI_RESID) tc_inv_rms(a0.epi, s_inv, et);  // read after the first barrier below
        int stage, t, kb_b, kb_e;
        bool arrived = false;
        for (int seg = 0; seg_of(seg, stage, t, kb_b, kb_e); ++seg) {
            if (stage == 1 && !arrived) {
                // this CTA's stage-0 output is written: arrive on the grid barrier
                __threadfence();
                epi_bar_sync();
                if (et == 0) atomicAdd(ch.bar, 1u);
                arrived = true;
            }
            const int st = seg & 1;
            if (et == 0) {
                if (!mbar_wait_bounded(smem_u32(&acc_full[st]), (uint32_t)((seg >> 1) & 1))) {
                    flags[0] = 1;
                    raise_err(a0.epi.err, YK_DEV_ERR_TIMEOUT);
                }
                flags[2 + st] = flags[0];
            }
            epi_bar_sync();
            if (flags[2 + st]) break;
            tc_fence_after();
            const uint32_t taddr = tmem + (uint32_t)st * a0.tmem_cols + ((uint32_t)(q * 32) << 16);
            const int tiles_m = stage == 0 ? a0.tiles_m : a1.tiles_m;
            const int tm = t % tiles_m, tn = t / tiles_m;
            const int n = tm * TC_BM + row;
            if (stage == 0) {
                if (kb_b == 0 && kb_e == a0.kb_total) tc_whole_tile<K0, F0>(a0.epi, taddr, n, tn * BN, BN, inv);
                else tc_cut_tile<K0, F0, 2>(a0, a0.epi, inv, c, t, taddr, row, et, flags);
            } else {
                if (kb_b == 0 && kb_e == a1.kb_total) tc_whole_tile<K1, F1>(a1.epi, taddr, n, tn * BN, BN, nullptr);
                else tc_cut_tile<K1, F1, 2>(a1, a1.epi, nullptr, c, t, taddr, row, et, flags);
            }
            tc_fence_before();
            mbar_arrive(smem_u32(&acc_empty[st]));
        }
        if (!arrived) {  // no stage-1 segment here (or an abort): arrive all the same
            __threadfence();
            epi_bar_sync();
            if (et == 0) atomicAdd(ch.bar, 1u);
        }
    }

    // ---------------- teardown ----------------
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 2 * a0.tmem_cols);
    if (threadIdx.x == 0) trace_mark(a0.tr, TR_END);
}

// ---------------------------------------------------------------------------
// SIMT GEMM: each warp owns an output-row pair, lanes stride over k; a CTA
// covers 16 rows x 8 tokens.  Used for fp32 weights.
// ---------------------------------------------------------------------------
template <int KIND, typename WT, typename XT>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const WT* __restrict__ W, const XT* __restrict__ X, int n_out,
                                                         int K, int m_tok, EpiParams ep) {
    constexpr int TOK = 8;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = (blockIdx.x * 8 + warp) * 2;
    const int j0 = blockIdx.y * TOK;
    if (n >= n_out) return;
    float acc0[TOK], acc1[TOK];
#pragma unroll
    for (int t = 0; t < TOK; ++t) { acc0[t] = 0.f; acc1[t] = 0.f; }
    const WT* w0 = W + (size_t)n * K;
    const WT* w1 = (n + 1 < n_out) ? w0 + K : w0;
    for (int k = lane; k < K; k += 32) {
        const float a0 = to_f32(w0[k]), a1 = to_f32(w1[k]);
#pragma unroll
        for (int t = 0; t < TOK; ++t) {
            if (j0 + t < m_tok) {
                const float x = to_f32(X[(size_t)(j0 + t) * K + k]);
                acc0[t] = fmaf(a0, x, acc0[t]);
                acc1[t] = fmaf(a1, x, acc1[t]);
            }
        }
    }
#pragma unroll
    for (int t = 0; t < TOK; ++t) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            acc0[t] += __shfl_xor_sync(0xffffffffu, acc0[t], o);
            acc1[t] += __shfl_xor_sync(0xffffffffu, acc1[t], o);
        }
    }
    if (lane == 0) {
#pragma unroll
        for (int t = 0; t < TOK; ++t)
            if (j0 + t < m_tok) epi_pair<KIND, XT>(ep, n, j0 + t, acc0[t], acc1[t]);
    }
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
yk_status make_weight_map(yk_engine* e, CUtensorMap* map, const void* W, int rows, int K) {
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {TC_BK, TC_BM};
    const cuuint32_t estr[2] = {1, 1};
    YK_ARG(((uintptr_t)W & 15) == 0 && (K * 2) % 16 == 0, "TMA operand must be 16-byte aligned");
    CUresult r = e->encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(W), dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        yk_set_error("cuTensorMapEncodeTiled(weight) failed: " + std::to_string((int)r));
        return YK_ERR_CUDA;
    }
    return YK_OK;
}

static yk_status get_x_map(yk_model* m, const void* X, int K, int BN, const CUtensorMap** out) {
    auto key = std::make_pair(X, BN * 100000 + K);
    auto it = m->xmaps.find(key);
    if (it == m->xmaps.end()) {
        CUtensorMap map;
        const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)m->cfg.max_tokens};
        const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
        const cuuint32_t box[2] = {TC_BK, (cuuint32_t)BN};
        const cuuint32_t estr[2] = {1, 1};
        CUresult r = m->e->encode_tiled(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(X), dims, strides,
                                        box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            yk_set_error("cuTensorMapEncodeTiled(activation) failed: " + std::to_string((int)r));
            return YK_ERR_CUDA;
        }
        it = m->xmaps.emplace(key, map).first;
    }
    *out = &it->second;
    return YK_OK;
}

template <int KIND>
static yk_status launch_tc(const cudaLaunchConfig_t& cfg, const CUtensorMap* tmW, const CUtensorMap* tmX,
                           const TcArgs& a, bool fn) {
    static bool attr = false;
    if (!attr) {
        YK_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<KIND, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           TC_SMEM_BUDGET + 16384 + TC_SMEM_TAIL));
        if constexpr (KIND == EPI_QKV || KIND == EPI_RESID || KIND == EPI_GLU)
            YK_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<KIND, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               TC_SMEM_BUDGET + 16384 + TC_SMEM_TAIL));
        attr = true;
    }
    if constexpr (KIND == EPI_QKV || KIND == EPI_RESID || KIND == EPI_GLU) {
        if (fn) {
            YK_CHECK_CUDA(cudaLaunchKernelEx(&cfg, gemm_tc_kernel<KIND, true>, *tmW, *tmX, a));
            return YK_OK;
        }
    }
    YK_CHECK_CUDA(cudaLaunchKernelEx(&cfg, gemm_tc_kernel<KIND, false>, *tmW, *tmX, a));
    return YK_OK;
}

// How many clusters of `s` GEMM CTAs (one per SM, full shared-memory budget) the
// device holds at once; queried once per size.
static int cluster_capacity(yk_engine* e, int s) {
    static int cap[9] = {0};
    static int dev = -1;
    if (dev != e->device) {
        for (int& c : cap) c = 0;
        dev = e->device;
    }
    if (cap[s] == 0) {
        cudaFuncSetAttribute(gemm_tc_kernel<EPI_STORE, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             TC_SMEM_BUDGET + 16384 + TC_SMEM_TAIL);
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(s * 64);
        cfg.blockDim = dim3(TC_THREADS);
        cfg.dynamicSmemBytes = TC_SMEM_BUDGET + TC_SMEM_TAIL;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = s;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, gemm_tc_kernel<EPI_STORE, false>, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = 1;
        }
        cap[s] = n;
    }
    return cap[s];
}

template <int KIND>
static void launch_simt(dim3 grid, cudaStream_t st, const void* W, const void* X, int n_out, int K, int m_tok,
                        const EpiParams& ep) {
    gemm_simt_kernel<KIND, float, float><<<grid, 256, 0, st>>>((const float*)W, (const float*)X, n_out, K, m_tok, ep);
}

// force_grid: 0 = heuristic; > 0 = stream-K with that many CTAs; < 0 = cluster
// split-K with -force_grid CTAs per tile (test hook).
yk_status gemm_run(yk_model* m, const void* W, const CUtensorMap* tmW, const void* X, int n_out, int K, int m_tok,
                   const EpiParams& ep_in, int force_grid) {
    yk_engine* e = m->e;
    EpiParams ep = ep_in;
    ep.n_out = n_out;
    ep.m_tok = m_tok;
    ep.err = e->d_err;
    YK_ARG(n_out % 4 == 0 && m_tok > 0 && m_tok <= m->cfg.max_tokens, "gemm shape");
    // Algorithmic traffic of this launch: weights + activations once, plus the epilogue's outputs.
    const double es = m->cfg.dtype == YK_DTYPE_BF16 ? 2.0 : 4.0;
    double out_bytes = (double)m_tok * n_out * 4.0;
    if (ep.kind == EPI_QKV) out_bytes = (double)m_tok * n_out * es;
    else if (ep.kind == EPI_RESID) out_bytes = (double)m_tok * n_out * 8.0;
    else if (ep.kind == EPI_GLU) out_bytes = (double)m_tok * (n_out / 2) * es;
    ProfScope prof(e, YK_PROF_GEMM, ((double)n_out + m_tok) * K * es + out_bytes, 2.0 * n_out * K * m_tok);
    if (m->cfg.dtype == YK_DTYPE_F32) {
        dim3 grid((n_out + 15) / 16, (m_tok + 7) / 8);
        switch (ep.kind) {
            case EPI_QKV: launch_simt<EPI_QKV>(grid, e->stream, W, X, n_out, K, m_tok, ep); break;
            case EPI_RESID: launch_simt<EPI_RESID>(grid, e->stream, W, X, n_out, K, m_tok, ep); break;
            case EPI_GLU: launch_simt<EPI_GLU>(grid, e->stream, W, X, n_out, K, m_tok, ep); break;
            case EPI_LOGITS: launch_simt<EPI_LOGITS>(grid, e->stream, W, X, n_out, K, m_tok, ep); break;
            default: launch_simt<EPI_STORE>(grid, e->stream, W, X, n_out, K, m_tok, ep); break;
        }
        e->launches++;
        YK_CHECK_CUDA(cudaGetLastError());
        return YK_OK;
    }
    // bf16: persistent tcgen05 path.
    const int BN = m_tok <= 256 ? ((m_tok + 15) / 16) * 16 : 256;
    const int tiles_n = (m_tok + BN - 1) / BN;
    const int tiles_m = (n_out + TC_BM - 1) / TC_BM;
    const int kb = (K + TC_BK - 1) / TC_BK;
    const long long tiles = (long long)tiles_m * tiles_n;
    const long long units = tiles * kb;
    // Few tiles (fewer than half the SMs): cluster split-K with the largest cluster
    // size whose clusters all run at once.  Otherwise stream-K with at least ~8
    // k-blocks per CTA so each pipeline fills before its epilogue.
    const uint32_t stage_bytes = 16384u + (uint32_t)BN * 128u;
    const int stages = std::max(2, std::min(8, (int)(TC_SMEM_BUDGET / stage_bytes)));
    // cluster split-K reuses the idle ring: the parked partial, plus with the
    // copy-engine exchange CS-1 receive slots (plus, QKV, the RoPE rows of a rank's tokens)
    const bool want_rope = ep.kind == EPI_QKV && ep.rope_tab != nullptr;
    const size_t ring = (size_t)stages * stage_bytes;
    const auto ring_need = [&](int s, bool push, bool rope) {
        const size_t slot = (size_t)((BN + s - 1) / s);
        return (size_t)(BN + (push ? (s - 1) * slot : 0)) * TC_BM * 4 + (rope ? slot * ep.head_dim * 4 : 0);
    };
    const auto cluster_fits = [&](int s) { return ring_need(s, false, false) <= ring; };
    int cs = 0;
    if (force_grid < 0) {
        for (int s = std::min(-force_grid, std::min(8, kb)); s >= 2 && cs == 0; --s)
            if (cluster_fits(s)) cs = s;
        YK_ARG(cs > 0, "no cluster size fits the shared-memory ring");
    } else if (force_grid == 0 && tiles * 2 < e->num_sms && !(e->gemm_variant & 32)) {
        for (int s = (int)std::min<long long>(std::min(8, kb), e->num_sms / tiles); s >= 2 && cs == 0; --s)
            if (tiles <= cluster_capacity(e, s) && cluster_fits(s)) cs = s;
    }
    // Otherwise: persistent CTAs (at least ~8 k-blocks each so each pipeline fills)
    // take whole tiles round-robin; the tiles left over after the full waves are
    // cut evenly over the CTAs (stream-K) and done first.
    int grid = (int)std::min<long long>(e->num_sms, std::max<long long>(1, units / 8));
    if (force_grid > 0) grid = (int)std::min<long long>(force_grid, units);
    int sk_tiles = 0, sk_ctas = 0;
    if (cs > 0) {
        grid = (int)(tiles * cs);
    } else {
        const long long waves = tiles / grid, rest = tiles % grid;
        if (waves == 0 || (e->gemm_variant & 1)) {
            sk_tiles = (int)tiles;
            sk_ctas = grid;
        } else if (rest > 0) {
            sk_tiles = (int)rest;
            sk_ctas = (int)std::min<long long>(grid, std::max<long long>(1, rest * kb / 8));
        }
    }
    YK_ARG((size_t)2 * sk_ctas * TC_BM * BN <= m->gemm_ws_floats, "split workspace too small");
    if (tiles > m->gemm_counter_cap) {
        YK_CHECK_CUDA(cudaStreamSynchronize(e->stream));
        if (m->gemm_counters) cudaFree(m->gemm_counters);
        m->gemm_counters = nullptr;
        m->gemm_counter_cap = 0;
        YK_CHECK_CUDA(cudaMalloc(&m->gemm_counters, (size_t)tiles * 2 * 4));
        YK_CHECK_CUDA(cudaMemset(m->gemm_counters, 0, (size_t)tiles * 2 * 4));
        m->gemm_counter_cap = (int)(tiles * 2);
    }
    const size_t smem = (size_t)stages * stage_bytes + TC_SMEM_TAIL;
    uint32_t cols = 32;
    while ((int)cols < BN) cols <<= 1;

    const CUtensorMap* tmX = nullptr;
    YK_TRY(get_x_map(m, X, K, BN, &tmX));
    TcArgs a;
    a.n_out = n_out; a.K = K; a.m_tok = m_tok;
    a.tiles_m = tiles_m; a.kb_total = kb;
    a.BN = BN; a.stages = stages;
    a.tiles = (int)tiles; a.grid = grid; a.cluster_s = cs;
    a.sk_tiles = sk_tiles; a.sk_ctas = sk_ctas;
    // large column shares: the copy engine moves them (distributed-shared-memory
    // loads of a large share need many loads in flight, a long unrolled epilogue body)
    a.push = cs > 0 && !(e->gemm_variant & 8) && (size_t)(BN / cs) * TC_BM * 4 >= (size_t)e->gemm_push_min &&
                     ring_need(cs, true, false) <= ring
                 ? 1
                 : 0;
    a.rope_stage = a.push && want_rope && ring_need(cs, true, true) <= ring ? 1 : 0;
    a.idesc = idesc_bf16_f32(TC_BM, BN);
    a.tmem_cols = cols;
    a.ws = m->gemm_ws;
    a.counters = m->gemm_counters;
    a.epi = ep;
    // trace kind: GEMM | epilogue << 4 | 128-row tiles << 8 | tokens / 16 << 24
    const uint32_t tkind = TK_GEMM | ((uint32_t)ep.kind << 4) | ((uint32_t)tiles_m << 8) |
                           ((uint32_t)((m_tok + 15) / 16) << 24);
    a.stamps = m->gemm_stamps;
    if (m->gemm_stamp_kind != 0) {  // test hook: stamps of the launches of one kind only
        if (m->gemm_stamp_kind == tkind && grid <= m->gemm_stamp_cap) m->gemm_stamp_grid = grid;
        else a.stamps = nullptr;
    }
    a.tr = trace_next(e, tkind);
    m->gemm_last_grid = grid;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(TC_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = e->stream;
    cudaLaunchAttribute at[3];
    int na = 0;
    at[na].id = cudaLaunchAttributeClusterDimension;
    at[na].val.clusterDim.x = cs > 0 ? cs : 1;
    at[na].val.clusterDim.y = 1;
    at[na].val.clusterDim.z = 1;
    ++na;
    if (cs > 0 && (e->gemm_variant & 4)) {  // (tuning knob) spread a cluster's CTAs over SMs
        at[na].id = cudaLaunchAttributeClusterSchedulingPolicyPreference;
        at[na].val.clusterSchedulingPolicyPreference = cudaClusterSchedulingPolicySpread;
        ++na;
    }
    if (e->pdl && !e->profiling) {
        at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    cfg.attrs = at;
    cfg.numAttrs = na;
    // fused norm: the residual kind writes x / sums of squares, QKV and gate/up consume them
    const bool fn = ep.kind == EPI_RESID ? ep.nx_out != nullptr : (ep.in_ss != nullptr);
    if (fn && ep.kind == EPI_RESID) YK_ARG(ep.nx_g && ep.nx_ss && ep.ss_ld >= m_tok, "fused norm: outputs");
    if (fn && ep.kind != EPI_RESID) YK_ARG(m_tok <= TC_QKV_STAGE_TOK && ep.ss_ld >= m_tok, "fused norm: input");
    switch (ep.kind) {
        case EPI_QKV: YK_TRY(launch_tc<EPI_QKV>(cfg, tmW, tmX, a, fn)); break;
        case EPI_RESID: YK_TRY(launch_tc<EPI_RESID>(cfg, tmW, tmX, a, fn)); break;
        case EPI_GLU: YK_TRY(launch_tc<EPI_GLU>(cfg, tmW, tmX, a, fn)); break;
        case EPI_LOGITS: YK_TRY(launch_tc<EPI_LOGITS>(cfg, tmW, tmX, a, false)); break;
        default: YK_TRY(launch_tc<EPI_STORE>(cfg, tmW, tmX, a, false)); break;
    }
    e->launches++;
    return YK_OK;
}

// Schedule of one chained stage: grid fixed at one CTA per SM, whole tiles
// round-robin with the remainder stream-K (or all stream-K), no clusters.
static yk_status chain_plan(yk_model* m, int n_out, int K, int m_tok, const EpiParams& ep_in, int grid, TcArgs* a) {
    yk_engine* e = m->e;
    EpiParams ep = ep_in;
    ep.n_out = n_out;
    ep.m_tok = m_tok;
    ep.err = e->d_err;
    YK_ARG(n_out % 4 == 0 && m_tok > 0 && m_tok <= 256 && m_tok <= m->cfg.max_tokens, "chained gemm shape");
    const int BN = ((m_tok + 15) / 16) * 16;
    const int tiles_m = (n_out + TC_BM - 1) / TC_BM;
    const int kb = (K + TC_BK - 1) / TC_BK;
    const long long tiles = tiles_m;
    const long long waves = tiles / grid, rest = tiles % grid;
    int sk_tiles = 0, sk_ctas = 0;
    if (waves == 0 || (e->gemm_variant & 1)) {
        // every stream-K CTA must get at least one k-block (a cut tile counts on a
        // partial from each CTA of its range)
        sk_tiles = (int)tiles;
        sk_ctas = (int)std::min<long long>(grid, tiles * kb);
    } else if (rest > 0) {
        sk_tiles = (int)rest;
        sk_ctas = (int)std::min<long long>(grid, std::max<long long>(1, rest * kb / 8));
    }
    YK_ARG((size_t)2 * sk_ctas * TC_BM * BN <= m->gemm_ws_floats, "split workspace too small");
    uint32_t cols = 32;
    while ((int)cols < BN) cols <<= 1;
    const uint32_t stage_bytes = 16384u + (uint32_t)BN * 128u;
    *a = TcArgs{};
    a->n_out = n_out; a->K = K; a->m_tok = m_tok;
    a->tiles_m = tiles_m; a->kb_total = kb;
    a->BN = BN;
    a->stages = std::max(2, std::min(8, (int)(TC_SMEM_BUDGET / stage_bytes)));
    a->tiles = (int)tiles; a->grid = grid; a->cluster_s = 0;
    a->sk_tiles = sk_tiles; a->sk_ctas = sk_ctas;
    a->idesc = idesc_bf16_f32(TC_BM, BN);
    a->tmem_cols = cols;
    a->ws = m->gemm_ws;
    a->epi = ep;
    a->stamps = nullptr;
    return YK_OK;
}

template <bool F0, bool F1>
static yk_status launch_chain(const cudaLaunchConfig_t& cfg, const CUtensorMap* w0, const CUtensorMap* x0,
                              const CUtensorMap* w1, const CUtensorMap* x1, const TcArgs& a0, const TcArgs& a1,
                              const ChainArgs& ch) {
    static bool attr = false;
    if (!attr) {
        YK_CHECK_CUDA(cudaFuncSetAttribute(gemm_chain_kernel<EPI_GLU, F0, EPI_RESID, F1>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           TC_SMEM_BUDGET + 16384 + TC_SMEM_TAIL));
        attr = true;
    }
    YK_CHECK_CUDA(cudaLaunchKernelEx(&cfg, gemm_chain_kernel<EPI_GLU, F0, EPI_RESID, F1>, *w0, *x0, *w1, *x1, a0, a1,
                                     ch));
    return YK_OK;
}

// gate/up (GLU epilogue, input X0) then down_proj (residual epilogue, input the
// GLU output X1) in one persistent launch of one CTA per SM.
yk_status gemm_chain_glu_down(yk_model* m, const void* Wgu, const CUtensorMap* tmWgu, const void* X0, int n_gu, int K0,
                              const void* Wd, const CUtensorMap* tmWd, const void* X1, int n_d, int K1, int m_tok,
                              const EpiParams& eg, const EpiParams& ed) {
    yk_engine* e = m->e;
    YK_ARG(m->cfg.dtype == YK_DTYPE_BF16, "chained GEMMs are bf16");
    const int grid = e->num_sms;
    TcArgs a0, a1;
    YK_TRY(chain_plan(m, n_gu, K0, m_tok, eg, grid, &a0));
    YK_TRY(chain_plan(m, n_d, K1, m_tok, ed, grid, &a1));
    const int need = a0.tiles + a1.tiles;
    if (need > m->gemm_counter_cap) {
        YK_CHECK_CUDA(cudaStreamSynchronize(e->stream));
        if (m->gemm_counters) cudaFree(m->gemm_counters);
        m->gemm_counters = nullptr;
        m->gemm_counter_cap = 0;
        YK_CHECK_CUDA(cudaMalloc(&m->gemm_counters, (size_t)need * 2 * 4));
        YK_CHECK_CUDA(cudaMemset(m->gemm_counters, 0, (size_t)need * 2 * 4));
        m->gemm_counter_cap = need * 2;
    }
    a0.counters = m->gemm_counters;
    a1.counters = m->gemm_counters + a0.tiles;
    const bool f0 = eg.in_ss != nullptr, f1 = ed.nx_out != nullptr;
    if (f0) YK_ARG(m_tok <= TC_QKV_STAGE_TOK && eg.ss_ld >= m_tok, "fused norm: input");
    if (f1) YK_ARG(ed.nx_g && ed.nx_ss && ed.ss_ld >= m_tok, "fused norm: outputs");
    const CUtensorMap *x0 = nullptr, *x1 = nullptr;
    YK_TRY(get_x_map(m, X0, K0, a0.BN, &x0));
    YK_TRY(get_x_map(m, X1, K1, a1.BN, &x1));
    if (!m->chain_bar) {
        YK_CHECK_CUDA(cudaMalloc(&m->chain_bar, 4));
        YK_CHECK_CUDA(cudaMemset(m->chain_bar, 0, 4));
        m->chain_epoch = 0;
    }
    ChainArgs ch;
    ch.bar = m->chain_bar;
    ch.target = m->chain_epoch + (uint32_t)grid;  // (every CTA adds 1 once, whatever path it takes)
    // trace kind: the gate/up shape (the launch covers both projections)
    a0.tr = trace_next(e, TK_GEMM | ((uint32_t)EPI_GLU << 4) | ((uint32_t)a0.tiles_m << 8) |
                              ((uint32_t)((m_tok + 15) / 16) << 24) | (1u << 31));
    const uint32_t stage_bytes = 16384u + (uint32_t)a0.BN * 128u;
    const size_t smem = (size_t)a0.stages * stage_bytes + TC_SMEM_TAIL;
    const double es = 2.0;
    ProfScope prof(e, YK_PROF_GEMM,
                   ((double)n_gu + m_tok) * K0 * es + ((double)n_d + m_tok) * K1 * es + (double)m_tok * (n_gu / 2) * es +
                       (double)m_tok * n_d * 8.0,
                   2.0 * ((double)n_gu * K0 + (double)n_d * K1) * m_tok);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(TC_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = e->stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = (e->pdl && !e->profiling) ? 1 : 0;
    if (f0 && f1) YK_TRY((launch_chain<true, true>(cfg, tmWgu, x0, tmWd, x1, a0, a1, ch)));
    else if (f0) YK_TRY((launch_chain<true, false>(cfg, tmWgu, x0, tmWd, x1, a0, a1, ch)));
    else if (f1) YK_TRY((launch_chain<false, true>(cfg, tmWgu, x0, tmWd, x1, a0, a1, ch)));
    else YK_TRY((launch_chain<false, false>(cfg, tmWgu, x0, tmWd, x1, a0, a1, ch)));
    m->chain_epoch = ch.target;  // only once the launch went in
    e->launches++;
    return YK_OK;
}

}  // namespace yk

// ---------------------------------------------------------------------------
// Test hooks (include/yk_testing.h): one tcgen05 GEMM with a plain fp32 store.
// ---------------------------------------------------------------------------
#include "../../include/yk_testing.h"

extern "C" yk_status ykt_gemm_bf16_timed(yk_engine* e, const uint16_t* W, const uint16_t* X, int32_t n_out,
                                         int32_t K, int32_t m_tok, int32_t grid, int32_t reps, float* Y,
                                         float* ms_per_rep, uint64_t* stamps, int32_t* grid_used) {
    YK_ARG(e && W && X && Y && n_out > 0 && K > 0 && m_tok > 0 && reps != 0, "arguments");
    const bool cold = reps < 0;
    if (cold) reps = -reps;
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    yk_model m;
    m.e = e;
    m.cfg.dtype = YK_DTYPE_BF16;
    m.cfg.max_tokens = m_tok;
    void *dW = nullptr, *dX = nullptr, *dY = nullptr, *dFlush = nullptr;
    constexpr size_t kFlushBytes = size_t(256) << 20;
    auto cleanup = [&]() {
        cudaStreamSynchronize(e->stream);
        if (dW) cudaFree(dW);
        if (dX) cudaFree(dX);
        if (dY) cudaFree(dY);
        if (dFlush) cudaFree(dFlush);
        if (m.gemm_ws) cudaFree(m.gemm_ws);
        if (m.gemm_counters) cudaFree(m.gemm_counters);
        if (m.gemm_stamps) cudaFree(m.gemm_stamps);
        m.gemm_counters = nullptr;
        m.gemm_stamps = nullptr;
    };
    // largest grid the launch can use: a forced stream-K grid, or a cluster grid
    // (tiles x CS with tiles < SMs/2 and CS <= 8, or a forced CS on any tile count)
    const int max_grid = std::max(std::max(grid, 4 * e->num_sms), 8 * ((n_out + 127) / 128) * ((m_tok + 255) / 256));
    m.gemm_ws_floats = (size_t)2 * std::max(grid, e->num_sms) * 128 * 256;
    m.gemm_counter_cap = 4096;
    if (cudaMalloc(&dW, (size_t)n_out * K * 2) != cudaSuccess || cudaMalloc(&dX, (size_t)m_tok * K * 2) != cudaSuccess ||
        cudaMalloc(&dY, (size_t)m_tok * n_out * 4) != cudaSuccess ||
        cudaMalloc(&m.gemm_ws, m.gemm_ws_floats * 4) != cudaSuccess ||
        cudaMalloc(&m.gemm_counters, (size_t)m.gemm_counter_cap * 4) != cudaSuccess ||
        (cold && cudaMalloc(&dFlush, kFlushBytes) != cudaSuccess)) {
        cleanup();
        yk_set_error("ykt_gemm_bf16: cudaMalloc failed");
        return YK_ERR_OOM;
    }
    cudaError_t up = cudaMemset(m.gemm_counters, 0, (size_t)m.gemm_counter_cap * 4);
    if (up == cudaSuccess) up = cudaMemcpy(dW, W, (size_t)n_out * K * 2, cudaMemcpyHostToDevice);
    if (up == cudaSuccess) up = cudaMemcpy(dX, X, (size_t)m_tok * K * 2, cudaMemcpyHostToDevice);
    if (up != cudaSuccess) {
        cleanup();
        yk_set_error(std::string("ykt_gemm_bf16: upload failed: ") + cudaGetErrorString(up));
        return YK_ERR_CUDA;
    }
    CUtensorMap tmW;
    yk_status s = yk::make_weight_map(e, &tmW, dW, n_out, K);
    yk::EpiParams ep;
    ep.kind = yk::EPI_STORE;
    ep.out = dY;
    if (s == YK_OK) s = yk::gemm_run(&m, dW, &tmW, dX, n_out, K, m_tok, ep, grid);  // result (and warm-up)
    if (s == YK_OK && (reps > 1 || ms_per_rep || stamps)) {
        if (stamps && cudaMalloc(&m.gemm_stamps, (size_t)max_grid * 8 * 8) != cudaSuccess) {
            m.gemm_stamps = nullptr;
            s = YK_ERR_OOM;
        }
        cudaEvent_t t0, t1;
        cudaEventCreate(&t0);
        cudaEventCreate(&t1);
        float ms = 0.f;
        if (cold) {
            for (int r = 0; r < reps && s == YK_OK; ++r) {
                cudaMemsetAsync(dFlush, r & 0xff, kFlushBytes, e->stream);
                cudaEventRecord(t0, e->stream);
                s = yk::gemm_run(&m, dW, &tmW, dX, n_out, K, m_tok, ep, grid);
                cudaEventRecord(t1, e->stream);
                cudaEventSynchronize(t1);
                float one = 0.f;
                cudaEventElapsedTime(&one, t0, t1);
                ms += one;
            }
        } else {
            cudaEventRecord(t0, e->stream);
            for (int r = 0; r < reps && s == YK_OK; ++r) s = yk::gemm_run(&m, dW, &tmW, dX, n_out, K, m_tok, ep, grid);
            cudaEventRecord(t1, e->stream);
            cudaEventSynchronize(t1);
            cudaEventElapsedTime(&ms, t0, t1);
        }
        if (ms_per_rep) *ms_per_rep = ms / reps;
        cudaEventDestroy(t0);
        cudaEventDestroy(t1);
        if (stamps && m.gemm_stamps)
            cudaMemcpy(stamps, m.gemm_stamps, (size_t)m.gemm_last_grid * 8 * 8, cudaMemcpyDeviceToHost);
    }
    if (grid_used) *grid_used = m.gemm_last_grid;
    if (s == YK_OK) {
        cudaError_t ce = cudaStreamSynchronize(e->stream);
        if (ce == cudaSuccess) ce = cudaMemcpy(Y, dY, (size_t)m_tok * n_out * 4, cudaMemcpyDeviceToHost);
        if (ce != cudaSuccess) {
            yk_set_error(std::string("ykt_gemm_bf16: ") + cudaGetErrorString(ce));
            s = YK_ERR_CUDA;
        }
        uint32_t err = 0;
        cudaMemcpy(&err, e->d_err, 4, cudaMemcpyDeviceToHost);
        if (s == YK_OK && err) {
            cudaMemset(e->d_err, 0, 4);
            yk_set_error("ykt_gemm_bf16: device error word " + std::to_string(err));
            s = (err & YK_DEV_ERR_TIMEOUT) ? YK_ERR_TIMEOUT : YK_ERR_DEVICE_CHECK;
        }
    }
    cleanup();
    return s;
}

extern "C" yk_status ykt_gemm_bf16(yk_engine* e, const uint16_t* W, const uint16_t* X, int32_t n_out, int32_t K,
                                   int32_t m_tok, int32_t grid, float* Y) {
    return ykt_gemm_bf16_timed(e, W, X, n_out, K, m_tok, grid, 1, Y, nullptr, nullptr, nullptr);
}

extern "C" yk_status ykt_gemm_bf16_epi_timed(yk_engine* e, const uint16_t* W, const uint16_t* X, int32_t n_out,
                                             int32_t K, int32_t m_tok, int32_t grid, int32_t reps, int32_t epi,
                                             int32_t head_dim, int32_t kv_dim, float* ms_per_rep, uint64_t* stamps,
                                             int32_t* grid_used) {
    YK_ARG(e && W && X && n_out > 0 && K > 0 && m_tok > 0 && reps != 0 && epi >= 0 && epi <= 4, "arguments");
    YK_ARG(epi != yk::EPI_QKV || (head_dim > 0 && kv_dim > 0 && n_out > 2 * kv_dim && kv_dim % head_dim == 0),
           "QKV split");
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    const bool cold = reps < 0;
    if (cold) reps = -reps;
    yk_model m;
    m.e = e;
    m.cfg.dtype = YK_DTYPE_BF16;
    m.cfg.max_tokens = m_tok;
    std::vector<void*> bufs;
    auto dmalloc = [&](size_t bytes) -> void* {
        void* ptr = nullptr;
        if (cudaMalloc(&ptr, bytes) != cudaSuccess) return nullptr;
        cudaMemset(ptr, 0, bytes);
        bufs.push_back(ptr);
        return ptr;
    };
    constexpr size_t kFlushBytes = size_t(256) << 20;
    const int max_grid = std::max(std::max(grid, 4 * e->num_sms), 8 * ((n_out + 127) / 128) * ((m_tok + 255) / 256));
    m.gemm_ws_floats = (size_t)2 * std::max(grid, e->num_sms) * 128 * 256;
    m.gemm_counter_cap = 4096;
    void* dW = dmalloc((size_t)n_out * K * 2);
    void* dX = dmalloc((size_t)m_tok * K * 2);
    void* dY = dmalloc((size_t)m_tok * n_out * 4);
    m.gemm_ws = (float*)dmalloc(m.gemm_ws_floats * 4);
    m.gemm_counters = (uint32_t*)dmalloc((size_t)m.gemm_counter_cap * 4);
    m.gemm_stamps = stamps ? (unsigned long long*)dmalloc((size_t)max_grid * 8 * 8) : nullptr;
    void* dFlush = cold ? dmalloc(kFlushBytes) : nullptr;
    yk::EpiParams ep;
    ep.kind = epi;
    ep.out = dY;
    ep.h = (float*)dY;
    ep.ld = n_out;
    ep.act = YK_ACT_SILU;
    int32_t *dpos = nullptr, *dslot = nullptr;
    float* dden = nullptr;
    void* dpool = nullptr;
    if (epi == yk::EPI_QKV) {
        const int n_kv = kv_dim / head_dim;
        ep.q_dim = n_out - 2 * kv_dim;
        ep.kv_dim = kv_dim;
        ep.head_dim = head_dim;
        ep.n_kv = n_kv;
        ep.block_elems = (long long)2 * n_kv * 16 * head_dim;
        ep.layer_off = 0;
        ep.pool_blocks = m_tok;
        dpool = dmalloc((size_t)ep.block_elems * m_tok * 2);
        dpos = (int32_t*)dmalloc((size_t)m_tok * 4);
        dslot = (int32_t*)dmalloc((size_t)m_tok * 4);
        dden = (float*)dmalloc((size_t)head_dim / 2 * 4);
        std::vector<int32_t> hp(m_tok), hs(m_tok);
        for (int t = 0; t < m_tok; ++t) {
            hp[t] = 1000 + t;
            hs[t] = t * 16;
        }
        std::vector<float> hd(head_dim / 2);
        for (int i = 0; i < head_dim / 2; ++i) hd[i] = powf(500000.0f, 2.0f * i / head_dim);
        if (dpos && dslot && dden) {
            cudaMemcpy(dpos, hp.data(), hp.size() * 4, cudaMemcpyHostToDevice);
            cudaMemcpy(dslot, hs.data(), hs.size() * 4, cudaMemcpyHostToDevice);
            cudaMemcpy(dden, hd.data(), hd.size() * 4, cudaMemcpyHostToDevice);
        }
        ep.pool = dpool;
        ep.pos = dpos;
        ep.slot = dslot;
        ep.rope_denom = dden;
    }
    yk_status s = YK_OK;
    for (void* b : bufs)
        if (!b) s = YK_ERR_OOM;
    if (!dW || !dX || !dY || !m.gemm_ws || !m.gemm_counters || (stamps && !m.gemm_stamps) || (cold && !dFlush) ||
        (epi == yk::EPI_QKV && (!dpool || !dpos || !dslot || !dden)))
        s = YK_ERR_OOM;
    CUtensorMap tmW;
    if (s == YK_OK) {
        cudaMemcpy(dW, W, (size_t)n_out * K * 2, cudaMemcpyHostToDevice);
        cudaMemcpy(dX, X, (size_t)m_tok * K * 2, cudaMemcpyHostToDevice);
        s = yk::make_weight_map(e, &tmW, dW, n_out, K);
    }
    if (s == YK_OK) s = yk::gemm_run(&m, dW, &tmW, dX, n_out, K, m_tok, ep, grid);  // warm-up
    float ms = 0.f;
    if (s == YK_OK) {
        cudaEvent_t t0, t1;
        cudaEventCreate(&t0);
        cudaEventCreate(&t1);
        for (int r = 0; r < reps && s == YK_OK; ++r) {
            if (cold) cudaMemsetAsync(dFlush, r & 0xff, kFlushBytes, e->stream);
            cudaEventRecord(t0, e->stream);
            s = yk::gemm_run(&m, dW, &tmW, dX, n_out, K, m_tok, ep, grid);
            cudaEventRecord(t1, e->stream);
            cudaEventSynchronize(t1);
            float one = 0.f;
            cudaEventElapsedTime(&one, t0, t1);
            ms += one;
        }
        cudaEventDestroy(t0);
        cudaEventDestroy(t1);
        const cudaError_t ce = cudaStreamSynchronize(e->stream);
        if (s == YK_OK && ce != cudaSuccess) {
            yk_set_error(std::string("ykt_gemm_bf16_epi_timed: ") + cudaGetErrorString(ce));
            s = YK_ERR_CUDA;
        }
        if (s == YK_OK && stamps)
            cudaMemcpy(stamps, m.gemm_stamps, (size_t)m.gemm_last_grid * 8 * 8, cudaMemcpyDeviceToHost);
    }
    if (ms_per_rep) *ms_per_rep = ms / reps;
    if (grid_used) *grid_used = m.gemm_last_grid;
    uint32_t err = 0;
    cudaMemcpy(&err, e->d_err, 4, cudaMemcpyDeviceToHost);
    if (s == YK_OK && err) {
        cudaMemset(e->d_err, 0, 4);
        yk_set_error("ykt_gemm_bf16_epi_timed: device error word " + std::to_string(err));
        s = (err & YK_DEV_ERR_TIMEOUT) ? YK_ERR_TIMEOUT : YK_ERR_DEVICE_CHECK;
    }
    cudaStreamSynchronize(e->stream);
    for (void* b : bufs)
        if (b) cudaFree(b);
    m.gemm_ws = nullptr;
    m.gemm_counters = nullptr;
    m.gemm_stamps = nullptr;
    return s;
}

extern "C" yk_status ykt_gemm_stamps_enable(yk_model* m, uint32_t kind) {
    YK_ARG(m, "arguments");
    YK_CHECK_CUDA(cudaSetDevice(m->e->device));
    YK_CHECK_CUDA(cudaStreamSynchronize(m->e->stream));
    if (m->gemm_stamps) cudaFree(m->gemm_stamps);
    m->gemm_stamps = nullptr;
    m->gemm_stamp_kind = 0;
    m->gemm_stamp_cap = 0;
    m->gemm_stamp_grid = 0;
    if (kind != 0) {
        const int cap = 2 * m->e->num_sms;
        YK_CHECK_CUDA(cudaMalloc(&m->gemm_stamps, (size_t)cap * 8 * 8));
        YK_CHECK_CUDA(cudaMemset(m->gemm_stamps, 0, (size_t)cap * 8 * 8));
        m->gemm_stamp_kind = kind;
        m->gemm_stamp_cap = cap;
    }
    return YK_OK;
}

extern "C" yk_status ykt_gemm_stamps_read(yk_model* m, uint64_t* host, int32_t cap, int32_t* n_ctas) {
    YK_ARG(m && host && n_ctas, "arguments");
    YK_ARG(m->gemm_stamps && m->gemm_stamp_kind, "GEMM stamps are not enabled");
    YK_CHECK_CUDA(cudaSetDevice(m->e->device));
    YK_CHECK_CUDA(cudaStreamSynchronize(m->e->stream));
    const int n = std::min(cap, m->gemm_stamp_grid);
    YK_CHECK_CUDA(cudaMemcpy(host, m->gemm_stamps, (size_t)n * 8 * 8, cudaMemcpyDeviceToHost));
    *n_ctas = n;
    return YK_OK;
}
