// yk_gemm.cu -- the verify-forward linear layers (replaces LinearLayer.forward /
// gemm_kernel, S/LinearLayer.swift:71-128, S/gemm.metal:6-34).
//
// bf16: swap-AB tcgen05 GEMM.  D[n][j] = sum_k W[n][k] * X[j][k]: the weight
// tile (128 output rows x 64 k) is the MMA "A" operand, the tokens (BN <= 256)
// are the MMA "N" dimension, so at verify batch sizes every weight byte is
// streamed from HBM exactly once.  TMA (no multicast) stages W and X tiles with
// 128-byte swizzle into a multi-stage mbarrier pipeline; one thread issues
// tcgen05.mma into a TMEM accumulator; all four warps drain TMEM through the
// fused epilogue.  Split-K spreads skinny layers over all SMs; the last CTA of
// a tile sums the fp32 partials in fixed split order (deterministic) and runs
// the epilogue.
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
constexpr int TC_THREADS = 128;  // 4 warps: TMA producer lane, MMA lane, 4 epilogue warps
constexpr int TC_SMEM_BUDGET = 200 * 1024;

struct TcArgs {
    int n_out, K, m_tok;
    int tiles_m, splits, kb_total;
    int BN, stages;
    uint32_t idesc, tmem_cols;
    float* ws;
    uint32_t* counters;
    EpiParams epi;
};

__global__ void __launch_bounds__(TC_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, const TcArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int BN = a.BN, S = a.stages;
    const uint32_t stage_bytes = 16384u + (uint32_t)BN * 128u;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)S * stage_bytes);
    uint64_t* full = bars;
    uint64_t* empty = bars + S;
    uint64_t* accb = bars + 2 * S;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 1);
    volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 1);  // [0] abort, [1] last

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int unit = blockIdx.x;
    const int split = unit % a.splits;
    const int tile = unit / a.splits;
    const int tm = tile % a.tiles_m, tn = tile / a.tiles_m;
    const int kb0 = (int)(((long long)split * a.kb_total) / a.splits);
    const int kb1 = (int)(((long long)(split + 1) * a.kb_total) / a.splits);
    const int nkb = kb1 - kb0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        mbar_init(smem_u32(accb), 1);
        flags[0] = 0;
        flags[1] = 0;
        mbar_fence_init();
    }
    if (warp == 0) tmem_alloc(smem_u32(tmem_slot), a.tmem_cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    int issued_round[8];
#pragma unroll
    for (int s = 0; s < 8; ++s) issued_round[s] = -1;

    if (threadIdx.x == 0) {
        // ---------------- TMA producer ----------------
        const uint64_t pol_w = policy_evict_first();
        const uint64_t pol_x = policy_evict_last();
        for (int i = 0; i < nkb; ++i) {
            const int s = i % S;
            const int r = i / S;
            if (r > 0 && !mbar_wait_bounded(smem_u32(&empty[s]), (uint32_t)((r - 1) & 1))) {
                flags[0] = 1;
                raise_err(a.epi.err, YK_DEV_ERR_TIMEOUT);
                break;
            }
            if (flags[0]) break;
            const uint32_t wdst = smem_u32(smem + (size_t)s * stage_bytes);
            const uint32_t xdst = wdst + 16384u;
            const uint32_t fb = smem_u32(&full[s]);
            mbar_arrive_expect_tx(fb, stage_bytes);
            tma_load_2d(wdst, &tmW, (kb0 + i) * TC_BK, tm * TC_BM, fb, pol_w);
            tma_load_2d(xdst, &tmX, (kb0 + i) * TC_BK, tn * BN, fb, pol_x);
            if (s < 8) issued_round[s] = r;
        }
    } else if (threadIdx.x == 32) {
        // ---------------- MMA issuer ----------------
        for (int i = 0; i < nkb; ++i) {
            const int s = i % S;
            const int r = i / S;
            if (!mbar_wait_bounded(smem_u32(&full[s]), (uint32_t)(r & 1))) {
                flags[0] = 1;
                raise_err(a.epi.err, YK_DEV_ERR_TIMEOUT);
                break;
            }
            tc_fence_after();
            const uint32_t wsm = smem_u32(smem + (size_t)s * stage_bytes);
            const uint32_t xsm = wsm + 16384u;
#pragma unroll
            for (int kk = 0; kk < TC_BK / 16; ++kk) {
                const uint64_t ad = sw128_kmajor_desc(wsm + kk * 32);
                const uint64_t bd = sw128_kmajor_desc(xsm + kk * 32);
                tc_mma_bf16(tmem, ad, bd, a.idesc, (i > 0 || kk > 0) ? 1u : 0u);
            }
            tc_commit(smem_u32(&empty[s]));
        }
        tc_commit(smem_u32(accb));
    }
    __syncwarp();

    // ---------------- epilogue: all 4 warps ----------------
    const bool acc_ok = mbar_wait_bounded(smem_u32(accb), 0);
    if (!acc_ok) {
        flags[0] = 1;
        raise_err(a.epi.err, YK_DEV_ERR_TIMEOUT);
    }
    tc_fence_after();
    __syncthreads();
    const bool aborted = flags[0] != 0;
    const int row = warp * 32 + lane;  // TMEM lane == output row within the tile
    const int n_base = tm * TC_BM;
    const int j_base = tn * BN;
    const uint32_t t_lane = tmem + ((uint32_t)(warp * 32) << 16);

    if (threadIdx.x == 0 && aborted) {
        // Let every TMA copy this CTA issued land before the stage buffers are reused.
        for (int s = 0; s < S && s < 8; ++s)
            if (issued_round[s] >= 0) (void)mbar_wait_bounded(smem_u32(&full[s]), (uint32_t)(issued_round[s] & 1));
    }
    __syncthreads();
    // Accumulator -> shared memory [BN][128] fp32 (the stage buffers are free now:
    // every TMA load was consumed and every MMA completed before accb fired).
    float* red = reinterpret_cast<float*>(smem);
    if (!aborted) {
        for (int c = 0; c < BN; c += 16) {
            uint32_t r[16];
            tmem_ld16(t_lane + (uint32_t)c, r);
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) red[(c + jj) * TC_BM + row] = __uint_as_float(r[jj]);
        }
    } else {
        for (int c = 0; c < BN; ++c) red[c * TC_BM + row] = 0.f;
    }
    // Split-K: the `splits` CTAs of a tile form one cluster.  After the barrier
    // each CTA reduces its share of the tile's columns over every CTA's partial
    // through distributed shared memory, always in rank order (deterministic),
    // and runs the epilogue for those columns.
    const int S_k = a.splits;
    const uint32_t rank = S_k > 1 ? cluster_ctarank() : 0u;
    if (S_k > 1) cluster_sync_all(); else __syncthreads();
    const int c0 = (int)((rank * (uint32_t)BN) / (uint32_t)S_k);
    const int c1 = (int)(((rank + 1) * (uint32_t)BN) / (uint32_t)S_k);
    const uint32_t red_addr = smem_u32(red);
    constexpr int NB = 8;
    for (int c = c0; c < c1; c += NB) {
        float v[NB], w[NB];
#pragma unroll
        for (int i = 0; i < NB; ++i) v[i] = 0.f;
        if (S_k == 1) {
#pragma unroll
            for (int i = 0; i < NB; ++i)
                if (c + i < c1) v[i] = red[(c + i) * TC_BM + row];
        } else {
            for (int sp = 0; sp < S_k; ++sp) {
                const uint32_t base = mapa_shared(red_addr, (uint32_t)sp);
                float t[NB];
#pragma unroll
                for (int i = 0; i < NB; ++i)
                    t[i] = (c + i < c1) ? ld_shared_cluster_f32(base + (uint32_t)(((c + i) * TC_BM + row) * 4)) : 0.f;
#pragma unroll
                for (int i = 0; i < NB; ++i) v[i] += t[i];
            }
        }
#pragma unroll
        for (int i = 0; i < NB; ++i) w[i] = __shfl_xor_sync(0xffffffffu, v[i], 1);
        if (!aborted && (lane & 1) == 0) {
            if (c + NB <= c1) {
                epi_batch<__nv_bfloat16, NB>(a.epi, n_base + row, j_base + c, v, w);
            } else {
                for (int i = 0; i < c1 - c; ++i) epi_pair<__nv_bfloat16>(a.epi, n_base + row, j_base + c + i, v[i], w[i]);
            }
        }
    }
    // No CTA may leave while a peer still reads its shared memory.
    if (S_k > 1) cluster_sync_all();

    // ---------------- teardown ----------------
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, a.tmem_cols);
}

// ---------------------------------------------------------------------------
// SIMT GEMM: each warp owns an output-row pair, lanes stride over k; a CTA
// covers 16 rows x 8 tokens.  Used for fp32 weights (and as the GPU-side
// cross-check of the tensor-core path in tests).
// ---------------------------------------------------------------------------
template <typename WT, typename XT>
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
            if (j0 + t < m_tok) epi_pair<XT>(ep, n, j0 + t, acc0[t], acc1[t]);
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

// How many clusters of `s` GEMM CTAs (one CTA per SM) the device runs at once.
static int cluster_capacity(yk_engine* e, int s) {
    static int cap[9] = {0};
    static int dev = -1;
    if (dev != e->device) {
        for (int i = 0; i < 9; ++i) cap[i] = 0;
        dev = e->device;
    }
    if (cap[s] == 0) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(s * 64);
        cfg.blockDim = dim3(TC_THREADS);
        cfg.dynamicSmemBytes = TC_SMEM_BUDGET + 1280;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = s;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, gemm_tc_kernel, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = std::max(1, e->num_sms / s / 2);
        }
        cap[s] = n;
    }
    return cap[s];
}

// Split-K choice (cluster size): minimise waves x (k-blocks per CTA + fixed cost).
static int choose_splits(yk_engine* e, int tiles, int kb) {
    int best = 1;
    double best_cost = 1e30;
    for (int s = 1; s <= std::min(kb, 8); ++s) {
        const int waves = (tiles + cluster_capacity(e, s) - 1) / cluster_capacity(e, s);
        const double cost = waves * ((double)((kb + s - 1) / s) + 3.0 + (s > 1 ? 1.0 : 0.0));
        if (cost < best_cost - 1e-9) { best_cost = cost; best = s; }
    }
    return best;
}

yk_status gemm_run(yk_model* m, const void* W, const CUtensorMap* tmW, const void* X, int n_out, int K, int m_tok,
                   const EpiParams& ep_in, int force_splits) {
    yk_engine* e = m->e;
    EpiParams ep = ep_in;
    ep.n_out = n_out;
    ep.m_tok = m_tok;
    ep.err = e->d_err;
    YK_ARG(n_out % 2 == 0 && m_tok > 0 && m_tok <= m->cfg.max_tokens, "gemm shape");
    // Algorithmic traffic of this launch: weights + activations once, plus the epilogue's outputs.
    const double es = m->cfg.dtype == YK_DTYPE_BF16 ? 2.0 : 4.0;
    double out_bytes = (double)m_tok * n_out * 4.0;
    if (ep.kind == EPI_QKV) out_bytes = (double)m_tok * n_out * es;
    else if (ep.kind == EPI_RESID) out_bytes = (double)m_tok * n_out * 8.0;
    else if (ep.kind == EPI_GLU) out_bytes = (double)m_tok * (n_out / 2) * es;
    ProfScope prof(e, YK_PROF_GEMM, ((double)n_out + m_tok) * K * es + out_bytes, 2.0 * n_out * K * m_tok);
    if (m->cfg.dtype == YK_DTYPE_F32) {
        dim3 grid((n_out + 15) / 16, (m_tok + 7) / 8);
        gemm_simt_kernel<float, float><<<grid, 256, 0, e->stream>>>((const float*)W, (const float*)X, n_out, K, m_tok, ep);
        e->launches++;
        YK_CHECK_CUDA(cudaGetLastError());
        return YK_OK;
    }
    // bf16: tcgen05 path.
    const int BN = m_tok <= 256 ? ((m_tok + 15) / 16) * 16 : 256;
    const int tiles_n = (m_tok + BN - 1) / BN;
    const int tiles_m = (n_out + TC_BM - 1) / TC_BM;
    const int kb = (K + TC_BK - 1) / TC_BK;
    const int tiles = tiles_m * tiles_n;
    static bool attr_set = false;
    if (!attr_set) {
        YK_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           TC_SMEM_BUDGET + 16384 + 2048));
        attr_set = true;
    }
    int splits = choose_splits(e, tiles, kb);
    if (force_splits > 0) {
        YK_ARG(force_splits <= kb && force_splits <= 8, "forced split count must be <= min(k-blocks, 8)");
        splits = force_splits;
    }
    const uint32_t stage_bytes = 16384u + (uint32_t)BN * 128u;
    int stages = std::min(8, (int)(TC_SMEM_BUDGET / stage_bytes));
    stages = std::max(2, std::min(stages, std::max(2, kb)));
    const size_t smem = (size_t)stages * stage_bytes + 1024 + 256;
    uint32_t cols = 32;
    while ((int)cols < BN) cols <<= 1;

    const CUtensorMap* tmX = nullptr;
    YK_TRY(get_x_map(m, X, K, BN, &tmX));
    TcArgs a;
    a.n_out = n_out; a.K = K; a.m_tok = m_tok;
    a.tiles_m = tiles_m; a.splits = splits; a.kb_total = kb;
    a.BN = BN; a.stages = stages;
    a.idesc = idesc_bf16_f32(TC_BM, BN);
    a.tmem_cols = cols;
    a.ws = m->gemm_ws;
    a.counters = m->gemm_counters;
    a.epi = ep;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(tiles * splits);
    cfg.blockDim = dim3(TC_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = e->stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = splits;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    YK_CHECK_CUDA(cudaLaunchKernelEx(&cfg, gemm_tc_kernel, *tmW, *tmX, a));
    e->launches++;
    return YK_OK;
}

}  // namespace yk

// ---------------------------------------------------------------------------
// Test hook (include/yk_testing.h): one tcgen05 GEMM with a plain fp32 store.
// ---------------------------------------------------------------------------
#include "../../include/yk_testing.h"

extern "C" yk_status ykt_gemm_bf16(yk_engine* e, const uint16_t* W, const uint16_t* X, int32_t n_out, int32_t K,
                                   int32_t m_tok, int32_t splits, float* Y) {
    YK_ARG(e && W && X && Y && n_out > 0 && K > 0 && m_tok > 0, "arguments");
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    yk_model m;
    m.e = e;
    m.cfg.dtype = YK_DTYPE_BF16;
    m.cfg.max_tokens = m_tok;
    void *dW = nullptr, *dX = nullptr, *dY = nullptr;
    auto cleanup = [&]() {
        cudaStreamSynchronize(e->stream);
        if (dW) cudaFree(dW);
        if (dX) cudaFree(dX);
        if (dY) cudaFree(dY);
        if (m.gemm_ws) cudaFree(m.gemm_ws);
        if (m.gemm_counters) cudaFree(m.gemm_counters);
    };
    m.gemm_ws_floats = (size_t)2 * e->num_sms * 128 * 256;
    m.gemm_counter_cap = 4096;
    if (cudaMalloc(&dW, (size_t)n_out * K * 2) != cudaSuccess || cudaMalloc(&dX, (size_t)m_tok * K * 2) != cudaSuccess ||
        cudaMalloc(&dY, (size_t)m_tok * n_out * 4) != cudaSuccess ||
        cudaMalloc(&m.gemm_ws, m.gemm_ws_floats * 4) != cudaSuccess ||
        cudaMalloc(&m.gemm_counters, (size_t)m.gemm_counter_cap * 4) != cudaSuccess) {
        cleanup();
        yk_set_error("ykt_gemm_bf16: cudaMalloc failed");
        return YK_ERR_OOM;
    }
    cudaMemset(m.gemm_counters, 0, (size_t)m.gemm_counter_cap * 4);
    cudaMemcpy(dW, W, (size_t)n_out * K * 2, cudaMemcpyHostToDevice);
    cudaMemcpy(dX, X, (size_t)m_tok * K * 2, cudaMemcpyHostToDevice);
    CUtensorMap tmW;
    yk_status s = yk::make_weight_map(e, &tmW, dW, n_out, K);
    if (s == YK_OK) {
        yk::EpiParams ep;
        ep.kind = yk::EPI_STORE;
        ep.out = dY;
        s = yk::gemm_run(&m, dW, &tmW, dX, n_out, K, m_tok, ep, splits);
    }
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
