// yk_kernels.cu -- embedding gather, RMSNorm, device random init.
#include "yk_common.cuh"
#include "yk_internal.h"

namespace yk {

// embedding_lookup_kernel (S/gemm.metal:326-341): h[t] = E[tokens[t]], fp32 residual stream.
// Also the step's RoPE table: rope[t][i] = (cos, sin)(pos[t] / denom[i]), the
// angle of dimension pair i at token t that every layer's QKV epilogue uses.
// dt.d: the last dt.nd tokens of each sequence are device-resident draft tokens.
// fn.g (fused RMSNorm): also the first GEMM's input x = bf16(h * g) and the sums
// of squares of h over each 32-element group, fn.ss[(i / 32) * T + t].
struct EmbedNorm {
    const float* g = nullptr;
    __nv_bfloat16* x = nullptr;
    float* ss = nullptr;
};
template <typename WT>
__global__ void embed_kernel(const WT* __restrict__ E, const int32_t* __restrict__ tokens, float* __restrict__ h,
                             int d, int V, const int32_t* __restrict__ pos, const float* __restrict__ denom,
                             float2* __restrict__ rope, int half_dh, uint32_t* err, Trace tr, DraftTokens dt,
                             const int32_t* __restrict__ seq_of, const int32_t* __restrict__ q_starts, EmbedNorm fn) {
    if (threadIdx.x == 0) trace_mark(tr, TR_ENTRY);
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x == 0) trace_mark(tr, TR_START);
    const int t = blockIdx.x;
    for (int i = threadIdx.x; i < half_dh; i += blockDim.x) {
        float sn, cs;
        sincosf(__fdiv_rn((float)pos[t], denom[i]), &sn, &cs);
        rope[(size_t)t * half_dh + i] = make_float2(cs, sn);
    }
    int tok = tokens[t];
    if (dt.d) {
        const int b = seq_of[t], qe = q_starts[b + 1];
        if (t >= qe - dt.nd) tok = (int)dt.d[(size_t)b * dt.k + dt.j0 + (t - (qe - dt.nd))];
    }
    if (tok < 0 || tok >= V) {
        if (threadIdx.x == 0) raise_err(err, YK_DEV_ERR_BOUNDS);
        return;
    }
    const WT* row = E + (size_t)tok * d;
    if constexpr (sizeof(WT) == 2) {
        if ((d & 31) == 0) {
            // bf16: 8 consecutive elements per thread (one 16-byte load), every load of
            // the row in flight at once; a 32-element group is 4 neighbouring lanes
            for (int i0 = threadIdx.x * 8; i0 - threadIdx.x * 8 < d; i0 += blockDim.x * 8) {
                const bool on = i0 < d;
                float v[8];
                if (on) {
                    const uint4 raw = *reinterpret_cast<const uint4*>(row + i0);
                    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        v[2 * k] = __uint_as_float(w[k] << 16);
                        v[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
                    }
                    float4* hr = reinterpret_cast<float4*>(h + (size_t)t * d + i0);
                    hr[0] = make_float4(v[0], v[1], v[2], v[3]);
                    hr[1] = make_float4(v[4], v[5], v[6], v[7]);
                } else {
#pragma unroll
                    for (int k = 0; k < 8; ++k) v[k] = 0.f;
                }
                if (fn.g) {
                    float ss = 0.f;
                    if (on) {
                        const float4 g0 = *reinterpret_cast<const float4*>(fn.g + i0);
                        const float4 g1 = *reinterpret_cast<const float4*>(fn.g + i0 + 4);
                        const __nv_bfloat162 x0 = __floats2bfloat162_rn(v[0] * g0.x, v[1] * g0.y);
                        const __nv_bfloat162 x1 = __floats2bfloat162_rn(v[2] * g0.z, v[3] * g0.w);
                        const __nv_bfloat162 x2 = __floats2bfloat162_rn(v[4] * g1.x, v[5] * g1.y);
                        const __nv_bfloat162 x3 = __floats2bfloat162_rn(v[6] * g1.z, v[7] * g1.w);
                        *reinterpret_cast<uint4*>(fn.x + (size_t)t * d + i0) =
                            make_uint4(*reinterpret_cast<const uint32_t*>(&x0), *reinterpret_cast<const uint32_t*>(&x1),
                                       *reinterpret_cast<const uint32_t*>(&x2), *reinterpret_cast<const uint32_t*>(&x3));
#pragma unroll
                        for (int k = 0; k < 8; ++k) ss += v[k] * v[k];
                    }
                    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
                    ss += __shfl_xor_sync(0xffffffffu, ss, 2);
                    if (on && (threadIdx.x & 3) == 0) fn.ss[(size_t)(i0 >> 5) * gridDim.x + t] = ss;
                }
            }
            if (threadIdx.x == 0) trace_mark(tr, TR_END);
            return;
        }
    }
    if (!fn.g) {
        for (int i = threadIdx.x; i < d; i += blockDim.x) h[(size_t)t * d + i] = to_f32(row[i]);
    } else {
        // every thread runs every pass (warp sums); a warp's 32 elements form one group
        for (int i0 = 0; i0 < d; i0 += blockDim.x) {
            const int i = i0 + threadIdx.x;
            float v = 0.f;
            if (i < d) {
                v = to_f32(row[i]);
                h[(size_t)t * d + i] = v;
                fn.x[(size_t)t * d + i] = __float2bfloat16_rn(v * fn.g[i]);
            }
            float ss = v * v;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            if ((threadIdx.x & 31) == 0 && i < d) fn.ss[(size_t)(i >> 5) * gridDim.x + t] = ss;
        }
    }
    if (threadIdx.x == 0) trace_mark(tr, TR_END);
}

// rmsnorm_kernel (S/gemm.metal:377-401): y = x * rsqrt(mean(x^2) + eps) * gamma,
// one CTA per row, fp32 statistics.  rows != nullptr gathers input rows.  The
// row stays in registers (float4 loads, up to RN_VEC vectors per thread): one
// read of x, one block reduction, one bf16/fp32 write.
// rows up to 8192 elements (the 70B shape's d_model) in registers; wider rows
// take the strided loop, which re-reads the row
constexpr int RN_THREADS = 256, RN_VEC = 8;
__device__ __forceinline__ void store4(float* y, float a, float b, float c, float d) {
    *reinterpret_cast<float4*>(y) = make_float4(a, b, c, d);
}
__device__ __forceinline__ void store4(__nv_bfloat16* y, float a, float b, float c, float d) {
    const __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
    *reinterpret_cast<uint2*>(y) =
        make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
}
template <typename AT>
__global__ void __launch_bounds__(RN_THREADS) rmsnorm_kernel(float* __restrict__ x, const float* __restrict__ g,
                                                            AT* __restrict__ y, int d, float eps,
                                                            const int32_t* __restrict__ rows,
                                                            const void* __restrict__ add, int add_bf16, Trace tr) {
    if (threadIdx.x == 0) trace_mark(tr, TR_ENTRY);
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x == 0) trace_mark(tr, TR_START);
    const int r = blockIdx.x;
    const int src = rows ? rows[r] : r;
    float* xr = x + (size_t)src * d;
    // pending residual (fp32, or bf16 when add_bf16): x += add first
    const float* ar = add && !add_bf16 ? reinterpret_cast<const float*>(add) + (size_t)src * d : nullptr;
    const __nv_bfloat16* ab =
        add && add_bf16 ? reinterpret_cast<const __nv_bfloat16*>(add) + (size_t)src * d : nullptr;
    __shared__ float red[RN_THREADS / 32];
    float ss = 0.f;
    const bool vec = (d & 3) == 0 && d <= RN_THREADS * 4 * RN_VEC;
    float4 xv[RN_VEC];
    if (vec) {
#pragma unroll
        for (int k = 0; k < RN_VEC; ++k) {
            const int i = (threadIdx.x + k * RN_THREADS) * 4;
            xv[k] = i < d ? *reinterpret_cast<const float4*>(xr + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            if ((ar || ab) && i < d) {
                float4 av;
                if (ar) {
                    av = *reinterpret_cast<const float4*>(ar + i);
                } else {
                    const uint2 raw = *reinterpret_cast<const uint2*>(ab + i);
                    const __nv_bfloat162 lo = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
                    const __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
                    av = make_float4(__low2float(lo), __high2float(lo), __low2float(hi), __high2float(hi));
                }
                xv[k] = make_float4(xv[k].x + av.x, xv[k].y + av.y, xv[k].z + av.z, xv[k].w + av.w);
                *reinterpret_cast<float4*>(xr + i) = xv[k];
            }
            ss += xv[k].x * xv[k].x + xv[k].y * xv[k].y + xv[k].z * xv[k].z + xv[k].w * xv[k].w;
        }
    } else {
        for (int i = threadIdx.x; i < d; i += RN_THREADS) {
            if (ar) xr[i] += ar[i];
            else if (ab) xr[i] += __bfloat162float(ab[i]);
            ss += xr[i] * xr[i];
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < RN_THREADS / 32; ++w) tot += red[w];
    const float rms = 1.0f / sqrtf(tot / (float)d + eps);
    AT* yr = y + (size_t)r * d;
    if (vec) {
#pragma unroll
        for (int k = 0; k < RN_VEC; ++k) {
            const int i = (threadIdx.x + k * RN_THREADS) * 4;
            if (i < d) {
                const float4 gv = *reinterpret_cast<const float4*>(g + i);
                store4(yr + i, xv[k].x * rms * gv.x, xv[k].y * rms * gv.y, xv[k].z * rms * gv.z,
                       xv[k].w * rms * gv.w);
            }
        }
    } else {
        for (int i = threadIdx.x; i < d; i += RN_THREADS) yr[i] = from_f32<AT>(xr[i] * rms * g[i]);
    }
    if (threadIdx.x == 0) trace_mark(tr, TR_END);
}

// N(0, std) from Philox (Box-Muller), counter = (index lo, index hi, stream, 0).
template <typename T>
__global__ void init_normal_kernel(T* __restrict__ out, size_t n, uint64_t seed, uint32_t stream, float std) {
    const uint2 key = make_uint2((uint32_t)seed, (uint32_t)(seed >> 32));
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const uint4 o = philox4x32_10(make_uint4((uint32_t)i, (uint32_t)(i >> 32), stream, 0u), key);
        const float u1 = ((float)(o.x >> 8) + 1.0f) * (1.0f / 16777216.0f);  // (0, 1]
        const float u2 = (float)(o.y >> 8) * (1.0f / 16777216.0f);
        const float z = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
        out[i] = from_f32<T>(z * std);
    }
}

template <typename T>
__global__ void fill_kernel(T* __restrict__ out, size_t n, float v) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = from_f32<T>(v);
}

// Host launchers -------------------------------------------------------------
yk_status launch_embed(yk_model* m, const int32_t* tokens, const int32_t* pos, int T, const DraftTokens& dt,
                       const float* norm_g) {
    const auto& c = m->cfg;
    EmbedNorm fn;
    if (norm_g) {  // fused RMSNorm of the first layer (bf16)
        fn.g = norm_g;
        fn.x = (__nv_bfloat16*)m->xn;
        fn.ss = m->norm_ss;
    }
    if (c.dtype == YK_DTYPE_BF16)
        YK_CHECK_CUDA(launch_pdl(m->e, embed_kernel<__nv_bfloat16>, T, 256, 0, (const __nv_bfloat16*)m->embed, tokens,
                                 m->h, c.d_model, c.vocab_size, pos, (const float*)m->rope_denom, m->rope_tab,
                                 c.head_dim / 2, m->e->d_err, trace_next(m->e, TK_EMBED), dt, m->cur.seq,
                                 m->cur.q_starts, fn));
    else
        YK_CHECK_CUDA(launch_pdl(m->e, embed_kernel<float>, T, 256, 0, (const float*)m->embed, tokens, m->h, c.d_model,
                                 c.vocab_size, pos, (const float*)m->rope_denom, m->rope_tab, c.head_dim / 2,
                                 m->e->d_err, trace_next(m->e, TK_EMBED), dt, m->cur.seq, m->cur.q_starts, EmbedNorm{}));
    m->e->launches++;
    return YK_OK;
}

yk_status launch_rmsnorm(yk_model* m, const float* g, int rows, const int32_t* row_idx, const void* add,
                         int add_bf16) {
    const auto& c = m->cfg;
    if (c.dtype == YK_DTYPE_BF16)
        YK_CHECK_CUDA(launch_pdl(m->e, rmsnorm_kernel<__nv_bfloat16>, rows, RN_THREADS, 0, m->h, g,
                                 (__nv_bfloat16*)m->xn, c.d_model, c.rms_eps, row_idx, add, add_bf16,
                                 trace_next(m->e, TK_RMSNORM)));
    else
        YK_CHECK_CUDA(launch_pdl(m->e, rmsnorm_kernel<float>, rows, RN_THREADS, 0, m->h, g, (float*)m->xn, c.d_model,
                                 c.rms_eps, row_idx, add, add_bf16, trace_next(m->e, TK_RMSNORM)));
    m->e->launches++;
    return YK_OK;
}

yk_status launch_init(yk_engine* e, void* p, size_t n, int dtype, uint64_t seed, uint32_t stream, float std,
                      bool constant) {
    const int blocks = 148 * 8;
    if (dtype == YK_DTYPE_BF16) {
        if (constant) fill_kernel<__nv_bfloat16><<<blocks, 256, 0, e->stream>>>((__nv_bfloat16*)p, n, std);
        else init_normal_kernel<__nv_bfloat16><<<blocks, 256, 0, e->stream>>>((__nv_bfloat16*)p, n, seed, stream, std);
    } else {
        if (constant) fill_kernel<float><<<blocks, 256, 0, e->stream>>>((float*)p, n, std);
        else init_normal_kernel<float><<<blocks, 256, 0, e->stream>>>((float*)p, n, seed, stream, std);
    }
    e->launches++;
    YK_CHECK_CUDA(cudaGetLastError());
    return YK_OK;
}

}  // namespace yk

// ---------------------------------------------------------------------------
// Test hook (include/yk_testing.h): the bounded-wait failure path.  One thread
// waits on a shared-memory mbarrier that nothing ever arrives at, with the same
// bounded wait every kernel uses but a budget of budget_ns; when the wait gives
// up it records the timeout in the engine's error word and the kernel returns.
// ---------------------------------------------------------------------------
namespace yk {
__global__ void wait_timeout_kernel(uint32_t* err, uint64_t budget_ns, unsigned long long* waited_ns) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    mbar_init(smem_u32(&bar), 1);
    mbar_fence_init();
    const uint64_t t0 = globaltimer_ns();
    if (!mbar_wait_bounded_ns(smem_u32(&bar), 0u, budget_ns)) raise_err(err, YK_DEV_ERR_TIMEOUT);
    *waited_ns = globaltimer_ns() - t0;
}
}  // namespace yk

#include "../../include/yk_testing.h"

extern "C" yk_status ykt_wait_timeout(yk_engine* e, int32_t budget_ms, double* waited_ms) {
    YK_ARG(e && budget_ms > 0 && budget_ms <= 2000, "arguments");
    YK_CHECK_CUDA(cudaSetDevice(e->device));
    unsigned long long* d = nullptr;
    YK_CHECK_CUDA(cudaMalloc(&d, sizeof(unsigned long long)));
    yk::wait_timeout_kernel<<<1, 32, 0, e->stream>>>(e->d_err, (uint64_t)budget_ms * 1000000ull, d);
    e->launches++;
    unsigned long long ns = 0;
    uint32_t err = 0;
    cudaError_t r = cudaGetLastError();
    if (r == cudaSuccess) r = cudaMemcpyAsync(&ns, d, sizeof(ns), cudaMemcpyDeviceToHost, e->stream);
    if (r == cudaSuccess) r = cudaMemcpyAsync(&err, e->d_err, 4, cudaMemcpyDeviceToHost, e->stream);
    if (r == cudaSuccess) r = cudaStreamSynchronize(e->stream);
    cudaFree(d);
    YK_CHECK_CUDA(r);
    if (waited_ms) *waited_ms = (double)ns / 1e6;
    if (err) {
        YK_CHECK_CUDA(cudaMemset(e->d_err, 0, 4));
        yk_set_error("a bounded device wait gave up (code " + std::to_string(err) + ")");
        return (err & YK_DEV_ERR_TIMEOUT) ? YK_ERR_TIMEOUT : YK_ERR_DEVICE_CHECK;
    }
    return YK_OK;
}
