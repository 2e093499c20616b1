// yk_kernels.cu -- embedding gather, RMSNorm, device random init.
#include "yk_common.cuh"
#include "yk_internal.h"

namespace yk {

// embedding_lookup_kernel (S/gemm.metal:326-341): h[t] = E[tokens[t]], fp32 residual stream.
template <typename WT>
__global__ void embed_kernel(const WT* __restrict__ E, const int32_t* __restrict__ tokens, float* __restrict__ h,
                             int d, int V, uint32_t* err) {
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.x;
    const int tok = tokens[t];
    if (tok < 0 || tok >= V) {
        if (threadIdx.x == 0) raise_err(err, YK_DEV_ERR_BOUNDS);
        return;
    }
    const WT* row = E + (size_t)tok * d;
    for (int i = threadIdx.x; i < d; i += blockDim.x) h[(size_t)t * d + i] = to_f32(row[i]);
}

// rmsnorm_kernel (S/gemm.metal:377-401): y = x * rsqrt(mean(x^2) + eps) * gamma,
// one CTA per row, fp32 statistics.  rows != nullptr gathers input rows.
template <typename AT>
__global__ void rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ g, AT* __restrict__ y, int d,
                               float eps, const int32_t* __restrict__ rows) {
    pdl_trigger();
    pdl_wait();
    const int r = blockIdx.x;
    const int src = rows ? rows[r] : r;
    const float* xr = x + (size_t)src * d;
    float ss = 0.f;
    for (int i = threadIdx.x; i < d; i += blockDim.x) ss += xr[i] * xr[i];
    __shared__ float red[32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    const float rms = 1.0f / sqrtf(red[0] / (float)d + eps);
    for (int i = threadIdx.x; i < d; i += blockDim.x) y[(size_t)r * d + i] = from_f32<AT>(xr[i] * rms * g[i]);
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
yk_status launch_embed(yk_model* m, const int32_t* tokens, int T) {
    const auto& c = m->cfg;
    if (c.dtype == YK_DTYPE_BF16)
        YK_CHECK_CUDA(launch_pdl(m->e, embed_kernel<__nv_bfloat16>, T, 256, 0, (const __nv_bfloat16*)m->embed, tokens,
                                 m->h, c.d_model, c.vocab_size, m->e->d_err));
    else
        YK_CHECK_CUDA(launch_pdl(m->e, embed_kernel<float>, T, 256, 0, (const float*)m->embed, tokens, m->h, c.d_model,
                                 c.vocab_size, m->e->d_err));
    m->e->launches++;
    return YK_OK;
}

yk_status launch_rmsnorm(yk_model* m, const float* g, int rows, const int32_t* row_idx) {
    const auto& c = m->cfg;
    if (c.dtype == YK_DTYPE_BF16)
        YK_CHECK_CUDA(launch_pdl(m->e, rmsnorm_kernel<__nv_bfloat16>, rows, 256, 0, (const float*)m->h, g,
                                 (__nv_bfloat16*)m->xn, c.d_model, c.rms_eps, row_idx));
    else
        YK_CHECK_CUDA(launch_pdl(m->e, rmsnorm_kernel<float>, rows, 256, 0, (const float*)m->h, g, (float*)m->xn,
                                 c.d_model, c.rms_eps, row_idx));
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
