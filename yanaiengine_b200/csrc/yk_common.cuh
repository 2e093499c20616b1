// yk_common.cuh -- device helpers shared by every kernel of libyk.so:
// Philox4x32-10, bf16 conversion, bounded mbarrier waits, and thin inline-PTX
// wrappers for the sm_100a async units (TMA, tcgen05 MMA / TMEM).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

// Device error word bits (read back by yk_engine_device_error).
#define YK_DEV_ERR_BOUNDS   0x1u  // index outside a buffer (checked, access skipped)
#define YK_DEV_ERR_TIMEOUT  0x2u  // a bounded wait gave up
#define YK_DEV_ERR_ARG      0x4u  // kernel-side argument check

// Wall-clock budget of any device-side wait before it gives up (ns).
#define YK_WAIT_BUDGET_NS 2000000000ull

namespace yk {

// ---------------------------------------------------------------------------
// Philox4x32-10 (Salmon et al., SC'11).  Counter = (step, seq, position, slot),
// key = seed.  The uniform is the top 24 bits of word 0 scaled by 2^-24.
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
#pragma unroll
    for (int r = 0; r < 10; ++r) {
#ifdef __CUDA_ARCH__
        const uint32_t hi0 = __umulhi(0xD2511F53u, c.x), lo0 = 0xD2511F53u * c.x;
        const uint32_t hi1 = __umulhi(0xCD9E8D57u, c.z), lo1 = 0xCD9E8D57u * c.z;
#else
        const uint64_t p0 = (uint64_t)0xD2511F53u * c.x, p1 = (uint64_t)0xCD9E8D57u * c.z;
        const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
        const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
#endif
        c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
        k.x += 0x9E3779B9u;
        k.y += 0xBB67AE85u;
    }
    return c;
}

__host__ __device__ __forceinline__ float u24(uint32_t x) { return (float)(x >> 8) * (1.0f / 16777216.0f); }

enum : uint32_t { SLOT_DRAFT = 0, SLOT_ACCEPT = 1, SLOT_RESAMPLE = 2, SLOT_BONUS = 3 };

__host__ __device__ __forceinline__ float uniform_at(uint64_t seed, uint32_t step, uint32_t seq, uint32_t pos,
                                                     uint32_t slot) {
    const uint4 o = philox4x32_10(make_uint4(step, seq, pos, slot),
                                  make_uint2((uint32_t)seed, (uint32_t)(seed >> 32)));
    return u24(o.x);
}

// ---------------------------------------------------------------------------
// Element types.
// ---------------------------------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// ---------------------------------------------------------------------------
// Clock and error word.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void raise_err(uint32_t* err, uint32_t bits) {
    if (err) atomicOr(err, bits);
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  Every kernel of the forward step is launched
// so that it may start while the previous kernel of the stream finishes:
// pdl_trigger lets the next kernel launch, pdl_wait blocks until the previous
// kernel has completed and its writes are visible.  Each kernel calls pdl_wait
// on every path before it reads or writes data another kernel touches (and
// before it exits), so completion stays ordered along the stream.  Both are
// no-ops for a kernel launched without the attribute.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------
// Launch trace (test hook).  With tracing on, every kernel of the forward step
// and the sampler records, for its launch, the first CTA's entry, the first
// CTA past its grid dependency wait and the last CTA's exit (%globaltimer ns),
// so gaps and overlap between launches can be read inside a real step.
// ---------------------------------------------------------------------------
struct TraceRec {
    unsigned long long entry, start, end, kind;
};
struct Trace {
    TraceRec* rec = nullptr;  // null: tracing off
    uint32_t id = 0, kind = 0;
};
enum : int { TR_ENTRY = 0, TR_START = 1, TR_END = 2 };
__device__ __forceinline__ void trace_mark(const Trace& t, int what) {
    if (t.rec == nullptr) return;
    TraceRec* r = t.rec + t.id;
    const unsigned long long now = globaltimer_ns();
    if (what == TR_ENTRY) {
        atomicMin(&r->entry, now);
        r->kind = t.kind;
    } else if (what == TR_START) {
        atomicMin(&r->start, now);
    } else {
        atomicMax(&r->end, now);
    }
}

// ---------------------------------------------------------------------------
// mbarrier (shared::cta) helpers.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Waits for the phase of parity `parity` to complete.  Gives up after
// budget_ns (returns false) so no wait can hang the GPU.
__device__ __forceinline__ bool mbar_wait_bounded_ns(uint32_t bar, uint32_t parity, uint64_t budget_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 0 && globaltimer_ns() - t0 > budget_ns) return false;
    }
}
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
    return mbar_wait_bounded_ns(bar, parity, YK_WAIT_BUDGET_NS);
}

// ---------------------------------------------------------------------------
// TMA: 2-D tiled bulk tensor load global -> shared (no multicast).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int32_t x, int32_t y,
                                            uint32_t bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
        "l"((uint64_t)map), "r"(x), "r"(y), "r"(bar), "l"(policy)
        : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// ---------------------------------------------------------------------------
// tcgen05 (5th-gen tensor core, TMEM accumulators), cta_group::1.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t slot_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot_smem), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc], bf16 inputs, fp32 accumulate.
__device__ __forceinline__ void tc_mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrives on `bar` once every tcgen05 op issued so far by this thread completes.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}
// 32 lanes x 16 columns of 32-bit: thread i of the warp gets TMEM lane (base+i).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Thread-block clusters: rank, barrier, distributed shared memory loads.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory location in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
__device__ __forceinline__ float ld_shared_cluster_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}
__device__ __forceinline__ float4 ld_shared_cluster_v4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}
// Acquire load of a global counter (gpu scope).
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Orders generic-proxy global writes (this thread's, and those it acquired) before
// its later async-proxy (TMA) reads of global memory.
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Non-binding prefetch of the 128-byte line holding p into L2.
__device__ __forceinline__ void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

// Bulk copy (copy engine) of `bytes` (a multiple of 16; both addresses 16-byte
// aligned) from this CTA's shared memory into the shared memory of a CTA of
// the cluster (dst and bar: shared::cluster addresses from mapa); completes
// with complete_tx on that CTA's mbarrier.  Point to point.
__device__ __forceinline__ void bulk_copy_to_peer(uint32_t dst, uint32_t src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "r"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
// Bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned) from
// global memory into this CTA's shared memory; completes with complete_tx on
// this CTA's mbarrier.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (bulk copy) reads of them.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ float4 lds_v4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}
// Cluster barrier that warps may reach divergently (no .aligned).
__device__ __forceinline__ void cluster_sync_any() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// The two halves of cluster_sync_any, for work that overlaps the barrier.
__device__ __forceinline__ void cluster_arrive_any() { asm volatile("barrier.cluster.arrive.release;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait_any() { asm volatile("barrier.cluster.wait.acquire;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major operand tile written by TMA with
// 128-byte swizzle: rows of 128 B, 8-row swizzle atoms of 1024 B stacked
// contiguously (stride byte offset 1024), sm_100 descriptor version 1.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)1 << 16;             // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;   // stride byte offset: next 8-row group
    d |= (uint64_t)1 << 46;             // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;             // SWIZZLE_128B
    return d;
}
// Instruction descriptor for kind::f16: bf16 A/B, fp32 D, both K-major, MxN.
__host__ __device__ __forceinline__ uint32_t idesc_bf16_f32(int M, int N) {
    return (1u << 4)                      // D format f32
           | (1u << 7)                    // A format bf16
           | (1u << 10)                   // B format bf16
           | ((uint32_t)(N >> 3) << 17)   // N
           | ((uint32_t)(M >> 4) << 24);  // M
}

}  // namespace yk
