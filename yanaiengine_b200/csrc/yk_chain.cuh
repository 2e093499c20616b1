// yk_chain.cuh -- the reference sampler's sequential fp32 sums, evaluated exactly
// by a whole thread block.
//
// SpeculativeSampler sums in index order: the residual normaliser
// (sum += diff, S/SpeculativeSampler.swift:40-45) and the CDF of
// sampleFromProbs (cdf += probs[i]; first i with r <= cdf, :63-73).  Both are
// chains c_{i+1} = fl(c_i + x_i) whose every rounding matters for bit-exact
// decisions.
//
// Exact parallel evaluation.  While c lies in one binade [2^E, 2^(E+1)), c is
// m*u with u = 2^(E-23) and integer m in [2^23, 2^24).  For x >= 0 with
// c + x still below 2^(E+1), round-to-nearest gives fl(c + x) = u*(m + k), k =
// x/u rounded to the nearest integer (x/u is exact: u is a power of two).  So a
// run of such steps is an integer prefix sum, which the block computes with a
// scan.  The steps where this does not hold are evaluated one at a time with
// the hardware add, in order:
//   * binade crossings (m + k would reach 2^24 - 1),
//   * negative, NaN or huge x, and states where c is 0, tiny or not finite.
// Exact ties (x/u = j + 1/2, rounded to even) are resolved inside the round:
// after a tie the running integer is even, so each tie's direction follows from
// the parity of the integer prefix since the previous tie.  A round covers 8192
// elements (512 threads x 16); a special step ends the round and the next round
// restarts right after it, reusing the terms already in the shared-memory ring.
// Every result is the one the sequential loop produces.
#pragma once
#include <climits>

#include "yk_common.cuh"

namespace yk {

constexpr int CHAIN_THREADS = 512;  // block size of every kernel that calls block_chain
constexpr int CHAIN_EPT = 16;       // elements per thread per round
constexpr int CHAIN_ROUND = CHAIN_THREADS * CHAIN_EPT;  // a power of two
constexpr int CHAIN_RING = CHAIN_ROUND + CHAIN_ROUND / 16;  // one pad word per 16 terms: conflict-free reads
constexpr int CHAIN_MAX_TIES = 256;  // rounding ties resolved inside one round; more end the round
constexpr uint32_t CHAIN_SAT = 1u << 30;    // saturation of the integer prefix sums
constexpr uint32_t CHAIN_TOP = (1u << 24) - 1;  // m + k at or above this: treat as a crossing
constexpr int CHAIN_SEQ_HEAD = 512;         // leading elements summed by one thread (many crossings)

struct ChainSmem {
    float ring[CHAIN_RING];  // terms [lo, hi) of the chain, term i at slot (i mod ROUND) + pad
    uint32_t wtot[CHAIN_THREADS / 32], wtie[CHAIN_THREADS / 32];   // per-warp totals
    uint32_t wpre[CHAIN_THREADS / 32], wtpre[CHAIN_THREADS / 32];  // inclusive warp prefixes
    long long wmin[CHAIN_THREADS / 32];
    uint8_t tie_par[CHAIN_MAX_TIES];    // parity of the integer prefix through each tie (ties excluded)
    uint8_t tie_delta[CHAIN_MAX_TIES];  // 1: the tie rounded up
    uint16_t tie_dcum[CHAIN_MAX_TIES + 1];  // ties rounded up before tie t
    uint32_t pex;
    int pure_hit;
    // sequential segment results
    float c_seq;
    long long pos_seq;
    long long found_seq;
    int n_rounds, n_special, n_seq, n_ties;  // work counters (read by the sampler's stamp test hook)
};

__device__ __forceinline__ uint32_t chain_sat(uint32_t a, uint32_t b) {
    const uint32_t s = a + b;
    return s > CHAIN_SAT ? CHAIN_SAT : s;
}

// Block-wide exclusive scans of two values per thread: a (saturating) and b
// (plain count); *ta / *tb = block totals.  Two barriers; the warp totals are
// rewritten only after the caller's next barrier.
__device__ __forceinline__ void chain_block_scan2(ChainSmem& cs, uint32_t a, uint32_t b, uint32_t* ea, uint32_t* eb,
                                                  uint32_t* ta, uint32_t* tb) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    uint32_t ia = a, ib = b;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t x = __shfl_up_sync(0xffffffffu, ia, o);
        const uint32_t y = __shfl_up_sync(0xffffffffu, ib, o);
        if (lane >= o) { ia = chain_sat(ia, x); ib += y; }
    }
    if (lane == 31) { cs.wtot[w] = ia; cs.wtie[w] = ib; }
    __syncthreads();
    if (w == 0) {
        uint32_t wa = lane < CHAIN_THREADS / 32 ? cs.wtot[lane] : 0u;
        uint32_t wb = lane < CHAIN_THREADS / 32 ? cs.wtie[lane] : 0u;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t x = __shfl_up_sync(0xffffffffu, wa, o);
            const uint32_t y = __shfl_up_sync(0xffffffffu, wb, o);
            if (lane >= o) { wa = chain_sat(wa, x); wb += y; }
        }
        if (lane < CHAIN_THREADS / 32) { cs.wpre[lane] = wa; cs.wtpre[lane] = wb; }  // inclusive warp prefixes
    }
    __syncthreads();
    const uint32_t pa = __shfl_up_sync(0xffffffffu, ia, 1), pb = __shfl_up_sync(0xffffffffu, ib, 1);
    *ea = chain_sat(w > 0 ? cs.wpre[w - 1] : 0u, lane > 0 ? pa : 0u);
    *eb = (w > 0 ? cs.wtpre[w - 1] : 0u) + (lane > 0 ? pb : 0u);
    *ta = cs.wpre[CHAIN_THREADS / 32 - 1];
    *tb = cs.wtpre[CHAIN_THREADS / 32 - 1];
}

// Block-wide minimum; one barrier (the per-warp slots are rewritten only after
// the caller's next barrier).
__device__ __forceinline__ long long chain_block_min(ChainSmem& cs, long long v) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) cs.wmin[w] = v;
    __syncthreads();
    long long r = cs.wmin[0];
#pragma unroll
    for (int i = 1; i < CHAIN_THREADS / 32; ++i) r = min(r, cs.wmin[i]);
    return r;
}

// Chain c = fl(c + f(i)), i = 0..n-1, c0 = +0.
// search: returns the first i with r <= c after step i (sampleFromProbs), or
// n-1 if there is none (:72).  !search: returns -1 and *sum = final c.
// Must be called by all CHAIN_THREADS threads of the block; f is evaluated
// once per index, cooperatively, into the shared-memory ring.
struct ChainNoPrefetch {
    __device__ void operator()(long long) const {}
};
// pf(i): optional prefetch into L2 of the sources of f(i .. i+31); each fill
// requests the round after the one it loads, so that round's loads hit L2.
template <class F, class P = ChainNoPrefetch>
__device__ long long block_chain(ChainSmem& cs, F f, long long n, bool search, float r, float* sum, P pf = P()) {
    enum { ZERO = 0, NORMAL = 1, SEQ = 2 };
    float c = 0.f;
    int mode = ZERO;
    uint32_t m = 0;
    float u = 0.f, scale = 0.f;
    long long pos = 0;
    long long found = -1;
    bool done = n <= 0;
    long long hi = 0;  // the ring holds the terms [pos, hi)

    auto slot = [&](long long i) -> float& {
        const int q = (int)(i & (CHAIN_ROUND - 1));
        return cs.ring[q + (q >> 4)];
    };
    // Ring := terms [pos, min(pos + ROUND, n)), loading only what is missing
    // (coalesced; a thread's up to CHAIN_EPT terms are all evaluated, their loads
    // in flight together, before any is stored).
    auto fill = [&]() {
        const long long want = min(pos + (long long)CHAIN_ROUND, n);
        const long long from = max(hi, pos) + threadIdx.x;
        float v[CHAIN_EPT];
#pragma unroll
        for (int u = 0; u < CHAIN_EPT; ++u) {
            const long long i = from + (long long)u * CHAIN_THREADS;
            v[u] = i < want ? f(i) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < CHAIN_EPT; ++u) {
            const long long i = from + (long long)u * CHAIN_THREADS;
            if (i < want) slot(i) = v[u];
        }
        // the next round's terms: one 32-element line per thread
        if (threadIdx.x < CHAIN_ROUND / 32) {
            const long long i = want + 32LL * threadIdx.x;
            if (i < n) pf(i);
        }
        hi = max(hi, want);
        __syncthreads();
    };

    auto set_state = [&](float cn) {
        c = cn;
        if (cn == 0.f) { mode = ZERO; return; }
        if (!isfinite(cn)) { mode = SEQ; return; }
        int e2;
        frexpf(cn, &e2);          // cn = f * 2^e2, f in [0.5, 1)
        const int E = e2 - 1;     // cn in [2^E, 2^(E+1))
        if (E < -100) { mode = SEQ; return; }
        mode = NORMAL;
        u = ldexpf(1.0f, E - 23);
        scale = ldexpf(1.0f, 23 - E);
        m = (uint32_t)__fmul_rn(cn, scale);  // exact integer in [2^23, 2^24)
    };

    // One thread sums up to `limit` (<= CHAIN_ROUND) terms in order (head of the
    // chain, and the rare zero / tiny / non-finite states), from the ring.  NaN
    // is absorbing.
    auto sequential = [&](long long limit) {
        if (threadIdx.x == 0) ++cs.n_seq;
        fill();
        const int cnt = (int)min(n - pos, limit);
        if (threadIdx.x == 0) {
            // SG terms loaded together, then their SG dependent additions, then one
            // test over the SG running values for the first step that reaches r or
            // turns NaN (the additions past it are discarded); a per-step test and
            // branch inside the chain cost about 70 cycles per term.
            constexpr int SG = 16;
            float cc = c;
            long long fnd = -1;
            int t = 0;
            for (int t0 = 0; t0 < cnt; t0 += SG) {
                const int nv = min(SG, cnt - t0);
                float v[SG], s[SG];
#pragma unroll
                for (int u = 0; u < SG; ++u) v[u] = u < nv ? slot(pos + t0 + u) : 0.f;
                float a = cc, last = cc;
#pragma unroll
                for (int u = 0; u < SG; ++u) {
                    a = __fadd_rn(a, v[u]);
                    s[u] = a;
                    if (u == nv - 1) last = a;
                }
                // (compile-time indices only: a runtime-indexed s[] would go to local memory)
                int first = SG;
                float at_first = 0.f;
#pragma unroll
                for (int u = SG - 1; u >= 0; --u)
                    if (u < nv && ((search && r <= s[u]) || isnan(s[u]))) {
                        first = u;
                        at_first = s[u];
                    }
                if (first < SG) {
                    cc = at_first;
                    if (search && r <= cc) {
                        fnd = pos + t0 + first;
                        t = t0 + first + 1;
                    } else {
                        t = (int)(n - pos);  // NaN is absorbing
                    }
                    break;
                }
                cc = last;
                t = t0 + nv;
            }
            cs.c_seq = cc;
            cs.pos_seq = pos + t;
            cs.found_seq = fnd;
        }
        __syncthreads();
        const float cc = cs.c_seq;
        pos = cs.pos_seq;
        found = cs.found_seq;
        __syncthreads();
        if (found >= 0 || pos >= n) { c = cc; done = true; return; }
        set_state(cc);
    };

    if (!done) sequential(CHAIN_SEQ_HEAD);
    while (!done) {
        if (mode == SEQ) {
            sequential(CHAIN_ROUND);
            continue;
        }
        const long long base = pos;
        const long long i0 = base + (long long)threadIdx.x * CHAIN_EPT;
        if (threadIdx.x == 0) ++cs.n_rounds;
        if (mode == ZERO) {
            // c stays +0 until the first non-zero element (x = -0 adds nothing).
            if (search && r <= 0.0f) {  // the next step decides; let the exact path take it
                sequential(CHAIN_ROUND);
                continue;
            }
            fill();
            long long cand = LLONG_MAX;
#pragma unroll
            for (int j = 0; j < CHAIN_EPT; ++j) {
                const long long i = i0 + j;
                if (i < n && cand == LLONG_MAX && slot(i) != 0.0f) cand = i;
            }
            const long long js = chain_block_min(cs, cand);
            if (js == LLONG_MAX) {
                pos = base + CHAIN_ROUND;
                if (pos >= n) done = true;
                continue;
            }
            const float cn = __fadd_rn(0.0f, slot(js));
            __syncthreads();  // all have read slot(js) before the next fill may reuse it
            pos = js + 1;
            if (search && r <= cn) { found = js; done = true; break; }
            set_state(cn);
            if (pos >= n) { done = true; break; }
            continue;
        }
        // NORMAL: c = m * u with m in [2^23, 2^24).  Term x adds y = x / u (exact);
        // round-to-nearest gives k = round(y) except at exact ties y = j + 1/2,
        // where the result is the even one of m + j, m + j + 1.  After a tie the
        // running integer is even, so a tie's direction is the parity of the
        // integer prefix since the previous tie: resolved in index order below.
        fill();
        uint32_t loc[CHAIN_EPT];
        uint32_t tie_mask = 0, sp_mask = 0;
        uint32_t run = 0, nties = 0;
#pragma unroll
        for (int j = 0; j < CHAIN_EPT; ++j) {
            const long long i = i0 + j;
            uint32_t k = 0;
            if (i < n) {
                const float x = slot(i);
                if (!(x >= 0.0f)) {  // negative or NaN
                    sp_mask |= 1u << j;
                    k = CHAIN_SAT;
                } else {
                    const float y = __fmul_rn(x, scale);  // exact: scale is a power of two
                    if (!(y < 16777216.0f)) {
                        sp_mask |= 1u << j;
                        k = CHAIN_SAT;
                    } else {
                        const float fl = floorf(y);
                        const float fr = __fsub_rn(y, fl);  // exact
                        k = (uint32_t)fl + (fr > 0.5f ? 1u : 0u);
                        if (fr == 0.5f) { tie_mask |= 1u << j; ++nties; }
                    }
                }
            }
            run = chain_sat(run, k);
            loc[j] = run;
        }
        uint32_t off, rank0, total, ntie;
        chain_block_scan2(cs, run, nties, &off, &rank0, &total, &ntie);
        // ties: rank in the round, parity of the prefix through each, resolved by thread 0
        uint32_t dstart = 0, dtotal = 0;
        if (ntie != 0) {
            if (threadIdx.x == 0) cs.n_ties += (int)ntie;
            uint32_t rk = rank0;
#pragma unroll
            for (int j = 0; j < CHAIN_EPT; ++j) {
                if (tie_mask & (1u << j)) {
                    if (rk < (uint32_t)CHAIN_MAX_TIES) cs.tie_par[rk] = (uint8_t)(chain_sat(off, loc[j]) & 1u);
                    ++rk;
                }
            }
            __syncthreads();
            const uint32_t nres = min(ntie, (uint32_t)CHAIN_MAX_TIES);
            if (threadIdx.x == 0) {
                uint32_t D = 0;
                for (uint32_t t = 0; t < nres; ++t) {
                    cs.tie_dcum[t] = (uint16_t)D;
                    const uint32_t d = (m + cs.tie_par[t] + D) & 1u;
                    cs.tie_delta[t] = (uint8_t)d;
                    D += d;
                }
                cs.tie_dcum[nres] = (uint16_t)D;
            }
            __syncthreads();
            dstart = cs.tie_dcum[min(rank0, nres)];
            dtotal = cs.tie_dcum[nres];
        }
        long long cand = LLONG_MAX;
        int cj = -1;
        bool pure = false;
        uint32_t pex_c = 0;
        uint32_t D = dstart, rk = rank0;
        // The prefix only grows along the segment, so a segment without special
        // terms or ties holds the candidate only if its end crosses the binade
        // or reaches r: every other thread skips the element loop.
        bool scan_seg = (sp_mask | tie_mask) != 0;
        if (!scan_seg && i0 < n) {
            const uint32_t pend = chain_sat(chain_sat(off, run), dstart);
            scan_seg = (m + pend >= CHAIN_TOP) || (search && r <= __fmul_rn((float)(m + pend), u));
        }
#pragma unroll
        for (int j = 0; j < CHAIN_EPT; ++j) {
            if (!scan_seg) break;
            const long long i = i0 + j;
            if (i < n && cand == LLONG_MAX) {
                bool special = (sp_mask >> j) & 1u;
                uint32_t delta = 0;
                if (tie_mask & (1u << j)) {
                    if (rk < (uint32_t)CHAIN_MAX_TIES) delta = cs.tie_delta[rk];
                    else special = true;
                    ++rk;
                }
                const uint32_t pexcl = chain_sat(j > 0 ? chain_sat(off, loc[j - 1]) : off, D);  // before element i
                const uint32_t pincl = chain_sat(chain_sat(off, loc[j]), D + delta);
                special = special || (m + pincl >= CHAIN_TOP);
                const bool hit = !special && search && (r <= __fmul_rn((float)(m + pincl), u));
                if (special || hit) { cand = i; cj = j; pure = !special; pex_c = pexcl; }
                D += delta;
            }
        }
        const long long js = chain_block_min(cs, cand);
        if (js == LLONG_MAX) {
            m += total + dtotal;  // stays below 2^24 - 1: no crossing in this round
            pos = base + CHAIN_ROUND;
            if (pos >= n) { c = __fmul_rn((float)m, u); done = true; }
            continue;
        }
        // every thread reads the special term before the barrier below: the next
        // round's fill may reuse its ring slot
        const float xs = slot(js);
        if (cand == js) {
            cs.pex = pex_c;
            cs.pure_hit = pure ? 1 : 0;
        }
        __syncthreads();  // (rewritten only after the next round's block minimum)
        const uint32_t pex = cs.pex;
        const int pure_hit = cs.pure_hit;
        (void)cj;
        if (pure_hit) { found = js; done = true; break; }
        if (threadIdx.x == 0) ++cs.n_special;
        const float cprev = __fmul_rn((float)(m + pex), u);
        const float cn = __fadd_rn(cprev, xs);
        pos = js + 1;
        if (search && r <= cn) { found = js; done = true; break; }
        set_state(cn);
        if (pos >= n) { done = true; break; }
    }
    if (sum) *sum = c;
    if (!search) return -1;
    return found >= 0 ? found : n - 1;
}

}  // namespace yk
