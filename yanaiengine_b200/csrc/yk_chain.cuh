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
//   * exact ties (x/u = j + 1/2: the result depends on the parity of m + j),
//   * negative, NaN or huge x, and states where c is 0, tiny or not finite.
// A round covers 8192 elements (512 threads x 16); a special step ends the round
// and the next round restarts right after it.  Every result is the one the
// sequential loop produces.
#pragma once
#include <climits>

#include "yk_common.cuh"

namespace yk {

constexpr int CHAIN_THREADS = 512;  // block size of every kernel that calls block_chain
constexpr int CHAIN_EPT = 16;       // elements per thread per round
constexpr int CHAIN_ROUND = CHAIN_THREADS * CHAIN_EPT;
constexpr uint32_t CHAIN_SAT = 1u << 30;    // saturation of the integer prefix sums
constexpr uint32_t CHAIN_TOP = (1u << 24) - 1;  // m + k at or above this: treat as a crossing
constexpr int CHAIN_SEQ_HEAD = 512;         // leading elements summed by one thread (many crossings)

struct ChainSmem {
    uint32_t wtot[CHAIN_THREADS / 32];
    long long wmin[CHAIN_THREADS / 32];
    long long jstar;
    float xstar;
    uint32_t pex;
    uint32_t total;
    int pure_hit;
    // sequential segment results
    float c_seq;
    long long pos_seq;
    long long found_seq;
    float seg[CHAIN_ROUND];  // terms of a sequential segment, staged by the whole block
    int n_rounds, n_special, n_seq;  // work counters (read by the sampler's stamp test hook)
};

__device__ __forceinline__ uint32_t chain_sat(uint32_t a, uint32_t b) {
    const uint32_t s = a + b;
    return s > CHAIN_SAT ? CHAIN_SAT : s;
}

// Block-wide exclusive scan (saturating) of one value per thread; *total = block sum.
__device__ __forceinline__ uint32_t chain_block_scan(ChainSmem& cs, uint32_t v, uint32_t* total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    uint32_t incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl = chain_sat(incl, t);
    }
    if (lane == 31) cs.wtot[w] = incl;
    __syncthreads();
    if (w == 0) {
        uint32_t wv = lane < CHAIN_THREADS / 32 ? cs.wtot[lane] : 0u;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t t = __shfl_up_sync(0xffffffffu, wv, o);
            if (lane >= o) wv = chain_sat(wv, t);
        }
        if (lane < CHAIN_THREADS / 32) cs.wtot[lane] = wv;  // inclusive warp prefix
    }
    __syncthreads();
    const uint32_t woff = w > 0 ? cs.wtot[w - 1] : 0u;
    *total = cs.wtot[CHAIN_THREADS / 32 - 1];
    const uint32_t prev = __shfl_up_sync(0xffffffffu, incl, 1);  // exact (saturated) exclusive prefix
    const uint32_t excl = chain_sat(woff, lane > 0 ? prev : 0u);
    __syncthreads();
    return excl;
}

__device__ __forceinline__ long long chain_block_min(ChainSmem& cs, long long v) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) cs.wmin[w] = v;
    __syncthreads();
    long long r = cs.wmin[0];
#pragma unroll
    for (int i = 1; i < CHAIN_THREADS / 32; ++i) r = min(r, cs.wmin[i]);
    __syncthreads();
    return r;
}

// Chain c = fl(c + f(i)), i = 0..n-1, c0 = +0.
// search: returns the first i with r <= c after step i (sampleFromProbs), or
// n-1 if there is none (:72).  !search: returns -1 and *sum = final c.
// Must be called by all CHAIN_THREADS threads of the block.
template <class F>
__device__ long long block_chain(ChainSmem& cs, F f, long long n, bool search, float r, float* sum) {
    enum { ZERO = 0, NORMAL = 1, SEQ = 2 };
    float c = 0.f;
    int mode = ZERO;
    uint32_t m = 0;
    float u = 0.f, scale = 0.f;
    long long pos = 0;
    long long found = -1;
    bool done = n <= 0;

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

    // One thread sums up to `limit` (<= CHAIN_ROUND) elements in order (head of
    // the chain, and the rare zero / tiny / non-finite states).  The block first
    // evaluates the terms into shared memory, so the ordered loop never waits on
    // global memory.  NaN is absorbing.
    auto sequential = [&](long long limit) {
        if (threadIdx.x == 0) ++cs.n_seq;
        const int cnt = (int)min(n - pos, limit);
        for (int t = threadIdx.x; t < cnt; t += CHAIN_THREADS) cs.seg[t] = f(pos + t);
        __syncthreads();
        if (threadIdx.x == 0) {
            float cc = c;
            long long fnd = -1;
            int t = 0;
            for (; t < cnt; ++t) {
                cc = __fadd_rn(cc, cs.seg[t]);
                if (search && r <= cc) { fnd = pos + t; ++t; break; }
                if (isnan(cc)) { t = (int)(n - pos); break; }
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
            long long cand = LLONG_MAX;
            float xc = 0.f;
#pragma unroll
            for (int j = 0; j < CHAIN_EPT; ++j) {
                const long long i = i0 + j;
                if (i < n && cand == LLONG_MAX) {
                    const float x = f(i);
                    if (x != 0.0f) { cand = i; xc = x; }
                }
            }
            const long long js = chain_block_min(cs, cand);
            if (js == LLONG_MAX) {
                pos = base + CHAIN_ROUND;
                if (pos >= n) done = true;
                continue;
            }
            if (cand == js) cs.xstar = xc;
            __syncthreads();
            const float cn = __fadd_rn(0.0f, cs.xstar);
            __syncthreads();
            pos = js + 1;
            if (search && r <= cn) { found = js; done = true; break; }
            set_state(cn);
            if (pos >= n) { done = true; break; }
            continue;
        }
        // NORMAL: integer increments k = round(x / u) with their flags
        float xv[CHAIN_EPT];
        uint32_t loc[CHAIN_EPT];
        bool sp[CHAIN_EPT];
        uint32_t run = 0;
#pragma unroll
        for (int j = 0; j < CHAIN_EPT; ++j) {
            const long long i = i0 + j;
            float x = 0.f;
            uint32_t k = 0;
            bool s = false;
            if (i < n) {
                x = f(i);
                if (!(x >= 0.0f)) {  // negative or NaN
                    s = true;
                    k = CHAIN_SAT;
                } else {
                    const float y = __fmul_rn(x, scale);  // exact: scale is a power of two
                    if (!(y < 16777216.0f)) {
                        s = true;
                        k = CHAIN_SAT;
                    } else {
                        const float fl = floorf(y);
                        const float fr = __fsub_rn(y, fl);  // exact
                        k = (uint32_t)fl + (fr > 0.5f ? 1u : 0u);
                        s = fr == 0.5f;                     // tie: parity decides
                    }
                }
            }
            xv[j] = x;
            sp[j] = s;
            run = chain_sat(run, k);
            loc[j] = run;
        }
        uint32_t total;
        const uint32_t off = chain_block_scan(cs, run, &total);
        long long cand = LLONG_MAX;
        int cj = -1;
        bool pure = false;
#pragma unroll
        for (int j = 0; j < CHAIN_EPT; ++j) {
            const long long i = i0 + j;
            if (i < n && cand == LLONG_MAX) {
                const uint32_t P = chain_sat(off, loc[j]);
                const bool special = sp[j] || (m + P >= CHAIN_TOP);
                const bool hit = !special && search && (r <= __fmul_rn((float)(m + P), u));
                if (special || hit) { cand = i; cj = j; pure = !special; }
            }
        }
        const long long js = chain_block_min(cs, cand);
        if (js == LLONG_MAX) {
            m += total;  // stays below 2^24 - 1: no crossing in this round
            pos = base + CHAIN_ROUND;
            if (pos >= n) { c = __fmul_rn((float)m, u); done = true; }
            continue;
        }
        if (cand == js) {
            cs.xstar = xv[cj];
            cs.pex = cj > 0 ? chain_sat(off, loc[cj - 1]) : off;
            cs.pure_hit = pure ? 1 : 0;
        }
        __syncthreads();
        const float xs = cs.xstar;
        const uint32_t pex = cs.pex;
        const int pure_hit = cs.pure_hit;
        __syncthreads();
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
