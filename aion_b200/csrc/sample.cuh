// Sampling beyond greedy (the reference only takes the argmax,
// src/kernel_simd.c:1236-1243; its PROB_EPSILON, :37, is unused).
//
// One CTA draws a token from logits[0..V) with temperature T, optional
// top-k and top-p, deterministically:
//   key_i = order-preserving bits of logit i (larger logit, larger key)
//   W_i   = floor(e^((l_i - max) / T) * 2^32) as an integer (e^x rounded to
//           float from the double exponential; W_max = 2^32)
//   top-k (0 < k < V): keep keys >= the k-th largest key (ties at the
//           threshold stay in);
//   top-p (p < 1): among those, keep keys >= the largest threshold whose
//           kept mass reaches ceil(p * mass);
//   draw:  u = the top 53 bits of SplitMix64(seed, counter) / 2^53,
//           r = floor(u * kept mass); the token is the first index (in
//           index order) where the running kept mass exceeds r.
// Thresholds come from 4-pass radix selection over the keys (8 bits per
// pass) with per-warp integer histograms, so the result does not depend on
// the order of any atomic update.  SplitMix64 is Steele, Lea and Flood's
// published generator (OOPSLA 2014), restated here.
#pragma once

#include "common.cuh"

namespace aion {

struct SamplerParams {
    float temperature;           // <= 0: greedy (the sampler is not called)
    float top_p;                 // (0, 1]; 1 = off
    int top_k;                   // 0 = off
    int pad;
    unsigned long long seed;
};

__host__ __device__ inline unsigned long long splitmix64(unsigned long long x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

// Uniform draw in [0, 1) for (seed, stream, position).
__host__ __device__ inline double sampler_uniform(unsigned long long seed, unsigned long long stream,
                                                  unsigned long long pos) {
    const unsigned long long h = splitmix64(splitmix64(seed ^ (stream * 0xD1B54A32D192ED03ull)) ^ pos);
    return (double)(h >> 11) * (1.0 / 9007199254740992.0);
}

constexpr int kSampleBins = 256;
// Shared scratch: per-warp histograms, the merged histogram, and a few words.
constexpr int kSampleScratch = (kComputeThreads / 32 + 1) * kSampleBins * 8 + 64 * 8;

__device__ __forceinline__ unsigned long long sample_weight(float l, float mx, float T) {
    const float w = (float)exp((double)__fdiv_rn(__fsub_rn(l, mx), T));
    return (unsigned long long)(w * 4294967296.0f);
}

// Radix selection over the keys with key >= lo (and, after each pass, the
// higher digits fixed): the largest key t such that the total of `val` over
// keys >= t reaches `need`.  MASS selects W_i as the value, else 1.
template <bool MASS>
__device__ uint32_t sample_select(const float* logits, int V, float mx, float T, uint32_t lo,
                                  unsigned long long need, unsigned long long* scratch) {
    const int tid = threadIdx.x, warp = tid >> 5, nw = kComputeThreads / 32;
    unsigned long long* hw = scratch + warp * kSampleBins;
    unsigned long long* hs = scratch + nw * kSampleBins;
    unsigned long long* sh = scratch + (nw + 1) * kSampleBins;   // [0] prefix, [1] need
    if (tid == 0) {
        sh[0] = 0;
        sh[1] = need;
    }
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = tid; i < nw * kSampleBins; i += kComputeThreads) scratch[i] = 0;
        csync();
        const uint32_t prefix = (uint32_t)sh[0];
        for (int i = tid; i < V; i += kComputeThreads) {
            const float l = __ldcg(logits + i);
            const uint32_t key = order_bits(l);
            if (key < lo) continue;
            if (shift < 24 && (key >> (shift + 8)) != prefix) continue;
            atomicAdd(hw + ((key >> shift) & 0xFF), MASS ? sample_weight(l, mx, T) : 1ull);
        }
        csync();
        for (int d = tid; d < kSampleBins; d += kComputeThreads) {
            unsigned long long v = 0;
            for (int w = 0; w < nw; w++) v += scratch[w * kSampleBins + d];
            hs[d] = v;
        }
        csync();
        if (tid == 0) {
            unsigned long long cum = 0, nd = sh[1];
            int sel = 0;
            for (int d = kSampleBins - 1; d >= 0; d--) {
                if (cum + hs[d] >= nd) {
                    sel = d;
                    break;
                }
                cum += hs[d];
            }
            sh[0] = ((unsigned long long)prefix << 8) | (unsigned long long)sel;
            sh[1] = nd - cum;
        }
        csync();
    }
    return (uint32_t)sh[0];
}

// Total weight of the keys >= lo (block reduction in a fixed order).
__device__ unsigned long long sample_mass(const float* logits, int V, float mx, float T, uint32_t lo,
                                          unsigned long long* scratch) {
    const int tid = threadIdx.x, nw = kComputeThreads / 32;
    unsigned long long s = 0;
    for (int i = tid; i < V; i += kComputeThreads) {
        const float l = __ldcg(logits + i);
        if (order_bits(l) >= lo) s += sample_weight(l, mx, T);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    csync();
    if ((tid & 31) == 0) scratch[tid >> 5] = s;
    csync();
    unsigned long long t = 0;
    for (int w = 0; w < nw; w++) t += scratch[w];
    csync();
    return t;
}

// Draws a token from logits[0..V) (all kComputeThreads threads of one CTA
// call this; every thread gets the result).  mx = the largest logit.
__device__ int sample_token(const float* logits, int V, float mx, const SamplerParams& sp, unsigned long long stream,
                            unsigned long long pos, unsigned long long* scratch) {
    const int tid = threadIdx.x, nw = kComputeThreads / 32;
    const float T = sp.temperature;
    uint32_t lo = 0;
    if (sp.top_k > 0 && sp.top_k < V) lo = sample_select<false>(logits, V, mx, T, 0, (unsigned long long)sp.top_k, scratch);
    if (sp.top_p < 1.0f) {
        const unsigned long long mk = sample_mass(logits, V, mx, T, lo, scratch);
        const unsigned long long need = (unsigned long long)ceil((double)sp.top_p * (double)mk);
        const uint32_t tp = sample_select<true>(logits, V, mx, T, lo, need > 0 ? need : 1ull, scratch);
        lo = tp > lo ? tp : lo;
    }
    const unsigned long long M = sample_mass(logits, V, mx, T, lo, scratch);
    const unsigned long long r = (unsigned long long)floor(sampler_uniform(sp.seed, stream, pos) * (double)M);
    // Contiguous index chunks per thread: chunk sums, an exclusive scan in
    // thread order, then the thread whose range holds r scans its chunk.
    const int per = (V + kComputeThreads - 1) / kComputeThreads;
    const int i0 = min(V, tid * per), i1 = min(V, i0 + per);
    unsigned long long cs = 0;
    for (int i = i0; i < i1; i++) {
        const float l = __ldcg(logits + i);
        if (order_bits(l) >= lo) cs += sample_weight(l, mx, T);
    }
    unsigned long long* sums = scratch;                   // [kComputeThreads]
    unsigned long long* res = scratch + kComputeThreads;  // [0] chosen index
    sums[tid] = cs;
    if (tid == 0) res[0] = (unsigned long long)(V - 1);
    csync();
    if (tid == 0) {
        unsigned long long run = 0;
        for (int t = 0; t < kComputeThreads; t++) {
            const unsigned long long v = sums[t];
            sums[t] = run;
            run += v;
        }
    }
    csync();
    const unsigned long long base = sums[tid];
    if (base <= r && r < base + cs) {
        unsigned long long run = base;
        for (int i = i0; i < i1; i++) {
            const float l = __ldcg(logits + i);
            if (order_bits(l) < lo) continue;
            run += sample_weight(l, mx, T);
            if (run > r) {
                res[0] = (unsigned long long)i;
                break;
            }
        }
    }
    csync();
    const int tok = (int)res[0];
    csync();
    (void)nw;
    return tok;
}

}  // namespace aion
