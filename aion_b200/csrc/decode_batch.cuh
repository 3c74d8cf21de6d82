// Lock-step batched decode: up to 32 sequences, each with its own KV cache
// and position, advance one greedy token per step in one persistent
// cooperative launch (W4A16).  Per sequence this is the forward of
// src/kernel_simd.c:1014-1169 and the greedy pick of :1236-1243; the
// reference itself only ever decodes one sequence.
//
// Every weight byte is read once per step for all sequences: each 16 x 32
// weight fragment feeds 3 MMAs (m16n8k32, s8) per 8 sequences.  Activations
// enter as three balanced base-256 digits of a 24-bit fixed-point value
// with one exponent per (group of 32, sequence):
//   X = round(x * 2^E), max |x| * 2^E in [2^21, 2^22) over the group,
//   X = d0 + 2^8 d1 + 2^16 d2, factor 2^-E / 16 (weights carry 16 * q).
// MMA 0 holds columns (d0, d1) of sequences 0-3, MMA 1 those of sequences
// 4-7, MMA 2 the d2 columns of all eight, so quad lane t accumulates
// sequences t and t + 4 for rows r and r + 8.
//
// The digits of a whole input do not fit in shared memory for 32 sequences,
// so each matvec is split along K: slice s covers groups [s*G/S, (s+1)*G/S)
// and a contiguous share of CTAs; a CTA digitises only its slice and its
// warps stream (tile, slice) units, writing 16 x nb8 partial rows per unit.
// The phase after the grid barrier sums the S partials of a row in slice
// order (deterministic), applies the RMSNorm factor of the input (a
// per-sequence scalar, so W (x * ss * w) = ss * W (x * w)) and runs the
// epilogue.  Phases per layer, each ending at a grid barrier:
//   QKV matvec | QKV sums, RoPE, KV append | attention | WO matvec |
//   x += WO sums | W13 matvec | SwiGLU -> hb | W2 matvec | x += W2 sums
// then per step: classifier matvec | logits, argmax per sequence, and at the
// start of the next step the embedding rows of the chosen tokens.
#pragma once

#include "decode_step.cuh"

namespace aion {

constexpr int kBMaxSeq = 32;
constexpr int kBChunkG = 8;                       // groups per bulk copy
constexpr int kBChunkBytes = kBChunkG * kGB;      // 2560
constexpr int kBBlockBytes = 768;                 // digits of 8 sequences for one group (3 B operands)
constexpr int kBFacBytes = 32;                    // factors of 8 sequences for one group
constexpr int kBDigitBudget = 112 * 1024;         // shared memory for one slice's digits + factors
constexpr int kBMaxResRows = 40;                  // residual rows per CTA (dim <= 40 * grid)

struct BOpDesc {
    MatDesc m;
    int kind, layer;
    int S;                 // K slices
    int pad;
};

// Slice of CTA c: groups [ga, gb), tiles [t0, t1).  CTA c serves slice
// floor(c * S / grid); the CTAs of a slice split its tiles evenly.
struct BSlice {
    int s, ga, gb, t0, t1;
};
__host__ __device__ inline BSlice bslice(const BOpDesc& o, int c, int grid) {
    BSlice r;
    const long long S = o.S;
    r.s = (int)(((long long)c * S) / grid);
    const int c_lo = (int)(((long long)r.s * grid + S - 1) / S);
    const int c_hi = (int)(((long long)(r.s + 1) * grid + S - 1) / S);
    const long long n = c_hi - c_lo, T = o.m.ntiles;
    r.t0 = (int)((c - c_lo) * T / n);
    r.t1 = (int)((c - c_lo + 1) * T / n);
    r.ga = (int)(r.s * (long long)o.m.G / S);
    r.gb = (int)((r.s + 1) * (long long)o.m.G / S);
    return r;
}

struct BatchArgs {
    const BOpDesc* ops;      // QKV, WO, W13, W2 per layer, then CLS
    int nops;
    MatDesc emb;
    int dim, hidden, n_layers, n_heads, kv_mul, head_size, kv_dim, q_dim, vocab, max_pos;
    const float *rms_att, *rms_ffn, *rms_final, *freq_re, *freq_im;
    int nb;                  // sequences; batch entry b uses KV cache b
    float *x, *q, *att, *hb, *logits;   // [nb][dim], [nb][q_dim] x2, [nb][hidden], [nb][vocab]
    float *kcache, *vcache;  // sequence b at + b * kv_seq: [L][max_pos][kv_dim]
    size_t kv_seq;
    float* part;             // [S][ntiles][nb8][16]: partial rows of the last matvec
    float* ssq;              // [grid][nb]: per CTA, sum of squares of its residual rows
    float* attn_part;        // [nb][n_heads][max_chunks][head_size + 4]
    int* attn_cnt;           // [nb][n_heads], zero between uses
    int max_chunks;
    StepState* step;         // barrier counter and error code
    unsigned long long* argmax;   // [2][kBMaxSeq] keys, by step parity
    const int32_t* first;    // [nb] tokens of step 0
    const int32_t* pos0;     // [nb] positions of step 0
    int32_t* tokens;         // [steps + 1][nb]: each step's input tokens, then the last step's pick
    int steps;
    int P;                   // ring slots per warp (kBChunkBytes each)
    int fac_off, ring_off, ops_off;   // dynamic shared memory: digits at 0
};

// ---------------------------------------------------------------------------
// Weight streaming: a warp's (tile, slice) units of one op, in chunks of up
// to kBChunkG groups.
// ---------------------------------------------------------------------------
struct BCursor {
    int s, tile, t1, g, ga, gb;
};
__device__ __forceinline__ bool bcur_begin(BCursor& cu, const BOpDesc& o, int warp) {
    const BSlice sl = bslice(o, blockIdx.x, gridDim.x);
    cu.s = sl.s;
    cu.tile = sl.t0 + warp;
    cu.t1 = sl.t1;
    cu.ga = cu.g = sl.ga;
    cu.gb = sl.gb;
    return cu.tile < cu.t1 && cu.ga < cu.gb;
}
__device__ __forceinline__ bool bcur_next(BCursor& cu) {
    cu.g += kBChunkG;
    if (cu.g >= cu.gb) {
        cu.g = cu.ga;
        cu.tile += kWarps;
    }
    return cu.tile < cu.t1;
}
__device__ __forceinline__ const uint8_t* bchunk_src(const MatDesc& m, const BCursor& cu, int& bytes) {
    bytes = min(kBChunkG, cu.gb - cu.g) * kGB;
    return m.w + (size_t)cu.tile * m.tile_bytes + (size_t)cu.g * kGB;
}

// Producer lane w: walks compute warp w's chunks over every op of every
// step (bounded like produce()).
__device__ void bproduce(const BatchArgs& a, const BOpDesc* ops, unsigned char* ring_base, uint64_t* bars, int w) {
    ProdRing pr;
    ring_init(pr.r, ring_base, bars, a.P, kBChunkBytes, w, false);
    pr.round = 0;
    int step = 0, op = 0;
    BCursor cu;
    bool have = false;
    auto enter = [&]() {
        have = false;
        while (step < a.steps) {
            while (op < a.nops) {
                if (bcur_begin(cu, ops[op], w)) {
                    have = true;
                    return;
                }
                op++;
            }
            op = 0;
            step++;
        }
    };
    enter();
    uint32_t spins = 0;
    while (have) {
        int bytes;
        const uint8_t* src = bchunk_src(ops[op].m, cu, bytes);
        if (prod_try_issue(pr, src, bytes)) {
            spins = 0;
            if (!bcur_next(cu)) {
                op++;
                enter();
            }
        } else if (++spins > (1u << 24) || ((spins & 4095u) == 0 && ld_relaxed_i32(&a.step->error) != 0)) {
            break;
        }
    }
    prod_drain(pr);
}

// ---------------------------------------------------------------------------
// Digits of this CTA's slice: groups [ga, gb) of every sequence's input
// src + b * ld, times the RMSNorm weight w when given (the per-sequence
// RMSNorm factor is applied to the sums).  Layout: group gl, block blk at
// (gl * NBLK + blk) * 768: B operands of MMA 0, 1, 2 (256 bytes each: column
// c at 32c, quad lane t at 8t, elements 4t..4t+3 then 16+4t..16+4t+3);
// factors at fac[((gl * NBLK + blk) * 4 + t) * 2 + hi] for sequence
// 8 blk + t + 4 hi.  Padding sequences (b >= nb) get zero digits and factors.
// ---------------------------------------------------------------------------
template <int NBLK>
__device__ void bbuild_digits(unsigned char* xd, float* fac, const float* src, int ld, const float* w, int ga, int gb,
                              int nb) {
    constexpr int NB8 = 8 * NBLK;
    const int total = (gb - ga) * NB8 * 8;
    for (int base = 0; base < total; base += kThreads) {   // uniform trip count: the shuffles see full warps
        const int i = base + threadIdx.x;
        const bool valid = i < total;
        const int q = i & 7, rest = i >> 3;
        const int b = rest % NB8, gl = rest / NB8;
        const int col = (ga + gl) * 32 + 4 * q;
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (valid && b < nb) {
            v = __ldcg(reinterpret_cast<const float4*>(src + (size_t)b * ld + col));
            if (w) {
                const float4 g = __ldg(reinterpret_cast<const float4*>(w + col));
                v.x = __fmul_rn(v.x, g.x);
                v.y = __fmul_rn(v.y, g.y);
                v.z = __fmul_rn(v.z, g.z);
                v.w = __fmul_rn(v.w, g.w);
            }
        }
        float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
        if (!valid) continue;
        const int ebits = (int)((__float_as_uint(m) >> 23) & 0xFF);
        const bool live = ebits >= 26;                    // groups below 2^-101 count as zero
        const int E = 148 - ebits;                        // max * 2^E in [2^21, 2^22)
        const float sa = __int_as_float((127 + E / 2) << 23), sb = __int_as_float((127 + E - E / 2) << 23);
        const float e[4] = {v.x, v.y, v.z, v.w};
        uint32_t Z[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int X = live ? __float2int_rn(__fmul_rn(__fmul_rn(e[k], sa), sb)) : 0;
            Z[k] = ((uint32_t)X + 0x8080u) ^ 0x8080u;      // bytes d0, d1, d2 as signed bytes
        }
        const uint32_t t01 = __byte_perm(Z[0], Z[1], 0x5140), t23 = __byte_perm(Z[2], Z[3], 0x5140);
        const uint32_t u01 = __byte_perm(Z[0], Z[1], 0x7362), u23 = __byte_perm(Z[2], Z[3], 0x7362);
        const int blk = b >> 3, j = b & 7, t = q & 3, h = q >> 2;
        unsigned char* blkp = xd + (size_t)(gl * NBLK + blk) * kBBlockBytes + 8 * t + 4 * h;
        unsigned char* lo = blkp + (j >> 2) * 256 + (2 * (j & 3)) * 32;
        *reinterpret_cast<uint32_t*>(lo) = __byte_perm(t01, t23, 0x5410);        // d0
        *reinterpret_cast<uint32_t*>(lo + 32) = __byte_perm(t01, t23, 0x7632);   // d1
        *reinterpret_cast<uint32_t*>(blkp + 512 + (2 * (j & 3) + (j >> 2)) * 32) = __byte_perm(u01, u23, 0x5410);
        if (q == 0) fac[((gl * NBLK + blk) * 4 + (j & 3)) * 2 + (j >> 2)] = live ? __int_as_float((123 - E) << 23) : 0.0f;
    }
}

// One matvec op on this CTA: consume its chunks, write each finished unit's
// 16 x nb8 partial rows.  False if a wait gave up (not uniform: the caller
// reduces it over the CTA).
template <int NBLK>
__device__ bool brun_op(const BOpDesc& op, Ring& ring, unsigned char* ring_base, const unsigned char* xd,
                        const float* fac, float* part) {
    constexpr int NB8 = 8 * NBLK;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, r = lane >> 2, t = lane & 3;
    BCursor cu;
    bool more = bcur_begin(cu, op, warp);
    float acc[NBLK][4];
#pragma unroll
    for (int k = 0; k < NBLK; k++) acc[k][0] = acc[k][1] = acc[k][2] = acc[k][3] = 0.0f;
    const size_t T = (size_t)op.m.ntiles;
    while (more) {
        const unsigned char* ch = ring_wait(ring, ring_base);
        if (!ch) return false;
        const int ng = min(kBChunkG, cu.gb - cu.g), gl0 = cu.g - cu.ga;
#pragma unroll 2
        for (int k = 0; k < ng; k++) {
            const uint2 wv = *reinterpret_cast<const uint2*>(ch + k * kGB + 8 * lane);
            const float2 sw = *reinterpret_cast<const float2*>(ch + k * kGB + 256 + 8 * r);
            const uint32_t a0 = lo16(wv.x), a1 = lo16(wv.y), a2 = hi16(wv.x), a3 = hi16(wv.y);
            const unsigned char* xb = xd + (size_t)(gl0 + k) * NBLK * kBBlockBytes + 8 * lane;
            const float* fb = fac + ((gl0 + k) * NBLK * 4 + t) * 2;
#pragma unroll
            for (int blk = 0; blk < NBLK; blk++) {
                const uint2 b0 = *reinterpret_cast<const uint2*>(xb + blk * kBBlockBytes);
                const uint2 b1 = *reinterpret_cast<const uint2*>(xb + blk * kBBlockBytes + 256);
                const uint2 b2 = *reinterpret_cast<const uint2*>(xb + blk * kBBlockBytes + 512);
                const float2 f = *reinterpret_cast<const float2*>(fb + blk * 8);
                int dl[4], dh[4], d2[4];
                mma_s8(dl, a0, a1, a2, a3, b0.x, b0.y);
                mma_s8(dh, a0, a1, a2, a3, b1.x, b1.y);
                mma_s8(d2, a0, a1, a2, a3, b2.x, b2.y);
                const float v0 = fmaf((float)d2[0], 65536.0f, (float)(dl[0] + 256 * dl[1]));   // seq t, row r
                const float v1 = fmaf((float)d2[2], 65536.0f, (float)(dl[2] + 256 * dl[3]));   // seq t, row r + 8
                const float v2 = fmaf((float)d2[1], 65536.0f, (float)(dh[0] + 256 * dh[1]));   // seq t + 4, row r
                const float v3 = fmaf((float)d2[3], 65536.0f, (float)(dh[2] + 256 * dh[3]));   // seq t + 4, row r + 8
                acc[blk][0] = fmaf(sw.x * f.x, v0, acc[blk][0]);
                acc[blk][1] = fmaf(sw.y * f.x, v1, acc[blk][1]);
                acc[blk][2] = fmaf(sw.x * f.y, v2, acc[blk][2]);
                acc[blk][3] = fmaf(sw.y * f.y, v3, acc[blk][3]);
            }
        }
        ring_release(ring, true);
        const int tile = cu.tile, s = cu.s;
        const bool last = cu.g + kBChunkG >= cu.gb;
        more = bcur_next(cu);
        if (last) {
            float* p = part + ((size_t)s * T + tile) * NB8 * kTR;
#pragma unroll
            for (int blk = 0; blk < NBLK; blk++) {
                float* pb = p + (size_t)(8 * blk + t) * kTR;
                __stcg(pb + r, acc[blk][0]);
                __stcg(pb + r + 8, acc[blk][1]);
                __stcg(pb + 4 * kTR + r, acc[blk][2]);
                __stcg(pb + 4 * kTR + r + 8, acc[blk][3]);
                acc[blk][0] = acc[blk][1] = acc[blk][2] = acc[blk][3] = 0.0f;
            }
        }
    }
    return true;
}

// Sum over the S slices (in slice order) of row `row` of sequence b.
__device__ __forceinline__ float bsum(const float* part, int S, int T, int nb8, int b, int row) {
    const size_t stride = (size_t)T * nb8 * kTR;
    const float* p = part + ((size_t)(row >> 4) * nb8 + b) * kTR + (row & 15);
    float v = 0.0f;
    for (int s = 0; s < S; s++) v += __ldcg(p + s * stride);
    return v;
}

// One element of the int4 embedding row `tok` (src/kernel_simd.c:1032-1040).
__device__ __forceinline__ float emb_elem(const MatDesc& emb, int tok, int i) {
    const int rr = tok % kTR, lr = rr & 7, half = rr >> 3, g = i >> 5, e = i & 31;
    const uint8_t* gp = emb.w + (size_t)(tok / kTR) * emb.tile_bytes + (size_t)g * kGB;
    const float sc = __ldg(reinterpret_cast<const float*>(gp + 256 + 8 * lr + 4 * half));
    const int t = (e & 15) >> 2;
    const uint32_t wd = __ldg(reinterpret_cast<const uint32_t*>(gp + 8 * (4 * lr + t) + 4 * half));
    const int nib = (int)((wd >> (8 * (e & 3) + (e >= 16 ? 4 : 0))) & 0xF);
    return (float)(nib - 8) * sc;
}

// RMSNorm factors of every sequence from the per-CTA sums of squares
// (fixed reduction order): s_ss[b] = 1 / sqrtf(sum / dim + 1e-5)
// (src/kernel_simd.c:793-813).
__device__ void bnorm_factors(const BatchArgs& a, float* s_ss) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int b = warp; b < a.nb; b += kWarps) {
        float v = 0.0f;
        for (int c = lane; c < (int)gridDim.x; c += 32) v += __ldcg(a.ssq + (size_t)c * a.nb + b);
        v = warp_sum(v);
        if (lane == 0) s_ss[b] = 1.0f / sqrtf(__fdiv_rn(v, (float)a.dim) + 1e-5f);
    }
    csync();
}

// Residual rows [r0, r1) of this CTA for every sequence: x = f(b, row)
// (the embedding, or x + the sums of the last matvec), then this CTA's sums
// of squares per sequence.
template <class F>
__device__ void bresidual(const BatchArgs& a, float* s_sq, F f) {
    const int G = gridDim.x, c = blockIdx.x;
    const int r0 = (int)((long long)c * a.dim / G), r1 = (int)((long long)(c + 1) * a.dim / G), nr = r1 - r0;
    for (int i = threadIdx.x; i < a.nb * nr; i += kThreads) {
        const int b = i / nr, row = r0 + i % nr;
        const float v = f(b, row);
        __stcg(a.x + (size_t)b * a.dim + row, v);
        s_sq[i] = v * v;
    }
    csync();
    if (threadIdx.x < a.nb) {
        float s = 0.0f;
        for (int k = 0; k < nr; k++) s += s_sq[threadIdx.x * nr + k];
        __stcg(a.ssq + (size_t)c * a.nb + threadIdx.x, s);
    }
}

// Attention of one layer for every sequence: units (b, head, 16-position
// chunk) spread over all warps of the grid, as in attention_layer; s_uoff[b]
// is the first unit of sequence b (s_uoff[nb] = total).
__device__ void battention(const BatchArgs& a, int layer, const int* s_pos, const int* s_uoff) {
    const int hs = a.head_size, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int hq = hs / 4, sub = lane & 3, pg = lane >> 2;
    const float rs = sqrtf((float)hs);
    const int pstride = hs + 4;
    const int nw = gridDim.x * kWarps;
    const bool vl = 4 * lane < hs;
    const float4 z4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const int units = s_uoff[a.nb];
    for (int u = warp * gridDim.x + blockIdx.x; u < units; u += nw) {
        int b = 0;
        while (s_uoff[b + 1] <= u) b++;
        const int pos = s_pos[b], nch = pos / kAttnUnit + 1;
        const int v = u - s_uoff[b], h = v / nch, k = v - h * nch;
        const int kvh = h / a.kv_mul;
        const size_t lkv = (size_t)b * a.kv_seq + (size_t)layer * a.max_pos * a.kv_dim;
        const float* kc = a.kcache + lkv;
        const float* vc = a.vcache + lkv;
        const int t0 = k * kAttnUnit, n = min(kAttnUnit, pos + 1 - t0);
        const float* qp = a.q + (size_t)b * a.q_dim + h * hs + sub * hq;
        const float* kr0 = kc + (size_t)(t0 + pg) * a.kv_dim + kvh * hs + sub * hq;
        const float* kr1 = kr0 + (size_t)8 * a.kv_dim;
        float4 qv[kQ4], k0[kQ4], k1[kQ4];
#pragma unroll
        for (int j = 0; j < kQ4; j++) {
            const bool in = 4 * j < hq;
            qv[j] = in ? __ldcg(reinterpret_cast<const float4*>(qp + 4 * j)) : z4;
            k0[j] = (in && pg < n) ? __ldcg(reinterpret_cast<const float4*>(kr0 + 4 * j)) : z4;
            k1[j] = (in && pg + 8 < n) ? __ldcg(reinterpret_cast<const float4*>(kr1 + 4 * j)) : z4;
        }
        float d0 = 0.0f, d1 = 0.0f;
#pragma unroll
        for (int j = 0; j < kQ4; j++) {
            d0 = fmaf(qv[j].x, k0[j].x, d0);
            d0 = fmaf(qv[j].y, k0[j].y, d0);
            d0 = fmaf(qv[j].z, k0[j].z, d0);
            d0 = fmaf(qv[j].w, k0[j].w, d0);
            d1 = fmaf(qv[j].x, k1[j].x, d1);
            d1 = fmaf(qv[j].y, k1[j].y, d1);
            d1 = fmaf(qv[j].z, k1[j].z, d1);
            d1 = fmaf(qv[j].w, k1[j].w, d1);
        }
        d0 += __shfl_xor_sync(0xffffffffu, d0, 1);
        d1 += __shfl_xor_sync(0xffffffffu, d1, 1);
        d0 += __shfl_xor_sync(0xffffffffu, d0, 2);
        d1 += __shfl_xor_sync(0xffffffffu, d1, 2);
        float sc[kAttnUnit];
#pragma unroll
        for (int pp = 0; pp < 8; pp++) {
            sc[pp] = __shfl_sync(0xffffffffu, d0, pp * 4);
            sc[8 + pp] = __shfl_sync(0xffffffffu, d1, pp * 4);
        }
        const float* vr = vc + (size_t)t0 * a.kv_dim + kvh * hs + 4 * lane;
        float4 vv[kAttnUnit];
#pragma unroll
        for (int p = 0; p < kAttnUnit; p++)
            vv[p] = (p < n && vl) ? __ldcg(reinterpret_cast<const float4*>(vr + (size_t)p * a.kv_dim)) : z4;
        float m = -INFINITY;
#pragma unroll
        for (int p = 0; p < kAttnUnit; p++) {
            sc[p] = p < n ? __fdiv_rn(sc[p], rs) : -INFINITY;
            m = fmaxf(m, sc[p]);
        }
        float l = 0.0f;
#pragma unroll
        for (int p = 0; p < kAttnUnit; p++) {
            sc[p] = p < n ? expf(sc[p] - m) : 0.0f;
            l += sc[p];
        }
        float4 o = z4;
#pragma unroll
        for (int p = 0; p < kAttnUnit; p++) {
            o.x = fmaf(sc[p], vv[p].x, o.x);
            o.y = fmaf(sc[p], vv[p].y, o.y);
            o.z = fmaf(sc[p], vv[p].z, o.z);
            o.w = fmaf(sc[p], vv[p].w, o.w);
        }
        float* ap = a.att + (size_t)b * a.q_dim + h * hs + 4 * lane;
        if (nch == 1) {
            const float inv = 1.0f / l;
            if (vl) __stcg(reinterpret_cast<float4*>(ap), make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv));
            continue;
        }
        const int bh = b * a.n_heads + h;
        float* part = a.attn_part + ((size_t)bh * a.max_chunks + k) * pstride;
        if (vl) __stcg(reinterpret_cast<float4*>(part + 4 + 4 * lane), o);
        if (lane == 0) {
            __stcg(part, m);
            __stcg(part + 1, l);
        }
        __threadfence();
        __syncwarp();
        int last = 0;
        if (lane == 0) last = atomicAdd(a.attn_cnt + bh, 1) == nch - 1;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (!last) continue;
        __threadfence();
        const float* ph = a.attn_part + (size_t)bh * a.max_chunks * pstride;
        float M = -INFINITY;
        for (int c0 = 0; c0 < nch; c0 += 32)
            if (c0 + lane < nch) M = fmaxf(M, __ldcg(ph + (size_t)(c0 + lane) * pstride));
        M = warp_max(M);
        float L = 0.0f;
        float4 acc = z4;
        for (int c0 = 0; c0 < nch; c0 += 32) {
            const int cn = min(32, nch - c0);
            float wl = 0.0f, ll = 0.0f;
            if (lane < cn) {
                wl = expf(__ldcg(ph + (size_t)(c0 + lane) * pstride) - M);
                ll = __ldcg(ph + (size_t)(c0 + lane) * pstride + 1);
            }
            for (int c = 0; c < cn; c++) {
                const float wgt = __shfl_sync(0xffffffffu, wl, c);
                const float lc = __shfl_sync(0xffffffffu, ll, c);
                L = fmaf(lc, wgt, L);
                if (vl) {
                    const float4 oc =
                        __ldcg(reinterpret_cast<const float4*>(ph + (size_t)(c0 + c) * pstride + 4 + 4 * lane));
                    acc.x = fmaf(oc.x, wgt, acc.x);
                    acc.y = fmaf(oc.y, wgt, acc.y);
                    acc.z = fmaf(oc.z, wgt, acc.z);
                    acc.w = fmaf(oc.w, wgt, acc.w);
                }
            }
        }
        const float inv = 1.0f / L;
        if (vl) __stcg(reinterpret_cast<float4*>(ap), make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv));
        if (lane == 0) a.attn_cnt[bh] = 0;
    }
}

// ---------------------------------------------------------------------------
// The batched decode kernel (NBLK blocks of 8 sequences).
// ---------------------------------------------------------------------------
template <int NBLK>
__global__ void __launch_bounds__(kDecodeThreads, 1) k_decode_batch(BatchArgs a) {
    constexpr int NB8 = 8 * NBLK;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bars[kWarps * 2 * 8];
    __shared__ float s_sq[kBMaxSeq * kBMaxResRows];
    __shared__ float s_ss[kBMaxSeq];
    __shared__ int s_tok[kBMaxSeq], s_pos[kBMaxSeq], s_uoff[kBMaxSeq + 1];
    __shared__ int s_bad;
    unsigned char* xd = smem;
    float* fac = reinterpret_cast<float*>(smem + a.fac_off);
    unsigned char* ring_base = smem + a.ring_off;
    BOpDesc* ops = reinterpret_cast<BOpDesc*>(smem + a.ops_off);
    static_assert(sizeof(BOpDesc) % 4 == 0, "BOpDesc copy");
    for (int i = threadIdx.x; i < a.nops * (int)(sizeof(BOpDesc) / 4); i += kDecodeThreads)
        reinterpret_cast<int*>(ops)[i] = __ldg(reinterpret_cast<const int*>(a.ops) + i);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    Ring ring;
    if (warp < kWarps) ring_init(ring, ring_base, bars, a.P, kBChunkBytes, warp, lane == 0);
    fence_mbar_init();
    __syncthreads();
    if (warp == kWarps) {
        if (lane < kWarps) bproduce(a, ops, ring_base, bars, lane);
        return;
    }

    uint32_t nbar = 0;
    bool ok = true;
    const int tid = threadIdx.x;
    // A matvec phase: digits of this CTA's slice, then its units.
    auto matvec = [&](const BOpDesc& op, const float* src, int ld, const float* nw) -> bool {
        const BSlice sl = bslice(op, blockIdx.x, gridDim.x);
        bbuild_digits<NBLK>(xd, fac, src, ld, nw, sl.ga, sl.gb, a.nb);
        csync();
        const bool fine = brun_op<NBLK>(op, ring, ring_base, xd, fac, a.part);
        if (csync_or(!fine)) {
            if (tid == 0) set_error(a.step, DEV_COPY_TIMEOUT);
            return false;
        }
        return grid_barrier(a.step, nbar);
    };

    for (int step = 0; step < a.steps && ok; step++) {
        // Tokens and positions of this step.
        const int par = step & 1;
        if (tid < a.nb) {
            const int tok = step == 0 ? a.first[tid] : (int)key_index(__ldcg(a.argmax + (par ^ 1) * kBMaxSeq + tid));
            const int pos = a.pos0[tid] + step;
            s_tok[tid] = tok;
            s_pos[tid] = pos;
        }
        csync();
        if (tid == 0) {
            int bad = 0;
            for (int b = 0; b < a.nb; b++)
                bad |= (s_tok[b] < 0 || s_tok[b] >= a.vocab || s_pos[b] < 0 || s_pos[b] >= a.max_pos);
            s_bad = bad;
            int u = 0;
            for (int b = 0; b < a.nb; b++) {
                s_uoff[b] = u;
                u += a.n_heads * (s_pos[b] / kAttnUnit + 1);
            }
            s_uoff[a.nb] = u;
        }
        csync();
        if (s_bad) {
            if (blockIdx.x == 0 && tid == 0) set_error(a.step, DEV_BAD_INPUT);
            break;
        }
        if (blockIdx.x == 0 && tid < a.nb) {
            a.tokens[(size_t)step * a.nb + tid] = s_tok[tid];
            a.argmax[par * kBMaxSeq + tid] = argmax_key(-1e9f, 0);   // this step's keys start here
        }
        bresidual(a, s_sq, [&](int b, int row) { return emb_elem(a.emb, s_tok[b], row); });
        if (!grid_barrier(a.step, nbar)) { ok = false; break; }

        for (int oi = 0; oi < a.nops && ok; oi++) {
            const BOpDesc op = ops[oi];
            const int T = op.m.ntiles, S = op.S;
            const int l = op.layer;
            if (op.kind == OP_QKV) {
                if (!(ok = matvec(op, a.x, a.dim, a.rms_att + (size_t)l * a.dim))) break;
                // q, k, v rows: RoPE on adjacent pairs (src/kernel_simd.c:1068-1085), KV append.
                bnorm_factors(a, s_ss);
                const int npair = (a.q_dim + 2 * a.kv_dim) / 2, h2 = a.head_size / 2;
                for (int i = blockIdx.x * kThreads + tid; i < a.nb * npair; i += gridDim.x * kThreads) {
                    const int b = i / npair, p = i - b * npair, row = 2 * p;
                    const float ss = s_ss[b];
                    const float v0 = __fmul_rn(bsum(a.part, S, T, NB8, b, row), ss);
                    const float v1 = __fmul_rn(bsum(a.part, S, T, NB8, b, row + 1), ss);
                    const int pos = s_pos[b];
                    const size_t lkv = (size_t)b * a.kv_seq + (size_t)l * a.max_pos * a.kv_dim + (size_t)pos * a.kv_dim;
                    if (row < a.q_dim + a.kv_dim) {
                        const bool is_q = row < a.q_dim;
                        const int base = is_q ? row : row - a.q_dim;
                        const int hd = base % a.head_size;
                        const float fr = __ldg(a.freq_re + (size_t)pos * h2 + hd / 2);
                        const float fi = __ldg(a.freq_im + (size_t)pos * h2 + hd / 2);
                        const float o0 = __fsub_rn(__fmul_rn(v0, fr), __fmul_rn(v1, fi));
                        const float o1 = __fadd_rn(__fmul_rn(v0, fi), __fmul_rn(v1, fr));
                        float* dst = is_q ? a.q + (size_t)b * a.q_dim + base : a.kcache + lkv + base;
                        __stcg(reinterpret_cast<float2*>(dst), make_float2(o0, o1));
                    } else {
                        const int base = row - a.q_dim - a.kv_dim;
                        __stcg(reinterpret_cast<float2*>(a.vcache + lkv + base), make_float2(v0, v1));
                    }
                }
                if (!grid_barrier(a.step, nbar)) { ok = false; break; }
                battention(a, l, s_pos, s_uoff);
                if (!grid_barrier(a.step, nbar)) { ok = false; break; }
            } else if (op.kind == OP_WO || op.kind == OP_W2) {
                const bool wo = op.kind == OP_WO;
                if (!(ok = matvec(op, wo ? a.att : a.hb, wo ? a.q_dim : a.hidden, nullptr))) break;
                bresidual(a, s_sq, [&](int b, int row) {
                    return __ldcg(a.x + (size_t)b * a.dim + row) + bsum(a.part, S, T, NB8, b, row);
                });
                if (!grid_barrier(a.step, nbar)) { ok = false; break; }
            } else if (op.kind == OP_W13) {
                if (!(ok = matvec(op, a.x, a.dim, a.rms_ffn + (size_t)l * a.dim))) break;
                // rows w1[2j], w1[2j+1], w3[2j], w3[2j+1]; SwiGLU (src/kernel_simd.c:836-841)
                bnorm_factors(a, s_ss);
                for (int i = blockIdx.x * kThreads + tid; i < a.nb * a.hidden; i += gridDim.x * kThreads) {
                    const int b = i / a.hidden, j = i - b * a.hidden;
                    const int row = 4 * (j >> 1) + (j & 1);
                    const float ss = s_ss[b];
                    const float g = __fmul_rn(bsum(a.part, S, T, NB8, b, row), ss);
                    const float u = __fmul_rn(bsum(a.part, S, T, NB8, b, row + 2), ss);
                    const float s = __fdiv_rn(g, __fadd_rn(1.0f, expf_cr(-g)));
                    __stcg(a.hb + (size_t)b * a.hidden + j, __fmul_rn(s, u));
                }
                if (!grid_barrier(a.step, nbar)) { ok = false; break; }
            } else {   // OP_CLS
                if (!(ok = matvec(op, a.x, a.dim, a.rms_final))) break;
                bnorm_factors(a, s_ss);
                const int G = gridDim.x, c = blockIdx.x;
                const int r0 = (int)((long long)c * a.vocab / G), r1 = (int)((long long)(c + 1) * a.vocab / G);
                for (int b = warp; b < a.nb; b += kWarps) {
                    const float ss = s_ss[b];
                    float best = -1e9f;
                    uint32_t bi = 0;
                    for (int row = r0 + lane; row < r1; row += 32) {
                        const float v = __fmul_rn(bsum(a.part, S, T, NB8, b, row), ss);
                        __stcg(a.logits + (size_t)b * a.vocab + row, v);
                        if (v > best) {
                            best = v;
                            bi = (uint32_t)row;
                        }
                    }
                    unsigned long long key = best > -1e9f ? argmax_key(best, bi) : 0ull;
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
                        const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
                        key = other > key ? other : key;
                    }
                    if (lane == 0 && key) atomicMax(a.argmax + par * kBMaxSeq + b, key);
                }
                if (!grid_barrier(a.step, nbar)) { ok = false; break; }
                if (step == a.steps - 1 && blockIdx.x == 0 && tid < a.nb)
                    a.tokens[(size_t)a.steps * a.nb + tid] = (int)key_index(__ldcg(a.argmax + par * kBMaxSeq + tid));
            }
        }
    }
}

}  // namespace aion
