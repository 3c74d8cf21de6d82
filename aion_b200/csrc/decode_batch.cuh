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
constexpr int kBDigitBudget = 112 * 1024;         // shared memory for one slice's digits + factors
constexpr int kBMaxResGroups = 40;                // residual groups of 32 per CTA (dim <= 1280 * grid)
constexpr int kBAttnStage = 16 * kMaxHead * 4;   // one warp's K and V rows of 8 positions
// Attention stages and partials, in the digit area (idle while attention runs).
constexpr int kBAttnScratch = kWarps * kBAttnStage + kWarps * (kMaxHead + 4) * 4;

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
    float *x, *q, *att, *logits;        // [nb][dim], [nb][q_dim] x2, [nb][vocab]
    unsigned char* dg;       // digits of the next matvec's input: [groups][NBLK][kBGroupBytes]
    float *kcache, *vcache;  // sequence b at + b * kv_seq: [L][max_pos][kv_dim]
    size_t kv_seq;
    float* part;             // [S][ntiles][nb8][16]: partial rows of the last matvec
    float* ssq;              // [grid][nb]: per CTA, sum of squares of its residual rows
    StepState* step;         // barrier counter and error code
    unsigned long long* argmax;   // [2][kBMaxSeq] keys, by step parity
    const int32_t* first;    // [nb] tokens of step 0
    const int32_t* pos0;     // [nb] positions of step 0
    int32_t* tokens;         // [steps + 1][nb]: each step's input tokens, then the last step's pick
    int steps;
    int P;                   // ring slots per warp (kBChunkBytes each)
    SamplerParams samp;      // used when sampling != 0 (else the greedy argmax)
    int sampling;
    int vocab_rows;          // classifier rows this GPU holds (logits stride): vocab, or vocab / tp_n
    // Tensor parallelism over tp_n GPUs (tp_n == 1: off), as in k_decode:
    // this rank holds q_dim query rows, kv_dim K/V rows, hidden FFN rows and
    // classifier rows [vocab_off, vocab_off + vocab_rows); WO and W2 give
    // partial sums over its slice of their inputs.  tp_peers[j] is rank j's
    // exchange region: partial rows u64 [2][tp_n][tp_nbmax][dim] at
    // tp_brecv_off (value | exchange count << 32, slot count & 1), argmax
    // keys u64 [tp_n][kBMaxSeq] at tp_bkeys_off, flags u32 [tp_n] at
    // tp_flags_off (shared with k_decode, as is StepState::tp_count).
    int tp_n, tp_rank, vocab_off, tp_nbmax;
    unsigned char* const* tp_peers;
    long long tp_brecv_off, tp_bkeys_off;
    int tp_flags_off;
    int ring_off, ops_off;   // dynamic shared memory: digits (or attention scratch) at 0
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
// Digit layout of an input vector, per group slot g and block blk of 8
// sequences, kBGroupBytes at (g * NBLK + blk) * kBGroupBytes: the B
// operands of MMA 0, 1, 2 (256 bytes each: column c at 32c, quad lane t at
// 8t, elements 4t..4t+3 then 16+4t..16+4t+3), then 8 fp32 factors, pair t
// = (sequence t, sequence t + 4).  The same layout serves the whole vector
// in global memory (slot = group) and one slice in shared memory (slot =
// group - first group of the slice).  Padding sequences (b >= nb) carry
// zero digits and factors.
// ---------------------------------------------------------------------------
constexpr int kBGroupBytes = 800;

// Largest magnitude of a group of 32 held by 8 consecutive lanes (4 each).
__device__ __forceinline__ float group_max8(float4 v) {
    float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    return fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
}

// Digits of elements 4q..4q+3 (v) of group slot g of sequence b, whose
// group maximum is m.
template <int NBLK>
__device__ __forceinline__ void bdigit_store(unsigned char* base, int g, int b, int q, float4 v, float m) {
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
    unsigned char* gp = base + (size_t)(g * NBLK + blk) * kBGroupBytes;
    unsigned char* lo = gp + (j >> 2) * 256 + (2 * (j & 3)) * 32 + 8 * t + 4 * h;
    *reinterpret_cast<uint32_t*>(lo) = __byte_perm(t01, t23, 0x5410);        // d0
    *reinterpret_cast<uint32_t*>(lo + 32) = __byte_perm(t01, t23, 0x7632);   // d1
    *reinterpret_cast<uint32_t*>(gp + 512 + (2 * (j & 3) + (j >> 2)) * 32 + 8 * t + 4 * h) =
        __byte_perm(u01, u23, 0x5410);                                       // d2
    if (q == 0)
        *reinterpret_cast<float*>(gp + 768 + ((j & 3) * 2 + (j >> 2)) * 4) =
            live ? __int_as_float((123 - E) << 23) : 0.0f;                  // 2^-E / 16
}

// Digits of groups [ga, gb) of every sequence's input src + b * ld into
// shared memory (slots from 0).  Item i = (local group, sequence, quarter);
// each pass loads four items per thread before digitising them, so the L2
// round trips overlap.
template <int NBLK>
__device__ void bbuild_digits(unsigned char* xd, const float* src, int ld, int ga, int gb, int nb) {
    constexpr int NB8 = 8 * NBLK, U = 4;
    const int total = (gb - ga) * NB8 * 8;
    for (int base = 0; base < total; base += U * kThreads) {   // uniform trip count: the shuffles see full warps
        float4 v[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int i = base + u * kThreads + threadIdx.x;
            const int q = i & 7, rest = i >> 3;
            const int b = rest % NB8, gl = rest / NB8;
            v[u] = (i < total && b < nb)
                       ? __ldcg(reinterpret_cast<const float4*>(src + (size_t)b * ld + (ga + gl) * 32 + 4 * q))
                       : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int i = base + u * kThreads + threadIdx.x;
            const float m = group_max8(v[u]);
            const int q = i & 7, rest = i >> 3;
            if (i < total) bdigit_store<NBLK>(xd, rest / NB8, rest % NB8, q, v[u], m);
        }
    }
}

// One matvec op on this CTA: consume its chunks, write each finished unit's
// 16 x nb8 partial rows.  False if a wait gave up (not uniform: the caller
// reduces it over the CTA).
template <int NBLK>
__device__ bool brun_op(const BOpDesc& op, Ring& ring, unsigned char* ring_base, const unsigned char* xd, float* part) {
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
            const unsigned char* gp = xd + (size_t)(gl0 + k) * NBLK * kBGroupBytes;
#pragma unroll
            for (int blk = 0; blk < NBLK; blk++) {
                const unsigned char* xb = gp + blk * kBGroupBytes + 8 * lane;
                const uint2 b0 = *reinterpret_cast<const uint2*>(xb);
                const uint2 b1 = *reinterpret_cast<const uint2*>(xb + 256);
                const uint2 b2 = *reinterpret_cast<const uint2*>(xb + 512);
                const float2 f = *reinterpret_cast<const float2*>(gp + blk * kBGroupBytes + 768 + 8 * t);
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

// Sum over the S slices (in slice order) of rows row4..row4+3 (row4 % 4 ==
// 0) of sequence b; four slices' loads are in flight at a time.
__device__ __forceinline__ float4 bsum4(const float* part, int S, int T, int nb8, int b, int row4) {
    const size_t stride = (size_t)T * nb8 * kTR;
    const float4* p = reinterpret_cast<const float4*>(part + ((size_t)(row4 >> 4) * nb8 + b) * kTR + (row4 & 15));
    const size_t st4 = stride / 4;
    float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    int s = 0;
    auto add = [&](float4 t) {
        v.x += t.x;
        v.y += t.y;
        v.z += t.z;
        v.w += t.w;
    };
    for (; s + 4 <= S; s += 4) {
        const float4 t0 = __ldcg(p + s * st4), t1 = __ldcg(p + (s + 1) * st4);
        const float4 t2 = __ldcg(p + (s + 2) * st4), t3 = __ldcg(p + (s + 3) * st4);
        add(t0);
        add(t1);
        add(t2);
        add(t3);
    }
    for (; s < S; s++) add(__ldcg(p + s * st4));
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
// The CTAs' partial sums ([grid][nb]) are staged into `scratch` (idle
// shared memory, grid * nb floats) in one coalesced pass, so the per-sequence
// sums below take no further L2 round trips; the order of the sums is fixed.
__device__ void bnorm_factors(const BatchArgs& a, float* s_ss, float* scratch) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = (int)gridDim.x * a.nb;
    for (int i = threadIdx.x; i < n; i += kThreads) scratch[i] = __ldcg(a.ssq + i);
    csync();
    for (int b = warp; b < a.nb; b += kWarps) {
        float v = 0.0f;
        for (int c = lane; c < (int)gridDim.x; c += 32) v += scratch[c * a.nb + b];
        v = warp_sum(v);
        if (lane == 0) s_ss[b] = 1.0f / sqrtf(__fdiv_rn(v, (float)a.dim) + 1e-5f);
    }
    csync();
}

// Tensor parallelism: this rank's partial rows d (rows row4..row4+3 of
// sequence b) go, tagged with the exchange count, into slot `count & 1` of
// every rank's receive rows; then the ranks' partials are summed in rank
// order as they arrive (bounded waits).  False if a wait gave up.
__device__ bool btp_sum4(const BatchArgs& a, float4& d, int b, int row4, uint32_t count) {
    const size_t nbm = (size_t)a.tp_nbmax, dim = (size_t)a.dim;
    const size_t slot = (size_t)(count & 1u) * a.tp_n;
    for (int j = 0; j < a.tp_n; j++) {
        uint64_t* r = reinterpret_cast<uint64_t*>(a.tp_peers[j] + a.tp_brecv_off) + ((slot + a.tp_rank) * nbm + b) * dim + row4;
        st_relaxed_sys_u64(r, tag_pack(d.x, count));
        st_relaxed_sys_u64(r + 1, tag_pack(d.y, count));
        st_relaxed_sys_u64(r + 2, tag_pack(d.z, count));
        st_relaxed_sys_u64(r + 3, tag_pack(d.w, count));
    }
    const uint64_t* own = reinterpret_cast<const uint64_t*>(a.tp_peers[a.tp_rank] + a.tp_brecv_off);
    float sum[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int j = 0; j < a.tp_n; j++) {
        // the rank's four words are loaded together, then only the untagged
        // ones polled again
        const uint64_t* p = own + ((slot + j) * nbm + b) * dim + row4;
        uint64_t t[4];
#pragma unroll
        for (int k = 0; k < 4; k++) t[k] = ld_relaxed_sys_u64(p + k);
#pragma unroll
        for (int k = 0; k < 4; k++) {
            for (uint32_t i = 0; tag_ep(t[k]) != count; i++) {
                if (i > (1u << 22)) return false;
                t[k] = ld_relaxed_sys_u64(p + k);
            }
            sum[k] += tag_val(t[k]);
        }
    }
    d = make_float4(sum[0], sum[1], sum[2], sum[3]);
    return true;
}

// The ranks' argmax keys: after a grid barrier CTA 0 raises this rank's flag
// to `count` in every rank's region and each CTA waits (bounded) until
// every rank's flag reached it (the keys were stored, fenced, before).
__device__ bool btp_exchange(const BatchArgs& a, uint32_t& nbar, uint32_t count) {
    __shared__ int s_xok;
    if (!grid_barrier(a.step, nbar)) return false;
    if (threadIdx.x == 0) {
        if (blockIdx.x == 0)
            for (int j = 0; j < a.tp_n; j++)
                st_release_sys_u32(reinterpret_cast<uint32_t*>(a.tp_peers[j] + a.tp_flags_off) + a.tp_rank, count);
        const volatile uint32_t* fl = reinterpret_cast<const volatile uint32_t*>(a.tp_peers[a.tp_rank] + a.tp_flags_off);
        int ok = 1;
        for (int j = 0; j < a.tp_n && ok; j++) {
            uint32_t i = 0;
            while ((int32_t)(fl[j] - count) < 0)
                if (++i > (1u << 24)) {
                    ok = 0;
                    break;
                }
        }
        __threadfence_system();
        if (!ok) set_error(a.step, DEV_BARRIER_TIMEOUT);
        s_xok = ok;
    }
    csync();
    return s_xok != 0;
}

// Residual update of this CTA's groups [g0, g1) of the model dimension for
// every sequence: x = f(b, row4) (float4 of rows row4..row4+3) when
// xcount == 0, else x + f(b, row4) summed over the ranks by exchange xcount;
// then this CTA's sums of squares per sequence, and the digits of x * nw
// (the RMSNorm weight of the op that reads x next) into the global digit
// buffer.  False if an exchange wait gave up.
template <int NBLK, class F>
__device__ bool bresidual(const BatchArgs& a, const float* nw, float* s_sq, uint32_t xcount, F f) {
    bool ok = true;
    constexpr int NB8 = 8 * NBLK;
    const int G = gridDim.x, c = blockIdx.x, Gd = a.dim / 32;
    const int g0 = (int)((long long)c * Gd / G), g1 = (int)((long long)(c + 1) * Gd / G), ng = g1 - g0;
    const int total = ng * NB8 * 8;
    for (int base = 0; base < total; base += kThreads) {
        const int i = base + threadIdx.x;
        const int q = i & 7, rest = i >> 3, b = rest % NB8, gl = rest / NB8;
        const bool live = i < total && b < a.nb;
        const int row4 = (g0 + gl) * 32 + 4 * q;
        float4 x = make_float4(0.0f, 0.0f, 0.0f, 0.0f), v = x;
        if (live) {
            x = f(b, row4);
            if (xcount) {
                if (a.tp_n > 1 && !btp_sum4(a, x, b, row4, xcount)) ok = false;
                const float4 xo = __ldcg(reinterpret_cast<const float4*>(a.x + (size_t)b * a.dim + row4));
                x = make_float4(xo.x + x.x, xo.y + x.y, xo.z + x.z, xo.w + x.w);
            }
            __stcg(reinterpret_cast<float4*>(a.x + (size_t)b * a.dim + row4), x);
            const float4 w = __ldg(reinterpret_cast<const float4*>(nw + row4));
            v = make_float4(__fmul_rn(x.x, w.x), __fmul_rn(x.y, w.y), __fmul_rn(x.z, w.z), __fmul_rn(x.w, w.w));
        }
        float sq = x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
        sq += __shfl_xor_sync(0xffffffffu, sq, 1);
        sq += __shfl_xor_sync(0xffffffffu, sq, 2);
        sq += __shfl_xor_sync(0xffffffffu, sq, 4);
        const float m = group_max8(v);
        if (i < total) {
            if (live && q == 0) s_sq[b * ng + gl] = sq;
            bdigit_store<NBLK>(a.dg, g0 + gl, b, q, v, m);
        }
    }
    const bool bad = csync_or(!ok);
    if (threadIdx.x < a.nb) {
        float s = 0.0f;
        for (int k = 0; k < ng; k++) s += s_sq[threadIdx.x * ng + k];
        __stcg(a.ssq + (size_t)c * a.nb + threadIdx.x, s);
    }
    if (bad && threadIdx.x == 0) set_error(a.step, DEV_BARRIER_TIMEOUT);
    return !bad;
}

// Attention of one layer for every sequence (src/kernel_simd.c:1099-1117):
// one CTA per (sequence b, head h) at a time.  Warp w takes the 8-position
// blocks w, w + 11, ... of positions 0..pos.  Its lane 0 bulk-copies the
// block's K and V rows (hs floats each) into the warp's stage in shared
// memory; the copies bypass the L1 path that a kernel with this much shared
// memory leaves narrow.  Then lane 4p + s scores position p on quarter s of
// the head (elements 4(s + 4j)..+3, j < hs/16), lane l accumulates V
// elements 4l..4l+3, and the warp folds the block into its running max, sum
// and weighted V sum (online softmax).  The warps' partials meet in shared
// memory and are merged in warp order.
// `area`: kWarps stages of kBAttnStage bytes, then kWarps * (hs + 4) floats.
__device__ bool battention(const BatchArgs& a, int layer, const int* s_pos, unsigned char* area, uint64_t* abar,
                           uint32_t& aphase) {
    const int hs = a.head_size, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int sub = lane & 3, pg = lane >> 2, nq = hs / 16;
    const float rs = sqrtf((float)hs);
    const bool vl = 4 * lane < hs;
    const float4 z4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const int pstride = hs + 4;
    const uint32_t rowb = (uint32_t)hs * 4;
    float* stage = reinterpret_cast<float*>(area + (size_t)warp * kBAttnStage);   // K rows [8][hs], V rows [8][hs]
    float* scratch = reinterpret_cast<float*>(area + (size_t)kWarps * kBAttnStage);
    const uint32_t bar = smem_addr(abar + warp);
    bool ok = true;
    const int units = a.nb * a.n_heads;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
        const int b = u / a.n_heads, h = u - b * a.n_heads;
        const int pos = s_pos[b], kvh = h / a.kv_mul;
        const size_t lkv = (size_t)b * a.kv_seq + (size_t)layer * a.max_pos * a.kv_dim + (size_t)kvh * hs;
        const float* kc = a.kcache + lkv;
        const float* vc = a.vcache + lkv;
        const float* qp = a.q + (size_t)b * a.q_dim + h * hs;
        float4 qv[kQ4];
#pragma unroll
        for (int j = 0; j < kQ4; j++)
            qv[j] = j < nq ? __ldcg(reinterpret_cast<const float4*>(qp + 4 * (sub + 4 * j))) : z4;
        float m = -INFINITY, l = 0.0f;
        float4 o = z4;
        for (int t0 = warp * 8; t0 <= pos && ok; t0 += kWarps * 8) {
            const int n = min(8, pos + 1 - t0);
            __syncwarp();   // every lane is done with the stage's previous rows
            if (lane == 0) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_arrive_expect_tx(bar, 2u * (uint32_t)n * rowb);
                for (int p = 0; p < n; p++) {
                    bulk_g2s(smem_addr(stage + p * hs), kc + (size_t)(t0 + p) * a.kv_dim, rowb, bar);
                    bulk_g2s(smem_addr(stage + (8 + p) * hs), vc + (size_t)(t0 + p) * a.kv_dim, rowb, bar);
                }
            }
            if (!mbar_wait(bar, aphase)) {
                // Give up on this warp's attention; let the copies in flight
                // land (bounded) before the stage is reused or the CTA ends.
                mbar_wait(bar, aphase, 1u << 20);
                ok = false;
                break;
            }
            aphase ^= 1u;
            float4 kv[kQ4], vv[8];
#pragma unroll
            for (int j = 0; j < kQ4; j++)
                kv[j] = (j < nq && pg < n) ? *reinterpret_cast<const float4*>(stage + pg * hs + 4 * (sub + 4 * j)) : z4;
#pragma unroll
            for (int p = 0; p < 8; p++)
                vv[p] = (p < n && vl) ? *reinterpret_cast<const float4*>(stage + (8 + p) * hs + 4 * lane) : z4;
            float d = 0.0f;
#pragma unroll
            for (int j = 0; j < kQ4; j++) {
                d = fmaf(qv[j].x, kv[j].x, d);
                d = fmaf(qv[j].y, kv[j].y, d);
                d = fmaf(qv[j].z, kv[j].z, d);
                d = fmaf(qv[j].w, kv[j].w, d);
            }
            d += __shfl_xor_sync(0xffffffffu, d, 1);
            d += __shfl_xor_sync(0xffffffffu, d, 2);
            const float sc_own = pg < n ? __fdiv_rn(d, rs) : -INFINITY;
            float sc[8];
            float mb = -INFINITY;
#pragma unroll
            for (int p = 0; p < 8; p++) {
                sc[p] = __shfl_sync(0xffffffffu, sc_own, 4 * p);
                mb = fmaxf(mb, sc[p]);
            }
            const float mn = fmaxf(m, mb);
            const float corr = expf(m - mn);
            l *= corr;
            o.x *= corr;
            o.y *= corr;
            o.z *= corr;
            o.w *= corr;
#pragma unroll
            for (int p = 0; p < 8; p++) {
                const float e = expf(sc[p] - mn);
                l += e;
                o.x = fmaf(e, vv[p].x, o.x);
                o.y = fmaf(e, vv[p].y, o.y);
                o.z = fmaf(e, vv[p].z, o.z);
                o.w = fmaf(e, vv[p].w, o.w);
            }
            m = mn;
        }
        float* wp = scratch + warp * pstride;
        if (lane == 0) {
            wp[0] = m;
            wp[1] = l;
        }
        if (vl) *reinterpret_cast<float4*>(wp + 4 + 4 * lane) = o;
        csync();
        for (int j = threadIdx.x; j < hs; j += kThreads) {
            float M = -INFINITY;
            for (int k = 0; k < kWarps; k++) M = fmaxf(M, scratch[k * pstride]);
            float L = 0.0f, O = 0.0f;
            for (int k = 0; k < kWarps; k++) {
                const float mk = scratch[k * pstride];
                if (mk == -INFINITY) continue;   // a warp with no positions
                const float wk = expf(mk - M);
                L = fmaf(scratch[k * pstride + 1], wk, L);
                O = fmaf(scratch[k * pstride + 4 + j], wk, O);
            }
            __stcg(a.att + (size_t)b * a.q_dim + h * hs + j, O / L);
        }
        csync();
    }
    return ok;
}

// ---------------------------------------------------------------------------
// The batched decode kernel (NBLK blocks of 8 sequences).
// ---------------------------------------------------------------------------
template <int NBLK>
__global__ void __launch_bounds__(kDecodeThreads, 1) k_decode_batch(BatchArgs a) {
    constexpr int NB8 = 8 * NBLK;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bars[kWarps * 2 * 8];
    __shared__ __align__(8) uint64_t s_dbar;          // the slice's digits, copied from the global buffer
    __shared__ __align__(8) uint64_t s_abar[kWarps];  // each warp's attention stage
    __shared__ float s_sq[kBMaxSeq * kBMaxResGroups];
    __shared__ float s_ss[kBMaxSeq];
    __shared__ int s_tok[kBMaxSeq], s_pos[kBMaxSeq];
    __shared__ int s_bad;
    unsigned char* xd = smem;
    unsigned char* ring_base = smem + a.ring_off;
    BOpDesc* ops = reinterpret_cast<BOpDesc*>(smem + a.ops_off);
    static_assert(sizeof(BOpDesc) % 4 == 0, "BOpDesc copy");
    for (int i = threadIdx.x; i < a.nops * (int)(sizeof(BOpDesc) / 4); i += kDecodeThreads)
        reinterpret_cast<int*>(ops)[i] = __ldg(reinterpret_cast<const int*>(a.ops) + i);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    Ring ring;
    if (warp < kWarps) ring_init(ring, ring_base, bars, a.P, kBChunkBytes, warp, lane == 0);
    if (threadIdx.x == 0) {
        mbar_init(smem_addr(&s_dbar), 1);
        for (int w = 0; w < kWarps; w++) mbar_init(smem_addr(&s_abar[w]), 1);
    }
    fence_mbar_init();
    __syncthreads();
    if (warp == kWarps) {
        if (lane < kWarps) bproduce(a, ops, ring_base, bars, lane);
        return;
    }

    uint32_t nbar = 0, dphase = 0, aphase = 0;
    bool ok = true;
    const int tid = threadIdx.x;
    __shared__ uint32_t s_xcount;
    if (tid == 0) s_xcount = *reinterpret_cast<volatile uint32_t*>(&a.step->tp_count);
    csync();
    uint32_t xcount = s_xcount;   // tensor-parallel exchanges so far (identical on every rank)
    // A matvec phase: the digits of this CTA's slice (built from att for WO,
    // else copied from the global buffer the previous phase wrote), then its
    // units.
    auto matvec = [&](const BOpDesc& op) -> bool {
        const BSlice sl = bslice(op, blockIdx.x, gridDim.x);
        bool fine = true;
        if (op.kind == OP_WO) {
            bbuild_digits<NBLK>(xd, a.att, a.q_dim, sl.ga, sl.gb, a.nb);
            csync();
        } else {
            if (tid == 0) {
                // The buffer was written by other CTAs' generic stores before
                // the grid barrier; the copy runs in the async proxy.
                asm volatile("fence.proxy.async;" ::: "memory");
                const uint32_t bytes = (uint32_t)((sl.gb - sl.ga) * NBLK * kBGroupBytes);
                mbar_arrive_expect_tx(smem_addr(&s_dbar), bytes);
                bulk_g2s(smem_addr(xd), a.dg + (size_t)sl.ga * NBLK * kBGroupBytes, bytes, smem_addr(&s_dbar));
            }
            fine = mbar_wait(smem_addr(&s_dbar), dphase);
            dphase ^= 1u;
        }
        if (fine) fine = brun_op<NBLK>(op, ring, ring_base, xd, a.part);
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
        bresidual<NBLK>(a, a.rms_att, s_sq, 0u, [&](int b, int row4) {
            return make_float4(emb_elem(a.emb, s_tok[b], row4), emb_elem(a.emb, s_tok[b], row4 + 1),
                               emb_elem(a.emb, s_tok[b], row4 + 2), emb_elem(a.emb, s_tok[b], row4 + 3));
        });
        if (!grid_barrier(a.step, nbar)) { ok = false; break; }

        for (int oi = 0; oi < a.nops && ok; oi++) {
            const BOpDesc op = ops[oi];
            const int T = op.m.ntiles, S = op.S;
            const int l = op.layer;
            if (!(ok = matvec(op))) break;
            if (op.kind == OP_QKV) {
                // q, k, v rows: RoPE on adjacent pairs (src/kernel_simd.c:1068-1085), KV append.
                bnorm_factors(a, s_ss, reinterpret_cast<float*>(xd));   // the slice's digits are used up
                const int nq = (a.q_dim + 2 * a.kv_dim) / 4, h2 = a.head_size / 2;
                const int nitems = a.nb * nq, gstride = gridDim.x * kThreads;
                auto rope_kv = [&](int i, float4 v) {
                    const int b = i / nq, row = 4 * (i - b * nq);
                    const float ss = s_ss[b];
                    v = make_float4(__fmul_rn(v.x, ss), __fmul_rn(v.y, ss), __fmul_rn(v.z, ss), __fmul_rn(v.w, ss));
                    const int pos = s_pos[b];
                    const size_t lkv = (size_t)b * a.kv_seq + (size_t)l * a.max_pos * a.kv_dim + (size_t)pos * a.kv_dim;
                    if (row < a.q_dim + a.kv_dim) {
                        const bool is_q = row < a.q_dim;
                        const int base = is_q ? row : row - a.q_dim;
                        const int hd = base % a.head_size;   // the quad's pairs: hd, hd + 2 in the same head
                        const float fr0 = __ldg(a.freq_re + (size_t)pos * h2 + hd / 2);
                        const float fi0 = __ldg(a.freq_im + (size_t)pos * h2 + hd / 2);
                        const float fr1 = __ldg(a.freq_re + (size_t)pos * h2 + hd / 2 + 1);
                        const float fi1 = __ldg(a.freq_im + (size_t)pos * h2 + hd / 2 + 1);
                        const float4 o = make_float4(__fsub_rn(__fmul_rn(v.x, fr0), __fmul_rn(v.y, fi0)),
                                                     __fadd_rn(__fmul_rn(v.x, fi0), __fmul_rn(v.y, fr0)),
                                                     __fsub_rn(__fmul_rn(v.z, fr1), __fmul_rn(v.w, fi1)),
                                                     __fadd_rn(__fmul_rn(v.z, fi1), __fmul_rn(v.w, fr1)));
                        float* dst = is_q ? a.q + (size_t)b * a.q_dim + base : a.kcache + lkv + base;
                        __stcg(reinterpret_cast<float4*>(dst), o);
                    } else {
                        __stcg(reinterpret_cast<float4*>(a.vcache + lkv + (row - a.q_dim - a.kv_dim)), v);
                    }
                };
                // Two items a pass: both items' partial sums are loaded before
                // either's stores, so their L2 round trips overlap.
                for (int i = blockIdx.x * kThreads + tid; i < nitems; i += 2 * gstride) {
                    const int j = i + gstride;
                    const int b0 = i / nq, b1 = j / nq;
                    const float4 v0 = bsum4(a.part, S, T, NB8, b0, 4 * (i - b0 * nq));
                    const float4 v1 = j < nitems ? bsum4(a.part, S, T, NB8, b1, 4 * (j - b1 * nq))
                                                 : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    rope_kv(i, v0);
                    if (j < nitems) rope_kv(j, v1);
                }
                if (!grid_barrier(a.step, nbar)) { ok = false; break; }
                if (csync_or(!battention(a, l, s_pos, xd, s_abar, aphase))) {
                    if (tid == 0) set_error(a.step, DEV_COPY_TIMEOUT);
                    ok = false;
                    break;
                }
                if (!grid_barrier(a.step, nbar)) { ok = false; break; }
            } else if (op.kind == OP_WO || op.kind == OP_W2) {
                // x += the op's sums; digits of x for the next op (W13 after
                // WO; the next layer's QKV, or the classifier, after W2).
                const float* nw = op.kind == OP_WO ? a.rms_ffn + (size_t)l * a.dim
                                  : (l + 1 < a.n_layers ? a.rms_att + (size_t)(l + 1) * a.dim : a.rms_final);
                // x += the op's sums (over the ranks' partials under tensor
                // parallelism, by exchange ++xcount).
                if (!bresidual<NBLK>(a, nw, s_sq, ++xcount,
                                     [&](int b, int row4) { return bsum4(a.part, S, T, NB8, b, row4); })) {
                    ok = false;
                    break;
                }
                if (!grid_barrier(a.step, nbar)) { ok = false; break; }
            } else if (op.kind == OP_W13) {
                // rows w1[2j], w1[2j+1], w3[2j], w3[2j+1]; SwiGLU (src/kernel_simd.c:836-841),
                // straight into the digits of W2's input.
                bnorm_factors(a, s_ss, reinterpret_cast<float*>(xd));   // the slice's digits are used up
                const int Gh = a.hidden / 32, total = Gh * NB8 * 8;
                for (int base = 0; base < total; base += gridDim.x * kThreads) {
                    const int i = base + blockIdx.x * kThreads + tid;
                    const int q = i & 7, rest = i >> 3, b = rest % NB8, g = rest / NB8;
                    float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    if (i < total && b < a.nb) {
                        const float ss = s_ss[b];
                        const int j0 = g * 32 + 4 * q;          // hidden units j0..j0+3: rows 2 j0 .. 2 j0 + 7
                        const float4 p0 = bsum4(a.part, S, T, NB8, b, 2 * j0);
                        const float4 p1 = bsum4(a.part, S, T, NB8, b, 2 * j0 + 4);
                        const float gv[4] = {p0.x, p0.y, p1.x, p1.y}, uv[4] = {p0.z, p0.w, p1.z, p1.w};
                        float hv[4];
#pragma unroll
                        for (int k = 0; k < 4; k++) {
                            const float gk = __fmul_rn(gv[k], ss), uk = __fmul_rn(uv[k], ss);
                            hv[k] = __fmul_rn(__fdiv_rn(gk, __fadd_rn(1.0f, expf_cr(-gk))), uk);
                        }
                        v = make_float4(hv[0], hv[1], hv[2], hv[3]);
                    }
                    const float m = group_max8(v);
                    if (i < total) bdigit_store<NBLK>(a.dg, g, b, q, v, m);
                }
                if (!grid_barrier(a.step, nbar)) { ok = false; break; }
            } else {   // OP_CLS
                bnorm_factors(a, s_ss, reinterpret_cast<float*>(xd));   // the slice's digits are used up
                const int G = gridDim.x, c = blockIdx.x, V4 = a.vocab_rows / 4;
                const int q0 = (int)((long long)c * V4 / G), q1 = (int)((long long)(c + 1) * V4 / G);
                for (int b = warp; b < a.nb; b += kWarps) {
                    const float ss = s_ss[b];
                    float best = -1e9f;
                    uint32_t bi = 0;
                    for (int qd = q0 + lane; qd < q1; qd += 32) {
                        const float4 s4 = bsum4(a.part, S, T, NB8, b, 4 * qd);
                        const float v[4] = {__fmul_rn(s4.x, ss), __fmul_rn(s4.y, ss), __fmul_rn(s4.z, ss),
                                            __fmul_rn(s4.w, ss)};
                        __stcg(reinterpret_cast<float4*>(a.logits + (size_t)b * a.vocab_rows + 4 * qd),
                               make_float4(v[0], v[1], v[2], v[3]));
#pragma unroll
                        for (int k = 0; k < 4; k++)
                            if (v[k] > best) {
                                best = v[k];
                                bi = (uint32_t)(a.vocab_off + 4 * qd + k);
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
                if (a.tp_n > 1) {
                    // The greedy token of each sequence is the largest of the ranks' keys.
                    if (blockIdx.x == 0 && tid < a.nb) {
                        const unsigned long long key = __ldcg(a.argmax + par * kBMaxSeq + tid);
                        for (int j = 0; j < a.tp_n; j++)
                            reinterpret_cast<unsigned long long*>(a.tp_peers[j] + a.tp_bkeys_off)[a.tp_rank * kBMaxSeq + tid] = key;
                        __threadfence_system();
                    }
                    if (!btp_exchange(a, nbar, ++xcount)) { ok = false; break; }
                    if (blockIdx.x == 0 && tid < a.nb) {
                        const unsigned long long* keys =
                            reinterpret_cast<const unsigned long long*>(a.tp_peers[a.tp_rank] + a.tp_bkeys_off);
                        unsigned long long m = 0;
                        for (int j = 0; j < a.tp_n; j++) {
                            const unsigned long long k = __ldcg(keys + j * kBMaxSeq + tid);
                            m = k > m ? k : m;
                        }
                        a.argmax[par * kBMaxSeq + tid] = m;
                        __threadfence();
                    }
                    if (!grid_barrier(a.step, nbar)) { ok = false; break; }
                }
                if (a.sampling) {
                    // CTA b draws sequence b's next token (stream b, its position)
                    // and leaves it in the key slot the next step reads.
                    for (int b = blockIdx.x; b < a.nb; b += gridDim.x) {
                        const float mx = key_value(__ldcg(a.argmax + par * kBMaxSeq + b));
                        const int t = sample_token(a.logits + (size_t)b * a.vocab_rows, a.vocab_rows, mx, a.samp,
                                                   (unsigned long long)b, (unsigned long long)s_pos[b],
                                                   reinterpret_cast<unsigned long long*>(xd));
                        if (tid == 0) a.argmax[par * kBMaxSeq + b] = argmax_key(0.0f, (uint32_t)t);
                    }
                    if (!grid_barrier(a.step, nbar)) { ok = false; break; }
                }
                if (step == a.steps - 1 && blockIdx.x == 0 && tid < a.nb)
                    a.tokens[(size_t)a.steps * a.nb + tid] = (int)key_index(__ldcg(a.argmax + par * kBMaxSeq + tid));
            }
        }
    }
    if (blockIdx.x == 0 && tid == 0) a.step->tp_count = xcount;
}

}  // namespace aion
