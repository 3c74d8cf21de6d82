// Streaming kernels: the persistent decode kernel and the standalone matvec.
//
// Persistent decode: `steps` greedy tokens of the int4 Llama-2 forward
// (src/kernel_simd.c:1014-1169 per token, :1223-1250 around it) in one
// cooperative launch, one CTA per SM.  Every weight matrix of a token is an
// "op"; the ops of all steps form one sequence.  Each warp streams its share
// of every op (see op_work) through its own ring of bulk copies, always P
// chunks ahead -- across op boundaries, grid barriers and tokens, since the
// weights never depend on the activations.  Between dependent ops the CTAs
// meet at a bounded grid barrier; the input of each op is rebuilt in shared
// memory as activation digits (matvec.cuh) with its fused prologue (RMSNorm,
// or the int4 embedding row).
//
// Per token (5 barriers per layer, 1 after the classifier):
//   [QKV: rmsnorm | q, k, v rows | RoPE, KV append]  barrier
//   [attention]  barrier
//   [wo: att | x += ]  barrier
//   [w1/w3: rmsnorm | SwiGLU -> hb]  barrier
//   [w2: hb | x += ]  barrier
//   ... [classifier: rmsnorm | logits, argmax key]  barrier (next token)
#pragma once

#include "matvec.cuh"
#include "sample.cuh"

namespace aion {

enum OpKind { OP_QKV = 0, OP_WO = 1, OP_W13 = 2, OP_W2 = 3, OP_CLS = 4, OP_STORE = 5 };

struct OpDesc {
    MatDesc m;
    int kind, layer;
};

constexpr int kMaxHead = 128;

// Inputs on which the host C library's expf differs from the correctly
// rounded e^x (see expf_host).
struct ExpTable {
    const uint32_t* x = nullptr;
    int n = 0;
    double delta = 0.0;
};

struct DecodeArgs {
    const OpDesc* ops;             // [nops]: QKV, WO, W13, W2 per layer, then CLS
    int nops;
    MatDesc emb;                   // tied embedding / classifier
    int dim, hidden, n_layers, n_heads, kv_mul, head_size, kv_dim, vocab, max_pos;
    const float *rms_att, *rms_ffn, *rms_final, *freq_re, *freq_im;
    float *x, *q, *att, *hb, *logits;
    float *kcache, *vcache;        // [L][max_pos][kv_dim]
    float* attn_part;              // [n_heads][max_chunks][head_size + 2]
    int* attn_cnt;                 // [n_heads], zero between uses
    int max_chunks;
    uint64_t* split_part;          // [max_tiles][16] tagged partial rows of tiles cut by CTA boundaries
    StepState* step;
    unsigned long long* argmax;
    int32_t* history;              // [max_pos]
    int steps;
    int P, slot_bytes, xbytes, xs_off;
    int ops_off;                   // shared-memory copy of ops[] (xbytes = ring offset)
    ExpTable exp_host;             // the host expf's deviations (W4A8), or empty
    int cr_exp;                    // SwiGLU's exp: 1 correctly rounded / host-table (W4A8, fp32), 0 CUDA expf (W4A16)
    SamplerParams samp;            // used when sampling != 0 (else the greedy argmax)
    int sampling;
    // Tensor parallelism over tp_n GPUs (tp_n == 1: off).  This rank holds
    // q_dim query rows (n_heads heads, kv_dim K/V rows), hidden FFN rows and
    // vocab rows [vocab_off, vocab_off + classifier rows); WO and W2 give
    // partial sums over its slice of their inputs.  tp_peers[j] is rank j's
    // exchange region (mapped into this process): recv u64 [2][tp_n][dim]
    // (partial rows tagged with the exchange count, slot count & 1), then
    // keys u64 [tp_n] at tp_keys_off, flags u32 [tp_n] at tp_flags_off.  A
    // rank rewrites a slot only after an exchange that needs this rank's
    // next partial rows, so no row is overwritten before it is read.
    int q_dim;
    int tp_n, tp_rank, vocab_off;
    unsigned long long wait_ns;    // bound of each wait on another rank (global timer ns)
    unsigned char* const* tp_peers;
    int tp_keys_off, tp_flags_off;
};

// ---------------------------------------------------------------------------
// Input sources of an op: an fp32 vector in global memory (written by other
// CTAs of this launch: read through L2), or the int4 embedding row of a
// token (src/kernel_simd.c:1032-1040: x[i] = (int8)(nibble - 8) * scale).
// ---------------------------------------------------------------------------
struct VecSrc {
    const float* p = nullptr;      // fp32 vector, or nullptr for the embedding row
    MatDesc emb;
    int tok = 0;
};

// Elements 4i..4i+3 of an fp32 tile row (the fp32 path's embedding row).
__device__ __forceinline__ float4 emb_load4_f32(const MatDesc& emb, int tok, int i) {
    const int g = i >> 3, e4 = i & 7;
    const int rr = tok % kTR, rl = rr & 7, half = rr >> 3;
    const int q = half * 2 + (e4 & 1), ln = 4 * rl + (e4 >> 1);
    const float* base = reinterpret_cast<const float*>(emb.w);
    return __ldg(reinterpret_cast<const float4*>(base + ((size_t)(tok / kTR) * emb.G + g) * 512 + (q * 32 + ln) * 4));
}

template <int MODE = MODE_W4A16>
__device__ __forceinline__ float4 src_load4(const VecSrc& s, int i) {
    if (s.p) return __ldcg(reinterpret_cast<const float4*>(s.p) + i);
    if (MODE == MODE_F32) return emb_load4_f32(s.emb, s.tok, i);
    // elements 4i..4i+3 of row tok: group g, elements k..k+3 of the group
    const int g = i >> 3, k = (i & 7) * 4;
    const long long R = s.tok;
    const int rr = (int)(R % kTR), lr = rr & 7, half = rr >> 3;
    const uint8_t* gp = s.emb.w + (R / kTR) * s.emb.tile_bytes + (size_t)g * kGB;
    const float sc = __ldg(reinterpret_cast<const float*>(gp + 256 + 8 * lr + 4 * half));
    // element e of the group: lane t = (e % 16) / 4, byte b = e % 4, high nibble if e >= 16
    const int t = (k & 15) >> 2;
    const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(gp + 8 * (4 * lr + t) + 4 * half));
    const int shift = k >= 16 ? 4 : 0;
    float4 v;
    v.x = (float)((int)((w >> shift) & 0xF) - 8) * sc;
    v.y = (float)((int)((w >> (8 + shift)) & 0xF) - 8) * sc;
    v.z = (float)((int)((w >> (16 + shift)) & 0xF) - 8) * sc;
    v.w = (float)((int)((w >> (24 + shift)) & 0xF) - 8) * sc;
    return v;
}

// e^x rounded once to float: the double-precision exponential rounded to
// the nearest float (CUDA exp() is accurate to < 1 double ulp, so only
// inputs within ~1e-16 relative of a float rounding boundary can differ
// from the correctly rounded value).
__device__ __forceinline__ float expf_cr(float x) { return (float)exp((double)x); }

// The host C library's expf, which the reference calls, is not correctly
// rounded: on a small set of inputs it returns the other float neighbour
// of e^x.  ExpTable lists those inputs (ascending bit patterns), found on
// the host by calling that expf on every float with a finite non-zero
// result; delta bounds how far (in result ulps) from a rounding midpoint
// e^x lies for any listed input.  expf_host() returns the correctly
// rounded value unless e^x is that close to a midpoint, and then looks the
// input up.  With no table it is expf_cr().
__device__ __forceinline__ float expf_host(float x, const ExpTable& t) {
    const double yd = exp((double)x);
    const float f = (float)yd;
    if (!t.x || !(f < INFINITY)) return f;
    const float other = (double)f < yd ? nextafterf(f, INFINITY) : nextafterf(f, 0.0f);
    const double mid = 0.5 * ((double)f + (double)other);
    const double ulp = fabs((double)other - (double)f);
    if (!(ulp > 0.0) || fabs(yd - mid) > t.delta * ulp) return f;
    const uint32_t key = __float_as_uint(x);
    int lo = 0, hi = t.n;
    while (lo < hi) {
        const int m = (lo + hi) >> 1;
        if (t.x[m] < key) lo = m + 1;
        else hi = m;
    }
    return (lo < t.n && t.x[lo] == key) ? other : f;
}

constexpr int kMaxVec = 10;       // float4 per thread of an op input: n <= 10 * 4 * kThreads
constexpr int kMaxNormVec = 4;    // float4 per thread of a normed input: dim <= 4 * 4 * kThreads

// Packs four signed values (the low bytes) into one word.
__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
    return (uint32_t)(a & 0xFF) | ((uint32_t)(b & 0xFF) << 8) | ((uint32_t)(c & 0xFF) << 16) | ((uint32_t)(d & 0xFF) << 24);
}

// Builds the activation digits of an op's input in one pass: thread j of
// the input holds float4 j (elements 4j..4j+3) in registers; the optional
// RMSNorm (src/kernel_simd.c:793-813: 1 / sqrtf(sum(x^2)/n + 1e-5), then
// (x * ss) * w) reduces over the CTA; the 8 threads of a 32-element group
// find its maximum with shuffles and each writes its own fragment words.
// W4A8 sums the squares in the reference's order (four lane sums of
// x[4m + l]^2, pairwise) from a copy of x staged in the digit area.
template <int MODE, int NV, bool NORM>
__device__ __forceinline__ void build_digits(unsigned char* xf, float* xs, const VecSrc& s, int n,
                                             const float* norm_w, float* red) {
    const int tid = threadIdx.x;
    const int nv = n / 4;
    float4 v[NV], w[NORM ? NV : 1];
    float norm_max = 0.0f;   // W4A16 with RMSNorm: max |input| from the fused reduction
#pragma unroll
    for (int i = 0; i < NV; i++) {
        const int j = tid + i * kThreads;
        v[i] = j < nv ? src_load4<MODE>(s, j) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (NORM) w[i] = j < nv ? __ldg(reinterpret_cast<const float4*>(norm_w) + j) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    if (NORM) {
        float ss;
        if (MODE == MODE_W4A8) {
            float4* stage = reinterpret_cast<float4*>(xf);
#pragma unroll
            for (int i = 0; i < NV; i++) {
                const int j = tid + i * kThreads;
                if (j < nv) stage[j] = v[i];
            }
            csync();
            if (tid < 4) {
                const float* sx = reinterpret_cast<const float*>(xf);
                float acc = 0.0f;
                for (int m = 0; m < nv; m++) {
                    const float e = sx[4 * m + tid];
                    acc = __fadd_rn(acc, __fmul_rn(e, e));
                }
                red[tid] = acc;
            }
            csync();
            const float sum = __fadd_rn(__fadd_rn(red[0], red[1]), __fadd_rn(red[2], red[3]));
            ss = 1.0f / sqrtf(__fdiv_rn(sum, (float)n) + 1e-5f);
            csync();
        } else if (MODE == MODE_W4A16) {
            // The sum of squares and max |x w| in one CTA exchange; max
            // |(x ss) w| is then max |x w| * ss to within two roundings, so
            // the exponent below is the exact one or one off, either way
            // with max |X| inside the four digits' range.
            float acc = 0.0f, mw = 0.0f;
#pragma unroll
            for (int i = 0; i < NV; i++) {
                acc += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
                mw = fmaxf(mw, fmaxf(fmaxf(fabsf(__fmul_rn(v[i].x, w[i].x)), fabsf(__fmul_rn(v[i].y, w[i].y))),
                                     fmaxf(fabsf(__fmul_rn(v[i].z, w[i].z)), fabsf(__fmul_rn(v[i].w, w[i].w)))));
            }
            const float2 r = block_sum_max(acc, mw, red);
            ss = 1.0f / sqrtf(__fdiv_rn(r.x, (float)n) + 1e-5f);
            norm_max = __fmul_rn(r.y, ss);
        } else {
            float acc = 0.0f;
#pragma unroll
            for (int i = 0; i < NV; i++) acc += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
            acc = block_sum(acc, red);
            ss = 1.0f / sqrtf(__fdiv_rn(acc, (float)n) + 1e-5f);
        }
#pragma unroll
        for (int i = 0; i < NV; i++) {
            v[i].x = __fmul_rn(__fmul_rn(v[i].x, ss), w[i].x);
            v[i].y = __fmul_rn(__fmul_rn(v[i].y, ss), w[i].y);
            v[i].z = __fmul_rn(__fmul_rn(v[i].z, ss), w[i].z);
            v[i].w = __fmul_rn(__fmul_rn(v[i].w, ss), w[i].w);
        }
    }
    if (MODE == MODE_F32) {
        // The fp32 path keeps the input as fp32, [G][32] in the digit area.
#pragma unroll
        for (int i = 0; i < NV; i++) {
            const int j = tid + i * kThreads;
            if (j < nv) reinterpret_cast<float4*>(xf)[j] = v[i];
        }
        return;
    }
    // W4A16: one exponent for the vector, from its largest magnitude M;
    // vectors with M < 2^-93 count as zero.
    int E = 0;
    bool live = false;
    float sa = 0.0f, sb = 0.0f;
    if (MODE == MODE_W4A16) {
        float mx = 0.0f;
        if (NORM) {
            mx = norm_max;
        } else {
#pragma unroll
            for (int i = 0; i < NV; i++)
                mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
            mx = block_max(mx, red);
        }
        const int ebits = (int)((__float_as_uint(mx) >> 23) & 0xFF);
        live = ebits >= 34;
        E = 156 - ebits;                                   // M * 2^E in [2^29, 2^30)
        sa = __int_as_float((127 + E / 2) << 23);
        sb = __int_as_float((127 + E - E / 2) << 23);
        if (tid == 0) xs[0] = live ? __int_as_float((127 - E - 4) << 23) : 0.0f;   // 2^-E / 16
    }
#pragma unroll
    for (int i = 0; i < NV; i++) {
        if (i * kThreads >= nv) break;                      // uniform across the CTA
        const int j = tid + i * kThreads;
        const bool valid = j < nv;                          // same for the 8 threads of a group
        const int g = j >> 3, q = j & 7;
        // element 4q + b sits in fragment lane t = q & 3, word (q >> 2)
        unsigned char* dst = xf + (size_t)g * kXF + (q & 3) * 8 + (q >> 2) * 4;
        const float e[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
        if (MODE == MODE_W4A16) {
            if (!valid) continue;
            // Balanced base-256 digits d0..d2 in [-128, 127] and d3: the bytes
            // of Z = (X + 0x808080) ^ 0x808080 are d0, d1, d2, d3 as signed
            // bytes (adding 128 per digit makes every digit a plain byte).
            // A 4x4 byte transpose then gives each digit column its word.
            uint32_t Z[4];
#pragma unroll
            for (int b = 0; b < 4; b++) {
                const int X = live ? __float2int_rn(__fmul_rn(__fmul_rn(e[b], sa), sb)) : 0;
                Z[b] = ((uint32_t)X + 0x808080u) ^ 0x808080u;
            }
            const uint32_t t0 = __byte_perm(Z[0], Z[1], 0x5140), t1 = __byte_perm(Z[0], Z[1], 0x7362);
            const uint32_t t2 = __byte_perm(Z[2], Z[3], 0x5140), t3 = __byte_perm(Z[2], Z[3], 0x7362);
            *reinterpret_cast<uint32_t*>(dst) = __byte_perm(t0, t2, 0x5410);
            *reinterpret_cast<uint32_t*>(dst + 32) = __byte_perm(t0, t2, 0x7632);
            *reinterpret_cast<uint32_t*>(dst + 64) = __byte_perm(t1, t3, 0x5410);
            *reinterpret_cast<uint32_t*>(dst + 96) = __byte_perm(t1, t3, 0x7632);
        } else {
            float m = fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w)));
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
            if (!valid) continue;
            // quantize_activations_neon (src/kernel_simd.c:186-227), bit-exact
            const bool big = m > 1e-9f;
            const float scale = big ? __fdiv_rn(127.0f, m) : 1.0f;
            int qv[4];
#pragma unroll
            for (int b = 0; b < 4; b++) qv[b] = (int)roundf(__fmul_rn(e[b], scale));
            *reinterpret_cast<uint32_t*>(dst) = pack4(qv[0], qv[1], qv[2], qv[3]);
            if (q == 0) xs[g] = big ? __fdiv_rn(m, 127.0f) : 1.0f;
        }
    }
}

// Norm inputs (the model dimension) take at most kMaxNormVec float4 per
// thread, with their RMSNorm weights loaded alongside; other inputs up to
// kMaxVec.
template <int MODE>
__device__ void build_input(unsigned char* xf, float* xs, const VecSrc& s, int n, const float* norm_w, float* red) {
    if (norm_w) build_digits<MODE, kMaxNormVec, true>(xf, xs, s, n, norm_w, red);
    else build_digits<MODE, kMaxVec, false>(xf, xs, s, n, nullptr, red);
}

// ---------------------------------------------------------------------------
// Producer position of a warp in the sequence of (step, op) chunk streams.
// ---------------------------------------------------------------------------
struct Seq {
    int step, op;                  // op == nops: end of the sequence
    OpWork w;
    OpCursor cu;
    MatDesc m;                     // copy of ops[op].m, kept in registers
};

__device__ __forceinline__ void seq_enter(Seq& s, const OpDesc* ops, int nops, int steps, int mode, int step, int op,
                                          int warp) {
    while (step < steps) {
        while (op < nops) {
            s.m = ops[op].m;
            s.w = op_work(s.m, mode);
            if (cursor_begin(s.cu, s.w, s.m, warp)) {
                s.step = step;
                s.op = op;
                return;
            }
            op++;
        }
        op = 0;
        step++;
    }
    s.step = steps;
    s.op = nops;
}

__device__ __forceinline__ void seq_issue_next(Seq& s, Ring& r, const OpDesc* ops, int nops, int steps, int mode) {
    if (s.step >= steps) return;
    int bytes;
    const uint8_t* src = chunk_src(s.m, s.cu.tile, s.cu.c, bytes);
    ring_issue(r, src, bytes);
    if (!cursor_next(s.cu, s.w, s.m)) seq_enter(s, ops, nops, steps, mode, s.step, s.op + 1, threadIdx.x >> 5);
}

// ---------------------------------------------------------------------------
// One op on this CTA: consume its chunks from the rings, reduce, combine the
// tiles cut by CTA boundaries, and hand every finished quad of rows to
// `epi(first_row, values[4])`.  Returns false if a wait gave up.
// ---------------------------------------------------------------------------
struct OpSmem {
    uint64_t cutw[kTR];                          // split: the partner's tagged words of the last cut tile, fetched early
    float part[kMaxLocalTiles * kWarps * kTR];   // split: warp partials per local tile
    float pre[kMaxLocalTiles * kTR];             // split: epilogue operands fetched ahead
    int state[2];
    int done;                                    // split: warps that have left the op's loop
};

// Split mode, a CTA whose range starts inside tile tf (it holds the
// tile's second part): every warp with units in tf arrives once it has
// left the tile, and the last of the n0 such warps sums the warps' partial
// rows (in warp order, as the full reduction does) and publishes them as
// 16 tagged 8-byte words (fp32 bits, the op's tag): one relaxed store each,
// read whole, so no fence or flag is needed.  The partner CTA thus finds
// the part as soon as this CTA's first tile is done, not after its op.
__device__ __forceinline__ void publish_cut_tile(OpSmem& os, int n0, int tf, uint64_t* split_part, uint32_t tag) {
    const int lane = threadIdx.x & 31;
    __threadfence_block();
    __syncwarp();
    int last = 0;
    if (lane == 0) last = atomicAdd(&os.state[1], 1) == n0 - 1;
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) return;
    __threadfence_block();
    if (lane < kTR) {
        float v = 0.0f;
        for (int k = 0; k < kWarps; k++) v += os.part[k * kTR + lane];
        st_relaxed_u64(split_part + (size_t)tf * kTR + lane, tag_pack(v, tag));
    }
}

// Clears the per-op shared state for the next op: run_op needs OpSmem::part
// zero and the counters reset on entry (kernels call this before their
// first op; run_op calls it on its way out).
__device__ __forceinline__ void reset_opsmem(OpSmem& os) {
    for (int i = threadIdx.x; i < kMaxLocalTiles * kWarps * kTR; i += kThreads) os.part[i] = 0.0f;
    if (threadIdx.x == 0) os.state[0] = os.state[1] = os.done = 0;
}

template <int MODE, bool PROD, class Epi>
__device__ bool run_op(const MatDesc& m, Ring& ring, unsigned char* ring_base, Seq& seq, const OpDesc* ops, int nops,
                       int steps, const unsigned char* xf, const float* xs, OpSmem& os, uint64_t* split_part,
                       uint32_t tag, Epi& epi, int pstep = 1 << 30, int pop = 0) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const float xfac = MODE == MODE_W4A16 ? xs[0] : 0.0f;
    const OpWork w = op_work(m, MODE);
    bool ok = true;
    OpCursor cu;
    bool more = cursor_begin(cu, w, m, warp);
    if (w.split) {
        const int tf = w.u0 / m.nch, tl = (w.u1 - 1) / m.nch, ntl = tl - tf + 1;
        const bool cut0 = (w.u0 % m.nch) != 0, cut1 = (w.u1 % m.nch) != 0;
        const int n0 = min(kWarps, min((tf + 1) * m.nch, w.u1) - w.u0);   // warps with units in tile tf
        // OpSmem was reset at the end of the previous op (or at kernel
        // start) and a CTA barrier has passed since, so no barrier here.
        epi.prefetch(tf * kTR, ntl * kTR, os.pre);
        float a0 = 0.0f, a1 = 0.0f;
        int cur = -1;
#ifdef AION_PHASE_TIMING
        unsigned long long tw_ = 0, tm_ = 0, nc_ = 0;
        PHASE_LOOP_START(pstep, pop);
#endif
        while (more) {
            const int tile = cu.tile, c = cu.c;
            if (tile != cur) {
                if (cur >= 0) {
                    quad_reduce<MODE>(a0, a1, xfac);
                    if ((lane & 3) == 0) {
                        float* p = os.part + ((cur - tf) * kWarps + warp) * kTR;
                        p[lane >> 2] = a0;
                        p[(lane >> 2) + 8] = a1;
                    }
                    if (cut0 && cur == tf) publish_cut_tile(os, n0, tf, split_part, tag);
                }
                a0 = a1 = 0.0f;
                cur = tile;
            }
#ifdef AION_PHASE_LOOP
            const unsigned long long q0_ = global_timer();
#endif
            const unsigned char* ch = ring_wait(ring, ring_base);
            if (!ch) { ok = false; break; }
#ifdef AION_PHASE_LOOP
            const unsigned long long q1_ = global_timer();
#endif
            const int g0 = chunk_g0(m, c), g1 = chunk_g0(m, c + 1);
            chunk_mma<MODE>(ch, g1 - g0, g0, xf, xs, a0, a1);
            __syncwarp();
#ifdef AION_PHASE_LOOP
            tw_ += q1_ - q0_;
            tm_ += global_timer() - q1_;
            nc_++;
#endif
            if (PROD) {
                ring_release(ring, true);
            } else {
                ring_release(ring);
                seq_issue_next(seq, ring, ops, nops, steps, MODE);
            }
            more = cursor_next(cu, w, m);
        }
#ifdef AION_PHASE_TIMING
        PHASE_W(pstep, pop, tw_, tm_, nc_);
#endif
        if (ok && cur >= 0) {
            quad_reduce<MODE>(a0, a1, xfac);
            if ((lane & 3) == 0) {
                float* p = os.part + ((cur - tf) * kWarps + warp) * kTR;
                p[lane >> 2] = a0;
                p[(lane >> 2) + 8] = a1;
            }
            if (cut0 && cur == tf) publish_cut_tile(os, n0, tf, split_part, tag);
        }
        if (ok && cut1) {
            // The first warp out of the loop fetches the partner's tagged
            // words of the last tile (published once the partner's warps
            // left that tile, long before) while the other warps compute,
            // so the epilogue seldom waits for them.
            int first = 0;
            if (lane == 0) first = atomicAdd(&os.done, 1) == 0;
            first = __shfl_sync(0xffffffffu, first, 0);
            if (first && lane < kTR) os.cutw[lane] = ld_relaxed_u64(split_part + (size_t)tl * kTR + lane);
        }
        cp_async_wait_all();
        if (csync_or(!ok)) return false;
        PHASE_T(pstep, pop, 2);
        PHASE_T(pstep, pop, 7);
        // The CTA's tiles are finished by quads of rows, one quad a thread:
        // the thread sums the warps' partials of its rows in warp order
        // (clearing them for the next op as it reads them), adds the
        // partner's part when the CTA boundary cuts the tile, and runs the
        // epilogue.  Tiles cut by a CTA boundary: local tile 0 when u0 is
        // inside a tile (this CTA has the tile's second part, published as
        // soon as its warps left the tile; the partner finishes the tile),
        // the last local tile when u1 is (this CTA has the first part: it
        // waits, bounded, for the partner's tagged words and adds first +
        // second in that order).  Publishing never waits, so the waits end.
        bool bad = false;
        for (int i = tid; i < ntl * (kTR / kRB); i += kThreads) {
            const int lt = i / (kTR / kRB), q = i % (kTR / kRB);
            float* p = os.part + lt * kWarps * kTR + q * kRB;
            if (lt == 0 && cut0) {
                for (int k = 0; k < kWarps; k++)
#pragma unroll
                    for (int r = 0; r < kRB; r++) p[k * kTR + r] = 0.0f;
                continue;
            }
            const bool cutq = cut1 && lt == ntl - 1;
            const uint64_t* cut_src = split_part + (size_t)tl * kTR + q * kRB;
            uint64_t w[kRB];
#pragma unroll
            for (int r = 0; r < kRB; r++) {
                // fetched as the first warp left the loop; if it was not this
                // op's yet, fetch again now, so the load overlaps the sums
                w[r] = cutq ? os.cutw[q * kRB + r] : 0ull;
                if (cutq && tag_ep(w[r]) != tag) w[r] = ld_relaxed_u64(cut_src + r);
            }
            float v[kRB];
#pragma unroll
            for (int r = 0; r < kRB; r++) v[r] = 0.0f;
            for (int k = 0; k < kWarps; k++)
#pragma unroll
                for (int r = 0; r < kRB; r++) {
                    v[r] += p[k * kTR + r];
                    p[k * kTR + r] = 0.0f;
                }
            if (cutq) {
#pragma unroll
                for (int r = 0; r < kRB; r++) {
                    uint32_t spins = 0;
                    while (tag_ep(w[r]) != tag && ++spins <= (1u << 22)) w[r] = ld_relaxed_u64(cut_src + r);
                    if (tag_ep(w[r]) == tag) v[r] = v[r] + tag_val(w[r]);
                    else bad = true;
                }
            }
            epi((tf + lt) * kTR + q * kRB, v);
        }
        if (cut1 && csync_or(bad)) return false;
        if (tid == 0) os.state[0] = os.state[1] = os.done = 0;
        PHASE_T(pstep, pop, 8);
    } else {
        float a0 = 0.0f, a1 = 0.0f;
        float* stage = os.part + warp * kTR;
        while (more) {
            const int tile = cu.tile, c = cu.c;
            const unsigned char* ch = ring_wait(ring, ring_base);
            if (!ch) { ok = false; break; }
            const int g0 = chunk_g0(m, c), g1 = chunk_g0(m, c + 1);
            chunk_mma<MODE>(ch, g1 - g0, g0, xf, xs, a0, a1);
            __syncwarp();
            if (PROD) {
                ring_release(ring, true);
            } else {
                ring_release(ring);
                seq_issue_next(seq, ring, ops, nops, steps, MODE);
            }
            if (c == m.nch - 1) {
                quad_reduce<MODE>(a0, a1, xfac);
                if ((lane & 3) == 0) {
                    stage[lane >> 2] = a0;
                    stage[(lane >> 2) + 8] = a1;
                }
                __syncwarp();
                if (lane < kTR / kRB) epi(tile * kTR + lane * kRB, stage + lane * kRB);
                __syncwarp();
                a0 = a1 = 0.0f;
            }
            more = cursor_next(cu, w, m);
        }
        if (csync_or(!ok)) return false;
        for (int i = tid; i < kWarps * kTR; i += kThreads) os.part[i] = 0.0f;   // the warps' stages
    }
    return true;
}

// ---------------------------------------------------------------------------
// Epilogue of the decode ops, per quad of rows.
// ---------------------------------------------------------------------------
struct DecodeEpi {
    const DecodeArgs* a;
    const OpDesc* op;
    int pos;
    const float* freq;             // shared: this position's RoPE cos[hs/2], sin[hs/2]
    float best;
    uint32_t best_i;
    uint32_t xcount = 0;           // tensor parallelism: the tag of this op's partial rows
    const float* pre = nullptr;    // shared: residual rows [pre_row0, ...) fetched ahead
    int pre_row0 = 0;

    // Split mode: rows [row0, row0 + rows) end on this CTA; WO / W2 fetch
    // their residual rows into shared memory while the op streams.
    __device__ __forceinline__ void prefetch(int row0, int rows, float* dst) {
        if ((op->kind != OP_WO && op->kind != OP_W2) || a->tp_n > 1) return;
        const int tid = threadIdx.x;
        if (4 * tid < rows) cp_async16(dst + 4 * tid, a->x + row0 + 4 * tid);
        pre = dst;
        pre_row0 = row0;
    }

    __device__ __forceinline__ void operator()(int r0, const float* v) {
        const DecodeArgs& A = *a;
        const int d = op->m.d;
        switch (op->kind) {
        case OP_QKV: {
            if (r0 >= d) break;
            const int hs = A.head_size;
            const size_t lkv = (size_t)op->layer * A.max_pos * A.kv_dim;
            if (r0 < A.q_dim + A.kv_dim) {
                // RoPE on adjacent pairs (src/kernel_simd.c:1068-1085)
                const bool is_q = r0 < A.q_dim;
                const int base = is_q ? r0 : r0 - A.q_dim;
                float out[kRB];
                for (int r = 0; r < kRB; r += 2) {
                    const int hd = (base + r) % hs;
                    const float fr = freq[hd / 2];
                    const float fi = freq[hs / 2 + hd / 2];
                    out[r] = __fsub_rn(__fmul_rn(v[r], fr), __fmul_rn(v[r + 1], fi));
                    out[r + 1] = __fadd_rn(__fmul_rn(v[r], fi), __fmul_rn(v[r + 1], fr));
                }
                float* dst = is_q ? A.q + base : A.kcache + lkv + (size_t)pos * A.kv_dim + base;
                __stcg(reinterpret_cast<float4*>(dst), make_float4(out[0], out[1], out[2], out[3]));
            } else {
                const int base = r0 - A.q_dim - A.kv_dim;
                __stcg(reinterpret_cast<float4*>(A.vcache + lkv + (size_t)pos * A.kv_dim + base),
                       make_float4(v[0], v[1], v[2], v[3]));
            }
            break;
        }
        case OP_WO:
        case OP_W2:
            if (A.tp_n > 1) {
                // Partial sums over this rank's slice of the input, tagged
                // with the exchange count: into slot tp_rank of every rank's
                // receive rows (one 8-byte store each, read whole).
                for (int j = 0; j < A.tp_n; j++) {
                    uint64_t* recv = reinterpret_cast<uint64_t*>(A.tp_peers[j]) +
                                     ((size_t)(xcount & 1u) * A.tp_n + A.tp_rank) * A.dim;
                    for (int r = 0; r < kRB; r++)
                        if (r0 + r < d) st_relaxed_sys_u64(recv + r0 + r, tag_pack(v[r], xcount));
                }
                break;
            }
            for (int r = 0; r < kRB; r++)
                if (r0 + r < d) {
                    const float xr = pre ? pre[r0 + r - pre_row0] : __ldcg(A.x + r0 + r);
                    __stcg(A.x + r0 + r, xr + v[r]);
                }
            break;
        case OP_W13: {
            // rows w1[2j], w1[2j+1], w3[2j], w3[2j+1]; swiglu (src/kernel_simd.c:836-841)
            const int h0 = r0 / 2;
            for (int r = 0; r < 2; r++)
                if (h0 + r < A.hidden) {
                    const float g = v[r];
                    const float e = A.cr_exp ? expf_host(-g, A.exp_host) : expf(-g);
                    const float s = __fdiv_rn(g, __fadd_rn(1.0f, e));
                    __stcg(A.hb + h0 + r, __fmul_rn(s, v[2 + r]));
                }
            break;
        }
        default:  // OP_CLS
            for (int r = 0; r < kRB; r++)
                if (r0 + r < d) {
                    __stcg(A.logits + r0 + r, v[r]);
                    if (v[r] > best) {
                        best = v[r];
                        best_i = (uint32_t)(A.vocab_off + r0 + r);
                    }
                }
            break;
        }
    }
};

// ---------------------------------------------------------------------------
// Attention of one layer, split into warp units: unit (head h, chunk k)
// covers positions [16k, 16k+16) ∩ [0, pos], one warp each, spread over every
// warp of the grid.  Scores (q . k_t) / sqrtf(head_size) (src/kernel_simd.c:
// 1099-1117), local max, e^(s - max), their sum and the weighted V sum; with
// a single chunk the warp writes att[h] directly, otherwise it writes a
// partial and the last warp to finish a head merges the partials in chunk
// order.  Unit u runs on CTA u mod G, warp u div G, so short contexts put one
// unit on each SM.  q and the unit's K rows are loaded into registers (4
// lanes per position, a quarter of the head each, 8 positions per pass); its
// V rows (4 consecutive elements of the head per lane) go by asynchronous
// copies into the warp's slice of the idle activation-digit buffer, issued
// with the K loads, so the unit makes one trip to memory (a warp whose slice
// does not fit loads V after the scores instead).  Lane p of the warp takes
// position p's score, scaling and exponential; the sum of the exponentials
// and the weighted V sum run over the positions in order, in every lane.
// Partial layout per (head, chunk): [max, sum, -, -, o[0..hs)].
// ---------------------------------------------------------------------------
constexpr int kAttnUnit = 16;
constexpr int kQ4 = kMaxHead / 16;     // float4 of K per lane per position

// One attention unit on one warp: scores of positions [t0, t0 + n) of
// head h against q, their max m, l = sum of e^(s - m), and o = sum of
// e^(s - m) v_t (4 head elements per lane: 4 * lane .. + 3, when vl).
struct AttnPart {
    float m, l;
    float4 o;
};

__device__ __forceinline__ AttnPart attn_unit(const DecodeArgs& a, const float* kc, const float* vc, int h, int t0, int n,
                                              float4* vstage) {
    const int hs = a.head_size, lane = threadIdx.x & 31;
    const int hq = hs / 4, sub = lane & 3, pg = lane >> 2;
    const int kvh = h / a.kv_mul;
    const float rs = sqrtf((float)hs);
    const bool vl = 4 * lane < hs;
    const float4 z4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const float* vr = vc + (size_t)t0 * a.kv_dim + kvh * hs + 4 * lane;
    if (vstage && vl)
        for (int p = 0; p < n; p++) cp_async16(vstage + p * 32 + lane, vr + (size_t)p * a.kv_dim);
    const float* qp = a.q + h * hs + sub * hq;
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
    // Lane p (and p + 16) takes position p: quad p % 8 holds its dot, in d0
    // for p < 8, in d1 above.
    const int pl = lane & 15;
    const float s0 = __shfl_sync(0xffffffffu, d0, (pl & 7) * 4), s1 = __shfl_sync(0xffffffffu, d1, (pl & 7) * 4);
    const float sc = pl < n ? __fdiv_rn(pl < 8 ? s0 : s1, rs) : -INFINITY;
    float m = sc;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float e = pl < n ? expf(sc - m) : 0.0f;
    float4 vv[kAttnUnit];
    if (vstage) {
        cp_async_wait_all();
        __syncwarp();
#pragma unroll
        for (int p = 0; p < kAttnUnit; p++) vv[p] = (p < n && vl) ? vstage[p * 32 + lane] : z4;
    } else {
#pragma unroll
        for (int p = 0; p < kAttnUnit; p++)
            vv[p] = (p < n && vl) ? __ldcg(reinterpret_cast<const float4*>(vr + (size_t)p * a.kv_dim)) : z4;
    }
    float l = 0.0f;
    float4 o = z4;
#pragma unroll
    for (int p = 0; p < kAttnUnit; p++) {
        const float w = __shfl_sync(0xffffffffu, e, p);
        l += w;
        o.x = fmaf(w, vv[p].x, o.x);
        o.y = fmaf(w, vv[p].y, o.y);
        o.z = fmaf(w, vv[p].z, o.z);
        o.w = fmaf(w, vv[p].w, o.w);
    }
    return AttnPart{m, l, o};
}

// Merges nch partials laid out [m, l, -, -, o[0..hs)] at stride pstride
// (chunk order; read through `ld`) into att[h]: the warp's lanes hold 32
// chunks' max and sum per pass; the o partials of kMergeBatch chunks are
// loaded before any of them is folded in (chunk order kept), so a merge
// of many chunks pays one memory round trip per batch, not per chunk.
constexpr int kMergeBatch = 8;
template <class Ld>
__device__ __forceinline__ void attn_merge(const DecodeArgs& a, int h, const float* ph, int nch, int pstride, Ld ld) {
    const int hs = a.head_size, lane = threadIdx.x & 31;
    const bool vl = 4 * lane < hs;
    float M = -INFINITY;
    for (int c0 = 0; c0 < nch; c0 += 32)
        if (c0 + lane < nch) M = fmaxf(M, ld(ph + (size_t)(c0 + lane) * pstride));
    M = warp_max(M);
    float L = 0.0f;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int c0 = 0; c0 < nch; c0 += 32) {
        const int cn = min(32, nch - c0);
        float wl = 0.0f, ll = 0.0f;
        if (lane < cn) {
            wl = expf(ld(ph + (size_t)(c0 + lane) * pstride) - M);
            ll = ld(ph + (size_t)(c0 + lane) * pstride + 1);
        }
        for (int cb = 0; cb < cn; cb += kMergeBatch) {
            float4 ov[kMergeBatch];
#pragma unroll
            for (int u = 0; u < kMergeBatch; u++) {
                ov[u] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (vl && cb + u < cn) {
                    const float* oc = ph + (size_t)(c0 + cb + u) * pstride + 4 + 4 * lane;
                    ov[u] = make_float4(ld(oc), ld(oc + 1), ld(oc + 2), ld(oc + 3));
                }
            }
#pragma unroll
            for (int u = 0; u < kMergeBatch; u++) {
                const int c = cb + u;
                const float wgt = __shfl_sync(0xffffffffu, wl, c & 31);
                const float lc = __shfl_sync(0xffffffffu, ll, c & 31);
                if (c < cn) {
                    L = fmaf(lc, wgt, L);
                    if (vl) {
                        acc.x = fmaf(ov[u].x, wgt, acc.x);
                        acc.y = fmaf(ov[u].y, wgt, acc.y);
                        acc.z = fmaf(ov[u].z, wgt, acc.z);
                        acc.w = fmaf(ov[u].w, wgt, acc.w);
                    }
                }
            }
        }
    }
    const float inv = 1.0f / L;
    if (vl) __stcg(reinterpret_cast<float4*>(a.att + h * hs + 4 * lane),
                   make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv));
}

// Asks L2 for the K and V rows [0, pos) of a layer (written by earlier
// steps, evicted by the weight stream since): spread over every compute
// thread of the grid, issued when the layer's QKV op starts so that its
// attention finds them in L2 instead of paying HBM latency under load.
__device__ __forceinline__ void prefetch_kv_l2(const DecodeArgs& a, int layer, int pos) {
    const size_t lkv = (size_t)layer * a.max_pos * a.kv_dim;
    const size_t bytes = (size_t)pos * a.kv_dim * 4;   // rows [0, pos) are contiguous
    const size_t lines = (bytes + 127) / 128;
    const char* kb = reinterpret_cast<const char*>(a.kcache + lkv);
    const char* vb = reinterpret_cast<const char*>(a.vcache + lkv);
    for (size_t i = (size_t)blockIdx.x * kThreads + threadIdx.x; i < lines; i += (size_t)gridDim.x * kThreads) {
        asm volatile("prefetch.global.L2 [%0];" ::"l"(kb + 128 * i));
        asm volatile("prefetch.global.L2 [%0];" ::"l"(vb + 128 * i));
    }
}

// Attention of one layer (src/kernel_simd.c:1099-1117, softmax :816-826),
// split into warp units: unit (head h, chunk k) covers positions [16k,
// 16k+16) ∩ [0, pos], one warp each, spread over every warp of the grid
// (unit u on CTA u mod G, warp u div G).  With a single chunk the warp
// writes att[h] directly; otherwise it writes a partial and the last warp
// of a head (atomic count) merges the partials in chunk order.
// `stage`: the activation-digit buffer (stage_bytes), idle between the QKV
// op and the WO op's input build; warp w stages V in bytes
// [w, w + 1) * kAttnUnit * 512 of it when they fit.
// `scratch`: zeroed shared memory (the op's warp partials, idle between
// ops) of scratch_floats; a head with 2..kWarps units runs them on warps
// 0..nch-1 of one CTA and merges their partials there, in chunk order, with
// no global round trips; the slots are zeroed again afterwards.
__device__ void attention_layer(const DecodeArgs& a, int layer, int pos, unsigned char* stage, int stage_bytes,
                                float* scratch, int scratch_floats) {
    const int hs = a.head_size, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int kStage = kAttnUnit * 32 * 16;   // bytes of V per warp
    float4* vstage = (warp + 1) * kStage <= stage_bytes ? reinterpret_cast<float4*>(stage + warp * kStage) : nullptr;
    const int nch = pos / kAttnUnit + 1;
    const size_t lkv = (size_t)layer * a.max_pos * a.kv_dim;
    const float* kc = a.kcache + lkv;
    const float* vc = a.vcache + lkv;
    const int pstride = hs + 4;
    const bool vl = 4 * lane < hs;
    if (nch >= 2 && nch <= kWarps && nch * pstride <= scratch_floats) {
        for (int h = blockIdx.x; h < a.n_heads; h += gridDim.x) {   // uniform in the CTA
            if (warp < nch) {
                const int t0 = warp * kAttnUnit, n = min(kAttnUnit, pos + 1 - t0);
                const AttnPart p = attn_unit(a, kc, vc, h, t0, n, vstage);
                float* sp = scratch + warp * pstride;
                if (vl) *reinterpret_cast<float4*>(sp + 4 + 4 * lane) = p.o;
                if (lane == 0) {
                    sp[0] = p.m;
                    sp[1] = p.l;
                }
            }
            csync();
            if (warp == 0) {
                attn_merge(a, h, scratch, nch, pstride, [](const float* x) { return *x; });
                __syncwarp();
                for (int i = lane; i < nch * pstride; i += 32) scratch[i] = 0.0f;
            }
            csync();
        }
        return;
    }
    const int units = a.n_heads * nch;
    const int nw = gridDim.x * kWarps;
    for (int u = warp * gridDim.x + blockIdx.x; u < units; u += nw) {
        const int h = u / nch, k = u - (u / nch) * nch;
        const int t0 = k * kAttnUnit, n = min(kAttnUnit, pos + 1 - t0);
        const AttnPart p = attn_unit(a, kc, vc, h, t0, n, vstage);
        if (nch == 1) {
            const float inv = 1.0f / p.l;
            if (vl) __stcg(reinterpret_cast<float4*>(a.att + h * hs + 4 * lane),
                           make_float4(p.o.x * inv, p.o.y * inv, p.o.z * inv, p.o.w * inv));
            continue;
        }
        float* part = a.attn_part + ((size_t)h * a.max_chunks + k) * pstride;
        if (vl) __stcg(reinterpret_cast<float4*>(part + 4 + 4 * lane), p.o);
        if (lane == 0) {
            __stcg(part, p.m);
            __stcg(part + 1, p.l);
        }
        __threadfence();
        __syncwarp();
        int last = 0;
        if (lane == 0) last = atomicAdd(a.attn_cnt + h, 1) == nch - 1;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (!last) continue;
        __threadfence();
        attn_merge(a, h, a.attn_part + (size_t)h * a.max_chunks * pstride, nch, pstride,
                   [](const float* x) { return __ldcg(x); });
        if (lane == 0) a.attn_cnt[h] = 0;
    }
}

// Attention of one layer in the reference's own order (src/kernel_simd.c:
// 1099-1117, softmax :816-826), one CTA per head: score_t = (sum_j q_j k_j
// sequentially) / sqrtf(head_size); max; e_t = e^(score_t - max); sum of e_t
// sequentially; a_t = e_t * (1 / sum); out_j = sum_t a_t v_t[j] sequentially.
// `sc` holds max_pos floats of shared memory.
__device__ void attention_layer_exact(const DecodeArgs& a, int layer, int pos, float* sc, float* red) {
    const int hs = a.head_size, tid = threadIdx.x;
    const size_t lkv = (size_t)layer * a.max_pos * a.kv_dim;
    const float* kc = a.kcache + lkv;
    const float* vc = a.vcache + lkv;
    const float rs = sqrtf((float)hs);
    __shared__ float s_q[kMaxHead];
    __shared__ float s_sum;
    for (int h = blockIdx.x; h < a.n_heads; h += gridDim.x) {
        const int kvh = h / a.kv_mul;
        for (int i = tid; i < hs; i += kThreads) s_q[i] = __ldcg(a.q + h * hs + i);
        csync();
        float m = -INFINITY;
        for (int t = tid; t <= pos; t += kThreads) {
            const float* kr = kc + (size_t)t * a.kv_dim + kvh * hs;
            float d = 0.0f;
            // 32 elements of the row are loaded before they are summed in
            // order (hs is a multiple of 16: one or more full batches of 16).
            for (int j0 = 0; j0 < hs; j0 += 32) {
                float4 kv[8];
#pragma unroll
                for (int u = 0; u < 8; u++)
                    kv[u] = j0 + 4 * u < hs ? __ldcg(reinterpret_cast<const float4*>(kr + j0 + 4 * u))
                                            : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    const int j = j0 + 4 * u;
                    if (j < hs) {
                        d = __fadd_rn(d, __fmul_rn(s_q[j], kv[u].x));
                        d = __fadd_rn(d, __fmul_rn(s_q[j + 1], kv[u].y));
                        d = __fadd_rn(d, __fmul_rn(s_q[j + 2], kv[u].z));
                        d = __fadd_rn(d, __fmul_rn(s_q[j + 3], kv[u].w));
                    }
                }
            }
            d = __fdiv_rn(d, rs);
            sc[t] = d;
            m = fmaxf(m, d);
        }
        m = block_max(m, red);
        for (int t = tid; t <= pos; t += kThreads) sc[t] = expf_host(__fsub_rn(sc[t], m), a.exp_host);
        csync();
        if (tid == 0) {
            float sum = 0.0f;
            for (int t = 0; t <= pos; t++) sum = __fadd_rn(sum, sc[t]);
            s_sum = sum;
        }
        csync();
        const float scale = __fdiv_rn(1.0f, s_sum);
        for (int t = tid; t <= pos; t += kThreads) sc[t] = __fmul_rn(sc[t], scale);
        csync();
        for (int j = tid; j < hs; j += kThreads) {
            // 16 positions' V elements are loaded before they are summed in order.
            const float* vj = vc + kvh * hs + j;
            float o = 0.0f;
            int t = 0;
            for (; t + 16 <= pos + 1; t += 16) {
                float v[16];
#pragma unroll
                for (int u = 0; u < 16; u++) v[u] = __ldcg(vj + (size_t)(t + u) * a.kv_dim);
#pragma unroll
                for (int u = 0; u < 16; u++) o = __fadd_rn(o, __fmul_rn(sc[t + u], v[u]));
            }
            for (; t <= pos; t++) o = __fadd_rn(o, __fmul_rn(sc[t], __ldcg(vj + (size_t)t * a.kv_dim)));
            __stcg(a.att + h * hs + j, o);
        }
        csync();
    }
}

// Sets the next step's position and/or forced token (negative: keep).
__global__ void k_set_step(StepState* s, int pos, int token) {
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        if (pos >= 0) s->pos_next = pos;
        if (token >= 0) s->forced_token = token;
    }
}

// Largest key of the CTA's threads -> one atomicMax.
__device__ __forceinline__ void cta_argmax(unsigned long long* dst, float best, uint32_t best_i, unsigned long long* red64) {
    unsigned long long k = best > -1e9f ? argmax_key(best, best_i) : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, k, o);
        k = other > k ? other : k;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red64[warp] = k;
    csync();
    if (threadIdx.x == 0) {
        unsigned long long m = 0;
        for (int i = 0; i < kWarps; i++) m = red64[i] > m ? red64[i] : m;
        if (m) atomicMax(dst, m);
    }
    csync();
}

// ---------------------------------------------------------------------------
// Tensor parallelism: the exchange after WO, W2 and the classifier.  Every
// thread makes its remote stores of the op visible system-wide, the CTAs
// meet at a grid barrier, CTA 0 raises this rank's flag to `count` in every
// rank's region, and each CTA waits (bounded) until every rank's flag in its
// own region reached `count`.
// ---------------------------------------------------------------------------
// The threads that stored to peers fence those stores (system scope) right
// after them; the flags are polled with plain volatile loads and one
// system-scope fence follows the last one.
__device__ bool tp_exchange(const DecodeArgs& a, uint32_t& nbar, uint32_t count) {
    __shared__ int s_xok;
    if (!grid_barrier(a.step, nbar)) return false;
    if (threadIdx.x == 0) {
        if (blockIdx.x == 0)
            for (int j = 0; j < a.tp_n; j++)
                st_release_sys_u32(reinterpret_cast<uint32_t*>(a.tp_peers[j] + a.tp_flags_off) + a.tp_rank, count);
        const volatile uint32_t* fl = reinterpret_cast<const volatile uint32_t*>(a.tp_peers[a.tp_rank] + a.tp_flags_off);
        int ok = 1;
        const unsigned long long t0 = global_timer();
        for (int j = 0; j < a.tp_n && ok; j++) {
            uint32_t i = 0;
            while ((int32_t)(fl[j] - count) < 0)
                if ((++i & 255u) == 0 && global_timer() - t0 > a.wait_ns) {
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

// x[row] += sum over ranks j (in rank order) of their partial rows, each
// read once its tag shows exchange `count` (bounded wait); rows are spread
// over all threads of the grid.  A thread issues the loads of all ranks'
// words of its row at once and re-polls only those not yet tagged, so the
// waits overlap instead of following one another.  False if a wait gave up.
constexpr int kMaxTpRanks = 8;
__device__ bool tp_reduce_residual(const DecodeArgs& a, uint32_t count) {
    const uint64_t* recv =
        reinterpret_cast<const uint64_t*>(a.tp_peers[a.tp_rank]) + (size_t)(count & 1u) * a.tp_n * a.dim;
    bool ok = true;
    const unsigned long long t0 = global_timer();
    for (int row = blockIdx.x * kThreads + threadIdx.x; row < a.dim && ok; row += gridDim.x * kThreads) {
        uint64_t t[kMaxTpRanks];
#pragma unroll
        for (int j = 0; j < kMaxTpRanks; j++)
            t[j] = j < a.tp_n ? ld_relaxed_sys_u64(recv + (size_t)j * a.dim + row) : ((uint64_t)count << 32);
        const float xr = __ldcg(a.x + row);
        float sum = 0.0f;
#pragma unroll
        for (int j = 0; j < kMaxTpRanks; j++) {
            for (uint32_t i = 0; ok && tag_ep(t[j]) != count; i++) {
                if ((i & 63u) == 63u && global_timer() - t0 > a.wait_ns) ok = false;
                else t[j] = ld_relaxed_sys_u64(recv + (size_t)j * a.dim + row);
            }
            if (j < a.tp_n) sum += tag_val(t[j]);
        }
        __stcg(a.x + row, xr + sum);
    }
    if (!ok) set_error(a.step, DEV_BARRIER_TIMEOUT);
    return ok;
}

// ---------------------------------------------------------------------------
// The persistent decode kernel.
// ---------------------------------------------------------------------------
// Warps 0..kWarps-1 compute; warp kWarps is the producer: its lane w walks compute warp
// w's chunk sequence and issues each chunk's bulk copy as soon as the slot
// it goes to is free, so the compute warps only wait, compute and release.
constexpr int kDecodeThreads = kThreads + 32;

// Producer lane `w` (bounded: gives up when a slot stays busy for 2^24 polls
// or a compute warp has recorded an error), then waits for its copies.
__device__ __forceinline__ void produce(const DecodeArgs& a, const OpDesc* ops, unsigned char* ring_base,
                                       uint64_t* bars, int w, int mode) {
    ProdRing pr;
    ring_init(pr.r, ring_base, bars, a.P, a.slot_bytes, w, false);
    pr.round = 0;
    Seq seq;
    seq_enter(seq, ops, a.nops, a.steps, mode, 0, 0, w);
    uint32_t spins = 0;
    while (seq.step < a.steps) {
        int bytes;
        const uint8_t* src = chunk_src(seq.m, seq.cu.tile, seq.cu.c, bytes);
        if (prod_try_issue(pr, src, bytes)) {
            spins = 0;
            if (!cursor_next(seq.cu, seq.w, seq.m)) seq_enter(seq, ops, a.nops, a.steps, mode, seq.step, seq.op + 1, w);
        } else if (++spins > (1u << 24) || ((spins & 4095u) == 0 && ld_relaxed_i32(&a.step->error) != 0)) {
            break;
        }
    }
    prod_drain(pr);
}

template <int MODE>
__global__ void __launch_bounds__(kDecodeThreads, 1) k_decode(DecodeArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bars[kWarps * 2 * 8];
    __shared__ float red[32];
    __shared__ unsigned long long red64[kWarps];
    __shared__ __align__(16) OpSmem os;
    __shared__ int s_tok, s_pos, s_bad;
    __shared__ float s_freq[kMaxHead];          // RoPE cos / sin of this step's position
    unsigned char* xf = smem;
    float* xs = reinterpret_cast<float*>(smem + a.xs_off);
    unsigned char* ring_base = smem + a.xbytes;

    // The op table lives in shared memory for the whole launch.
    OpDesc* ops = reinterpret_cast<OpDesc*>(smem + a.ops_off);
    static_assert(sizeof(OpDesc) % 4 == 0, "OpDesc copy");
    for (int i = threadIdx.x; i < a.nops * (int)(sizeof(OpDesc) / 4); i += kDecodeThreads)
        reinterpret_cast<int*>(ops)[i] = __ldg(reinterpret_cast<const int*>(a.ops) + i);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    Ring ring;
    if (warp < kWarps) {
        ring_init(ring, ring_base, bars, a.P, a.slot_bytes, warp, lane == 0);
        reset_opsmem(os);
    }
    fence_mbar_init();
    __syncthreads();   // all kDecodeThreads: the op table, the barriers and OpSmem are ready
    if (warp == kWarps) {
        if (lane < kWarps) produce(a, ops, ring_base, bars, lane, MODE);
        return;
    }
    Seq seq;   // unused: the producer warp issues every chunk
    __shared__ uint32_t s_xcount, s_opseq;
    if (threadIdx.x == 0) {
        s_xcount = *reinterpret_cast<volatile uint32_t*>(&a.step->tp_count);
        s_opseq = *reinterpret_cast<volatile uint32_t*>(&a.step->op_seq);
    }
    csync();
    uint32_t xcount = s_xcount;   // tensor-parallel exchanges so far (identical on every rank)
    const uint32_t op_seq = s_opseq;

    uint32_t nbar = 0;
    bool ok = true;
    for (int step = 0; step < a.steps && ok; step++) {
        // Resolve this step's position and token (identical in every CTA).
        if (threadIdx.x == 0) {
            volatile StepState* st = a.step;
            const int pos = st->pos_next;
            const int forced = st->forced_token;
            const int tok = forced >= 0 ? forced : (int)key_index(__ldcg(a.argmax));
            s_bad = (tok < 0 || tok >= a.vocab || pos < 0 || pos >= a.max_pos);
            s_tok = tok;
            s_pos = pos;
        }
        csync();
        if (s_bad) {
            if (blockIdx.x == 0 && threadIdx.x == 0) set_error(a.step, DEV_BAD_INPUT);
            break;
        }
        const int pos = s_pos, tok = s_tok;
        {
            const int h2 = a.head_size / 2;
            if (threadIdx.x < 2 * h2)
                s_freq[threadIdx.x] = threadIdx.x < h2 ? __ldg(a.freq_re + (size_t)pos * h2 + threadIdx.x)
                                                       : __ldg(a.freq_im + (size_t)pos * h2 + threadIdx.x - h2);
        }
        VecSrc emb_src;
        emb_src.p = nullptr;
        emb_src.emb = a.emb;
        emb_src.tok = tok;
        if (blockIdx.x == 0)   // x = embedding row, for the residual stream
            for (int i = threadIdx.x; i < a.dim / 4; i += kThreads)
                __stcg(reinterpret_cast<float4*>(a.x) + i, src_load4<MODE>(emb_src, i));

        for (int oi = 0; oi < a.nops && ok; oi++) {
            const OpDesc op = ops[oi];
            VecSrc src;
            src.emb = a.emb;
            src.tok = tok;
            src.p = nullptr;
            const float* nw = nullptr;
            if (op.kind == OP_QKV) {
                nw = a.rms_att + (size_t)op.layer * a.dim;
                if (op.layer > 0) src.p = a.x;
            } else if (op.kind == OP_W13) {
                nw = a.rms_ffn + (size_t)op.layer * a.dim;
                src.p = a.x;
            } else if (op.kind == OP_CLS) {
                nw = a.rms_final;
                src.p = a.x;
            } else {
                src.p = op.kind == OP_WO ? a.att : a.hb;
            }
            PHASE_T(step, oi, 0);
            // Tag of this op's cut-tile parts: unique over every decode launch
            // of the context (op_seq counts all ops before this launch), never 0.
            const uint32_t ctag = (op_seq + (uint32_t)(step * a.nops + oi)) % 0xFFFFFFFFu + 1u;
            if (op.kind == OP_QKV && MODE != MODE_W4A8) prefetch_kv_l2(a, op.layer, pos);
            build_input<MODE>(xf, xs, src, op.m.n, nw, red);
            csync();
            PHASE_T(step, oi, 1);
            DecodeEpi epi{&a, &op, pos, s_freq, -1e9f, 0u};
            if (a.tp_n > 1 && (op.kind == OP_WO || op.kind == OP_W2)) epi.xcount = ++xcount;
            if (!run_op<MODE, true>(op.m, ring, ring_base, seq, ops, a.nops, a.steps, xf, xs, os, a.split_part, ctag,
                                    epi, step, oi)) {
                set_error(a.step, DEV_COPY_TIMEOUT);
                ok = false;
                break;
            }
            PHASE_T(step, oi, 3);
            if (op.kind == OP_CLS) cta_argmax(a.argmax, epi.best, epi.best_i, red64);
            if (a.tp_n > 1 && (op.kind == OP_WO || op.kind == OP_W2)) {
                // Sum the ranks' partial rows into the residual stream.
                if (csync_or(!tp_reduce_residual(a, epi.xcount))) { ok = false; break; }
                if (!grid_barrier(a.step, nbar)) { ok = false; break; }
                continue;
            }
            if (a.tp_n > 1 && op.kind == OP_CLS) {
                // The greedy token is the largest of the ranks' argmax keys.
                if (!grid_barrier(a.step, nbar)) { ok = false; break; }
                if (blockIdx.x == 0 && threadIdx.x == 0) {
                    const unsigned long long key = __ldcg(a.argmax);
                    for (int j = 0; j < a.tp_n; j++)
                        reinterpret_cast<unsigned long long*>(a.tp_peers[j] + a.tp_keys_off)[a.tp_rank] = key;
                    __threadfence_system();
                }
                if (!tp_exchange(a, nbar, ++xcount)) { ok = false; break; }
                if (blockIdx.x == 0 && threadIdx.x == 0) {
                    const unsigned long long* keys =
                        reinterpret_cast<const unsigned long long*>(a.tp_peers[a.tp_rank] + a.tp_keys_off);
                    unsigned long long m = 0;
                    for (int j = 0; j < a.tp_n; j++) {
                        const unsigned long long k = __ldcg(keys + j);
                        m = k > m ? k : m;
                    }
                    *a.argmax = m;
                    __threadfence();
                }
            }
            if (op.kind == OP_CLS && a.sampling) {
                // Every logit and the argmax key are in place: CTA 0 draws the
                // next token and hands it to the next step as a forced token.
                if (!grid_barrier(a.step, nbar)) { ok = false; break; }
                if (blockIdx.x == 0) {
                    const float mx = key_value(__ldcg(a.argmax));
                    const int t = sample_token(a.logits, a.vocab, mx, a.samp, 0ull, (unsigned long long)pos,
                                               reinterpret_cast<unsigned long long*>(xf));
                    if (threadIdx.x == 0) {
                        a.step->forced_token = t;
                        __threadfence();
                    }
                }
            }
            if (oi == a.nops - 1 && step == a.steps - 1) break;   // nothing after the last classifier
            if (!grid_barrier(a.step, nbar)) { ok = false; break; }
            PHASE_T(step, oi, 4);
            if (op.kind == OP_QKV) {
                if (op.layer == 0 && blockIdx.x == 0 && threadIdx.x == 0) {
                    // Every CTA has read the step state and the argmax key.
                    StepState* st = a.step;
                    st->pos = pos;
                    st->token = tok;
                    st->pos_next = pos + 1;
                    st->forced_token = -1;
                    a.history[pos] = tok;
                    *a.argmax = argmax_key(-1e9f, 0);
                    __threadfence();
                }
                if (MODE == MODE_W4A8)
                    attention_layer_exact(a, op.layer, pos, reinterpret_cast<float*>(xf), red);
                else
                    attention_layer(a, op.layer, pos, xf, a.ops_off, os.part, kMaxLocalTiles * kWarps * kTR);
                PHASE_T(step, oi, 5);
                if (!grid_barrier(a.step, nbar)) { ok = false; break; }
                PHASE_T(step, oi, 6);
            }
        }
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        a.step->tp_count = xcount;
        a.step->op_seq = op_seq + (uint32_t)(a.steps * a.nops);   // every tag this launch could have used
    }
}

// ---------------------------------------------------------------------------
// Standalone matvec y = W x (kernel-level entry points): the same streaming
// and epilogue machinery as one op of the decode kernel.
// ---------------------------------------------------------------------------
struct StandaloneArgs {
    uint32_t epoch;                // tag of this call's cut-tile flags (nonzero)
    OpDesc op;
    const float* x;
    float* y;
    uint64_t* split_part;
    int P, slot_bytes, xbytes, xs_off;
    int* error;
};

struct StoreEpi {
    float* y;
    int d;
    __device__ __forceinline__ void prefetch(int, int, float*) {}
    __device__ __forceinline__ void operator()(int r0, const float* v) {
        for (int r = 0; r < kRB; r++)
            if (r0 + r < d) y[r0 + r] = v[r];
    }
};

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1) k_matvec(StandaloneArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bars[kWarps * 2 * 8];
    __shared__ __align__(16) OpSmem os;
    __shared__ OpDesc s_op;
    unsigned char* xf = smem;
    float* xs = reinterpret_cast<float*>(smem + a.xs_off);
    unsigned char* ring_base = smem + a.xbytes;
    if (threadIdx.x == 0) s_op = a.op;
    Ring ring;
    ring_init(ring, ring_base, bars, a.P, a.slot_bytes, threadIdx.x >> 5, (threadIdx.x & 31) == 0);
    reset_opsmem(os);
    fence_mbar_init();
    csync();
    Seq seq;
    seq_enter(seq, &s_op, 1, 1, MODE, 0, 0, threadIdx.x >> 5);
    for (int i = 0; i < a.P; i++) seq_issue_next(seq, ring, &s_op, 1, 1, MODE);
    pdl_launch_dependents();
    pdl_wait();
    VecSrc src;
    src.p = a.x;
    src.tok = 0;
    src.emb = a.op.m;
    __shared__ float red[32];
    build_input<MODE>(xf, xs, src, s_op.m.n, nullptr, red);
    csync();
    StoreEpi epi{a.y, a.op.m.d};
    if (!run_op<MODE, false>(s_op.m, ring, ring_base, seq, &s_op, 1, 1, xf, xs, os, a.split_part, a.epoch, epi))
        if (threadIdx.x == 0) atomicCAS(a.error, 0, DEV_COPY_TIMEOUT);
    ring_drain(ring);
}

}  // namespace aion
