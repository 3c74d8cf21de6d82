// Persistent decode kernel: `steps` greedy tokens of the int4 Llama-2
// forward (src/kernel_simd.c:1014-1169 per token, :1223-1250 around it) in
// one cooperative launch, one CTA per SM.
//
// Every weight matrix of a token is an "op"; the ops of all steps form one
// sequence.  CTA c owns tiles [c*T/G, (c+1)*T/G) of every op; warp w of the
// CTA streams tiles t0 + w, t0 + w + 8, ... of each op, chunk by chunk,
// through its own ring of bulk copies, always P chunks ahead -- across op
// boundaries, grid barriers and tokens, since the weights never depend on
// the activations.  Between dependent ops the CTAs meet at a bounded grid
// barrier; the input vector of each op is rebuilt in shared memory ("x'")
// with its fused prologue (RMSNorm, or the int4 embedding row).
//
// Per token (5 barriers per layer, 1 after the classifier):
//   [QKV: rmsnorm x' | q, k, v rows | RoPE, KV append]  barrier
//   [attention: (head, 64-position chunk) units, last CTA per head combines] barrier
//   [wo: att x' | x += ]  barrier
//   [w1/w3: rmsnorm x' | SwiGLU -> hb]  barrier
//   [w2: hb x' | x += ]  barrier
//   ... [classifier: rmsnorm x' | logits, argmax key]  barrier (next token)
#pragma once

#include "matvec.cuh"

namespace aion {

enum OpKind { OP_QKV = 0, OP_WO = 1, OP_W13 = 2, OP_W2 = 3, OP_CLS = 4 };

struct OpDesc {
    MatDesc m;
    int kind, layer;
};

constexpr int kAttnLen = 64;       // positions per attention unit
constexpr int kMaxHead = 256;

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
    StepState* step;
    unsigned long long* argmax;
    int32_t* history;              // [max_pos]
    int steps;
    int P, slot_bytes, xbytes;
};

// ---------------------------------------------------------------------------
// Input sources of an op's x': an fp32 vector in global memory (written by
// other CTAs of this launch: read through L2), or the int4 embedding row of
// a token (src/kernel_simd.c:1032-1040: x[i] = (int8)(nibble - 8) * scale).
// ---------------------------------------------------------------------------
struct VecSrc {
    const float* p;                // fp32 vector, or nullptr for the embedding row
    const uint8_t* emb_w;
    MatDesc emb;
    int tok;
};

__device__ __forceinline__ float4 src_load4(const VecSrc& s, int i) {
    if (s.p) return __ldcg(reinterpret_cast<const float4*>(s.p) + i);
    const int e = 4 * i, g = e / 32;
    const float sc = __ldg(reinterpret_cast<const float*>(s.emb_w + scale_offset(s.emb, s.tok, g)));
    const uint16_t b = __ldg(reinterpret_cast<const uint16_t*>(s.emb_w + group_offset(s.emb, s.tok, g) + (e % 32) / 2));
    float4 v;
    v.x = (float)((int)(b & 0xF) - 8) * sc;
    v.y = (float)((int)((b >> 4) & 0xF) - 8) * sc;
    v.z = (float)((int)((b >> 8) & 0xF) - 8) * sc;
    v.w = (float)((int)((b >> 12) & 0xF) - 8) * sc;
    return v;
}

__device__ __forceinline__ float src_rms_scale(const VecSrc& s, int n, float* red) {
    float acc = 0.0f;
    for (int i = threadIdx.x; i < n / 4; i += blockDim.x) {
        const float4 v = src_load4(s, i);
        acc += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    acc = block_sum(acc, red);
    return 1.0f / sqrtf(__fdiv_rn(acc, (float)n) + 1e-5f);
}

// The rmsnorm scale in the reference's own order (src/kernel_simd.c:793-803):
// four lane sums of x[4m + l]^2 (product rounded, then added), reduced
// pairwise, then mean, + 1e-5, 1 / sqrtf.  A sequential chain of n/4 adds
// per lane: used where bit-exact parity with the reference is the contract.
__device__ __forceinline__ float src_rms_scale_exact(const VecSrc& s, int n, float* red) {
    if (threadIdx.x < 4) {
        float acc = 0.0f;
        for (int i = 0; i < n / 4; i++) {
            const float4 v = src_load4(s, i);
            const float e = threadIdx.x == 0 ? v.x : threadIdx.x == 1 ? v.y : threadIdx.x == 2 ? v.z : v.w;
            acc = __fadd_rn(acc, __fmul_rn(e, e));
        }
        red[threadIdx.x] = acc;
    }
    __syncthreads();
    const float sum = __fadd_rn(__fadd_rn(red[0], red[1]), __fadd_rn(red[2], red[3]));
    __syncthreads();
    return 1.0f / sqrtf(__fdiv_rn(sum, (float)n) + 1e-5f);
}

// e^x rounded once to float: the double-precision exponential rounded to
// the nearest float (CUDA exp() is accurate to < 1 double ulp, so only
// inputs within ~1e-16 relative of a float rounding boundary can differ
// from the correctly rounded value).
__device__ __forceinline__ float expf_cr(float x) { return (float)exp((double)x); }

template <int MODE>
__device__ __forceinline__ void src_build_x(unsigned char* xbuf, const VecSrc& s, int n, const float* norm_w, float ss) {
    const int G = n / 32;
    if (MODE == MODE_W4A16) {
        float4* xs4 = reinterpret_cast<float4*>(xbuf);
        for (int i = threadIdx.x; i < n / 4; i += blockDim.x) {
            float4 v = src_load4(s, i);
            if (norm_w) {
                const float4 w = __ldg(reinterpret_cast<const float4*>(norm_w) + i);
                v.x = __fmul_rn(__fmul_rn(v.x, ss), w.x);
                v.y = __fmul_rn(__fmul_rn(v.y, ss), w.y);
                v.z = __fmul_rn(__fmul_rn(v.z, ss), w.z);
                v.w = __fmul_rn(__fmul_rn(v.w, ss), w.w);
            }
            const int e0 = (i & 1) * 4;
            v.x *= prescale(e0);
            v.y *= prescale(e0 + 1);
            v.z *= prescale(e0 + 2);
            v.w *= prescale(e0 + 3);
            xs4[xperm(i >> 3, i & 7)] = v;
        }
    } else {
        const int chunks = (G + 31) / 32;
        uint4* qx = reinterpret_cast<uint4*>(xbuf);
        float* xsc = reinterpret_cast<float*>(xbuf + chunks * 2 * 32 * 16);
        for (int g = threadIdx.x; g < G; g += blockDim.x) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                float4 t = src_load4(s, g * 8 + j);
                if (norm_w) {
                    const float4 w = __ldg(reinterpret_cast<const float4*>(norm_w) + g * 8 + j);
                    t.x = __fmul_rn(__fmul_rn(t.x, ss), w.x);
                    t.y = __fmul_rn(__fmul_rn(t.y, ss), w.y);
                    t.z = __fmul_rn(__fmul_rn(t.z, ss), w.z);
                    t.w = __fmul_rn(__fmul_rn(t.w, ss), w.w);
                }
                v[4 * j] = t.x; v[4 * j + 1] = t.y; v[4 * j + 2] = t.z; v[4 * j + 3] = t.w;
            }
            float amax = 0.0f;
#pragma unroll
            for (int k = 0; k < 32; k++) amax = fmaxf(amax, fabsf(v[k]));
            const bool big = amax > 1e-9f;
            const float scale = big ? __fdiv_rn(127.0f, amax) : 1.0f;
            xsc[g] = big ? __fdiv_rn(amax, 127.0f) : 1.0f;
            uint32_t words[8];
#pragma unroll
            for (int wd = 0; wd < 4; wd++) {
                uint32_t ev = 0, od = 0;
#pragma unroll
                for (int b = 0; b < 4; b++) {
                    const int qe = (int)roundf(__fmul_rn(v[8 * wd + 2 * b], scale));
                    const int qo = (int)roundf(__fmul_rn(v[8 * wd + 2 * b + 1], scale));
                    ev |= (uint32_t)(qe & 0xFF) << (8 * b);
                    od |= (uint32_t)(qo & 0xFF) << (8 * b);
                }
                words[2 * wd] = ev;
                words[2 * wd + 1] = od;
            }
            qx[((g >> 5) * 2 + 0) * 32 + (g & 31)] = make_uint4(words[0], words[1], words[2], words[3]);
            qx[((g >> 5) * 2 + 1) * 32 + (g & 31)] = make_uint4(words[4], words[5], words[6], words[7]);
        }
    }
}

// ---------------------------------------------------------------------------
// Producer position of a warp in the op sequence (all lanes keep it).
// ---------------------------------------------------------------------------
struct Seq {
    int step, op, t, c, t1;        // op == nops: end of the sequence
};

__device__ __forceinline__ void seq_enter(Seq& s, const DecodeArgs& a, int step, int op) {
    const int warp = threadIdx.x >> 5;
    while (step < a.steps) {
        while (op < a.nops) {
            const int T = a.ops[op].m.ntiles;
            int t0, t1;
            t0 = (int)(((long long)blockIdx.x * T) / gridDim.x);
            t1 = (int)(((long long)(blockIdx.x + 1) * T) / gridDim.x);
            if (t0 + warp < t1) {
                s.step = step; s.op = op; s.t = t0 + warp; s.c = 0; s.t1 = t1;
                return;
            }
            op++;
        }
        op = 0;
        step++;
    }
    s.step = a.steps; s.op = a.nops;
}

__device__ __forceinline__ void seq_issue_next(Seq& s, Ring& r, const DecodeArgs& a) {
    if (s.step >= a.steps) return;
    const MatDesc& m = a.ops[s.op].m;
    ring_issue(r, m.w + (size_t)s.t * m.tile_bytes + (size_t)s.c * m.chunk_bytes, m.chunk_bytes);
    if (++s.c == m.nch) {
        s.c = 0;
        s.t += kWarps;
        if (s.t >= s.t1) seq_enter(s, a, s.step, s.op + 1);
    }
}

// ---------------------------------------------------------------------------
// Epilogue of one finished tile (runs on lane 0).
// ---------------------------------------------------------------------------
struct TokenCtx {
    int pos, tok;
    float best;
    uint32_t best_i;
};

__device__ __forceinline__ void decode_epilogue(const DecodeArgs& a, const OpDesc& op, int r0, const float* v,
                                                TokenCtx& tc) {
    const int d = op.m.d;
    switch (op.kind) {
    case OP_QKV: {
        const int hs = a.head_size, pos = tc.pos;
        const size_t lkv = (size_t)op.layer * a.max_pos * a.kv_dim;
        if (r0 < a.dim + a.kv_dim) {
            // RoPE on adjacent pairs (src/kernel_simd.c:1068-1085)
            const bool is_q = r0 < a.dim;
            const int base = is_q ? r0 : r0 - a.dim;
            float out[kRB];
            for (int r = 0; r < kRB; r += 2) {
                const int hd = (base + r) % hs;
                const float fr = __ldg(a.freq_re + pos * (hs / 2) + hd / 2);
                const float fi = __ldg(a.freq_im + pos * (hs / 2) + hd / 2);
                out[r] = __fsub_rn(__fmul_rn(v[r], fr), __fmul_rn(v[r + 1], fi));
                out[r + 1] = __fadd_rn(__fmul_rn(v[r], fi), __fmul_rn(v[r + 1], fr));
            }
            float* dst = is_q ? a.q + base : a.kcache + lkv + (size_t)pos * a.kv_dim + base;
            __stcg(reinterpret_cast<float4*>(dst), make_float4(out[0], out[1], out[2], out[3]));
        } else {
            const int base = r0 - a.dim - a.kv_dim;
            __stcg(reinterpret_cast<float4*>(a.vcache + lkv + (size_t)pos * a.kv_dim + base),
                   make_float4(v[0], v[1], v[2], v[3]));
        }
        break;
    }
    case OP_WO:
    case OP_W2:
        for (int r = 0; r < kRB; r++)
            if (r0 + r < d) __stcg(a.x + r0 + r, __ldcg(a.x + r0 + r) + v[r]);
        break;
    case OP_W13: {
        // tile rows w1[2t], w1[2t+1], w3[2t], w3[2t+1]; swiglu (src/kernel_simd.c:836-841)
        const int h0 = r0 / 2;
        for (int r = 0; r < 2; r++)
            if (h0 + r < a.hidden) {
                const float g = v[r];
                const float s = __fdiv_rn(g, __fadd_rn(1.0f, expf_cr(-g)));
                __stcg(a.hb + h0 + r, __fmul_rn(s, v[2 + r]));
            }
        break;
    }
    default:  // OP_CLS
        for (int r = 0; r < kRB; r++)
            if (r0 + r < d) {
                __stcg(a.logits + r0 + r, v[r]);
                if (v[r] > tc.best) { tc.best = v[r]; tc.best_i = (uint32_t)(r0 + r); }
            }
        break;
    }
}

// ---------------------------------------------------------------------------
// Attention of one layer (CTA-wide).  Unit (head h, chunk k) covers
// positions [64k, 64k+64) ∩ [0, pos]: scores (q . k_t) / sqrtf(head_size)
// (src/kernel_simd.c:1099-1117), local max, e^(s - max), their sum and the
// weighted V sum are written as a partial; the last CTA to finish a head
// merges the partials in chunk order into att[h].
// ---------------------------------------------------------------------------
struct AttnSmem {
    float q[kMaxHead];
    float s[kAttnLen];
    float o[kThreads];             // groups * head_size <= kThreads
    float red[32];
    int last;
};

__device__ void attention_layer(const DecodeArgs& a, int layer, int pos, AttnSmem& sm) {
    const int hs = a.head_size, tid = threadIdx.x;
    const int nch = (pos + kAttnLen) / kAttnLen;
    const int units = a.n_heads * nch;
    const size_t lkv = (size_t)layer * a.max_pos * a.kv_dim;
    const float* kc = a.kcache + lkv;
    const float* vc = a.vcache + lkv;
    const float rs = sqrtf((float)hs);
    const int groups = blockDim.x / hs;           // position groups for the V sum (>= 1)
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
        const int h = u / nch, k = u % nch;
        const int kvh = h / a.kv_mul;
        const int t0 = k * kAttnLen, n = min(kAttnLen, pos + 1 - t0);
        for (int i = tid; i < hs; i += blockDim.x) sm.q[i] = __ldcg(a.q + h * hs + i);
        __syncthreads();
        // scores: 4 threads per position, each a quarter of the head
        {
            const int p = tid >> 2, part = tid & 3;
            float dot = 0.0f;
            if (p < n) {
                const float* kr = kc + (size_t)(t0 + p) * a.kv_dim + kvh * hs;
                const int q4 = hs / 4;
                if ((q4 & 3) == 0) {
                    for (int i = part * q4; i < (part + 1) * q4; i += 4) {
                        const float4 kv4 = __ldcg(reinterpret_cast<const float4*>(kr + i));
                        dot = fmaf(sm.q[i], kv4.x, dot);
                        dot = fmaf(sm.q[i + 1], kv4.y, dot);
                        dot = fmaf(sm.q[i + 2], kv4.z, dot);
                        dot = fmaf(sm.q[i + 3], kv4.w, dot);
                    }
                } else {
                    for (int i = part; i < hs; i += 4) dot = fmaf(sm.q[i], __ldcg(kr + i), dot);
                }
            }
            dot += __shfl_xor_sync(0xffffffffu, dot, 1);
            dot += __shfl_xor_sync(0xffffffffu, dot, 2);
            if (part == 0 && p < kAttnLen) sm.s[p] = p < n ? __fdiv_rn(dot, rs) : -INFINITY;
        }
        __syncthreads();
        float m = tid < n ? sm.s[tid] : -INFINITY;
        m = block_max(m, sm.red);
        float e = 0.0f;
        if (tid < n) {
            e = expf_cr(sm.s[tid] - m);
            sm.s[tid] = e;
        }
        const float l = block_sum(e, sm.red);   // contains a __syncthreads before its smem use
        __syncthreads();
        // V: thread (group gi, dim i) sums positions gi, gi + groups, ...;
        // the group sums are added in group order.
        {
            const int gi = tid / hs, i = tid % hs;
            if (gi < groups) {
                float o = 0.0f;
                for (int p = gi; p < n; p += groups)
                    o = fmaf(sm.s[p], __ldcg(vc + (size_t)(t0 + p) * a.kv_dim + kvh * hs + i), o);
                sm.o[gi * hs + i] = o;
            }
        }
        __syncthreads();
        float* part = a.attn_part + ((size_t)h * a.max_chunks + k) * (hs + 2);
        for (int i = tid; i < hs; i += blockDim.x) {
            float o = sm.o[i];
            for (int g = 1; g < groups; g++) o += sm.o[g * hs + i];
            __stcg(part + 2 + i, o);
        }
        if (tid == 0) {
            __stcg(part, m);
            __stcg(part + 1, l);
        }
        __threadfence();
        __syncthreads();
        if (tid == 0) sm.last = (atomicAdd(a.attn_cnt + h, 1) == nch - 1);
        __syncthreads();
        if (sm.last) {
            __threadfence();
            const float* ph = a.attn_part + (size_t)h * a.max_chunks * (hs + 2);
            float M = -INFINITY;
            for (int c = 0; c < nch; c++) M = fmaxf(M, __ldcg(ph + (size_t)c * (hs + 2)));
            float L = 0.0f;
            for (int c = 0; c < nch; c++) L = fmaf(__ldcg(ph + (size_t)c * (hs + 2) + 1), expf(__ldcg(ph + (size_t)c * (hs + 2)) - M), L);
            const float inv = 1.0f / L;
            for (int i = tid; i < hs; i += blockDim.x) {
                float o = 0.0f;
                for (int c = 0; c < nch; c++)
                    o = fmaf(__ldcg(ph + (size_t)c * (hs + 2) + 2 + i), expf(__ldcg(ph + (size_t)c * (hs + 2)) - M), o);
                __stcg(a.att + h * hs + i, o * inv);
            }
            if (tid == 0) a.attn_cnt[h] = 0;
        }
        __syncthreads();
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
        for (int i = tid; i < hs; i += blockDim.x) s_q[i] = __ldcg(a.q + h * hs + i);
        __syncthreads();
        float m = -INFINITY;
        for (int t = tid; t <= pos; t += blockDim.x) {
            const float* kr = kc + (size_t)t * a.kv_dim + kvh * hs;
            float d = 0.0f;
            for (int j = 0; j < hs; j++) d = __fadd_rn(d, __fmul_rn(s_q[j], __ldcg(kr + j)));
            d = __fdiv_rn(d, rs);
            sc[t] = d;
            m = fmaxf(m, d);
        }
        m = block_max(m, red);
        for (int t = tid; t <= pos; t += blockDim.x) sc[t] = expf_cr(__fsub_rn(sc[t], m));
        __syncthreads();
        if (tid == 0) {
            float sum = 0.0f;
            for (int t = 0; t <= pos; t++) sum = __fadd_rn(sum, sc[t]);
            s_sum = sum;
        }
        __syncthreads();
        const float scale = __fdiv_rn(1.0f, s_sum);
        for (int t = tid; t <= pos; t += blockDim.x) sc[t] = __fmul_rn(sc[t], scale);
        __syncthreads();
        for (int j = tid; j < hs; j += blockDim.x) {
            float o = 0.0f;
            for (int t = 0; t <= pos; t++)
                o = __fadd_rn(o, __fmul_rn(sc[t], __ldcg(vc + (size_t)t * a.kv_dim + kvh * hs + j)));
            __stcg(a.att + h * hs + j, o);
        }
        __syncthreads();
    }
}

// Sets the next step's position and/or forced token (negative: keep).
__global__ void k_set_step(StepState* s, int pos, int token) {
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        if (pos >= 0) s->pos_next = pos;
        if (token >= 0) s->forced_token = token;
    }
}

// ---------------------------------------------------------------------------
// The kernel.
// ---------------------------------------------------------------------------
template <int MODE>
__global__ void __launch_bounds__(kThreads, 1) k_decode(DecodeArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bars[kWarps * 8];
    __shared__ float red[32];
    __shared__ AttnSmem attn;
    __shared__ int s_tok, s_pos, s_bad;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    unsigned char* xbuf = smem;
    unsigned char* ring_base = smem + a.xbytes;

    Ring ring;
    ring_init(ring, ring_base, bars, a.P, a.slot_bytes);
    Seq seq;
    seq_enter(seq, a, 0, 0);
    for (int i = 0; i < a.P; i++) seq_issue_next(seq, ring, a);

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
        __syncthreads();
        if (s_bad) {
            if (blockIdx.x == 0 && threadIdx.x == 0) set_error(a.step, DEV_BAD_INPUT);
            break;
        }
        TokenCtx tc;
        tc.pos = s_pos;
        tc.tok = s_tok;
        tc.best = -1e9f;
        tc.best_i = 0;
        VecSrc emb_src;
        emb_src.p = nullptr;
        emb_src.emb_w = a.emb.w;
        emb_src.emb = a.emb;
        emb_src.tok = tc.tok;
        if (blockIdx.x == 0)   // x = embedding row, for the residual stream
            for (int i = threadIdx.x; i < a.dim / 4; i += blockDim.x)
                __stcg(reinterpret_cast<float4*>(a.x) + i, src_load4(emb_src, i));

        for (int oi = 0; oi < a.nops && ok; oi++) {
            const OpDesc op = a.ops[oi];
            // ---- input x' of this op
            VecSrc src;
            src.p = nullptr; src.emb_w = a.emb.w; src.emb = a.emb; src.tok = tc.tok;
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
            const float ss = !nw ? 1.0f
                             : (MODE == MODE_W4A8 ? src_rms_scale_exact(src, op.m.n, red) : src_rms_scale(src, op.m.n, red));
            src_build_x<MODE>(xbuf, src, op.m.n, nw, ss);
            __syncthreads();
            // ---- this warp's tiles of the op
            int t0, t1;
            t0 = (int)(((long long)blockIdx.x * op.m.ntiles) / gridDim.x);
            t1 = (int)(((long long)(blockIdx.x + 1) * op.m.ntiles) / gridDim.x);
            for (int t = t0 + warp; t < t1 && ok; t += kWarps) {
                float acc[kRB] = {0.0f, 0.0f, 0.0f, 0.0f};
                for (int c = 0; c < op.m.nch; c++) {
                    const unsigned char* ch = ring_wait(ring, ring_base);
                    if (!ch) {
                        set_error(a.step, DEV_COPY_TIMEOUT);
                        ok = false;
                        break;
                    }
                    chunk_compute<MODE>(ch, op.m.kc, c * (op.m.kc / 32), xbuf, op.m.n, acc);
                    __syncwarp();
                    ring.consumed++;
                    seq_issue_next(seq, ring, a);
                }
                if (!ok) break;
                finish_rows<MODE>(acc);
                if (lane == 0) decode_epilogue(a, op, t * kRB, acc, tc);
            }
            if (op.kind == OP_CLS && lane == 0 && tc.best > -1e9f)
                atomicMax(a.argmax, argmax_key(tc.best, tc.best_i));
            // An error in one warp must stop the whole CTA consistently.
            if (__syncthreads_or(!ok)) ok = false;
            if (!ok) break;
            if (oi == a.nops - 1 && step == a.steps - 1) break;   // nothing after the last classifier
            if (!grid_barrier(a.step, nbar)) { ok = false; break; }
            if (op.kind == OP_QKV) {
                if (op.layer == 0 && blockIdx.x == 0 && threadIdx.x == 0) {
                    // Every CTA has read the step state and the argmax key.
                    StepState* st = a.step;
                    st->pos = tc.pos;
                    st->token = tc.tok;
                    st->pos_next = tc.pos + 1;
                    st->forced_token = -1;
                    a.history[tc.pos] = tc.tok;
                    *a.argmax = argmax_key(-1e9f, 0);
                    __threadfence();
                }
                if (MODE == MODE_W4A8)
                    attention_layer_exact(a, op.layer, tc.pos, reinterpret_cast<float*>(xbuf), red);
                else
                    attention_layer(a, op.layer, tc.pos, attn);
                if (!grid_barrier(a.step, nbar)) { ok = false; break; }
            }
        }
    }
    ring_drain(ring);
}

}  // namespace aion
