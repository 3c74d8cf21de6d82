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

namespace aion {

enum OpKind { OP_QKV = 0, OP_WO = 1, OP_W13 = 2, OP_W2 = 3, OP_CLS = 4, OP_STORE = 5 };

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
    float* split_part;             // [max_tiles][2][16] partial rows of tiles cut by CTA boundaries
    int* split_cnt;                // [max_tiles], zero between uses
    StepState* step;
    unsigned long long* argmax;
    int32_t* history;              // [max_pos]
    int steps;
    int P, slot_bytes, xbytes, xs_off;
};

// ---------------------------------------------------------------------------
// Input sources of an op: an fp32 vector in global memory (written by other
// CTAs of this launch: read through L2), or the int4 embedding row of a
// token (src/kernel_simd.c:1032-1040: x[i] = (int8)(nibble - 8) * scale).
// ---------------------------------------------------------------------------
struct VecSrc {
    const float* p;                // fp32 vector, or nullptr for the embedding row
    MatDesc emb;
    int tok;
};

__device__ __forceinline__ float4 src_load4(const VecSrc& s, int i) {
    if (s.p) return __ldcg(reinterpret_cast<const float4*>(s.p) + i);
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

// Activation digits of an op's input (optionally RMS-normalised as
// (x * ss) * w, src/kernel_simd.c:805-813).  Thread per group.
template <int MODE>
__device__ __forceinline__ void src_build_digits(unsigned char* xf, float* xs, const VecSrc& s, int n,
                                                 const float* norm_w, float ss) {
    for (int g = threadIdx.x; g < n / 32; g += blockDim.x) {
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
        group_digits<MODE>(xf, xs, g, v);
    }
}

// ---------------------------------------------------------------------------
// Producer position of a warp in the sequence of (step, op) chunk streams.
// ---------------------------------------------------------------------------
struct Seq {
    int step, op;                  // op == nops: end of the sequence
    OpWork w;
    OpCursor cu;
};

__device__ __forceinline__ void seq_enter(Seq& s, const OpDesc* ops, int nops, int steps, int mode, int step, int op) {
    while (step < steps) {
        while (op < nops) {
            s.w = op_work(ops[op].m, mode);
            if (cursor_begin(s.cu, s.w)) {
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
    const MatDesc& m = ops[s.op].m;
    int tile, c, bytes;
    cursor_tc(s.cu, s.w, m, tile, c);
    const uint8_t* src = chunk_src(m, tile, c, bytes);
    ring_issue(r, src, bytes);
    if (!cursor_next(s.cu, s.w, m)) seq_enter(s, ops, nops, steps, mode, s.step, s.op + 1);
}

// ---------------------------------------------------------------------------
// One op on this CTA: consume its chunks from the rings, reduce, combine the
// tiles cut by CTA boundaries, and hand every finished quad of rows to
// `epi(first_row, values[4])`.  Returns false if a wait gave up.
// ---------------------------------------------------------------------------
struct OpSmem {
    float part[kMaxLocalTiles * kWarps * kTR];   // split: warp partials per local tile
    float vals[kMaxLocalTiles * kTR];            // split: finished rows per local tile
    int state[2];
};

template <int MODE, class Epi>
__device__ bool run_op(const MatDesc& m, Ring& ring, unsigned char* ring_base, Seq& seq, const OpDesc* ops, int nops,
                       int steps, const unsigned char* xf, const float* xs, OpSmem& os, float* split_part,
                       int* split_cnt, Epi& epi) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const float lf = MODE == MODE_W4A16 ? w4a16_lane_factor() : 0.0f;
    const OpWork w = op_work(m, MODE);
    bool ok = true;
    OpCursor cu;
    bool more = cursor_begin(cu, w);
    if (w.split) {
        const int tf = w.u0 / m.nch, tl = (w.u1 - 1) / m.nch, ntl = tl - tf + 1;
        for (int i = tid; i < ntl * kWarps * kTR; i += blockDim.x) os.part[i] = 0.0f;
        __syncthreads();
        float a0 = 0.0f, a1 = 0.0f;
        int cur = -1;
        while (more) {
            int tile, c;
            cursor_tc(cu, w, m, tile, c);
            if (tile != cur) {
                if (cur >= 0) {
                    quad_reduce<MODE>(a0, a1);
                    if ((lane & 3) == 0) {
                        float* p = os.part + ((cur - tf) * kWarps + warp) * kTR;
                        p[lane >> 2] = a0;
                        p[(lane >> 2) + 8] = a1;
                    }
                }
                a0 = a1 = 0.0f;
                cur = tile;
            }
            const unsigned char* ch = ring_wait(ring, ring_base);
            if (!ch) { ok = false; break; }
            const int g0 = chunk_g0(m, c), g1 = chunk_g0(m, c + 1);
            chunk_mma<MODE>(ch, g1 - g0, g0, xf, xs, lf, a0, a1);
            __syncwarp();
            ring.consumed++;
            seq_issue_next(seq, ring, ops, nops, steps, MODE);
            more = cursor_next(cu, w, m);
        }
        if (ok && cur >= 0) {
            quad_reduce<MODE>(a0, a1);
            if ((lane & 3) == 0) {
                float* p = os.part + ((cur - tf) * kWarps + warp) * kTR;
                p[lane >> 2] = a0;
                p[(lane >> 2) + 8] = a1;
            }
        }
        if (__syncthreads_or(!ok)) return false;
        for (int i = tid; i < ntl * kTR; i += blockDim.x) {
            const int lt = i / kTR, r = i % kTR;
            float v = 0.0f;
            for (int k = 0; k < kWarps; k++) v += os.part[(lt * kWarps + k) * kTR + r];
            os.vals[i] = v;
        }
        __syncthreads();
        // Tiles cut by a CTA boundary: local tile 0 when u0 is inside a tile
        // (this CTA has the tile's second part), the last local tile when u1
        // is (this CTA has the first part).  The CTA arriving second adds
        // first + second and finishes the tile.
        int finish[2] = {1, 1};
        for (int k = 0; k < 2; k++) {
            const bool cut = k == 0 ? (w.u0 % m.nch) != 0 : (w.u1 % m.nch) != 0;
            if (!cut) continue;
            const int lt = k == 0 ? 0 : ntl - 1, partno = k == 0 ? 1 : 0, tile = tf + lt;
            if (tid < kTR) __stcg(split_part + ((size_t)tile * 2 + partno) * kTR + tid, os.vals[lt * kTR + tid]);
            __threadfence();
            __syncthreads();
            if (tid == 0) os.state[k] = atomicAdd(split_cnt + tile, 1);
            __syncthreads();
            if (os.state[k] == 1) {
                __threadfence();
                if (tid < kTR) {
                    const float mine = os.vals[lt * kTR + tid];
                    const float other = __ldcg(split_part + ((size_t)tile * 2 + (1 - partno)) * kTR + tid);
                    os.vals[lt * kTR + tid] = partno == 0 ? mine + other : other + mine;
                }
                if (tid == 0) split_cnt[tile] = 0;
            } else {
                finish[k] = 0;
            }
            __syncthreads();
        }
        for (int i = tid; i < ntl * (kTR / kRB); i += blockDim.x) {
            const int lt = i / (kTR / kRB), q = i % (kTR / kRB);
            if (lt == 0 && (w.u0 % m.nch) != 0 && !finish[0]) continue;
            if (lt == ntl - 1 && (w.u1 % m.nch) != 0 && !finish[1]) continue;
            epi((tf + lt) * kTR + q * kRB, os.vals + lt * kTR + q * kRB);
        }
    } else {
        float a0 = 0.0f, a1 = 0.0f;
        float* stage = os.part + warp * kTR;
        while (more) {
            int tile, c;
            cursor_tc(cu, w, m, tile, c);
            const unsigned char* ch = ring_wait(ring, ring_base);
            if (!ch) { ok = false; break; }
            const int g0 = chunk_g0(m, c), g1 = chunk_g0(m, c + 1);
            chunk_mma<MODE>(ch, g1 - g0, g0, xf, xs, lf, a0, a1);
            __syncwarp();
            ring.consumed++;
            seq_issue_next(seq, ring, ops, nops, steps, MODE);
            if (c == m.nch - 1) {
                quad_reduce<MODE>(a0, a1);
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
        if (__syncthreads_or(!ok)) return false;
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
    float best;
    uint32_t best_i;

    __device__ __forceinline__ void operator()(int r0, const float* v) {
        const DecodeArgs& A = *a;
        const int d = op->m.d;
        switch (op->kind) {
        case OP_QKV: {
            if (r0 >= d) break;
            const int hs = A.head_size;
            const size_t lkv = (size_t)op->layer * A.max_pos * A.kv_dim;
            if (r0 < A.dim + A.kv_dim) {
                // RoPE on adjacent pairs (src/kernel_simd.c:1068-1085)
                const bool is_q = r0 < A.dim;
                const int base = is_q ? r0 : r0 - A.dim;
                float out[kRB];
                for (int r = 0; r < kRB; r += 2) {
                    const int hd = (base + r) % hs;
                    const float fr = __ldg(A.freq_re + pos * (hs / 2) + hd / 2);
                    const float fi = __ldg(A.freq_im + pos * (hs / 2) + hd / 2);
                    out[r] = __fsub_rn(__fmul_rn(v[r], fr), __fmul_rn(v[r + 1], fi));
                    out[r + 1] = __fadd_rn(__fmul_rn(v[r], fi), __fmul_rn(v[r + 1], fr));
                }
                float* dst = is_q ? A.q + base : A.kcache + lkv + (size_t)pos * A.kv_dim + base;
                __stcg(reinterpret_cast<float4*>(dst), make_float4(out[0], out[1], out[2], out[3]));
            } else {
                const int base = r0 - A.dim - A.kv_dim;
                __stcg(reinterpret_cast<float4*>(A.vcache + lkv + (size_t)pos * A.kv_dim + base),
                       make_float4(v[0], v[1], v[2], v[3]));
            }
            break;
        }
        case OP_WO:
        case OP_W2:
            for (int r = 0; r < kRB; r++)
                if (r0 + r < d) __stcg(A.x + r0 + r, __ldcg(A.x + r0 + r) + v[r]);
            break;
        case OP_W13: {
            // rows w1[2j], w1[2j+1], w3[2j], w3[2j+1]; swiglu (src/kernel_simd.c:836-841)
            const int h0 = r0 / 2;
            for (int r = 0; r < 2; r++)
                if (h0 + r < A.hidden) {
                    const float g = v[r];
                    const float s = __fdiv_rn(g, __fadd_rn(1.0f, expf_cr(-g)));
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
                        best_i = (uint32_t)(r0 + r);
                    }
                }
            break;
        }
    }
};

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
        const float l = block_sum(e, sm.red);
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
            for (int c = 0; c < nch; c++)
                L = fmaf(__ldcg(ph + (size_t)c * (hs + 2) + 1), expf_cr(__ldcg(ph + (size_t)c * (hs + 2)) - M), L);
            const float inv = 1.0f / L;
            for (int i = tid; i < hs; i += blockDim.x) {
                float o = 0.0f;
                for (int c = 0; c < nch; c++)
                    o = fmaf(__ldcg(ph + (size_t)c * (hs + 2) + 2 + i), expf_cr(__ldcg(ph + (size_t)c * (hs + 2)) - M), o);
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
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long m = 0;
        for (int i = 0; i < (int)(blockDim.x >> 5); i++) m = red64[i] > m ? red64[i] : m;
        if (m) atomicMax(dst, m);
    }
    __syncthreads();
}

// ---------------------------------------------------------------------------
// The persistent decode kernel.
// ---------------------------------------------------------------------------
template <int MODE>
__global__ void __launch_bounds__(kThreads, 1) k_decode(DecodeArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bars[kWarps * 8];
    __shared__ float red[32];
    __shared__ unsigned long long red64[kWarps];
    __shared__ AttnSmem attn;
    __shared__ OpSmem os;
    __shared__ int s_tok, s_pos, s_bad;
    unsigned char* xf = smem;
    float* xs = reinterpret_cast<float*>(smem + a.xs_off);
    unsigned char* ring_base = smem + a.xbytes;

    Ring ring;
    ring_init(ring, ring_base, bars, a.P, a.slot_bytes);
    Seq seq;
    seq_enter(seq, a.ops, a.nops, a.steps, MODE, 0, 0);
    for (int i = 0; i < a.P; i++) seq_issue_next(seq, ring, a.ops, a.nops, a.steps, MODE);

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
        const int pos = s_pos, tok = s_tok;
        VecSrc emb_src;
        emb_src.p = nullptr;
        emb_src.emb = a.emb;
        emb_src.tok = tok;
        if (blockIdx.x == 0)   // x = embedding row, for the residual stream
            for (int i = threadIdx.x; i < a.dim / 4; i += blockDim.x)
                __stcg(reinterpret_cast<float4*>(a.x) + i, src_load4(emb_src, i));

        for (int oi = 0; oi < a.nops && ok; oi++) {
            const OpDesc op = a.ops[oi];
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
            const float ss = !nw ? 1.0f
                             : (MODE == MODE_W4A8 ? src_rms_scale_exact(src, op.m.n, red) : src_rms_scale(src, op.m.n, red));
            src_build_digits<MODE>(xf, xs, src, op.m.n, nw, ss);
            __syncthreads();
            DecodeEpi epi{&a, &op, pos, -1e9f, 0u};
            if (!run_op<MODE>(op.m, ring, ring_base, seq, a.ops, a.nops, a.steps, xf, xs, os, a.split_part, a.split_cnt,
                              epi)) {
                set_error(a.step, DEV_COPY_TIMEOUT);
                ok = false;
                break;
            }
            if (op.kind == OP_CLS) cta_argmax(a.argmax, epi.best, epi.best_i, red64);
            if (oi == a.nops - 1 && step == a.steps - 1) break;   // nothing after the last classifier
            if (!grid_barrier(a.step, nbar)) { ok = false; break; }
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
                    attention_layer(a, op.layer, pos, attn);
                if (!grid_barrier(a.step, nbar)) { ok = false; break; }
            }
        }
    }
    ring_drain(ring);
}

// ---------------------------------------------------------------------------
// Standalone matvec y = W x (kernel-level entry points): the same streaming
// and epilogue machinery as one op of the decode kernel.
// ---------------------------------------------------------------------------
struct StandaloneArgs {
    OpDesc op;
    const float* x;
    float* y;
    float* split_part;
    int* split_cnt;
    int P, slot_bytes, xbytes, xs_off;
    int* error;
};

struct StoreEpi {
    float* y;
    int d;
    __device__ __forceinline__ void operator()(int r0, const float* v) {
        for (int r = 0; r < kRB; r++)
            if (r0 + r < d) y[r0 + r] = v[r];
    }
};

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1) k_matvec(StandaloneArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bars[kWarps * 8];
    __shared__ OpSmem os;
    __shared__ OpDesc s_op;
    unsigned char* xf = smem;
    float* xs = reinterpret_cast<float*>(smem + a.xs_off);
    unsigned char* ring_base = smem + a.xbytes;
    if (threadIdx.x == 0) s_op = a.op;
    __syncthreads();
    Ring ring;
    ring_init(ring, ring_base, bars, a.P, a.slot_bytes);
    Seq seq;
    seq_enter(seq, &s_op, 1, 1, MODE, 0, 0);
    for (int i = 0; i < a.P; i++) seq_issue_next(seq, ring, &s_op, 1, 1, MODE);
    pdl_launch_dependents();
    pdl_wait();
    VecSrc src;
    src.p = a.x;
    src.tok = 0;
    src.emb = a.op.m;
    src_build_digits<MODE>(xf, xs, src, a.op.m.n, nullptr, 1.0f);
    __syncthreads();
    StoreEpi epi{a.y, a.op.m.d};
    if (!run_op<MODE>(s_op.m, ring, ring_base, seq, &s_op, 1, 1, xf, xs, os, a.split_part, a.split_cnt, epi))
        if (threadIdx.x == 0) atomicCAS(a.error, 0, DEV_COPY_TIMEOUT);
    ring_drain(ring);
}

}  // namespace aion
