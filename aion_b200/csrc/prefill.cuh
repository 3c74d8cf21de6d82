// Batched prefill: S sequences of T tokens through every layer at once, the
// matrix products on the tensor cores (gemm_tc.cuh).  Row m = s*T + t of
// every activation matrix is token t of sequence s (position t).
//
// Operands of a product C = A B^T reach the GEMM as bf16 with K padded to a
// multiple of 64 (Kp) and split in two parts to keep fp32-like accuracy:
//   A row = [hi(a) | lo(a) | hi(a)],  B row = [hi(b) | hi(b) | lo(b)]
// with hi(v) = bf16(v), lo(v) = bf16(v - hi(v)); the 3*Kp-long dot is
// hi(a)hi(b) + lo(a)hi(b) + hi(a)lo(b), which leaves out lo(a)lo(b), about
// 2^-16 of each product.  Weights are (nibble - 8) * scale from the int4
// tiles (no other copy of them exists); rows and columns past the real
// sizes are zero.
#pragma once

#include <cuda_bf16.h>

#include "decode_step.cuh"

namespace aion {

// A operand row: [hi | lo | hi].
__device__ __forceinline__ void split_store(__nv_bfloat16* row, int kp, int k, float v) {
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    const __nv_bfloat16 lo = __float2bfloat16_rn(v - __bfloat162float(hi));
    row[k] = hi;
    row[kp + k] = lo;
    row[2 * kp + k] = hi;
}
// Eight consecutive values k0..k0+7 (k0 % 8 == 0) of an A row ([hi|lo|hi])
// or a B row ([hi|hi|lo]) as three 16-byte stores.
template <bool B>
__device__ __forceinline__ void split8_store(__nv_bfloat16* row, int kp, int k0, const float (&v)[8]) {
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
        const float2 hf = __bfloat1622float2(h);
        const __nv_bfloat162 l = __floats2bfloat162_rn(v[2 * i] - hf.x, v[2 * i + 1] - hf.y);
        hi[i] = *reinterpret_cast<const uint32_t*>(&h);
        lo[i] = *reinterpret_cast<const uint32_t*>(&l);
    }
    const uint4 H = make_uint4(hi[0], hi[1], hi[2], hi[3]), Lo = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    *reinterpret_cast<uint4*>(row + k0) = H;
    *reinterpret_cast<uint4*>(row + kp + k0) = B ? H : Lo;
    *reinterpret_cast<uint4*>(row + 2 * kp + k0) = B ? Lo : H;
}


// B operand of an int4 matrix: out[n][3*kp] for n < np (zero past the
// matrix), from the tile layout of matvec.cuh.  One thread per (row, 8
// consecutive columns).
__global__ void k_pf_dequant(MatDesc m, int np, int kp, __nv_bfloat16* out) {
    const long long tasks = (long long)np * (kp / 8);
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < tasks;
         i += (long long)gridDim.x * blockDim.x) {
        const int n = (int)(i / (kp / 8)), c8 = (int)(i % (kp / 8));
        const int k0 = c8 * 8;
        __nv_bfloat16* row = out + (size_t)n * 3 * kp;
        float v[8];
        if (n >= m.d || k0 >= m.n) {
#pragma unroll
            for (int e = 0; e < 8; e++) v[e] = 0.0f;
            split8_store<true>(row, kp, k0, v);
            continue;
        }
        const int g = k0 >> 5, j = (k0 & 31) >> 3;   // group, eighth of the group
        const int tr = n % kTR, lr = tr & 7, half = tr >> 3;
        const uint8_t* gp = m.w + (size_t)(n / kTR) * m.tile_bytes + (size_t)g * kGB;
        const float sc = *reinterpret_cast<const float*>(gp + 256 + 8 * lr + 4 * half);
        // elements 8j..8j+7: lanes t0, t0+1 of row tr, low nibbles for j < 2
        const int t0 = (j & 1) * 2, shift = (j >> 1) * 4;
        const uint32_t w0 = *reinterpret_cast<const uint32_t*>(gp + 8 * (4 * lr + t0) + 4 * half);
        const uint32_t w1 = *reinterpret_cast<const uint32_t*>(gp + 8 * (4 * lr + t0 + 1) + 4 * half);
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const uint32_t w = e < 4 ? w0 : w1;
            v[e] = (float)((int)((w >> (8 * (e & 3) + shift)) & 0xF) - 8) * sc;
        }
        split8_store<true>(row, kp, k0, v);
    }
}

// Embedding rows of the prompt tokens: x[m][dim] (src/kernel_simd.c:1032-1040).
__global__ void k_pf_embed(const int32_t* tokens, int mrows, MatDesc emb, int dim, float* x) {
    const int m = blockIdx.x;
    if (m >= mrows) return;
    VecSrc src;
    src.p = nullptr;
    src.emb = emb;
    src.tok = tokens[m];
    for (int i = threadIdx.x; i < dim / 4; i += blockDim.x)
        reinterpret_cast<float4*>(x + (size_t)m * dim)[i] = src_load4(src, i);
}

// A operand of an RMSNorm'd input (src/kernel_simd.c:793-813): row m of
// out from row map[m] (or m) of x; rows >= mrows are zero.
__global__ void k_pf_norm_split(const float* x, const int* map, int mrows, int k, int kp, const float* w,
                                __nv_bfloat16* out) {
    __shared__ float red[32];
    const int m = blockIdx.x;
    __nv_bfloat16* row = out + (size_t)m * 3 * kp;
    if (m >= mrows) {
        const float z[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int i = 8 * threadIdx.x; i < kp; i += 8 * blockDim.x) split8_store<false>(row, kp, i, z);
        return;
    }
    const float* xr = x + (size_t)(map ? map[m] : m) * k;
    float acc = 0.0f;
    for (int i = threadIdx.x; i < k; i += blockDim.x) acc += xr[i] * xr[i];
    acc = warp_sum(acc);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    float tot = 0.0f;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) tot += red[i];
    const float ss = 1.0f / sqrtf(tot / (float)k + 1e-5f);
    for (int i = 8 * threadIdx.x; i < kp; i += 8 * blockDim.x) {
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; e++) v[e] = i + e < k ? (xr[i + e] * ss) * w[i + e] : 0.0f;
        split8_store<false>(row, kp, i, v);
    }
}

// QKV output (ld columns per row) -> RoPE'd q rows, and K / V rows of each
// sequence's cache at positions 0..T-1 (src/kernel_simd.c:1068-1092).
struct PfRopeArgs {
    const float* c;
    int ldc, mrows, T, dim, kv_dim, hs;
    const float *freq_re, *freq_im;   // [pos][hs/2]
    float* q;                         // [mrows][dim]
    float *kcache, *vcache;           // sequence 0, layer l; sequence stride seq_stride
    size_t seq_stride;
};
__global__ void k_pf_rope_kv(PfRopeArgs a) {
    const int m = blockIdx.x;
    if (m >= a.mrows) return;
    const int s = m / a.T, t = m % a.T;
    const float* cr = a.c + (size_t)m * a.ldc;
    float* kc = a.kcache + s * a.seq_stride + (size_t)t * a.kv_dim;
    float* vc = a.vcache + s * a.seq_stride + (size_t)t * a.kv_dim;
    for (int i = 2 * threadIdx.x; i < a.dim + a.kv_dim; i += 2 * blockDim.x) {
        const bool is_q = i < a.dim;
        const int base = is_q ? i : i - a.dim;
        const int hd = base % a.hs;
        const float fr = a.freq_re[(size_t)t * (a.hs / 2) + hd / 2], fi = a.freq_im[(size_t)t * (a.hs / 2) + hd / 2];
        const float v0 = cr[i], v1 = cr[i + 1];
        const float o0 = __fsub_rn(__fmul_rn(v0, fr), __fmul_rn(v1, fi));
        const float o1 = __fadd_rn(__fmul_rn(v0, fi), __fmul_rn(v1, fr));
        float* dst = is_q ? a.q + (size_t)m * a.dim + base : kc + base;
        dst[0] = o0;
        dst[1] = o1;
    }
    for (int i = threadIdx.x; i < a.kv_dim; i += blockDim.x) vc[i] = cr[a.dim + a.kv_dim + i];
}

// Causal attention of every (sequence, head) over its T positions
// (src/kernel_simd.c:1099-1117: scores q.k / sqrt(hs), softmax over
// positions 0..t, weighted sum of V rows), on the tensor cores.  The output
// goes straight into the A operand of WO.
//
// CTA = (query block of 128, head, sequence), longest blocks first; warp w
// holds rows 16w..16w+15 of the block.  Keys come in blocks of 64.  The fp32
// K and V rows of the next block stream into a raw stage with cp.async
// while the current block is processed; at the top of each block the CTA
// converts the raw stage into bf16 hi/lo parts, K as [key][d] and V as
// [d][key], so both are B operands of mma.sync.m16n8k16 read with 32-bit
// loads (K rows padded by 8 elements; V^T words XOR-swizzled, vt_word):
// every fragment read and conversion store hits 32 distinct banks.
// Each product takes three MMAs, hi.hi + lo.hi + hi.lo, as in the prefill
// GEMMs (lo.lo, about 2^-16 of a product, is left out): S = Q K^T with Q's
// fragments held in registers, then an online softmax in fp32 on the S
// fragments (rows g and g + 8 of a lane, the quad's four lanes reduced by
// shuffles), then O += P V with P's fragments taken straight from S's
// accumulator layout.  A warp whose rows all precede the key block skips it.
constexpr int kPfTQ = 128, kPfTK = 64, kPfAttnThreads = 256;
constexpr int kPfKs = kMaxHead + 8;   // K row stride (bf16 elements)
constexpr int kPfVs = kPfTK + 8;      // V^T row stride
constexpr int kPfAttnImage = 2 * (kPfTK * kPfKs + kMaxHead * kPfVs) * 2;   // bf16 K and V^T, hi and lo
constexpr int kPfAttnRaw = 2 * kPfTK * kMaxHead * 4;                        // fp32 K and V rows
constexpr int kPfAttnSmem = kPfAttnImage + kPfAttnRaw;
struct PfAttnArgs {
    const float* q;                   // [mrows][dim]
    const float *kcache, *vcache;     // sequence 0, layer l
    size_t seq_stride;
    int T, dim, kv_dim, hs, kv_mul;
    int kp;
    __nv_bfloat16* out;               // [mpad][3*kp]
};
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// (x, y) as packed bf16 pairs: hi = bf16(v), lo = bf16(v - hi); x in the low half.
__device__ __forceinline__ void split2(float x, float y, uint32_t& hi, uint32_t& lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(x - hf.x, y - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}
// 16-byte cp.async; zero-fills the destination when !valid (nothing is read).
__device__ __forceinline__ void cp_async16_zfill(void* dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
// 32-bit word of V^T row d holding keys 2 kp, 2 kp + 1.  The XOR of the
// pair index with bits 3..5 of d spreads a warp's stores (32 rows d, one
// kp) over 32 banks; a fragment read (rows 8n + g, pairs 8j + t) sees one
// XOR constant, so its 32 lanes still hit 4g + (pair ^ c): 32 banks.
__device__ __forceinline__ int vt_word(int d, int kp) { return d * (kPfVs / 2) + (kp ^ ((d >> 3) & 7)); }
__global__ void __launch_bounds__(kPfAttnThreads, 1) k_pf_attention(PfAttnArgs a) {
    constexpr int NK = kMaxHead / 16, ND = kMaxHead / 8, NT = kPfTK / 8;
    extern __shared__ __align__(16) unsigned char pf_smem[];
    __nv_bfloat16* kh = reinterpret_cast<__nv_bfloat16*>(pf_smem);   // [key][kPfKs]
    __nv_bfloat16* kl = kh + kPfTK * kPfKs;
    __nv_bfloat16* vh = kl + kPfTK * kPfKs;                          // [d][kPfVs], words at vt_word
    __nv_bfloat16* vl = vh + kMaxHead * kPfVs;
    float* rk = reinterpret_cast<float*>(pf_smem + kPfAttnImage);   // raw K rows [kPfTK][hs]
    float* rv = rk + kPfTK * kMaxHead;                               // raw V rows [kPfTK][hs]
    const int nqb = (a.T + kPfTQ - 1) / kPfTQ;
    const int qb = nqb - 1 - (int)blockIdx.x, h = blockIdx.y, s = blockIdx.z;
    const int hs = a.hs, nk = hs / 16, nd = hs / 8, h4 = hs / 4, h2 = hs / 2, kvh = h / a.kv_mul;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int q0 = qb * kPfTQ;
    const int wr0 = q0 + 16 * warp;                  // the warp's first row
    const int r0 = wr0 + g, r1 = r0 + 8;             // this lane's rows (positions)
    const int t_last = min(a.T, q0 + kPfTQ) - 1;     // the last key any row of the CTA sees
    const float* kc = a.kcache + s * a.seq_stride + (size_t)kvh * hs;
    const float* vc = a.vcache + s * a.seq_stride + (size_t)kvh * hs;
    const float2 z2 = make_float2(0.0f, 0.0f);

    // Raw stage: fp32 K and V rows of keys k0..k0+63 (zero past t_last).
    auto stage_raw = [&](int k0) {
        for (int i = threadIdx.x; i < kPfTK * h4; i += kPfAttnThreads) {
            const int key = i / h4, d = 4 * (i - key * h4);
            const bool in = k0 + key <= t_last;
            const size_t off = (size_t)(in ? k0 + key : 0) * a.kv_dim + d;
            cp_async16_zfill(rk + key * hs + d, kc + off, in);
            cp_async16_zfill(rv + key * hs + d, vc + off, in);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    stage_raw(0);

    // Q arrives scaled by log2(e) / sqrt(hs): the scores are then in base-2
    // units and the softmax uses exp2 (the same weights up to rounding).
    const float qscale = 1.4426950408889634f / sqrtf((float)hs);
    uint32_t qh[NK][4], ql[NK][4];
    {
        const float* q0p = a.q + ((size_t)s * a.T + min(r0, a.T - 1)) * a.dim + h * hs;
        const float* q1p = a.q + ((size_t)s * a.T + min(r1, a.T - 1)) * a.dim + h * hs;
#pragma unroll
        for (int kk = 0; kk < NK; kk++) {
            if (kk < nk) {
                const int c = 16 * kk + 2 * t;
                const float2 x0 = r0 < a.T ? *reinterpret_cast<const float2*>(q0p + c) : z2;
                const float2 x1 = r1 < a.T ? *reinterpret_cast<const float2*>(q1p + c) : z2;
                const float2 x2 = r0 < a.T ? *reinterpret_cast<const float2*>(q0p + c + 8) : z2;
                const float2 x3 = r1 < a.T ? *reinterpret_cast<const float2*>(q1p + c + 8) : z2;
                split2(x0.x * qscale, x0.y * qscale, qh[kk][0], ql[kk][0]);
                split2(x1.x * qscale, x1.y * qscale, qh[kk][1], ql[kk][1]);
                split2(x2.x * qscale, x2.y * qscale, qh[kk][2], ql[kk][2]);
                split2(x3.x * qscale, x3.y * qscale, qh[kk][3], ql[kk][3]);
            }
        }
    }
    float o[ND][4];
#pragma unroll
    for (int n = 0; n < ND; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;   // l: this lane's share of the row sums

    for (int k0 = 0; k0 <= t_last; k0 += kPfTK) {
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        __syncthreads();   // the raw stage holds block k0; the previous image is read
        for (int i = threadIdx.x; i < kPfTK * h4; i += kPfAttnThreads) {
            const int key = i / h4, d = 4 * (i - key * h4);
            const float4 v = *reinterpret_cast<const float4*>(rk + key * hs + d);
            uint32_t h01, l01, h23, l23;
            split2(v.x, v.y, h01, l01);
            split2(v.z, v.w, h23, l23);
            *reinterpret_cast<uint2*>(kh + key * kPfKs + d) = make_uint2(h01, h23);
            *reinterpret_cast<uint2*>(kl + key * kPfKs + d) = make_uint2(l01, l23);
        }
        for (int i = threadIdx.x; i < (kPfTK / 2) * h2; i += kPfAttnThreads) {
            const int kp = i / h2, d = 2 * (i - kp * h2);
            const float2 va = *reinterpret_cast<const float2*>(rv + (2 * kp) * hs + d);
            const float2 vb = *reinterpret_cast<const float2*>(rv + (2 * kp + 1) * hs + d);
            uint32_t hi, lo;
            split2(va.x, vb.x, hi, lo);
            reinterpret_cast<uint32_t*>(vh)[vt_word(d, kp)] = hi;
            reinterpret_cast<uint32_t*>(vl)[vt_word(d, kp)] = lo;
            split2(va.y, vb.y, hi, lo);
            reinterpret_cast<uint32_t*>(vh)[vt_word(d + 1, kp)] = hi;
            reinterpret_cast<uint32_t*>(vl)[vt_word(d + 1, kp)] = lo;
        }
        __syncthreads();   // the image is complete; the raw stage is free
        if (k0 + kPfTK <= t_last) stage_raw(k0 + kPfTK);
        if (k0 > wr0 + 15) continue;   // every row of this warp precedes the block

        // S = Q K^T: 16 rows x 64 keys per warp.
        float sc[NT][4];
#pragma unroll
        for (int n = 0; n < NT; n++) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.0f;
#pragma unroll
        for (int kk = 0; kk < NK; kk++) {
            if (kk < nk) {
#pragma unroll
                for (int n = 0; n < NT; n++) {
                    const int off = (n * 8 + g) * kPfKs + 16 * kk + 2 * t;
                    const uint32_t bh0 = *reinterpret_cast<const uint32_t*>(kh + off);
                    const uint32_t bh1 = *reinterpret_cast<const uint32_t*>(kh + off + 8);
                    const uint32_t bl0 = *reinterpret_cast<const uint32_t*>(kl + off);
                    const uint32_t bl1 = *reinterpret_cast<const uint32_t*>(kl + off + 8);
                    mma_bf16(sc[n], qh[kk], bh0, bh1);
                    mma_bf16(sc[n], ql[kk], bh0, bh1);
                    mma_bf16(sc[n], qh[kk], bl0, bl1);
                }
            }
        }
        // Online softmax: causal mask (blocks reaching past the warp's first
        // row only), block max per row.
        if (k0 + kPfTK - 1 > wr0) {
#pragma unroll
            for (int n = 0; n < NT; n++) {
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    const int key = k0 + n * 8 + 2 * t + e;
                    if (key > r0) sc[n][e] = -INFINITY;
                    if (key > r1) sc[n][2 + e] = -INFINITY;
                }
            }
        }
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int n = 0; n < NT; n++) {
            mx0 = fmaxf(mx0, fmaxf(sc[n][0], sc[n][1]));
            mx1 = fmaxf(mx1, fmaxf(sc[n][2], sc[n][3]));
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        // Key 0 is seen by every row in the first block, so the running maxima
        // are finite from then on; a row with no key in this block keeps its max.
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        const float c0 = exp2f(m0 - mn0), c1 = exp2f(m1 - mn1);
        l0 *= c0;
        l1 *= c1;
#pragma unroll
        for (int n = 0; n < ND; n++) {
            o[n][0] *= c0;
            o[n][1] *= c0;
            o[n][2] *= c1;
            o[n][3] *= c1;
        }
#pragma unroll
        for (int n = 0; n < NT; n++) {
#pragma unroll
            for (int e = 0; e < 2; e++) {
                sc[n][e] = exp2f(sc[n][e] - mn0);
                sc[n][2 + e] = exp2f(sc[n][2 + e] - mn1);
                l0 += sc[n][e];
                l1 += sc[n][2 + e];
            }
        }
        m0 = mn0;
        m1 = mn1;
        // O += P V, P's 16 x 16 fragments from the accumulators of S tiles 2j, 2j + 1.
#pragma unroll
        for (int j = 0; j < kPfTK / 16; j++) {
            uint32_t ph[4], pl[4];
            split2(sc[2 * j][0], sc[2 * j][1], ph[0], pl[0]);
            split2(sc[2 * j][2], sc[2 * j][3], ph[1], pl[1]);
            split2(sc[2 * j + 1][0], sc[2 * j + 1][1], ph[2], pl[2]);
            split2(sc[2 * j + 1][2], sc[2 * j + 1][3], ph[3], pl[3]);
#pragma unroll
            for (int n = 0; n < ND; n++) {
                if (n < nd) {
                    const int w0 = vt_word(n * 8 + g, 8 * j + t), w1 = vt_word(n * 8 + g, 8 * j + 4 + t);
                    const uint32_t bh0 = reinterpret_cast<const uint32_t*>(vh)[w0];
                    const uint32_t bh1 = reinterpret_cast<const uint32_t*>(vh)[w1];
                    const uint32_t bl0 = reinterpret_cast<const uint32_t*>(vl)[w0];
                    const uint32_t bl1 = reinterpret_cast<const uint32_t*>(vl)[w1];
                    mma_bf16(o[n], ph, bh0, bh1);
                    mma_bf16(o[n], pl, bh0, bh1);
                    mma_bf16(o[n], ph, bl0, bl1);
                }
            }
        }
    }
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    const float inv0 = 1.0f / l0, inv1 = 1.0f / l1;
#pragma unroll
    for (int half = 0; half < 2; half++) {
        const int r = half ? r1 : r0;
        if (r >= a.T) continue;
        const float inv = half ? inv1 : inv0;
        __nv_bfloat16* row = a.out + ((size_t)s * a.T + r) * 3 * a.kp;
#pragma unroll
        for (int n = 0; n < ND; n++) {
            if (n < nd) {
                const int col = h * hs + n * 8 + 2 * t;
                uint32_t hi, lo;
                split2(o[n][2 * half] * inv, o[n][2 * half + 1] * inv, hi, lo);
                *reinterpret_cast<uint32_t*>(row + col) = hi;
                *reinterpret_cast<uint32_t*>(row + a.kp + col) = lo;
                *reinterpret_cast<uint32_t*>(row + 2 * a.kp + col) = hi;
            }
        }
    }
}

// x[m][0:dim] += c[m][0:dim] (residual, src/kernel_simd.c:1126,1153).
__global__ void k_pf_residual(float* x, const float* c, int ldc, int mrows, int dim) {
    const int m = blockIdx.x;
    if (m >= mrows) return;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) x[(size_t)m * dim + i] += c[(size_t)m * ldc + i];
}

// SwiGLU of the W13 output (rows interleaved per quad: w1[2j], w1[2j+1],
// w3[2j], w3[2j+1]) into the A operand of W2 (src/kernel_simd.c:836-843).
__global__ void k_pf_swiglu_split(const float* c, int ldc, int mrows, int hidden, int kp, __nv_bfloat16* out) {
    const int m = blockIdx.x;
    __nv_bfloat16* row = out + (size_t)m * 3 * kp;
    for (int j0 = 8 * threadIdx.x; j0 < kp; j0 += 8 * blockDim.x) {
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const int j = j0 + e;
            v[e] = 0.0f;
            if (m < mrows && j < hidden) {
                const int col = 4 * (j >> 1) + (j & 1);
                const float g = c[(size_t)m * ldc + col], u = c[(size_t)m * ldc + col + 2];
                v[e] = (g / (1.0f + expf(-g))) * u;
            }
        }
        split8_store<false>(row, kp, j0, v);
    }
}

}  // namespace aion
