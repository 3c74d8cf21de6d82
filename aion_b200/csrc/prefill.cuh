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

// Causal attention of every (sequence, head) over its T positions, online
// softmax, fp32 on the CUDA cores; the output goes straight into the A
// operand of WO.  CTA = (query block of 32, head, sequence); warp w takes
// queries 4w..4w+3 of the block; keys come in blocks of 32 through shared
// memory (K rows padded by one float against bank conflicts).  Dynamic
// shared memory: kPfAttnSmem bytes.
constexpr int kPfQB = 32, kPfKB = 32;
constexpr int kPfAttnSmem = (kPfQB * kMaxHead + kPfKB * (kMaxHead + 1) + kPfKB * kMaxHead) * 4;
struct PfAttnArgs {
    const float* q;                   // [mrows][dim]
    const float *kcache, *vcache;     // sequence 0, layer l
    size_t seq_stride;
    int T, dim, kv_dim, hs, kv_mul;
    int kp;
    __nv_bfloat16* out;               // [mpad][3*kp]
};
__global__ void __launch_bounds__(256) k_pf_attention(PfAttnArgs a) {
    extern __shared__ float pf_smem[];
    float(*sq)[kMaxHead] = reinterpret_cast<float(*)[kMaxHead]>(pf_smem);
    float(*sk)[kMaxHead + 1] = reinterpret_cast<float(*)[kMaxHead + 1]>(pf_smem + kPfQB * kMaxHead);
    float(*sv)[kMaxHead] = reinterpret_cast<float(*)[kMaxHead]>(pf_smem + kPfQB * kMaxHead + kPfKB * (kMaxHead + 1));
    const int qb = blockIdx.x, h = blockIdx.y, s = blockIdx.z;
    const int hs = a.hs, kvh = h / a.kv_mul;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t_first = qb * kPfQB, t_last = min(a.T, t_first + kPfQB) - 1;
    const float* kc = a.kcache + s * a.seq_stride + (size_t)kvh * hs;
    const float* vc = a.vcache + s * a.seq_stride + (size_t)kvh * hs;
    for (int i = threadIdx.x; i < kPfQB * hs; i += blockDim.x) {
        const int r = i / hs, d = i % hs, t = t_first + r;
        sq[r][d] = t < a.T ? a.q[((size_t)s * a.T + t) * a.dim + h * hs + d] : 0.0f;
    }
    const float rs = sqrtf((float)hs);
    float mx[4], l[4], acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        mx[i] = -INFINITY;
        l[i] = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;
    }
    for (int k0 = 0; k0 <= t_last; k0 += kPfKB) {
        __syncthreads();
        for (int i = threadIdx.x; i < kPfKB * hs; i += blockDim.x) {
            const int r = i / hs, d = i % hs, t = k0 + r;
            sk[r][d] = t <= t_last ? kc[(size_t)t * a.kv_dim + d] : 0.0f;
            sv[r][d] = t <= t_last ? vc[(size_t)t * a.kv_dim + d] : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int r = 4 * warp + i, t = t_first + r;
            if (t > t_last) continue;                       // uniform per warp
            const int key = k0 + lane;
            float sc = -INFINITY;
            if (key <= t) {
                float d = 0.0f;
                for (int j = 0; j < hs; j++) d = fmaf(sq[r][j], sk[lane][j], d);
                sc = d / rs;
            }
            const float bm = warp_max(sc);
            const float mnew = fmaxf(mx[i], bm);
            const float p = key <= t ? expf(sc - mnew) : 0.0f;
            const float corr = expf(mx[i] - mnew);
            l[i] = l[i] * corr + warp_sum(p);
#pragma unroll
            for (int j = 0; j < 4; j++) acc[i][j] *= corr;
            for (int kk = 0; kk < kPfKB; kk++) {
                const float pk = __shfl_sync(0xffffffffu, p, kk);   // every lane takes part
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int d = lane + 32 * j;
                    if (d < hs) acc[i][j] = fmaf(pk, sv[kk][d], acc[i][j]);
                }
            }
            mx[i] = mnew;
        }
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int r = 4 * warp + i, t = t_first + r;
        if (t > t_last) continue;
        __nv_bfloat16* row = a.out + ((size_t)s * a.T + t) * 3 * a.kp;
        const float inv = 1.0f / l[i];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int d = lane + 32 * j;
            if (d < hs) split_store(row, a.kp, h * hs + d, acc[i][j] * inv);
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
