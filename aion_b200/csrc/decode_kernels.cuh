// Device code of the int4 Llama-2 decode path for sm_100a.
//
// Weight layout in HBM ("tiled"): a matrix [d][n] (n % 32 == 0) is stored as
// ceil(d / kRB) tiles of kRB consecutive rows.  Tile t occupies kRB*n*5/8
// bytes: first the fp32 group scales of its rows, row-major [kRB][n/32], then
// the packed nibbles of its rows, row-major [kRB][n/2], each row's bytes in
// the quantize.c order (low nibble = even element, stored value q + 8).
// Every tile starts on a 16-byte boundary and every group is one 16-byte
// vector, so a warp reading consecutive groups of a row issues fully
// coalesced 128-bit loads.  Rows past d (padding) have scale 0, nibbles 0x88.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace aion {

constexpr int kRB = 4;           // rows per tile
constexpr int kMvThreads = 256;  // threads per matvec CTA
constexpr int kMvWarps = kMvThreads / 32;

// Argmax over logits is reduced on the device through one 64-bit key per
// sequence: (order-preserving float bits << 32) | (0xFFFFFFFF - index), so a
// max over keys picks the largest logit and, among equal logits, the
// smallest index -- the first-max rule of the reference greedy loop
// (src/kernel_simd.c:1236-1243).  The initial key encodes (-1e9, index 0).
__host__ __device__ inline uint32_t order_bits(float f) {
    uint32_t u;
#ifdef __CUDA_ARCH__
    u = __float_as_uint(f);
#else
    memcpy(&u, &f, 4);
#endif
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__host__ __device__ inline unsigned long long argmax_key(float v, uint32_t idx) {
    return ((unsigned long long)order_bits(v) << 32) | (unsigned long long)(0xFFFFFFFFu - idx);
}
__host__ __device__ inline uint32_t key_index(unsigned long long k) {
    return 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull);
}

// Per-step state shared by the kernels of one decode step.  The embedding
// kernel starts a step: it takes pos from pos_next, the token from
// forced_token (>= 0) or from the previous step's argmax key, records it in
// the token history and publishes pos/token for the rest of the step.
struct StepState {
    int32_t pos_next;
    int32_t forced_token;
    int32_t pos;
    int32_t token;
    int32_t error;         // nonzero: a kernel rejected its input (bad token / position)
    int32_t pad[3];
};

// ---------------------------------------------------------------------------
// Programmatic dependent launch helpers (griddepcontrol, sm_90+).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Bulk prefetch of [p, p + bytes) into L2 (bytes a multiple of 16, p 16-aligned).
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Streaming 128-bit load: weights are read once per step, keep them out of L1.
__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ---------------------------------------------------------------------------
// int4 -> fp32 dequant-dot for one 32-bit word (8 nibbles, element e at bits
// 4e..4e+3).  A nibble n placed in the low mantissa bits of 2^23 gives the
// float 2^23 + n * 16^p exactly (p = its nibble position inside the mantissa);
// subtracting 2^23 + 8 * 16^p yields (n - 8) * 16^p exactly.  Elements 0..4
// are masked in place (p = 0..4), elements 5..7 after one shift by 12 bits
// (p = 2..4).  The activations are pre-scaled by 16^-p (exact powers of two),
// so each product is q * x.  Two elements per packed fp32x2 instruction.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float2 dq_dot8(uint32_t w, float4 xa, float4 xb, float2 acc) {
    const uint32_t M = 0x4B000000u;
    const uint32_t w2 = w >> 12;
    const float2 f01 = make_float2(__uint_as_float((w & 0xFu) | M), __uint_as_float((w & 0xF0u) | M));
    const float2 f23 = make_float2(__uint_as_float((w & 0xF00u) | M), __uint_as_float((w & 0xF000u) | M));
    const float2 f45 = make_float2(__uint_as_float((w & 0xF0000u) | M), __uint_as_float((w2 & 0xF00u) | M));
    const float2 f67 = make_float2(__uint_as_float((w2 & 0xF000u) | M), __uint_as_float((w2 & 0xF0000u) | M));
    const float2 c01 = make_float2(-8388616.0f, -8388736.0f);   // 2^23 + 8*16^0, 2^23 + 8*16^1
    const float2 c23 = make_float2(-8390656.0f, -8421376.0f);   // 2^23 + 8*16^2, 2^23 + 8*16^3
    const float2 c45 = make_float2(-8912896.0f, -8390656.0f);   // 2^23 + 8*16^4, 2^23 + 8*16^2
    const float2 c67 = make_float2(-8421376.0f, -8912896.0f);   // 2^23 + 8*16^3, 2^23 + 8*16^4
    acc = __ffma2_rn(__fadd2_rn(f01, c01), make_float2(xa.x, xa.y), acc);
    acc = __ffma2_rn(__fadd2_rn(f23, c23), make_float2(xa.z, xa.w), acc);
    acc = __ffma2_rn(__fadd2_rn(f45, c45), make_float2(xb.x, xb.y), acc);
    acc = __ffma2_rn(__fadd2_rn(f67, c67), make_float2(xb.z, xb.w), acc);
    return acc;
}

// Pre-scale factor of element e (0..7) of an 8-element word.
__device__ __forceinline__ float prescale(int e) {
    // 16^-p for p = 0,1,2,3,4,2,3,4
    const float t[8] = {1.0f, 0.0625f, 0.00390625f, 0.000244140625f, 1.52587890625e-05f,
                        0.00390625f, 0.000244140625f, 1.52587890625e-05f};
    return t[e];
}

// Index (in float4 units) of float4 j (0..7) of group g inside the permuted
// shared-memory copy of x: lane l reading group l + 32*i touches consecutive
// 16-byte words for every j (no bank conflicts).
__device__ __forceinline__ int xperm(int g, int j) { return ((g >> 5) * 8 + j) * 32 + (g & 31); }

// ---------------------------------------------------------------------------
// Matvec kernel arguments.  One struct for all fused variants.
// ---------------------------------------------------------------------------
enum Prologue { PRO_PLAIN = 0, PRO_RMSNORM = 1 };
enum Epilogue { EPI_STORE = 0, EPI_RESIDUAL = 1, EPI_QKV = 2, EPI_SWIGLU = 3, EPI_LOGITS = 4 };
enum Mode { MODE_W4A16 = 0, MODE_W4A8 = 1 };

struct MatvecArgs {
    const uint8_t* w;        // tiled matrix
    long long tile_bytes;
    int n;                   // columns
    int ntiles;              // tiles (rows padded to kRB)
    int d;                   // logical rows
    const float* x;          // input [n]
    const float* norm_w;     // RMSNorm weight [n] (PRO_RMSNORM)
    float* y;                // output (STORE / RESIDUAL / LOGITS / SWIGLU)
    // EPI_QKV
    float* q_out;
    float* kcache;           // layer base, [max_pos][kv_dim]
    float* vcache;
    const float* freq_re;    // [seq_len][head_size/2]
    const float* freq_im;
    int dim, kv_dim, head_size;
    // EPI_LOGITS
    unsigned long long* argmax;
    StepState* step;
    int prefetch_tiles;      // tiles of this CTA to prefetch into L2 before the dependency wait
};

// Shared-memory bytes of the matvec kernel for n columns.
__host__ __device__ inline int matvec_smem_bytes(int n, int mode) {
    int G = n / 32;
    int chunks = (G + 31) / 32;
    if (mode == MODE_W4A16) return chunks * 8 * 32 * 16;
    return chunks * 2 * 32 * 16 + chunks * 32 * 4;   // permuted int8 x + per-group scales
}

// Block-wide sum (all threads receive the result).
__device__ __forceinline__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = (lane < (int)(blockDim.x >> 5)) ? red[lane] : 0.0f;
    return warp_sum(t);
}

// Builds the (optionally RMS-normalised) input in shared memory.
// W4A16: x' = pre-scaled fp32, permuted per xperm().
// W4A8: per-32 int8 quantization, bit-exact with quantize_activations_neon
// (src/kernel_simd.c:186-227): amax; scale = 127/amax (amax > 1e-9) else 1;
// stored scale amax/127 (else 1); q = round-half-away(x * scale).  The int8
// values of each 8-element word are stored as [e0 e2 e4 e6][e1 e3 e5 e7] to
// match the nibble split of dq_dot_i8().
template <int MODE, int PRO>
__device__ __forceinline__ void build_input(const MatvecArgs& a, unsigned char* smem, float* red) {
    const int n = a.n, G = n / 32;
    float ss = 1.0f;
    if (PRO == PRO_RMSNORM) {
        float s = 0.0f;
        for (int i = threadIdx.x; i < n / 4; i += blockDim.x) {
            float4 v = reinterpret_cast<const float4*>(a.x)[i];
            s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
        s = block_sum(s, red);
        // rmsnorm (src/kernel_simd.c:802-803): mean, + 1e-5, 1/sqrtf
        ss = 1.0f / sqrtf(__fdiv_rn(s, (float)n) + 1e-5f);
    }
    if (MODE == MODE_W4A16) {
        float4* xs4 = reinterpret_cast<float4*>(smem);
        for (int i = threadIdx.x; i < n / 4; i += blockDim.x) {
            float4 v = reinterpret_cast<const float4*>(a.x)[i];
            if (PRO == PRO_RMSNORM) {
                float4 wv = reinterpret_cast<const float4*>(a.norm_w)[i];
                v.x = __fmul_rn(__fmul_rn(v.x, ss), wv.x);
                v.y = __fmul_rn(__fmul_rn(v.y, ss), wv.y);
                v.z = __fmul_rn(__fmul_rn(v.z, ss), wv.z);
                v.w = __fmul_rn(__fmul_rn(v.w, ss), wv.w);
            }
            const int e0 = (i & 1) * 4;
            v.x *= prescale(e0 + 0);
            v.y *= prescale(e0 + 1);
            v.z *= prescale(e0 + 2);
            v.w *= prescale(e0 + 3);
            xs4[xperm(i >> 3, i & 7)] = v;
        }
    } else {
        const int chunks = (G + 31) / 32;
        uint4* qx = reinterpret_cast<uint4*>(smem);
        float* xsc = reinterpret_cast<float*>(smem + chunks * 2 * 32 * 16);
        for (int g = threadIdx.x; g < G; g += blockDim.x) {
            float v[32];
            const float4* src = reinterpret_cast<const float4*>(a.x) + g * 8;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                float4 t = src[j];
                v[4 * j] = t.x; v[4 * j + 1] = t.y; v[4 * j + 2] = t.z; v[4 * j + 3] = t.w;
            }
            if (PRO == PRO_RMSNORM) {
                const float4* wsrc = reinterpret_cast<const float4*>(a.norm_w) + g * 8;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    float4 t = wsrc[j];
                    v[4 * j] = __fmul_rn(__fmul_rn(v[4 * j], ss), t.x);
                    v[4 * j + 1] = __fmul_rn(__fmul_rn(v[4 * j + 1], ss), t.y);
                    v[4 * j + 2] = __fmul_rn(__fmul_rn(v[4 * j + 2], ss), t.z);
                    v[4 * j + 3] = __fmul_rn(__fmul_rn(v[4 * j + 3], ss), t.w);
                }
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
                    int qe = (int)roundf(__fmul_rn(v[8 * wd + 2 * b], scale));
                    int qo = (int)roundf(__fmul_rn(v[8 * wd + 2 * b + 1], scale));
                    ev |= (uint32_t)(qe & 0xFF) << (8 * b);
                    od |= (uint32_t)(qo & 0xFF) << (8 * b);
                }
                words[2 * wd] = ev;
                words[2 * wd + 1] = od;
            }
            const int ch = g >> 5, l = g & 31;
            qx[(ch * 2 + 0) * 32 + l] = make_uint4(words[0], words[1], words[2], words[3]);
            qx[(ch * 2 + 1) * 32 + l] = make_uint4(words[4], words[5], words[6], words[7]);
        }
    }
}

// int4 x int8 dot of one 8-element word, returned times 16: the nibbles are
// moved to the high half of each byte and XORed with 0x80, which yields the
// signed byte 16 * (n - 8).
__device__ __forceinline__ int dq_dot_i8(uint32_t w, uint32_t xe, uint32_t xo, int acc) {
    const uint32_t lo = ((w << 4) & 0xF0F0F0F0u) ^ 0x80808080u;   // elements 0,2,4,6
    const uint32_t hi = (w & 0xF0F0F0F0u) ^ 0x80808080u;          // elements 1,3,5,7
    acc = __dp4a((int)lo, (int)xe, acc);
    acc = __dp4a((int)hi, (int)xo, acc);
    return acc;
}

// Epilogue for one finished tile (rows r0..r0+kRB-1, values v[]).  Runs on
// lane 0 of the warp.
template <int EPI>
__device__ __forceinline__ void epilogue(const MatvecArgs& a, int r0, const float* v, float& best, uint32_t& best_i) {
    if (EPI == EPI_STORE) {
        for (int r = 0; r < kRB; r++) if (r0 + r < a.d) a.y[r0 + r] = v[r];
    } else if (EPI == EPI_RESIDUAL) {
        for (int r = 0; r < kRB; r++) if (r0 + r < a.d) a.y[r0 + r] += v[r];
    } else if (EPI == EPI_LOGITS) {
        for (int r = 0; r < kRB; r++)
            if (r0 + r < a.d) {
                a.y[r0 + r] = v[r];
                if (v[r] > best) { best = v[r]; best_i = (uint32_t)(r0 + r); }
            }
    } else if (EPI == EPI_SWIGLU) {
        // tile rows: w1[2t], w1[2t+1], w3[2t], w3[2t+1] -> hb[2t], hb[2t+1]
        // swiglu (src/kernel_simd.c:836-841): v / (1 + e^-v) * w3x
        const int h0 = r0 / 2;
        for (int r = 0; r < 2; r++)
            if (h0 + r < a.d) {
                float g = v[r];
                float s = __fdiv_rn(g, 1.0f + expf(-g));
                a.y[h0 + r] = __fmul_rn(s, v[2 + r]);
            }
    } else if (EPI == EPI_QKV) {
        const int pos = a.step->pos;
        const int hs = a.head_size;
        if (r0 < a.dim + a.kv_dim) {
            // RoPE on adjacent pairs (src/kernel_simd.c:1068-1085)
            const bool is_q = r0 < a.dim;
            const int base = is_q ? r0 : r0 - a.dim;
            float out[kRB];
            for (int r = 0; r < kRB; r += 2) {
                const int i = base + r;
                const int hd = i % hs;
                const float fr = a.freq_re[pos * (hs / 2) + hd / 2];
                const float fi = a.freq_im[pos * (hs / 2) + hd / 2];
                out[r] = __fsub_rn(__fmul_rn(v[r], fr), __fmul_rn(v[r + 1], fi));
                out[r + 1] = __fadd_rn(__fmul_rn(v[r], fi), __fmul_rn(v[r + 1], fr));
            }
            float* dst = is_q ? a.q_out + base : a.kcache + (size_t)pos * a.kv_dim + base;
            for (int r = 0; r < kRB; r++) dst[r] = out[r];
        } else {
            const int base = r0 - a.dim - a.kv_dim;
            float* dst = a.vcache + (size_t)pos * a.kv_dim + base;
            for (int r = 0; r < kRB; r++) dst[r] = v[r];
        }
    }
}

// ---------------------------------------------------------------------------
// Batch-1 matvec over the tiled layout, with fused prologue / epilogue.
// Each warp owns whole tiles (kRB rows); lanes stride over the row's groups
// (lane l takes groups l, l+32, ...); weights stream through 128-bit loads,
// double-buffered in registers; partial row sums reduce with warp shuffles.
// ---------------------------------------------------------------------------
template <int MODE, int PRO, int EPI>
__global__ void __launch_bounds__(kMvThreads) k_matvec(MatvecArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ float red[32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = a.n / 32;
    const int gw = blockIdx.x * kMvWarps + warp;
    const int nw = gridDim.x * kMvWarps;

    // Weights do not depend on the previous kernel: pull this CTA's first
    // tiles into L2 while the producer of x is still finishing.
    if (threadIdx.x == 0 && a.prefetch_tiles > 0) {
        const int t0 = blockIdx.x * kMvWarps;
        int cnt = min(a.prefetch_tiles, a.ntiles - t0);
        if (cnt > 0) prefetch_l2(a.w + (size_t)t0 * a.tile_bytes, (uint32_t)(cnt * a.tile_bytes));
    }
    pdl_launch_dependents();
    pdl_wait();

    build_input<MODE, PRO>(a, smem, red);
    __syncthreads();

    float best = -1e9f;
    uint32_t best_i = 0;
    const int scale_bytes = kRB * G * 4;

    for (int t = gw; t < a.ntiles; t += nw) {
        const uint8_t* base = a.w + (size_t)t * a.tile_bytes;
        const float* sc = reinterpret_cast<const float*>(base);
        const uint4* pk = reinterpret_cast<const uint4*>(base + scale_bytes);
        float acc[kRB];
#pragma unroll
        for (int r = 0; r < kRB; r++) acc[r] = 0.0f;

        if (MODE == MODE_W4A16) {
            const float4* xs4 = reinterpret_cast<const float4*>(smem);
            uint4 wcur[kRB];
            float scur[kRB];
            int g = lane;
            if (g < G) {
#pragma unroll
                for (int r = 0; r < kRB; r++) { wcur[r] = ldg_stream(pk + r * G + g); scur[r] = __ldg(sc + r * G + g); }
            }
            for (; g < G; g += 32) {
                uint4 wnext[kRB];
                float snext[kRB];
                const int gn = g + 32;
                if (gn < G) {
#pragma unroll
                    for (int r = 0; r < kRB; r++) { wnext[r] = ldg_stream(pk + r * G + gn); snext[r] = __ldg(sc + r * G + gn); }
                }
                float4 xv[8];
#pragma unroll
                for (int j = 0; j < 8; j++) xv[j] = xs4[xperm(g, j)];
#pragma unroll
                for (int r = 0; r < kRB; r++) {
                    float2 p = make_float2(0.0f, 0.0f);
                    p = dq_dot8(wcur[r].x, xv[0], xv[1], p);
                    p = dq_dot8(wcur[r].y, xv[2], xv[3], p);
                    p = dq_dot8(wcur[r].z, xv[4], xv[5], p);
                    p = dq_dot8(wcur[r].w, xv[6], xv[7], p);
                    acc[r] = fmaf(scur[r], p.x + p.y, acc[r]);
                }
                if (gn < G) {
#pragma unroll
                    for (int r = 0; r < kRB; r++) { wcur[r] = wnext[r]; scur[r] = snext[r]; }
                }
            }
#pragma unroll
            for (int r = 0; r < kRB; r++) acc[r] = warp_sum(acc[r]);
        } else {
            // W4A8: exact int32 group dots, then the reference's epilogue
            // row += (float)dot * (w_scale * x_scale), sequential over the
            // groups of the row in order (src/kernel_simd.c:250-335).
            const int chunks = (G + 31) / 32;
            const uint4* qx = reinterpret_cast<const uint4*>(smem);
            const float* xsc = reinterpret_cast<const float*>(smem + chunks * 2 * 32 * 16);
            for (int c = 0; c < chunks; c++) {
                const int g = c * 32 + lane;
                float prod[kRB];
                if (g < G) {
                    const uint4 xa = qx[(c * 2 + 0) * 32 + lane];
                    const uint4 xb = qx[(c * 2 + 1) * 32 + lane];
                    const float xscale = xsc[g];
#pragma unroll
                    for (int r = 0; r < kRB; r++) {
                        const uint4 w = ldg_stream(pk + r * G + g);
                        int s16 = 0;
                        s16 = dq_dot_i8(w.x, xa.x, xa.y, s16);
                        s16 = dq_dot_i8(w.y, xa.z, xa.w, s16);
                        s16 = dq_dot_i8(w.z, xb.x, xb.y, s16);
                        s16 = dq_dot_i8(w.w, xb.z, xb.w, s16);
                        const int dot = s16 >> 4;
                        const float comb = __fmul_rn(__ldg(sc + r * G + g), xscale);
                        prod[r] = __fmul_rn((float)dot, comb);
                    }
                } else {
#pragma unroll
                    for (int r = 0; r < kRB; r++) prod[r] = 0.0f;
                }
                const int cnt = min(32, G - c * 32);
                for (int j = 0; j < cnt; j++) {
#pragma unroll
                    for (int r = 0; r < kRB; r++) acc[r] = __fadd_rn(acc[r], __shfl_sync(0xffffffffu, prod[r], j));
                }
            }
        }
        if (lane == 0) epilogue<EPI>(a, t * kRB, acc, best, best_i);
    }
    if (EPI == EPI_LOGITS && lane == 0 && best_i != 0xFFFFFFFFu) {
        if (best > -1e9f) atomicMax(a.argmax, argmax_key(best, best_i));
    }
}

// ---------------------------------------------------------------------------
// Step start: resolve the token, publish pos/token, record history, reset the
// argmax key, and dequantize the embedding row (src/kernel_simd.c:1032-1040):
// x[i] = (int8)(nibble - 8) * scale[i / 32].
// ---------------------------------------------------------------------------
struct EmbedArgs {
    const uint8_t* emb;          // tiled [vocab][dim]
    long long tile_bytes;
    int dim, vocab, max_pos;
    float* x;
    StepState* step;
    unsigned long long* argmax;
    int32_t* history;            // [max_pos] input token of each position
};

__global__ void __launch_bounds__(256) k_embed(EmbedArgs a) {
    __shared__ int s_tok;
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x == 0) {
        StepState st = *a.step;
        int pos = st.pos_next;
        int tok = st.forced_token >= 0 ? st.forced_token : (int)key_index(*a.argmax);
        if (tok < 0 || tok >= a.vocab || pos < 0 || pos >= a.max_pos) {
            a.step->error = 1;
            tok = 0;
            pos = pos < 0 ? 0 : (pos >= a.max_pos ? a.max_pos - 1 : pos);
        }
        a.step->pos = pos;
        a.step->token = tok;
        a.step->pos_next = pos + 1;
        a.step->forced_token = -1;
        a.history[pos] = tok;
        *a.argmax = argmax_key(-1e9f, 0);
        s_tok = tok;
    }
    __syncthreads();
    const int tok = s_tok;
    const int G = a.dim / 32;
    const uint8_t* base = a.emb + (size_t)(tok / kRB) * a.tile_bytes;
    const int r = tok % kRB;
    const float* sc = reinterpret_cast<const float*>(base) + r * G;
    const uint8_t* pk = base + kRB * G * 4 + (size_t)r * (a.dim / 2);
    for (int i = threadIdx.x; i < a.dim / 2; i += blockDim.x) {
        const uint8_t b = pk[i];
        const float s = sc[(2 * i) / 32];
        const int v0 = (int)(b & 0xF) - 8, v1 = (int)(b >> 4) - 8;
        a.x[2 * i] = (float)v0 * s;
        a.x[2 * i + 1] = (float)v1 * s;
    }
}

// ---------------------------------------------------------------------------
// Decode attention for one layer, split over positions (flash-decoding):
// CTA (head h, split s) scores positions [s*L, s*L+L) ∩ [0, pos], keeps the
// running max / sum / weighted V of its slice, and the last CTA of the head
// to finish combines the slices in split order.  Per position the score is
// (q . k) / sqrtf(head_size) (src/kernel_simd.c:1099-1117).
// ---------------------------------------------------------------------------
struct AttnArgs {
    const float* q;          // [dim] (RoPE applied)
    const float* kcache;     // layer base [max_pos][kv_dim]
    const float* vcache;
    float* out;              // [dim]
    float* partial;          // [n_heads][n_splits][head_size + 2]
    int* counters;           // [n_heads], zero between launches
    const StepState* step;
    int n_heads, kv_mul, head_size, kv_dim, split_len, n_splits;
};

constexpr int kAttnThreads = 128;
constexpr int kMaxSplitLen = 256;
constexpr int kMaxHeadSize = 256;

__global__ void __launch_bounds__(kAttnThreads) k_attention(AttnArgs a) {
    __shared__ float s_q[kMaxHeadSize];
    __shared__ float s_p[kMaxSplitLen];
    __shared__ float red[32];
    __shared__ int s_last;
    pdl_launch_dependents();
    pdl_wait();
    const int h = blockIdx.x, split = blockIdx.y;
    const int pos = a.step->pos;
    const int t0 = split * a.split_len;
    if (t0 > pos) return;                          // inactive split
    const int t1 = min(t0 + a.split_len, pos + 1);
    const int n_active = pos / a.split_len + 1;
    const int hs = a.head_size;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    const int kvh = h / a.kv_mul;
    for (int i = threadIdx.x; i < hs; i += blockDim.x) s_q[i] = a.q[h * hs + i];
    __syncthreads();
    const float rs = sqrtf((float)hs);
    for (int t = t0 + warp; t < t1; t += nwarps) {
        const float* k = a.kcache + (size_t)t * a.kv_dim + kvh * hs;
        float d = 0.0f;
        for (int i = lane; i < hs; i += 32) d = fmaf(s_q[i], k[i], d);
        d = warp_sum(d);
        if (lane == 0) s_p[t - t0] = __fdiv_rn(d, rs);
    }
    __syncthreads();
    float m = -INFINITY;
    for (int i = threadIdx.x; i < t1 - t0; i += blockDim.x) m = fmaxf(m, s_p[i]);
    m = warp_max(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = -INFINITY;
    for (int i = 0; i < nwarps; i++) m = fmaxf(m, red[i]);
    __syncthreads();
    float l = 0.0f;
    for (int i = threadIdx.x; i < t1 - t0; i += blockDim.x) {
        const float p = expf(s_p[i] - m);
        s_p[i] = p;
        l += p;
    }
    l = block_sum(l, red);
    float* part = a.partial + ((size_t)h * a.n_splits + split) * (hs + 2);
    for (int i = threadIdx.x; i < hs; i += blockDim.x) {
        float o = 0.0f;
        for (int t = t0; t < t1; t++) o = fmaf(s_p[t - t0], a.vcache[(size_t)t * a.kv_dim + kvh * hs + i], o);
        part[2 + i] = o;
    }
    if (threadIdx.x == 0) { part[0] = m; part[1] = l; }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = (atomicAdd(&a.counters[h], 1) == n_active - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const float* ph = a.partial + (size_t)h * a.n_splits * (hs + 2);
    float M = -INFINITY;
    for (int s = 0; s < n_active; s++) M = fmaxf(M, __ldcg(ph + (size_t)s * (hs + 2)));
    float L = 0.0f;
    for (int s = 0; s < n_active; s++) {
        const float* p = ph + (size_t)s * (hs + 2);
        L = fmaf(__ldcg(p + 1), expf(__ldcg(p) - M), L);
    }
    const float inv = 1.0f / L;
    for (int i = threadIdx.x; i < hs; i += blockDim.x) {
        float o = 0.0f;
        for (int s = 0; s < n_active; s++) {
            const float* p = ph + (size_t)s * (hs + 2);
            o = fmaf(__ldcg(p + 2 + i), expf(__ldcg(p) - M), o);
        }
        a.out[h * hs + i] = o * inv;
    }
    if (threadIdx.x == 0) a.counters[h] = 0;
}

// ---------------------------------------------------------------------------
// Re-tile: quantize.c layout rows -> tiled rows, and the exact inverse.
// Thread per (row, group): one fp32 scale + one 16-byte group.
// dst_row(r) = row_offset + r               (interleave == 0)
//            = (r / 2) * 4 + (r % 2) + slot * 2   (interleave == 1: w1/w3)
// ---------------------------------------------------------------------------
struct RetileArgs {
    const float* src_scales;     // [rows][n/32]
    const uint8_t* src_packed;   // [rows][n/2]
    uint8_t* dst;                // tiled
    long long tile_bytes;
    long long rows;
    int n;
    int row_offset, interleave, slot;
    int inverse;                 // 1: tiled -> quantize.c layout (src_* become outputs)
};

__device__ __forceinline__ long long retile_dst_row(const RetileArgs& a, long long r) {
    if (a.interleave) return (r / 2) * 4 + (r % 2) + a.slot * 2;
    return a.row_offset + r;
}

__global__ void k_retile(RetileArgs a) {
    const int G = a.n / 32;
    const long long total = a.rows * G;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / G;
        const int g = (int)(i % G);
        const long long R = retile_dst_row(a, r);
        uint8_t* base = a.dst + (R / kRB) * a.tile_bytes;
        const int rr = (int)(R % kRB);
        float* dsc = reinterpret_cast<float*>(base) + rr * G + g;
        uint4* dpk = reinterpret_cast<uint4*>(base + kRB * G * 4 + (size_t)rr * (a.n / 2) + 16 * g);
        float* ssc = const_cast<float*>(a.src_scales) + r * G + g;
        uint4* spk = reinterpret_cast<uint4*>(const_cast<uint8_t*>(a.src_packed) + r * (a.n / 2) + 16 * g);
        if (!a.inverse) { *dsc = *ssc; *dpk = *spk; }
        else { *ssc = *dsc; *spk = *dpk; }
    }
}

// Padding rows of the last tile: scale 0, nibbles 0x88 (q = 0).
__global__ void k_fill_pad(uint8_t* dst, long long tile_bytes, long long rows, long long rows_pad, int n) {
    const int G = n / 32;
    const long long total = (rows_pad - rows) * G;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const long long R = rows + i / G;
        const int g = (int)(i % G);
        uint8_t* base = dst + (R / kRB) * tile_bytes;
        const int rr = (int)(R % kRB);
        reinterpret_cast<float*>(base)[rr * G + g] = 0.0f;
        *reinterpret_cast<uint4*>(base + kRB * G * 4 + (size_t)rr * (n / 2) + 16 * g) =
            make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);
    }
}

// Sets the next step's position and/or forced token (negative: keep).
__global__ void k_set_step(StepState* s, int pos, int token) {
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        if (pos >= 0) s->pos_next = pos;
        if (token >= 0) s->forced_token = token;
    }
}

// Standalone activation quantization (bit-exact with the reference).
__global__ void k_quantize_act(const float* x, int8_t* qx, float* xs, long long n) {
    const long long G = n / 32;
    for (long long g = blockIdx.x * (long long)blockDim.x + threadIdx.x; g < G; g += (long long)gridDim.x * blockDim.x) {
        float amax = 0.0f;
        for (int k = 0; k < 32; k++) amax = fmaxf(amax, fabsf(x[g * 32 + k]));
        const bool big = amax > 1e-9f;
        const float scale = big ? __fdiv_rn(127.0f, amax) : 1.0f;
        xs[g] = big ? __fdiv_rn(amax, 127.0f) : 1.0f;
        for (int k = 0; k < 32; k++) qx[g * 32 + k] = (int8_t)(int)roundf(__fmul_rn(x[g * 32 + k], scale));
    }
}

}  // namespace aion
