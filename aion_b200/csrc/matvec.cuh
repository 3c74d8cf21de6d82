// int4 matvec core for sm_100a: HBM layout, per-warp bulk-copy rings, the
// W4A16 / W4A8 dequant-dot of one chunk, and the standalone streaming kernel.
//
// HBM layout ("tiled, chunked").  A matrix [d][n] (n % 32 == 0) is stored as
// ceil(d / kRB) tiles of kRB consecutive rows; each tile is n / kc chunks of
// kc columns; chunk c of tile t starts at t * tile_bytes + c * chunk_bytes and
// holds the fp32 group scales of its rows, row-major [kRB][kc/32], then the
// packed nibbles, row-major [kRB][kc/2], in the quantize.c order (low nibble
// = even element, stored value q + 8).  A chunk is one contiguous,
// 16-byte-aligned span of kRB*kc*5/8 bytes: one bulk copy.  Padding rows
// (past d) have scale 0 and nibbles 0x88.
#pragma once

#include "common.cuh"

namespace aion {

constexpr int kRB = 4;             // rows per tile
constexpr int kWarps = 8;          // consumer warps per CTA
constexpr int kThreads = kWarps * 32;
constexpr int kMaxChunkBytes = 6656;

struct MatDesc {
    const uint8_t* w;
    long long tile_bytes;
    int n, kc, nch, chunk_bytes;
    int ntiles, d;                 // tiles, logical rows
};

// Largest kc dividing n (multiple of 32) whose chunk fits kMaxChunkBytes.
__host__ __device__ inline int choose_kc(int n) {
    const int G = n / 32;
    int best = 1;
    for (int g = 1; g <= G; g++)
        if (G % g == 0 && kRB * g * 32 * 5 / 8 <= kMaxChunkBytes) best = g;
    return best * 32;
}

__host__ __device__ inline MatDesc make_desc(const uint8_t* w, long long rows, int n) {
    MatDesc m;
    m.w = w;
    m.n = n;
    m.kc = choose_kc(n);
    m.nch = n / m.kc;
    m.chunk_bytes = kRB * m.kc / 32 * 4 + kRB * m.kc / 2;
    m.tile_bytes = (long long)m.chunk_bytes * m.nch;
    m.ntiles = (int)((rows + kRB - 1) / kRB);
    m.d = (int)rows;
    return m;
}

__host__ __device__ inline long long desc_bytes(const MatDesc& m) { return m.tile_bytes * m.ntiles; }

// Byte offset of (row R, group g) scale / 16-byte group inside the layout.
__host__ __device__ inline long long scale_offset(const MatDesc& m, long long R, int g) {
    const int c = g / (m.kc / 32), gg = g % (m.kc / 32);
    return (R / kRB) * m.tile_bytes + (long long)c * m.chunk_bytes + ((R % kRB) * (m.kc / 32) + gg) * 4;
}
__host__ __device__ inline long long group_offset(const MatDesc& m, long long R, int g) {
    const int c = g / (m.kc / 32), gg = g % (m.kc / 32);
    return (R / kRB) * m.tile_bytes + (long long)c * m.chunk_bytes + kRB * (m.kc / 32) * 4 +
           (R % kRB) * (m.kc / 2) + 16 * gg;
}

// ---------------------------------------------------------------------------
// Dequant-dot of one 32-bit word (8 nibbles, element e at bits 4e..4e+3).
// A nibble v placed in the low mantissa bits of 2^23 gives the float
// 2^23 + v * 16^p exactly (p = its nibble position in the mantissa);
// subtracting 2^23 + 8 * 16^p yields (v - 8) * 16^p exactly.  Elements 0..4
// are masked in place (p = 0..4), elements 5..7 after one 12-bit shift
// (p = 2..4); the activations are pre-scaled by 16^-p (exact powers of two),
// so each product is q * x.  Two elements per packed fp32x2 instruction.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float2 dq_dot8(uint32_t w, float4 xa, float4 xb, float2 acc) {
    const uint32_t M = 0x4B000000u;
    const uint32_t w2 = w >> 12;
    const float2 f01 = make_float2(__uint_as_float((w & 0xFu) | M), __uint_as_float((w & 0xF0u) | M));
    const float2 f23 = make_float2(__uint_as_float((w & 0xF00u) | M), __uint_as_float((w & 0xF000u) | M));
    const float2 f45 = make_float2(__uint_as_float((w & 0xF0000u) | M), __uint_as_float((w2 & 0xF00u) | M));
    const float2 f67 = make_float2(__uint_as_float((w2 & 0xF000u) | M), __uint_as_float((w2 & 0xF0000u) | M));
    const float2 c01 = make_float2(-8388616.0f, -8388736.0f);   // -(2^23 + 8*16^0), -(2^23 + 8*16^1)
    const float2 c23 = make_float2(-8390656.0f, -8421376.0f);   // -(2^23 + 8*16^2), -(2^23 + 8*16^3)
    const float2 c45 = make_float2(-8912896.0f, -8390656.0f);   // -(2^23 + 8*16^4), -(2^23 + 8*16^2)
    const float2 c67 = make_float2(-8421376.0f, -8912896.0f);   // -(2^23 + 8*16^3), -(2^23 + 8*16^4)
    acc = __ffma2_rn(__fadd2_rn(f01, c01), make_float2(xa.x, xa.y), acc);
    acc = __ffma2_rn(__fadd2_rn(f23, c23), make_float2(xa.z, xa.w), acc);
    acc = __ffma2_rn(__fadd2_rn(f45, c45), make_float2(xb.x, xb.y), acc);
    acc = __ffma2_rn(__fadd2_rn(f67, c67), make_float2(xb.z, xb.w), acc);
    return acc;
}

// 16^-p for the element positions p = 0,1,2,3,4,2,3,4 of an 8-element word,
// built directly as the float exponent 127 - 4p.
__device__ __forceinline__ float prescale(int e) {
    const int p = e < 5 ? e : e - 3;
    return __int_as_float((127 - 4 * p) << 23);
}

// int4 x int8 dot of one 8-element word, times 16: the nibbles are moved to
// the high half of each byte and XORed with 0x80, giving the signed byte
// 16 * (v - 8).  xe / xo hold the int8 activations of elements 0,2,4,6 and
// 1,3,5,7.
__device__ __forceinline__ int dq_dot_i8(uint32_t w, uint32_t xe, uint32_t xo, int acc) {
    const uint32_t lo = ((w << 4) & 0xF0F0F0F0u) ^ 0x80808080u;
    const uint32_t hi = (w & 0xF0F0F0F0u) ^ 0x80808080u;
    acc = __dp4a((int)lo, (int)xe, acc);
    acc = __dp4a((int)hi, (int)xo, acc);
    return acc;
}

enum Mode { MODE_W4A16 = 0, MODE_W4A8 = 1 };

// ---------------------------------------------------------------------------
// Input vector in shared memory ("x'").
// W4A16: fp32, pre-scaled by prescale(), stored so that lane l reading group
//        l + 32*i touches consecutive 16-byte words: float4 j of group g at
//        ((g/32)*8 + j)*32 + g%32.
// W4A8:  per-32 int8 quantization, bit-exact with quantize_activations_neon
//        (src/kernel_simd.c:186-227): amax; scale 127/amax if amax > 1e-9
//        else 1; stored scale amax/127 (else 1); q = round-half-away(x*scale).
//        The int8 values of each 8-element word are stored as
//        [e0 e2 e4 e6][e1 e3 e5 e7]; uint4 h (0/1) of group g at
//        ((g/32)*2 + h)*32 + g%32, followed by the fp32 group scales.
// ---------------------------------------------------------------------------
__host__ __device__ inline int xbuf_bytes(int n, int mode) {
    const int chunks = (n / 32 + 31) / 32;
    return mode == MODE_W4A16 ? chunks * 8 * 32 * 16 : chunks * 2 * 32 * 16 + chunks * 32 * 4;
}

__device__ __forceinline__ int xperm(int g, int j) { return ((g >> 5) * 8 + j) * 32 + (g & 31); }

// Loads an fp32 vector that may have been written by other CTAs of the same
// kernel: through L2, never a stale L1 line.
__device__ __forceinline__ float4 ld_vec(const float* p, int i) { return __ldcg(reinterpret_cast<const float4*>(p) + i); }

// rmsnorm scale of src/kernel_simd.c:793-803: 1 / sqrtf(sum(x^2) / n + 1e-5).
__device__ __forceinline__ float rms_scale(const float* x, int n, float* red) {
    float s = 0.0f;
    for (int i = threadIdx.x; i < n / 4; i += blockDim.x) {
        const float4 v = ld_vec(x, i);
        s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    s = block_sum(s, red);
    return 1.0f / sqrtf(__fdiv_rn(s, (float)n) + 1e-5f);
}

// Writes x' for input x (optionally times ss * norm_w, elementwise as
// (x * ss) * w, src/kernel_simd.c:805-813).  All threads of the CTA call it.
template <int MODE>
__device__ __forceinline__ void build_x(unsigned char* xbuf, const float* x, int n, const float* norm_w, float ss) {
    const int G = n / 32;
    if (MODE == MODE_W4A16) {
        float4* xs4 = reinterpret_cast<float4*>(xbuf);
        for (int i = threadIdx.x; i < n / 4; i += blockDim.x) {
            float4 v = ld_vec(x, i);
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
                const float4 t = ld_vec(x, g * 8 + j);
                v[4 * j] = t.x; v[4 * j + 1] = t.y; v[4 * j + 2] = t.z; v[4 * j + 3] = t.w;
            }
            if (norm_w) {
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const float4 t = __ldg(reinterpret_cast<const float4*>(norm_w) + g * 8 + j);
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
// Per-warp bulk-copy ring.  Each warp streams its own chunk sequence through
// P slots: lane 0 issues one bulk copy per slot (mbarrier expect_tx), the
// warp waits on the slot's mbarrier, computes, and lane 0 refills the slot
// with the chunk P positions further on.  No cross-warp coordination.
// ---------------------------------------------------------------------------
struct Ring {
    uint32_t slots;      // shared address of this warp's slot 0
    uint32_t bars;       // shared address of this warp's mbarrier 0
    int P, slot_bytes;
    uint32_t issued, consumed;
};

__device__ __forceinline__ void ring_init(Ring& r, unsigned char* ring_base, uint64_t* bar_base, int P, int slot_bytes) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    r.P = P;
    r.slot_bytes = slot_bytes;
    r.slots = smem_addr(ring_base + (size_t)warp * P * slot_bytes);
    r.bars = smem_addr(bar_base + warp * P);
    r.issued = r.consumed = 0;
    if (lane == 0)
        for (int i = 0; i < P; i++) mbar_init(r.bars + 8 * i, 1);
    fence_mbar_init();
    __syncwarp();
}

// Lane 0: issue the next chunk into the next free slot.
__device__ __forceinline__ void ring_issue(Ring& r, const uint8_t* src, int bytes) {
    const int slot = r.issued % r.P;
    if ((threadIdx.x & 31) == 0) {
        const uint32_t bar = r.bars + 8 * slot;
        mbar_arrive_expect_tx(bar, (uint32_t)bytes);
        bulk_g2s(r.slots + slot * r.slot_bytes, src, (uint32_t)bytes, bar);
    }
    r.issued++;
}

// Waits for the oldest issued chunk; returns its generic shared pointer, or
// nullptr on timeout.
__device__ __forceinline__ const unsigned char* ring_wait(Ring& r, unsigned char* ring_base) {
    const int slot = r.consumed % r.P;
    const uint32_t parity = (r.consumed / r.P) & 1;
    if (!mbar_wait(r.bars + 8 * slot, parity)) return nullptr;
    const int warp = threadIdx.x >> 5;
    return ring_base + ((size_t)warp * r.P + slot) * r.slot_bytes;
}

// Drains every chunk still in flight (bounded), so the CTA may exit safely.
__device__ __forceinline__ void ring_drain(Ring& r) {
    while (r.consumed < r.issued) {
        const int slot = r.consumed % r.P;
        mbar_wait(r.bars + 8 * slot, (r.consumed / r.P) & 1, 1u << 20);
        r.consumed++;
    }
}

// ---------------------------------------------------------------------------
// Compute of one chunk (kRB rows x kc columns) held in shared memory.
// acc[r] accumulates row r.  g0 = first group of the chunk within the row.
// W4A16: per group fp32 dot of q*x, then acc += scale * dot (lanes in
//        parallel; rows reduce across lanes after the last chunk).
// W4A8:  per group exact int32 dot; the reference epilogue
//        row += (float)dot * (w_scale * x_scale) runs sequentially over the
//        groups of the row in order (src/kernel_simd.c:250-335), lanes
//        broadcasting their products through shuffles.
// ---------------------------------------------------------------------------
template <int MODE>
__device__ __forceinline__ void chunk_compute(const unsigned char* chunk, int kc, int g0, const unsigned char* xbuf,
                                              int n, float* acc) {
    const int lane = threadIdx.x & 31;
    const int gk = kc / 32;
    const float* sc = reinterpret_cast<const float*>(chunk);
    const uint4* pk = reinterpret_cast<const uint4*>(chunk + kRB * gk * 4);
    if (MODE == MODE_W4A16) {
        const float4* xs4 = reinterpret_cast<const float4*>(xbuf);
        for (int gg = lane; gg < gk; gg += 32) {
            const int g = g0 + gg;
            float4 xv[8];
#pragma unroll
            for (int j = 0; j < 8; j++) xv[j] = xs4[xperm(g, j)];
#pragma unroll
            for (int r = 0; r < kRB; r++) {
                const uint4 w = pk[r * gk + gg];
                float2 p = make_float2(0.0f, 0.0f);
                p = dq_dot8(w.x, xv[0], xv[1], p);
                p = dq_dot8(w.y, xv[2], xv[3], p);
                p = dq_dot8(w.z, xv[4], xv[5], p);
                p = dq_dot8(w.w, xv[6], xv[7], p);
                acc[r] = fmaf(sc[r * gk + gg], p.x + p.y, acc[r]);
            }
        }
    } else {
        const int chunks = (n / 32 + 31) / 32;
        const uint4* qx = reinterpret_cast<const uint4*>(xbuf);
        const float* xsc = reinterpret_cast<const float*>(xbuf + chunks * 2 * 32 * 16);
        for (int base = 0; base < gk; base += 32) {
            const int gg = base + lane;
            float prod[kRB];
            if (gg < gk) {
                const int g = g0 + gg;
                const uint4 xa = qx[((g >> 5) * 2 + 0) * 32 + (g & 31)];
                const uint4 xb = qx[((g >> 5) * 2 + 1) * 32 + (g & 31)];
                const float xscale = xsc[g];
#pragma unroll
                for (int r = 0; r < kRB; r++) {
                    const uint4 w = pk[r * gk + gg];
                    int s16 = 0;
                    s16 = dq_dot_i8(w.x, xa.x, xa.y, s16);
                    s16 = dq_dot_i8(w.y, xa.z, xa.w, s16);
                    s16 = dq_dot_i8(w.z, xb.x, xb.y, s16);
                    s16 = dq_dot_i8(w.w, xb.z, xb.w, s16);
                    const float comb = __fmul_rn(sc[r * gk + gg], xscale);
                    prod[r] = __fmul_rn((float)(s16 >> 4), comb);
                }
            } else {
#pragma unroll
                for (int r = 0; r < kRB; r++) prod[r] = 0.0f;
            }
            const int cnt = min(32, gk - base);
            for (int j = 0; j < cnt; j++) {
#pragma unroll
                for (int r = 0; r < kRB; r++) acc[r] = __fadd_rn(acc[r], __shfl_sync(0xffffffffu, prod[r], j));
            }
        }
    }
}

// Rows of a finished tile: W4A16 reduces the lane partial sums (every lane
// receives the totals); W4A8 rows are already complete and lane-uniform.
template <int MODE>
__device__ __forceinline__ void finish_rows(float* acc) {
    if (MODE == MODE_W4A16) {
#pragma unroll
        for (int r = 0; r < kRB; r++) acc[r] = warp_sum(acc[r]);
    }
}

// ---------------------------------------------------------------------------
// Standalone matvec y = W x over all rows, streaming through the per-warp
// rings.  One CTA per SM; CTA c owns tiles [c*T/G, (c+1)*T/G), its warps take
// every kWarps-th tile of that range.  Weight chunks are requested before
// the grid-dependency wait (weights never depend on the previous kernel).
// ---------------------------------------------------------------------------
struct StandaloneArgs {
    MatDesc m;
    const float* x;
    float* y;
    int P, slot_bytes;
};

__device__ __forceinline__ void cta_tile_range(int ntiles, int& t0, int& t1) {
    t0 = (int)(((long long)blockIdx.x * ntiles) / gridDim.x);
    t1 = (int)(((long long)(blockIdx.x + 1) * ntiles) / gridDim.x);
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1) k_matvec(StandaloneArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bars[kWarps * 8];
    __shared__ float red[32];
    const int warp = threadIdx.x >> 5;
    const MatDesc& m = a.m;
    unsigned char* xbuf = smem;
    unsigned char* ring_base = smem + ((xbuf_bytes(m.n, MODE) + 127) & ~127);
    Ring ring;
    ring_init(ring, ring_base, bars, a.P, a.slot_bytes);
    int t0, t1;
    cta_tile_range(m.ntiles, t0, t1);
    // This warp's chunk sequence: tiles t0 + warp, t0 + warp + kWarps, ...
    int pt = t0 + warp, pc = 0;
    const int total = t1 > t0 + warp ? ((t1 - t0 - warp + kWarps - 1) / kWarps) * m.nch : 0;
    for (int i = 0; i < a.P && (int)ring.issued < total; i++) {
        ring_issue(ring, m.w + (size_t)pt * m.tile_bytes + (size_t)pc * m.chunk_bytes, m.chunk_bytes);
        if (++pc == m.nch) { pc = 0; pt += kWarps; }
    }
    pdl_launch_dependents();
    pdl_wait();
    build_x<MODE>(xbuf, a.x, m.n, nullptr, 1.0f);
    __syncthreads();
    (void)red;
    for (int t = t0 + warp; t < t1; t += kWarps) {
        float acc[kRB] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int c = 0; c < m.nch; c++) {
            const unsigned char* ch = ring_wait(ring, ring_base);
            if (!ch) { ring_drain(ring); return; }
            chunk_compute<MODE>(ch, m.kc, c * (m.kc / 32), xbuf, m.n, acc);
            __syncwarp();
            ring.consumed++;
            if ((int)ring.issued < total) {
                ring_issue(ring, m.w + (size_t)pt * m.tile_bytes + (size_t)pc * m.chunk_bytes, m.chunk_bytes);
                if (++pc == m.nch) { pc = 0; pt += kWarps; }
            }
        }
        finish_rows<MODE>(acc);
        if ((threadIdx.x & 31) == 0)
            for (int r = 0; r < kRB; r++)
                if (t * kRB + r < m.d) a.y[t * kRB + r] = acc[r];
    }
}

// ---------------------------------------------------------------------------
// Re-tile: quantize.c layout rows -> chunked tiles, and the exact inverse.
// Thread per (row, group): one fp32 scale + one 16-byte group.
//   dst_row(r) = row_offset + r                         (interleave == 0)
//              = (r / 2) * 4 + (r % 2) + slot * 2        (interleave == 1:
//                w1 rows in slot 0, w3 rows in slot 1, so a tile holds
//                w1[2t], w1[2t+1], w3[2t], w3[2t+1])
// ---------------------------------------------------------------------------
struct RetileArgs {
    const float* src_scales;     // [rows][n/32]
    const uint8_t* src_packed;   // [rows][n/2]
    MatDesc m;                   // destination layout (m.w is written)
    long long rows;
    int row_offset, interleave, slot;
    int inverse;                 // 1: chunked tiles -> quantize.c layout
};

__global__ void k_retile(RetileArgs a) {
    const int G = a.m.n / 32;
    const long long total = a.rows * G;
    uint8_t* base = const_cast<uint8_t*>(a.m.w);
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / G;
        const int g = (int)(i % G);
        const long long R = a.interleave ? (r / 2) * 4 + (r % 2) + a.slot * 2 : a.row_offset + r;
        float* dsc = reinterpret_cast<float*>(base + scale_offset(a.m, R, g));
        uint4* dpk = reinterpret_cast<uint4*>(base + group_offset(a.m, R, g));
        float* ssc = const_cast<float*>(a.src_scales) + r * G + g;
        uint4* spk = reinterpret_cast<uint4*>(const_cast<uint8_t*>(a.src_packed) + r * (a.m.n / 2) + 16 * g);
        if (!a.inverse) { *dsc = *ssc; *dpk = *spk; }
        else { *ssc = *dsc; *spk = *dpk; }
    }
}

// Padding rows of the last tile: scale 0, nibbles 0x88 (q = 0).
__global__ void k_fill_pad(MatDesc m) {
    const int G = m.n / 32;
    const long long rows_pad = (long long)m.ntiles * kRB;
    const long long total = (rows_pad - m.d) * G;
    uint8_t* base = const_cast<uint8_t*>(m.w);
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long R = m.d + i / G;
        const int g = (int)(i % G);
        *reinterpret_cast<float*>(base + scale_offset(m, R, g)) = 0.0f;
        *reinterpret_cast<uint4*>(base + group_offset(m, R, g)) =
            make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);
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
