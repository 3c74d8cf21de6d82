// int4 matvec core for sm_100a: HBM layout, per-warp bulk-copy rings, the
// tensor-pipe group dot, and the shared pieces of the streaming kernels.
//
// HBM layout.  A matrix [d][n] (n % 32 == 0, G = n/32 groups per row) is
// stored as ceil(d/16) tiles of 16 rows.  Group g of tile T occupies the 320
// bytes at T*G*320 + g*320: 256 bytes of packed nibbles in the order the
// MMA A fragment wants them (lane l = 4*r + t holds 8 bytes: one 32-bit word
// for row r and one for row r + 8; byte b of a word holds, low nibble,
// element 4t + b and, high nibble, element 16 + 4t + b of that row's group),
// then the 16 fp32 group scales as pairs (row r, row r + 8), r = 0..7.
// Nibble values are the stored quantize.c values q + 8.  A transfer "chunk"
// is any run of consecutive groups of one tile: one contiguous, 16-byte
// aligned span, one bulk copy.  Rows past d have scale 0 and nibbles 8.
//
// Group dot.  mma.sync.m16n8k32 s8 x s8 -> s32 multiplies A = the 16 rows'
// int8 weights of one group by B = up to 3 int8 "digit" columns of the
// activations (the other columns of B are zero), giving exact int32 dots.
// Weights enter as 16 * (v - 8): each nibble moved to the high half of its
// byte and XORed with 0x80.
//   W4A16: x of a group is scaled by 2^E (E = 22 - exponent of its max) and
//          rounded to an integer X (|X| <= 2^22), split into signed digits
//          X = X0 + 256 X1 + 65536 X2; the dots of the three digits are
//          recombined in int32 / fp32 and scaled by w_scale * 2^-E / 16,
//          accumulated in fp32.  The activation keeps 22 bits relative to its
//          group maximum; the dot of those values is exact.
//   W4A8:  B holds the reference's int8 activations (one digit); the row sum
//          row += (float)dot * (w_scale * x_scale) runs over the groups in
//          order (src/kernel_simd.c:250-335): bit-exact with the reference.
#pragma once

#include "common.cuh"

namespace aion {

constexpr int kTR = 16;              // rows per tile (MMA M)
constexpr int kRB = 4;               // rows per epilogue quad
constexpr int kGB = 320;             // bytes per (tile, group)
constexpr int kWarps = 11;           // compute warps per CTA
constexpr int kThreads = kWarps * 32;
static_assert(kThreads == kComputeThreads, "compute threads");
constexpr int kTargetChunk = 6400;   // bytes per bulk copy, about
constexpr int kXF = 128;             // bytes of activation digits per group (4 columns)
constexpr int kMaxLocalTiles = 24;   // tiles of one op per CTA (split mode)

enum Mode { MODE_W4A16 = 0, MODE_W4A8 = 1, MODE_F32 = 2 };

// fp32 tiles (the reference's fp32 path): per (tile, group) 4 x 32 float4,
// entry (q, lane) = row r (q < 2) or r + 8 (q >= 2), columns 8t + 4(q & 1)
// .. +3 of the group, for lane = 4r + t; 2048 bytes.
constexpr int kGBF = 2048;

struct MatDesc {
    const uint8_t* w;
    long long tile_bytes;          // G * gbytes
    int n, G, nch;                 // columns, groups per row, chunks per tile
    int cg, cr, gq;                // chunk c spans gq * cg groups, gq more for c < cr
    int ntiles, d;                 // tiles, logical rows
    int gbytes;                    // bytes per (tile, group): kGB (int4) or kGBF (fp32)
};

// Cuts every tile into nch chunks of whole granules (gq groups); the tile
// layout in memory does not depend on it.
__host__ __device__ inline void set_chunks(MatDesc& m, int nch) {
    const int Q = m.G / m.gq;
    m.nch = nch < 1 ? 1 : nch > Q ? Q : nch;
    m.cg = Q / m.nch;
    m.cr = Q % m.nch;
}

__host__ __device__ inline MatDesc make_desc(const uint8_t* w, long long rows, int n, int gbytes = kGB) {
    MatDesc m;
    m.w = w;
    m.n = n;
    m.G = n / 32;
    m.gbytes = gbytes;
    m.tile_bytes = (long long)m.G * gbytes;
    // fp32 groups are 6.4x larger: about two per copy, so two ring slots per
    // warp still fit next to an 11008-wide fp32 input.  int4 chunks are cut
    // in whole quads of groups where G allows it (the group dot takes four
    // groups per step, so no step of a chunk is padded).
    const int target = gbytes == kGB ? kTargetChunk : 2 * gbytes;
    m.gq = (gbytes == kGB && m.G % 4 == 0) ? 4 : 1;
    m.ntiles = (int)((rows + kTR - 1) / kTR);
    m.d = (int)rows;
    set_chunks(m, (int)((m.tile_bytes + target - 1) / target));
    return m;
}

__host__ __device__ inline long long desc_bytes(const MatDesc& m) { return m.tile_bytes * m.ntiles; }
__host__ __device__ inline int chunk_g0(const MatDesc& m, int c) { return m.gq * (c * m.cg + (c < m.cr ? c : m.cr)); }
__host__ __device__ inline int max_chunk_bytes(const MatDesc& m) { return m.gq * (m.cg + (m.cr ? 1 : 0)) * m.gbytes; }

// ---------------------------------------------------------------------------
// Activation digits in shared memory: group g at g*128: digit column p
// (0..3), lane t (0..3): 8 bytes = the B-fragment words (elements 4t..4t+3
// and 16+4t..16+4t+3), so lane l of a warp loads its fragment at
// g*128 + 8*(l % 16) (lanes 16..31 repeat columns 0..3 as columns 4..7,
// whose products no lane uses).  Then G fp32 group factors: W4A8's
// activation scales; W4A16 keeps one factor for the whole vector in xs[0].
//   W4A16: X = round(x * 2^E) with one E per vector (max |x| * 2^E in
//     [2^29, 2^30)), written as four signed bytes X = d0 + 2^8 d1 + 2^16 d2
//     + 2^24 d3; factor 2^-E / 16 (the weight bytes carry 16 * q).
//   W4A8: column 0 holds the reference's int8 activations; the other
//     columns are not read for any output.
// ---------------------------------------------------------------------------
__host__ __device__ inline int xbuf_bytes(int n) { return (n / 32) * (kXF + 4); }

// ---------------------------------------------------------------------------
// Tensor-pipe group dot.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// int8 bytes 16 * (v - 8) of the low / high nibbles of a packed word.
__device__ __forceinline__ uint32_t lo16(uint32_t w) { return ((w << 4) & 0xF0F0F0F0u) ^ 0x80808080u; }
__device__ __forceinline__ uint32_t hi16(uint32_t w) { return (w & 0xF0F0F0F0u) ^ 0x80808080u; }

// Accumulates groups [0, ng) of one chunk of one tile held in shared memory
// (group k of the chunk at chunk + k*320; g0 = its first group in the row).
// acc0 / acc1 belong to rows r and r + 8 of the tile (r = lane / 4).  Four
// groups per step: their operand loads and MMAs are independent, only the
// final accumulation is a chain.
//   W4A16: quad lane t = 0 holds columns 0, 1 (digits d0 + 2^8 d1), t = 1
//     columns 2, 3 (d2 + 2^8 d3); each adds weight scale * that integer.
//   W4A8: lane t = 0 adds (column 0 / 16) * (weight scale * activation
//     scale) in the reference's order.
template <int MODE>
__device__ __forceinline__ void group_accumulate(const int (&d)[4], float2 sw, float f, float& acc0, float& acc1) {
    if (MODE == MODE_W4A16) {
        acc0 = fmaf(sw.x, (float)(d[0] + 256 * d[1]), acc0);
        acc1 = fmaf(sw.y, (float)(d[2] + 256 * d[3]), acc1);
    } else {
        acc0 = __fadd_rn(acc0, __fmul_rn((float)(d[0] >> 4), __fmul_rn(sw.x, f)));
        acc1 = __fadd_rn(acc1, __fmul_rn((float)(d[2] >> 4), __fmul_rn(sw.y, f)));
    }
}

template <int MODE>
__device__ __forceinline__ void chunk_mma(const unsigned char* chunk, int ng, int g0, const unsigned char* xf,
                                          const float* xs, float& acc0, float& acc1) {
    if constexpr (MODE == MODE_F32) {
        // fp32 tiles on the CUDA cores: lane 4r + t adds rows r and r + 8
        // over columns 8t..8t+7 of every group; xf holds x as fp32 [G][32].
        const int ln = threadIdx.x & 31, tq = ln & 3;
        const float4* wp = reinterpret_cast<const float4*>(chunk) + ln;
        const float* xp = reinterpret_cast<const float*>(xf) + (size_t)g0 * 32 + 8 * tq;
#pragma unroll 2
        for (int k = 0; k < ng; k++) {
            const float4 w0 = wp[k * 128], w1 = wp[k * 128 + 32], w2 = wp[k * 128 + 64], w3 = wp[k * 128 + 96];
            const float4 x0 = *reinterpret_cast<const float4*>(xp + k * 32);
            const float4 x1 = *reinterpret_cast<const float4*>(xp + k * 32 + 4);
            acc0 = fmaf(w0.x, x0.x, acc0);
            acc0 = fmaf(w0.y, x0.y, acc0);
            acc0 = fmaf(w0.z, x0.z, acc0);
            acc0 = fmaf(w0.w, x0.w, acc0);
            acc0 = fmaf(w1.x, x1.x, acc0);
            acc0 = fmaf(w1.y, x1.y, acc0);
            acc0 = fmaf(w1.z, x1.z, acc0);
            acc0 = fmaf(w1.w, x1.w, acc0);
            acc1 = fmaf(w2.x, x0.x, acc1);
            acc1 = fmaf(w2.y, x0.y, acc1);
            acc1 = fmaf(w2.z, x0.z, acc1);
            acc1 = fmaf(w2.w, x0.w, acc1);
            acc1 = fmaf(w3.x, x1.x, acc1);
            acc1 = fmaf(w3.y, x1.y, acc1);
            acc1 = fmaf(w3.z, x1.z, acc1);
            acc1 = fmaf(w3.w, x1.w, acc1);
        }
        return;
    }
    const int lane = threadIdx.x & 31;
    const int r = lane >> 2;
    const unsigned char* wp = chunk + 8 * lane;
    const unsigned char* sp = chunk + 256 + 8 * r;
    const unsigned char* xp = xf + (size_t)g0 * kXF + 8 * (lane & 15);
    const float* fp = xs + g0;
    int k = 0;
    for (; k + 4 <= ng; k += 4) {
        uint2 wv[4], xv[4];
        float2 sw[4];
        float f[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            wv[j] = *reinterpret_cast<const uint2*>(wp + (k + j) * kGB);
            sw[j] = *reinterpret_cast<const float2*>(sp + (k + j) * kGB);
            xv[j] = *reinterpret_cast<const uint2*>(xp + (k + j) * kXF);
            f[j] = MODE == MODE_W4A8 ? fp[k + j] : 0.0f;
        }
        int d[4][4];
#pragma unroll
        for (int j = 0; j < 4; j++)
            mma_s8(d[j], lo16(wv[j].x), lo16(wv[j].y), hi16(wv[j].x), hi16(wv[j].y), xv[j].x, xv[j].y);
#pragma unroll
        for (int j = 0; j < 4; j++) group_accumulate<MODE>(d[j], sw[j], f[j], acc0, acc1);
    }
    if (k < ng) {
        // Last 1-3 groups as one step of four; the missing groups read the
        // chunk's last group with all-zero weights (nibbles 8), whose
        // products add exactly zero.
        uint2 wv[4], xv[4];
        float2 sw[4];
        float f[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int kk = min(k + j, ng - 1);
            wv[j] = *reinterpret_cast<const uint2*>(wp + kk * kGB);
            if (k + j >= ng) wv[j] = make_uint2(0x88888888u, 0x88888888u);
            sw[j] = *reinterpret_cast<const float2*>(sp + kk * kGB);
            xv[j] = *reinterpret_cast<const uint2*>(xp + kk * kXF);
            f[j] = MODE == MODE_W4A8 ? fp[kk] : 0.0f;
        }
        int d[4][4];
#pragma unroll
        for (int j = 0; j < 4; j++)
            mma_s8(d[j], lo16(wv[j].x), lo16(wv[j].y), hi16(wv[j].x), hi16(wv[j].y), xv[j].x, xv[j].y);
#pragma unroll
        for (int j = 0; j < 4; j++) group_accumulate<MODE>(d[j], sw[j], f[j], acc0, acc1);
    }
}

// Finishes a tile's lane accumulators: afterwards lane 4r (t = 0) holds rows
// r (acc0) and r + 8 (acc1).  W4A16 joins the quad's low and high digit
// halves and applies the vector factor; W4A8 rows are complete in lane t = 0
// already.
template <int MODE>
__device__ __forceinline__ void quad_reduce(float& acc0, float& acc1, float xfactor) {
    if (MODE == MODE_F32) {
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
    }
    if (MODE == MODE_W4A16) {
        const float h0 = __shfl_xor_sync(0xffffffffu, acc0, 1);
        const float h1 = __shfl_xor_sync(0xffffffffu, acc1, 1);
        acc0 = fmaf(h0, 65536.0f, acc0) * xfactor;
        acc1 = fmaf(h1, 65536.0f, acc1) * xfactor;
    }
}

// ---------------------------------------------------------------------------
// Per-warp bulk-copy ring of P slots.  Slot s has a "full" mbarrier (armed
// with the chunk's byte count, completed by the bulk copy) and an "empty"
// mbarrier (one arrival when the consuming warp is done with the slot).
// The chunks are issued either by the consuming warp's lane 0 right after it
// frees a slot (ring_issue), or by a producer lane that waits for the slot's
// empty barrier (ProdRing).
// ---------------------------------------------------------------------------
struct Ring {
    uint32_t slots;      // shared address of this warp's slot 0
    uint32_t bars;       // shared address of this warp's full mbarrier 0
    uint32_t ebars;      // shared address of this warp's empty mbarrier 0
    int P, slot_bytes;
    uint32_t issued, consumed;
    int islot, cslot;    // issued % P, consumed % P
    uint32_t cphase;     // (consumed / P) & 1
};

// Ring of warp `warp`; its lane 0 initialises the barriers when init is set.
__device__ __forceinline__ void ring_init(Ring& r, unsigned char* ring_base, uint64_t* bar_base, int P, int slot_bytes,
                                          int warp, bool init) {
    r.P = P;
    r.slot_bytes = slot_bytes;
    r.slots = smem_addr(ring_base + (size_t)warp * P * slot_bytes);
    r.bars = smem_addr(bar_base + warp * 2 * P);
    r.ebars = r.bars + 8 * P;
    r.issued = r.consumed = 0;
    r.islot = r.cslot = 0;
    r.cphase = 0;
    if (init)
        for (int i = 0; i < P; i++) {
            mbar_init(r.bars + 8 * i, 1);
            mbar_init(r.ebars + 8 * i, 1);
        }
}

// Consumer-issued chunk (lane 0 of the consuming warp).
__device__ __forceinline__ void ring_issue(Ring& r, const uint8_t* src, int bytes) {
    const int slot = r.islot;
    if ((threadIdx.x & 31) == 0) {
        const uint32_t bar = r.bars + 8 * slot;
        mbar_arrive_expect_tx(bar, (uint32_t)bytes);
        bulk_g2s(r.slots + slot * r.slot_bytes, src, (uint32_t)bytes, bar);
    }
    r.issued++;
    r.islot = slot + 1 == r.P ? 0 : slot + 1;
}

// Waits for the oldest issued chunk; returns its generic shared pointer, or
// nullptr on timeout.  ring_release() then frees the slot.
__device__ __forceinline__ const unsigned char* ring_wait(Ring& r, unsigned char* ring_base) {
    if (!mbar_wait(r.bars + 8 * r.cslot, r.cphase)) return nullptr;
    const int warp = threadIdx.x >> 5;
    return ring_base + ((size_t)warp * r.P + r.cslot) * r.slot_bytes;
}
// Frees the oldest slot; with a producer, tells it so through the slot's
// empty barrier (after every lane of the warp is done reading).
__device__ __forceinline__ void ring_release(Ring& r, bool producer = false) {
    if (producer) {
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive(r.ebars + 8 * r.cslot);
    }
    r.consumed++;
    if (++r.cslot == r.P) {
        r.cslot = 0;
        r.cphase ^= 1u;
    }
}

// Drains every chunk still in flight (bounded), so the CTA may exit safely.
__device__ __forceinline__ void ring_drain(Ring& r) {
    while (r.consumed < r.issued) {
        mbar_wait(r.bars + 8 * r.cslot, r.cphase, 1u << 20);
        ring_release(r);
    }
}

// Producer side of one warp's ring, run by a single producer lane: issue k
// goes to slot k % P after the consumer has released issue k - P there.
struct ProdRing {
    Ring r;
    uint32_t round;      // issued / P
};

// Non-blocking: issues the chunk if its slot is free; false otherwise.
__device__ __forceinline__ bool prod_try_issue(ProdRing& p, const uint8_t* src, int bytes) {
    const int slot = p.r.islot;
    if (p.round > 0 && !mbar_try_wait(p.r.ebars + 8 * slot, (p.round - 1) & 1)) return false;
    const uint32_t bar = p.r.bars + 8 * slot;
    mbar_arrive_expect_tx(bar, (uint32_t)bytes);
    bulk_g2s(p.r.slots + slot * p.r.slot_bytes, src, (uint32_t)bytes, bar);
    p.r.issued++;
    if (++p.r.islot == p.r.P) {
        p.r.islot = 0;
        p.round++;
    }
    return true;
}

// Waits (bounded) until every chunk this producer issued has landed.
__device__ __forceinline__ void prod_drain(ProdRing& p) {
    const uint32_t n = p.r.issued < (uint32_t)p.r.P ? p.r.issued : (uint32_t)p.r.P;
    for (uint32_t i = 0; i < n; i++) {
        // the last issue into slot s was number issued - 1 - i
        const uint32_t k = p.r.issued - 1 - i;
        mbar_wait(p.r.bars + 8 * (k % p.r.P), (k / p.r.P) & 1, 1u << 20);
    }
}

// ---------------------------------------------------------------------------
// Work split of one op over the CTAs and warps.
//   split (W4A16 with at least as many tiles as CTAs): the op is
//     ntiles * nch (tile, chunk) units; CTA c takes the contiguous units
//     [c*U/G, (c+1)*U/G), so every CTA streams the same bytes (to one chunk);
//     its warps take every 8th unit.  A tile cut by a CTA boundary gets two
//     partial sums, added in a fixed order by the CTA that finishes second.
//   whole (W4A8, or fewer tiles than CTAs): CTA c takes tiles
//     [c*T/G, (c+1)*T/G); warp w takes every 8th of them with all their
//     chunks in order (the W4A8 row sum is sequential over the groups).
// ---------------------------------------------------------------------------
struct OpWork {
    int split;
    int u0, u1;          // split: unit range; whole: tile range
};

__host__ __device__ inline OpWork op_work_at(const MatDesc& m, int mode, int c, int G) {
    OpWork w;
    w.split = (mode != MODE_W4A8 && m.ntiles >= G && m.ntiles <= (kMaxLocalTiles - 2) * G) ? 1 : 0;
    const long long U = w.split ? (long long)m.ntiles * m.nch : m.ntiles;
    if (U * G < (1LL << 31)) {   // 32-bit division when the products fit
        const uint32_t u = (uint32_t)U;
        w.u0 = (int)(((uint32_t)c * u) / (uint32_t)G);
        w.u1 = (int)(((uint32_t)(c + 1) * u) / (uint32_t)G);
    } else {
        w.u0 = (int)(((long long)c * U) / G);
        w.u1 = (int)(((long long)(c + 1) * U) / G);
    }
    return w;
}
__device__ __forceinline__ OpWork op_work(const MatDesc& m, int mode) { return op_work_at(m, mode, blockIdx.x, gridDim.x); }

// Position in a warp's chunk sequence of one op: unit index a (split) or
// tile index (whole), and the tile / chunk it stands for.
struct OpCursor {
    int a, tile, c;
};

__host__ __device__ inline bool cursor_begin(OpCursor& cu, const OpWork& w, const MatDesc& m, int warp) {
    cu.a = w.u0 + warp;
    if (w.split) {
        cu.tile = cu.a / m.nch;
        cu.c = cu.a - cu.tile * m.nch;
    } else {
        cu.tile = cu.a;
        cu.c = 0;
    }
    return cu.a < w.u1;
}
__host__ __device__ inline bool cursor_next(OpCursor& cu, const OpWork& w, const MatDesc& m) {
    if (w.split) {
        cu.a += kWarps;
        cu.c += kWarps;
        while (cu.c >= m.nch) {
            cu.c -= m.nch;
            cu.tile++;
        }
    } else if (++cu.c == m.nch) {
        cu.c = 0;
        cu.a += kWarps;
        cu.tile = cu.a;
    }
    return cu.a < w.u1;
}

__device__ __forceinline__ const uint8_t* chunk_src(const MatDesc& m, int tile, int c, int& bytes) {
    const int g0 = chunk_g0(m, c), g1 = chunk_g0(m, c + 1);
    bytes = (g1 - g0) * m.gbytes;
    return m.w + (size_t)tile * m.tile_bytes + (size_t)g0 * m.gbytes;
}

// ---------------------------------------------------------------------------
// Re-tile: quantize.c layout rows -> tiles, and the exact inverse.
// Thread per (row, group): one fp32 scale + 16 bytes of nibbles.
//   dst_row(r) = row_offset + r                       (interleave == 0)
//              = (r / 2) * 4 + (r % 2) + slot * 2      (interleave == 1: w1
//                rows in slot 0, w3 rows in slot 1, so each aligned quad of
//                rows holds w1[2j], w1[2j+1], w3[2j], w3[2j+1])
// ---------------------------------------------------------------------------
struct RetileArgs {
    const float* src_scales;     // [rows][src_G] (source rows of src_G groups)
    const uint8_t* src_packed;   // [rows][src_G * 16]
    MatDesc m;                   // destination layout (m.w is written)
    long long rows;
    int row_offset, interleave, slot;
    int inverse;                 // 1: tiles -> quantize.c layout
    int src_G, src_g0;           // source groups per row, first source group of the tiles' columns
};

__device__ __forceinline__ int nib(const uint8_t* b, int e) { return (e & 1) ? (b[e >> 1] >> 4) : (b[e >> 1] & 0xF); }

__global__ void k_retile(RetileArgs a) {
    const int G = a.m.G;
    const long long total = a.rows * G;
    uint8_t* base = const_cast<uint8_t*>(a.m.w);
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / G;
        const int g = (int)(i % G);
        const long long R = a.interleave ? (r / 2) * 4 + (r % 2) + a.slot * 2 : a.row_offset + r;
        const int rr = (int)(R % kTR), lr = rr & 7, half = rr >> 3;
        uint8_t* gp = base + (R / kTR) * a.m.tile_bytes + (size_t)g * kGB;
        float* dsc = reinterpret_cast<float*>(gp + 256 + 8 * lr + 4 * half);
        float* ssc = const_cast<float*>(a.src_scales) + r * a.src_G + a.src_g0 + g;
        uint8_t* spk = const_cast<uint8_t*>(a.src_packed) + r * (16LL * a.src_G) + 16 * (a.src_g0 + g);
        if (!a.inverse) {
            uint8_t src[16];
            *reinterpret_cast<uint4*>(src) = *reinterpret_cast<const uint4*>(spk);
            for (int t = 0; t < 4; t++) {
                uint32_t w = 0;
                for (int b = 0; b < 4; b++)
                    w |= (uint32_t)(nib(src, 4 * t + b) | (nib(src, 16 + 4 * t + b) << 4)) << (8 * b);
                *reinterpret_cast<uint32_t*>(gp + 8 * (4 * lr + t) + 4 * half) = w;
            }
            *dsc = *ssc;
        } else {
            uint8_t out[16] = {0};
            for (int t = 0; t < 4; t++) {
                const uint32_t w = *reinterpret_cast<const uint32_t*>(gp + 8 * (4 * lr + t) + 4 * half);
                for (int b = 0; b < 4; b++) {
                    const int lo = (w >> (8 * b)) & 0xF, hi = (w >> (8 * b + 4)) & 0xF;
                    const int e0 = 4 * t + b, e1 = 16 + 4 * t + b;   // both even or both odd with b
                    if (e0 & 1) out[e0 >> 1] = (uint8_t)((out[e0 >> 1] & 0x0F) | (lo << 4));
                    else out[e0 >> 1] = (uint8_t)((out[e0 >> 1] & 0xF0) | lo);
                    if (e1 & 1) out[e1 >> 1] = (uint8_t)((out[e1 >> 1] & 0x0F) | (hi << 4));
                    else out[e1 >> 1] = (uint8_t)((out[e1 >> 1] & 0xF0) | hi);
                }
            }
            *reinterpret_cast<uint4*>(spk) = *reinterpret_cast<const uint4*>(out);
            *ssc = *dsc;
        }
    }
}

// fp32 rows -> fp32 tiles (same row mapping as k_retile).  Thread per
// (row, group, 4 columns).
struct RetileF32Args {
    const float* src;            // [rows][src_n]
    MatDesc m;
    long long rows;
    int row_offset, interleave, slot;
    int src_n, src_g0;           // source row length, first source group of the tiles' columns
};

__global__ void k_retile_f32(RetileF32Args a) {
    const int G = a.m.G;
    const long long total = a.rows * G * 8;
    float* base = reinterpret_cast<float*>(const_cast<uint8_t*>(a.m.w));
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / (8LL * G);
        const int g = (int)((i / 8) % G), e4 = (int)(i % 8);
        const long long R = a.interleave ? (r / 2) * 4 + (r % 2) + a.slot * 2 : a.row_offset + r;
        const int rr = (int)(R % kTR), rl = rr & 7, half = rr >> 3;
        const int q = half * 2 + (e4 & 1), ln = 4 * rl + (e4 >> 1);
        float* dst = base + ((R / kTR) * G + g) * 512 + (q * 32 + ln) * 4;
        const float* src = a.src + r * a.src_n + (a.src_g0 + g) * 32 + 4 * e4;
        *reinterpret_cast<float4*>(dst) = *reinterpret_cast<const float4*>(src);
    }
}

// quantize_buffer (quantize.c:59-109) on the device, bit for bit: per group
// of 32 values scale = max|w| / 7 (0 becomes 1.0), q = clamp(roundf(w *
// (1 / scale)), -7, 7) stored as q + 8, even element in the low nibble.
// One thread per group (its 128 input bytes are whole cache lines).
__global__ void k_quantize_groups(const float* in, uint8_t* packed, float* scales, long long groups) {
    for (long long g = blockIdx.x * (long long)blockDim.x + threadIdx.x; g < groups;
         g += (long long)gridDim.x * blockDim.x) {
        float w[32];
        const float4* src = reinterpret_cast<const float4*>(in + g * 32);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const float4 v = __ldcs(src + i);
            w[4 * i] = v.x;
            w[4 * i + 1] = v.y;
            w[4 * i + 2] = v.z;
            w[4 * i + 3] = v.w;
        }
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < 32; i++) {
            const float a = fabsf(w[i]);
            if (a > amax) amax = a;
        }
        float scale = __fdiv_rn(amax, 7.0f);
        if (scale == 0.0f) scale = 1.0f;
        scales[g] = scale;
        const float inv = __fdiv_rn(1.0f, scale);
        uint32_t words[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            uint32_t wd = 0;
#pragma unroll
            for (int b = 0; b < 4; b++) {
                const int i = 8 * k + 2 * b;
                int q0 = (int)roundf(__fmul_rn(w[i], inv)), q1 = (int)roundf(__fmul_rn(w[i + 1], inv));
                q0 = q0 < -7 ? -7 : (q0 > 7 ? 7 : q0);
                q1 = q1 < -7 ? -7 : (q1 > 7 ? 7 : q1);
                wd |= (uint32_t)(((q0 + 8) & 0xF) | (((q1 + 8) & 0xF) << 4)) << (8 * b);
            }
            words[k] = wd;
        }
        *reinterpret_cast<uint4*>(packed + g * 16) = make_uint4(words[0], words[1], words[2], words[3]);
    }
}

// Padding rows of the last tile: scale 0, nibbles 8 (q = 0).
__global__ void k_fill_pad(MatDesc m) {
    const long long rows_pad = (long long)m.ntiles * kTR;
    const long long total = (rows_pad - m.d) * m.G;
    uint8_t* base = const_cast<uint8_t*>(m.w);
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long R = m.d + i / m.G;
        const int g = (int)(i % m.G);
        const int rr = (int)(R % kTR), lr = rr & 7, half = rr >> 3;
        uint8_t* gp = base + (R / kTR) * m.tile_bytes + (size_t)g * kGB;
        *reinterpret_cast<float*>(gp + 256 + 8 * lr + 4 * half) = 0.0f;
        for (int t = 0; t < 4; t++) *reinterpret_cast<uint32_t*>(gp + 8 * (4 * lr + t) + 4 * half) = 0x88888888u;
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
