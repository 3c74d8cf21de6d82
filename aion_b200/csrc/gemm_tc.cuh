// Dense bf16 GEMM on the 5th-generation tensor cores (sm_100a), for the
// batched prefill: C[M][N] (fp32) = A[M][K] * B[N][K]^T, A and B bf16 with K
// contiguous.  The int4 weights reach it as bf16 tiles written by
// k_pf_dequant (prefill.cuh); the activations as bf16 rows.
//
// A persistent kernel: one CTA per SM walks the 128 x 256 tiles of C in a
// grouped order (kGemmGroupM row tiles a group, column tile by column tile,
// so the CTAs resident at one time share operand tiles in L2):
//   warp 0     TMA producer: 128 x 64 tile of A and 256 x 64 tile of B per
//              K block into a ring of kStages shared-memory stages (128-byte
//              swizzle), completion counted on the stage's full mbarrier; it
//              runs ahead across tile boundaries;
//   warp 1     allocates 2 x 256 TMEM columns (two accumulators), then one
//              thread issues tcgen05.mma (M 128, N 256, K 16; bf16 x bf16 ->
//              fp32 in TMEM) four times per K block, commits each stage back
//              to its empty mbarrier and each finished tile to its
//              accumulator's full mbarrier;
//   warps 2-5  epilogue: tcgen05.ld of a finished accumulator (each warp its
//              TMEM lane quarter, 16 columns at a time), fp32 stores to C,
//              then one arrive per warp on the accumulator's empty mbarrier,
//              while the MMAs of the next tile run into the other one.
// Every wait is bounded; a wait that gives up records an error code in
// *err and the CTA finishes without further work.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "common.cuh"

namespace aion {

constexpr int kGemmBM = 128, kGemmBN = 256, kGemmBK = 64;
constexpr int kGemmStages = 4;
constexpr int kGemmThreads = 192;
constexpr int kGemmABytes = kGemmBM * kGemmBK * 2;   // 16 KB
constexpr int kGemmBBytes = kGemmBN * kGemmBK * 2;   // 32 KB
constexpr int kGemmStageBytes = kGemmABytes + kGemmBBytes;
constexpr int kGemmSmem = kGemmStages * kGemmStageBytes + 1024;   // + room to align to 1024
constexpr uint32_t kGemmWaitLimit = 1u << 26;

// UMMA shared-memory matrix descriptor, K-major with the 128-byte swizzle:
// rows of 128 bytes, 8-row groups 1024 bytes apart (SBO), version 1.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor: bf16 A and B (K-major), fp32 D, M 128, N 256.
constexpr uint32_t kGemmIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kGemmBN >> 3) << 17) |
                                ((uint32_t)(kGemmBM >> 4) << 24);

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

constexpr int kGemmGroupM = 16;   // row tiles per rasterisation group

struct GemmArgs {
    float* C;          // [M][ldc]
    int M, N, K;       // multiples of 128, 256 and 64
    int ldc;
    int* err;          // first error code of any CTA (0 = none)
};

// Origin of tile `id` in the grouped order.
__device__ __forceinline__ void gemm_tile(const GemmArgs& g, int id, int& m0, int& n0) {
    const int mt = g.M / kGemmBM, nt = g.N / kGemmBN;
    const int per_group = kGemmGroupM * nt, gi = id / per_group, first = gi * kGemmGroupM;
    const int gm = min(mt - first, kGemmGroupM), r = id - gi * per_group;
    m0 = (first + r % gm) * kGemmBM;
    n0 = (r / gm) * kGemmBN;
}

__global__ void __launch_bounds__(kGemmThreads, 1)
k_gemm_bf16_tn(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, GemmArgs g) {
    extern __shared__ __align__(1024) unsigned char gsm_raw[];
    __shared__ __align__(8) uint64_t full_bar[kGemmStages], empty_bar[kGemmStages];
    __shared__ __align__(8) uint64_t tfull_bar[2], tempty_bar[2], done_bar;
    __shared__ uint32_t s_tmem, s_issued;
    __shared__ volatile int s_fail;
    unsigned char* gsm =
        gsm_raw + ((1024u - (smem_addr(gsm_raw) & 1023u)) & 1023u);   // stages start 1024-aligned
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntiles = (g.M / kGemmBM) * (g.N / kGemmBN);
    const int nkb = g.K / kGemmBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kGemmStages; s++) {
            mbar_init(smem_addr(&full_bar[s]), 1);
            mbar_init(smem_addr(&empty_bar[s]), 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(smem_addr(&tfull_bar[b]), 1);
            mbar_init(smem_addr(&tempty_bar[b]), 4);   // one arrive per epilogue warp
        }
        mbar_init(smem_addr(&done_bar), 1);
        s_fail = 0;
        s_issued = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&s_tmem)),
                     "r"(2 * kGemmBN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;

    if (warp == 0 && lane == 0) {
        // Producer.  Stage s is reused after the MMAs that read it commit.
        uint32_t it = 0;
        for (int id = blockIdx.x; id < ntiles && !s_fail; id += gridDim.x) {
            int m0, n0;
            gemm_tile(g, id, m0, n0);
            bool ok = true;
            for (int kb = 0; kb < nkb; kb++, it++) {
                const int s = it % kGemmStages;
                const uint32_t round = it / kGemmStages;
                if (round > 0 && !mbar_wait(smem_addr(&empty_bar[s]), (round - 1) & 1, kGemmWaitLimit)) {
                    ok = false;
                    break;
                }
                const uint32_t sa = smem_addr(gsm + s * kGemmStageBytes);
                mbar_arrive_expect_tx(smem_addr(&full_bar[s]), kGemmStageBytes);
                tma_load_2d(sa, &map_a, kb * kGemmBK, m0, smem_addr(&full_bar[s]));
                tma_load_2d(sa + kGemmABytes, &map_b, kb * kGemmBK, n0, smem_addr(&full_bar[s]));
            }
            if (!ok) {
                s_fail = 1;
                break;
            }
        }
        s_issued = it;
    } else if (warp == 1 && lane == 0) {
        // MMA issuer: tile j of this CTA accumulates into buffer j & 1.
        bool ok = true;
        uint32_t it = 0;
        int j = 0;
        for (int id = blockIdx.x; id < ntiles && ok && !s_fail; id += gridDim.x, j++) {
            const int b = j & 1;
            if (j >= 2 && !mbar_wait(smem_addr(&tempty_bar[b]), ((j >> 1) - 1) & 1, kGemmWaitLimit)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t acc = tmem + (uint32_t)(b * kGemmBN);
            for (int kb = 0; kb < nkb; kb++, it++) {
                const int s = it % kGemmStages;
                if (!mbar_wait(smem_addr(&full_bar[s]), (it / kGemmStages) & 1, kGemmWaitLimit)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t sa = smem_addr(gsm + s * kGemmStageBytes);
                const uint64_t adesc = umma_desc_sw128(sa), bdesc = umma_desc_sw128(sa + kGemmABytes);
#pragma unroll
                for (int k = 0; k < kGemmBK / 16; k++)   // 32 bytes of K per step inside the swizzle atom
                    umma_bf16(acc, adesc + 2 * k, bdesc + 2 * k, kGemmIdesc, (kb | k) != 0);
                umma_commit(smem_addr(&empty_bar[s]));
            }
            if (!ok) break;
            umma_commit(smem_addr(&tfull_bar[b]));
        }
        if (!ok) s_fail = 1;
        umma_commit(smem_addr(&done_bar));   // arrives once every issued MMA is complete
    } else if (warp >= 2) {
        // Epilogue: TMEM lane quarter q = warp % 4 holds rows m0 + 32q ..
        const int q = warp & 3;
        int j = 0;
        for (int id = blockIdx.x; id < ntiles; id += gridDim.x, j++) {
            const int b = j & 1;
            const bool full = mbar_wait(smem_addr(&tfull_bar[b]), (j >> 1) & 1, kGemmWaitLimit);
            tc_fence_after();
            if (!full) {
                if (lane == 0) s_fail = 1;
                break;
            }
            int m0, n0;
            gemm_tile(g, id, m0, n0);
            const int row = m0 + 32 * q + lane;
            float* crow = g.C + (size_t)row * g.ldc + n0;
            const uint32_t src = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(b * kGemmBN);
#pragma unroll 1
            for (int c = 0; c < kGemmBN; c += 16) {
                float v[16];
                tmem_ld16(src + (uint32_t)c, v);
#pragma unroll
                for (int i = 0; i < 16; i += 4)
                    *reinterpret_cast<float4*>(crow + c + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_addr(&tempty_bar[b]));
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0 && lane == 0) {
        // Let every issued copy land before the CTA's shared memory goes.
        const uint32_t n = s_issued;
        for (uint32_t it = (n > (uint32_t)kGemmStages ? n - kGemmStages : 0); it < n; it++)
            mbar_wait(smem_addr(&full_bar[it % kGemmStages]), (it / kGemmStages) & 1, 1u << 20);
    }
    if (warp == 1) {
        // Every issued MMA is complete before the accumulators go.
        mbar_wait(smem_addr(&done_bar), 0, kGemmWaitLimit);
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * kGemmBN) : "memory");
    }
    if (threadIdx.x == 0 && s_fail) atomicCAS(g.err, 0, DEV_COPY_TIMEOUT);
}

}  // namespace aion
