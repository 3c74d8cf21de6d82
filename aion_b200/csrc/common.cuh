// Shared device helpers for sm_100a: PDL, mbarriers, bulk (TMA) copies,
// bounded grid barrier, warp reductions, the device-side argmax key and the
// per-step state.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

namespace aion {

// Error codes a kernel can leave in StepState::error (first one wins).
enum DeviceError : int32_t {
    DEV_OK = 0,
    DEV_BAD_INPUT = 1,       // token or position out of range
    DEV_BARRIER_TIMEOUT = 2, // a grid barrier wait gave up
    DEV_COPY_TIMEOUT = 3,    // a bulk-copy mbarrier wait gave up
};

// Per-step state shared by the kernels of one decode step.  A step takes
// pos from pos_next, the token from forced_token (>= 0) or from the previous
// step's argmax key, records the token in the history and publishes
// pos/token for the rest of the step.
struct StepState {
    int32_t pos_next;
    int32_t forced_token;
    int32_t pos;
    int32_t token;
    int32_t error;
    uint32_t barrier;        // grid-barrier arrival counter of the persistent decode kernel
    uint32_t tp_count;       // tensor parallelism: exchanges completed so far (same on every rank)
    uint32_t op_seq;         // ops run by all decode launches so far (tags of the cut-tile parts)
};

// Argmax key: (order-preserving float bits << 32) | (0xFFFFFFFF - index).
// The max over keys picks the largest logit and, among equal logits, the
// smallest index: the first-max rule of the reference greedy loop
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
// The logit a key was made from.
__host__ __device__ inline float key_value(unsigned long long k) {
    const uint32_t ob = (uint32_t)(k >> 32);
    const uint32_t u = (ob & 0x80000000u) ? (ob & 0x7FFFFFFFu) : ~ob;
    float f;
#ifdef __CUDA_ARCH__
    f = __uint_as_float(u);
#else
    memcpy(&f, &u, 4);
#endif
    return f;
}

// ---------------------------------------------------------------------------
// Phase timestamps (profiling builds only, -DAION_PHASE_TIMING): thread 0 of
// every CTA records the global timer at fixed points of each op of the
// first kPhaseSteps steps of a decode launch; aion_phase_dump() copies them
// out.  Normal builds compile PHASE_T to nothing.
// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned long long global_timer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

#ifdef AION_PHASE_TIMING
constexpr int kPhaseSteps = 8, kPhaseOps = 168, kPhaseCtas = 160, kPhaseSlots = 12;
__device__ unsigned long long g_phase[(size_t)kPhaseSteps * kPhaseOps * kPhaseCtas * kPhaseSlots];
// per (step, op, cta): ring-wait ns and group-dot ns summed over the warps,
// chunks, then the latest loop end, loop start and per-warp busy time
__device__ unsigned long long g_phase_w[(size_t)kPhaseSteps * kPhaseOps * kPhaseCtas * 8];
#define PHASE_T(step, op, slot)                                                                               \
    do {                                                                                                      \
        if (threadIdx.x == 0 && (step) < kPhaseSteps && (op) < kPhaseOps && blockIdx.x < kPhaseCtas)          \
            g_phase[(((size_t)(step) * kPhaseOps + (op)) * kPhaseCtas + blockIdx.x) * kPhaseSlots + (slot)] = \
                global_timer();                                                                               \
    } while (0)
#define PHASE_LOOP_START(step, op)                                                              \
    do {                                                                                        \
        if ((threadIdx.x & 31) == 0 && (step) < kPhaseSteps && (op) < kPhaseOps && blockIdx.x < kPhaseCtas) \
            atomicMax(g_phase_w + (((size_t)(step) * kPhaseOps + (op)) * kPhaseCtas + blockIdx.x) * 8 + 4, global_timer()); \
    } while (0)
#define PHASE_W(step, op, wait_ns, mma_ns, n)                                                  \
    do {                                                                                        \
        if ((threadIdx.x & 31) == 0 && (step) < kPhaseSteps && (op) < kPhaseOps && blockIdx.x < kPhaseCtas) { \
            unsigned long long* w_ = g_phase_w + (((size_t)(step) * kPhaseOps + (op)) * kPhaseCtas + blockIdx.x) * 8; \
            atomicAdd(w_, (wait_ns));                                                          \
            atomicAdd(w_ + 1, (mma_ns));                                                       \
            atomicAdd(w_ + 2, (n));                                                            \
            atomicMax(w_ + 3, global_timer());                                                 \
            atomicMax(w_ + 5, (wait_ns) + (mma_ns));                                           \
        }                                                                                       \
    } while (0)
#else
#define PHASE_W(step, op, wait_ns, mma_ns, n) \
    do {                                      \
    } while (0)
#define PHASE_LOOP_START(step, op) \
    do {                           \
    } while (0)
#define PHASE_T(step, op, slot) \
    do {                        \
    } while (0)
#endif

// ---------------------------------------------------------------------------
// Programmatic dependent launch.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------
// Memory helpers.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte asynchronous copy global -> shared (L2 only), and the wait for
// all of this thread's copies.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// ---------------------------------------------------------------------------
// mbarrier + bulk copy (global -> shared, completion counted in bytes).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: false after `limit` unsuccessful polls (each poll itself
// suspends for a hardware-defined interval).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint32_t limit = (1u << 24)) {
    for (uint32_t i = 0; i < limit; i++)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

// ---------------------------------------------------------------------------
// CTA barrier of the compute threads: named barrier 1 over the first
// kComputeThreads threads, so a kernel may run extra (producer) warps that
// never join it.
// ---------------------------------------------------------------------------
constexpr int kComputeThreads = 352;
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(kComputeThreads) : "memory"); }
__device__ __forceinline__ int csync_or(int pred) {
    int r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.s32 p, %1, 0;\n\t"
        "bar.red.or.pred q, 1, %2, p;\n\t"
        "selp.s32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(pred), "n"(kComputeThreads)
        : "memory");
    return r;
}

// ---------------------------------------------------------------------------
// Grid barrier for a kernel whose CTAs are all co-resident (cooperative
// launch).  The counter only grows within a launch; barrier k (0-based)
// completes when it reaches (k + 1) * gridDim.x.  Bounded: after `limit`
// polls the waiting thread records DEV_BARRIER_TIMEOUT and returns false.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_release_u32(uint32_t* p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t ld_relaxed_u64(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_u64(uint64_t* p, uint64_t v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Tagged 64-bit entries: fp32 bits in the low half, a counter in the high half.
__device__ __forceinline__ uint64_t tag_pack(float v, uint32_t ep) {
    return ((uint64_t)ep << 32) | (uint64_t)__float_as_uint(v);
}
__device__ __forceinline__ float tag_val(uint64_t t) { return __uint_as_float((uint32_t)t); }
__device__ __forceinline__ uint32_t tag_ep(uint64_t t) { return (uint32_t)(t >> 32); }
__device__ __forceinline__ int32_t ld_relaxed_i32(const int32_t* p) {
    int32_t v;
    asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void set_error(StepState* st, int32_t code) { atomicCAS(&st->error, 0, code); }

// All threads of the CTA call this; returns false (uniformly) on timeout or
// when another CTA already recorded an error.
__device__ __forceinline__ bool grid_barrier(StepState* st, uint32_t& k, uint32_t limit = (1u << 24)) {
    __shared__ int s_ok;
    csync();
    if (threadIdx.x == 0) {
        // bar.sync orders the CTA's writes before this release, and the
        // release is cumulative, so no separate fence is needed; likewise
        // the acquire below orders every later read of the CTA.
        red_release_add(&st->barrier, 1u);
        const uint32_t target = (k + 1) * gridDim.x;
        int ok = 1;
        uint32_t i = 0;
        while (ld_acquire_u32(&st->barrier) < target) {
            if (++i > limit || ((i & 1023u) == 0 && ld_relaxed_i32(&st->error) != 0)) {
                ok = 0;
                break;
            }
        }
        if (!ok) set_error(st, DEV_BARRIER_TIMEOUT);
        s_ok = ok;
    }
    csync();
    k++;
    return s_ok != 0;
}

// ---------------------------------------------------------------------------
// Reductions.
// ---------------------------------------------------------------------------
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
// Block-wide sum; every thread receives the result.  red: >= 32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    csync();
    if (lane == 0) red[warp] = v;
    csync();
    float t = (lane < kComputeThreads / 32) ? red[lane] : 0.0f;
    return warp_sum(t);
}
// Sum of s and max of m over the compute threads in one exchange (red
// holds at least 16 + kComputeThreads / 32 floats).
__device__ __forceinline__ float2 block_sum_max(float s, float m, float* red) {
    s = warp_sum(s);
    m = warp_max(m);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    csync();
    if (lane == 0) {
        red[warp] = s;
        red[16 + warp] = m;
    }
    csync();
    const bool in = lane < kComputeThreads / 32;
    return make_float2(warp_sum(in ? red[lane] : 0.0f), warp_max(in ? red[16 + lane] : -INFINITY));
}
__device__ __forceinline__ float block_max(float v, float* red) {
    v = warp_max(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    csync();
    if (lane == 0) red[warp] = v;
    csync();
    float t = (lane < kComputeThreads / 32) ? red[lane] : -INFINITY;
    return warp_max(t);
}

}  // namespace aion
