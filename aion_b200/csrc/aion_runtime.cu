// Host side of libaion: the C ABI declared in include/aion.h.
//
// Replaces the reference's loader, run state, thread pool and forward driver
// (src/kernel_simd.c:631-787, 906-1169).  The int4 checkpoint is uploaded
// once and re-tiled in HBM; decode runs as one persistent cooperative kernel
// per launch (one CTA per SM) that executes `steps` greedy tokens; one
// decode step is captured once as a CUDA graph and replayed per token.  No
// host thread spins; nothing here exits the process.
#include <cuda_runtime.h>
#include <errno.h>
#include <fcntl.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>
#include <sys/stat.h>
#include <time.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include <cudaTypedefs.h>

#include "../../include/aion.h"
#include "decode_batch.cuh"
#include "decode_step.cuh"
#include "gemm_tc.cuh"
#include "prefill.cuh"

using namespace aion;

// ---------------------------------------------------------------------------
// Errors
// ---------------------------------------------------------------------------
static thread_local std::string g_thread_err;

static void set_err(std::string* dst, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    if (dst) *dst = buf;
    g_thread_err = buf;
}

static aion_status cuda_status(cudaError_t e) {
    return e == cudaErrorMemoryAllocation ? AION_ERR_OOM : AION_ERR_CUDA;
}

#define CK_RET(errp, call)                                                                          \
    do {                                                                                            \
        cudaError_t e_ = (call);                                                                    \
        if (e_ != cudaSuccess) {                                                                    \
            set_err(errp, "CUDA error %s (%s) at %s:%d", cudaGetErrorName(e_), cudaGetErrorString(e_), \
                    __FILE__, __LINE__);                                                            \
            return cuda_status(e_);                                                                 \
        }                                                                                           \
    } while (0)

// ---------------------------------------------------------------------------
// Device properties and launch geometry
// ---------------------------------------------------------------------------
struct DevInfo {
    int sms = 0, smem_optin = 0;
};
static DevInfo g_dev[64];

static const DevInfo& dev_info(int dev) {
    static DevInfo fallback = {148, 227 * 1024};
    if (dev < 0 || dev >= 64) return fallback;
    DevInfo& d = g_dev[dev];
    if (!d.sms) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
        d.sms = v;
        v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess || v <= 0)
            v = 227 * 1024;
        d.smem_optin = v;
    }
    return d;
}

static int round128(int b) { return (b + 127) & ~127; }

// Opts a kernel into `bytes` of dynamic shared memory on the current device
// once per (device, kernel slot); thread-safe.  The attribute belongs to the
// device's context, so a second device needs its own call; devices beyond
// the table get the call every time.
enum AttrSlot { ATTR_MATVEC_W4A16 = 0, ATTR_MATVEC_W4A8 = 1, ATTR_GEMM = 2, ATTR_SLOTS = 3 };
constexpr int kMaxAttrDevices = 64;
static cudaError_t ensure_smem_attr(const void* fn, int slot, int dev, int bytes) {
    static std::mutex mu;
    static bool done[kMaxAttrDevices][ATTR_SLOTS] = {};
    if (dev < 0 || dev >= kMaxAttrDevices)
        return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    std::lock_guard<std::mutex> lock(mu);
    if (done[dev][slot]) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) done[dev][slot] = true;
    return e;
}

// Dynamic shared memory plan of the streaming kernels: activation digits
// (G * 128 bytes) and group factors (G * 4), the op table (decode kernel),
// then the per-warp rings of P slots.
struct SmemPlan {
    int xbytes = 0, xs_off = 0, ring_off = 0, slot_bytes = 0, P = 0, total = 0;
};

static SmemPlan plan_smem(int max_n, int max_chunk_bytes, int smem_optin, int static_bytes, int min_xbytes = 0,
                          int ops_bytes = 0) {
    SmemPlan p;
    const int G = max_n / 32;
    p.xs_off = G * kXF;
    p.xbytes = round128(std::max(xbuf_bytes(max_n), min_xbytes));
    p.ring_off = p.xbytes + round128(ops_bytes);
    p.slot_bytes = round128(max_chunk_bytes);
    const int avail = smem_optin - static_bytes - 1024 - p.ring_off;
    p.P = std::min(8, avail / (kWarps * p.slot_bytes));
    p.total = p.ring_off + kWarps * std::max(p.P, 0) * p.slot_bytes;
    return p;
}

// Chunk count of a matrix streamed by the decode / matvec kernels in split
// mode: among the cuts into nch0 .. 3 nch0 chunks per tile whose largest
// chunk is no larger than the default cut's (the ring slot), the one whose
// busiest warp of any CTA has the least work under the kernels' own split,
// counting a chunk as kChunkCost groups more than its groups (its ring round
// trip and bookkeeping).  Ties keep fewer chunks.  With 7B shapes on 148
// SMs: QKV 7 -> 8, WO 7 -> 11, W2 18 -> 19, classifier 7 -> 8, W13 stays 7.
constexpr int kChunkCost = 4;

static void tune_chunks(MatDesc& m, int mode, int grid) {
    if (grid <= 0 || !op_work_at(m, mode, 0, grid).split) return;   // whole tiles: the cut does not split the work
    const int nch0 = m.nch, max_bytes = max_chunk_bytes(m);
    int best = nch0;
    long long best_cost = -1;
    for (int nch = nch0; nch <= 3 * nch0; nch++) {
        MatDesc t = m;
        set_chunks(t, nch);
        if (t.nch != nch || max_chunk_bytes(t) > max_bytes) continue;
        long long worst = 0;
        for (int c = 0; c < grid; c++) {
            const OpWork w = op_work_at(t, mode, c, grid);
            for (int k = 0; k < kWarps; k++) {
                OpCursor cu;
                long long cost = 0;
                for (bool more = cursor_begin(cu, w, t, k); more; more = cursor_next(cu, w, t))
                    cost += chunk_g0(t, cu.c + 1) - chunk_g0(t, cu.c) + kChunkCost;
                worst = std::max(worst, cost);
            }
        }
        if (best_cost < 0 || worst < best_cost) {
            best_cost = worst;
            best = nch;
        }
    }
    set_chunks(m, best);
}

template <typename... KArgs, typename... Args>
static cudaError_t launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                             bool coop, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        na++;
    }
    if (coop) {
        attr[na].id = cudaLaunchAttributeCooperative;
        attr[na].val.cooperative = 1;
        na++;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Source rows hold src_G groups; the tiles take groups [src_g0, src_g0 + m.G)
// of each (src_G = 0: the tiles' own width).
// fp32 rows [rows][src_n] (columns from group src_g0) into fp32 tiles.
static cudaError_t retile_f32(const MatDesc& m, const float* src, long long rows, int row_offset, int interleave,
                              int slot, int src_n, int src_g0, cudaStream_t st) {
    RetileF32Args a;
    a.src = src;
    a.m = m;
    a.rows = rows;
    a.row_offset = row_offset;
    a.interleave = interleave;
    a.slot = slot;
    a.src_n = src_n;
    a.src_g0 = src_g0;
    const long long total = rows * m.G * 8;
    int grid = (int)std::min<long long>((total + 255) / 256, 65535);
    if (grid < 1) grid = 1;
    k_retile_f32<<<grid, 256, 0, st>>>(a);
    return cudaGetLastError();
}

static cudaError_t retile(const MatDesc& m, const float* scales, const uint8_t* packed, long long rows, int row_offset,
                          int interleave, int slot, int inverse, cudaStream_t st, int src_G = 0, int src_g0 = 0) {
    RetileArgs a;
    a.src_G = src_G > 0 ? src_G : m.G;
    a.src_g0 = src_g0;
    a.src_scales = scales;
    a.src_packed = packed;
    a.m = m;
    a.rows = rows;
    a.row_offset = row_offset;
    a.interleave = interleave;
    a.slot = slot;
    a.inverse = inverse;
    const long long total = rows * m.G;
    int grid = (int)std::min<long long>((total + 255) / 256, 65535);
    if (grid < 1) grid = 1;
    k_retile<<<grid, 256, 0, st>>>(a);
    return cudaGetLastError();
}

static cudaError_t fill_pad(const MatDesc& m, cudaStream_t st) {
    if ((long long)m.ntiles * kTR == m.d) return cudaSuccess;
    k_fill_pad<<<8, 256, 0, st>>>(m);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Standalone matvec (kernel-level API)
// ---------------------------------------------------------------------------
struct Scratch {
    uint64_t* split_part = nullptr;   // [ntiles][16] tagged partial rows of cut tiles
    int* error = nullptr;
};

// `epoch` tags this call's cut-tile flags (nonzero, different from the
// previous call's on the same scratch), so a flag that a call which gave up
// left behind is never taken for the next call's.
template <int MODE>
static cudaError_t launch_standalone(const MatDesc& m, const Scratch& sc, const float* x, float* y, int dev,
                                     cudaStream_t st, uint32_t epoch) {
    const DevInfo& di = dev_info(dev);
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, k_matvec<MODE>);
    if (e != cudaSuccess) return e;
    SmemPlan p = plan_smem(m.n, max_chunk_bytes(m), di.smem_optin, (int)fa.sharedSizeBytes);
    if (p.P < 1) return cudaErrorInvalidConfiguration;
    e = ensure_smem_attr((const void*)k_matvec<MODE>, MODE == MODE_W4A8 ? ATTR_MATVEC_W4A8 : ATTR_MATVEC_W4A16, dev,
                         di.smem_optin - (int)fa.sharedSizeBytes);
    if (e != cudaSuccess) return e;
    StandaloneArgs a;
    a.epoch = epoch;
    a.op.m = m;
    a.op.kind = OP_STORE;
    a.op.layer = 0;
    a.x = x;
    a.y = y;
    a.split_part = sc.split_part;
    a.error = sc.error;
    a.P = p.P;
    a.slot_bytes = p.slot_bytes;
    a.xbytes = p.ring_off;
    a.xs_off = p.xs_off;
    return launch_ex(k_matvec<MODE>, dim3(di.sms), dim3(kThreads), (size_t)p.total, st, true, false, a);
}

// ---------------------------------------------------------------------------
// Context
// ---------------------------------------------------------------------------
struct aion_ctx {
    std::string err;
    aion_opts opts;
    aion_config cfg;
    int dev = 0, mode = 0;
    int nseq = 1;                  // sequences (KV caches) held; opts.max_batch
    int cur_seq = 0;               // the sequence decode / forward calls run on
    size_t kv_seq = 0;             // floats per sequence in kcache / vcache
    struct PrefillBufs {           // grown on demand by aion_prefill
        __nv_bfloat16 *a = nullptr, *b = nullptr;
        float *c = nullptr, *x = nullptr, *q = nullptr;
        int32_t* tok = nullptr;
        int* map = nullptr;
        size_t a_cap = 0, b_cap = 0, c_cap = 0, x_cap = 0, q_cap = 0, tok_cap = 0, map_cap = 0;
    } pf;
    struct BatchBufs {             // lock-step batched decode, allocated on first use
        float *x = nullptr, *q = nullptr, *att = nullptr, *logits = nullptr;
        float *part = nullptr, *ssq = nullptr;
        unsigned char* dg = nullptr;
        unsigned long long* argmax = nullptr;
        int32_t *first = nullptr, *pos0 = nullptr, *tokens = nullptr;
        size_t part_cap = 0, tok_cap = 0;
        int nb = 0;                // sequences the fixed buffers hold
        struct Plan {
            BOpDesc* ops = nullptr;
            int P = 0, ring_off = 0, ops_off = 0, total = 0;
            size_t part_floats = 0;
        } plan[kBMaxSeq / 8 + 1];
    } bt;
    uint32_t* exp_tab = nullptr;   // W4A8: inputs where the host expf is not correctly rounded
    int exp_n = 0;
    double exp_delta = 0.0;
    long long dim = 0, hidden = 0, L = 0, nh = 0, nkv = 0, vocab = 0, seq = 0, hs = 0, kv_dim = 0, kv_mul = 0;
    // This rank's share under tensor parallelism (the full sizes when tp_n == 1).
    int tp_n = 1, tp_rank = 0;
    long long q_l = 0, kv_l = 0, hid_l = 0, nh_l = 0, vocab_l = 0, vocab_off = 0;
    MatDesc cls;                   // classifier rows of this rank: a view of emb
    unsigned char* xr = nullptr;   // exchange region (receive rows, keys, flags)
    size_t xr_bytes = 0;
    int xr_keys_off = 0, xr_flags_off = 0;
    long long xr_brecv_off = 0, xr_bkeys_off = 0;   // batched decode: partial rows, argmax keys
    int xr_nbmax = 0;
    std::vector<unsigned char*> peers;           // exchange regions of every rank (IPC-mapped)
    unsigned char** peers_dev = nullptr;         // the same pointers in device memory
    bool tp_connected = false;
    int max_pos = 0;
    cudaStream_t stream = nullptr;
    uint8_t* arena = nullptr;
    size_t arena_bytes = 0, arena_used = 0;
    MatDesc emb;
    std::vector<MatDesc> qkv, wo, w13, w2;
    float *rms_att = nullptr, *rms_ffn = nullptr, *rms_final = nullptr, *freq_re = nullptr, *freq_im = nullptr;
    float *kcache = nullptr, *vcache = nullptr;
    float *x = nullptr, *q = nullptr, *att = nullptr, *hb = nullptr, *logits = nullptr;
    float* attn_part = nullptr;
    int* attn_cnt = nullptr;
    int max_chunks = 1;
    uint64_t* split_part = nullptr;
    int max_tiles = 0;
    StepState* step = nullptr;
    unsigned long long* argmax = nullptr;
    int32_t* history = nullptr;
    OpDesc* ops = nullptr;
    int nops = 0;
    SmemPlan plan;
    int grid = 0;
    StepState* h_step = nullptr;   // pinned
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t gexec = nullptr;
    SamplerParams samp = {};       // sampling (aion_set_sampler); off: greedy
    int sampling = 0;
};

static uint8_t* arena_take(aion_ctx* c, size_t bytes) {
    size_t off = (c->arena_used + 255) & ~(size_t)255;
    if (off + bytes > c->arena_bytes) return nullptr;
    c->arena_used = off + bytes;
    return c->arena + off;
}

static size_t align256(size_t b) { return (b + 255) & ~(size_t)255; }

extern "C" AION_API void aion_default_opts(aion_opts* o) {
    if (!o) return;
    memset(o, 0, sizeof(*o));
    o->mode = AION_MODE_W4A16;
    o->max_batch = 1;
    o->tp_size = 1;
    o->use_graph = 1;
}

extern "C" AION_API const char* aion_last_error(const aion_ctx* ctx) {
    if (ctx) return ctx->err.c_str();
    return g_thread_err.c_str();
}

// ---------------------------------------------------------------------------
// The host C library's expf, tabulated.  The reference's softmax and SwiGLU
// call expf; its results are correctly rounded except on a small set of
// inputs.  Calling it on every float x with a finite non-zero result and
// comparing with the correctly rounded e^x finds that set once per process
// (about 2^31 calls, spread over the host's cores).  The device keeps the
// sorted list and the largest distance of e^x from a rounding midpoint over
// the listed inputs (see expf_host).  If the library ever returned a value
// other than one of the two floats around e^x, the table could not express
// it and is not used.
// ---------------------------------------------------------------------------
struct HostExpTable {
    std::vector<uint32_t> x;
    double delta = 0.0;
    bool usable = false;
};

// Correctly rounded e^x: the double exponential rounded to float, or, when
// that lands within 1e-6 result ulp of a midpoint, the long double one.
static float cr_expf_host(float x) {
    const double d = std::exp((double)x);
    const float f = (float)d;
    if (!std::isfinite(f)) return f;
    const float o = (double)f < d ? std::nextafterf(f, INFINITY) : std::nextafterf(f, 0.0f);
    const double mid = 0.5 * ((double)f + (double)o), ulp = std::fabs((double)o - (double)f);
    if (ulp > 0.0 && std::fabs(d - mid) > 1e-6 * ulp) return f;
    return (float)expl((long double)x);
}

static const HostExpTable& host_exp_table() {
    static HostExpTable t;
    static std::once_flag once;
    std::call_once(once, [] {
        // x in [0, 88.75) and (-104, -0]: every float whose e^x is a finite,
        // non-zero float lies in these bit ranges.
        const uint64_t ranges[2][2] = {{0x00000000u, 0x42B20000u}, {0x80000000u, 0xC2D00000u}};
        const int nt = std::max(1u, std::thread::hardware_concurrency());
        std::vector<std::vector<uint32_t>> found(nt);
        std::vector<double> dmax(nt, 0.0);
        std::vector<int> bad(nt, 0);
        std::vector<std::thread> th;
        for (int k = 0; k < nt; k++)
            th.emplace_back([&, k] {
                for (const auto& r : ranges) {
                    const uint64_t len = r[1] - r[0], b0 = r[0] + len * k / nt, b1 = r[0] + len * (k + 1) / nt;
                    for (uint64_t b = b0; b < b1; b++) {
                        float x;
                        const uint32_t u = (uint32_t)b;
                        memcpy(&x, &u, 4);
                        const float g = expf(x);
                        const double d = std::exp((double)x);
                        const float f = (float)d;
                        if (g == f) {
                            // f may still be off when d sits on a midpoint;
                            // then the long double value decides.
                            const float o = (double)f < d ? std::nextafterf(f, INFINITY) : std::nextafterf(f, 0.0f);
                            const double ulp = std::fabs((double)o - (double)f);
                            if (!(ulp > 0.0) || std::fabs(d - 0.5 * ((double)f + (double)o)) > 1e-6 * ulp) continue;
                        }
                        const float c = cr_expf_host(x);
                        if (g == c) continue;
                        if (std::nextafterf(c, g) != g) {
                            bad[k]++;
                            continue;
                        }
                        const long double e = expl((long double)x);
                        const long double mid = 0.5L * ((long double)c + (long double)g);
                        const long double ulp = fabsl((long double)g - (long double)c);
                        dmax[k] = std::max(dmax[k], (double)(fabsl(e - mid) / ulp));
                        found[k].push_back(u);
                    }
                }
            });
        for (auto& h : th) h.join();
        int nbad = 0;
        for (int k = 0; k < nt; k++) {
            t.x.insert(t.x.end(), found[k].begin(), found[k].end());
            t.delta = std::max(t.delta, dmax[k]);
            nbad += bad[k];
        }
        std::sort(t.x.begin(), t.x.end());
        t.delta += 1e-6;   // room for the device's double exponential
        t.usable = nbad == 0 && t.x.size() < (1u << 30);
    });
    return t;
}

static void ctx_destroy(aion_ctx* c) {
    if (!c) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(c->dev);
    if (c->stream) cudaStreamSynchronize(c->stream);
    if (c->gexec) cudaGraphExecDestroy(c->gexec);
    if (c->graph) cudaGraphDestroy(c->graph);
    if (c->arena) cudaFree(c->arena);
    if (c->exp_tab) cudaFree(c->exp_tab);
    for (int j = 0; j < (int)c->peers.size(); j++)
        if (j != c->tp_rank && c->peers[j]) cudaIpcCloseMemHandle(c->peers[j]);
    if (c->peers_dev) cudaFree(c->peers_dev);
    if (c->xr) cudaFree(c->xr);
    for (void* p : {(void*)c->pf.a, (void*)c->pf.b, (void*)c->pf.c, (void*)c->pf.x, (void*)c->pf.q,
                    (void*)c->pf.tok, (void*)c->pf.map})
        if (p) cudaFree(p);
    for (void* p : {(void*)c->bt.x, (void*)c->bt.q, (void*)c->bt.att, (void*)c->bt.dg, (void*)c->bt.logits,
                    (void*)c->bt.part, (void*)c->bt.ssq, (void*)c->bt.argmax, (void*)c->bt.first, (void*)c->bt.pos0, (void*)c->bt.tokens})
        if (p) cudaFree(p);
    for (auto& pl : c->bt.plan)
        if (pl.ops) cudaFree(pl.ops);
    if (c->h_step) cudaFreeHost(c->h_step);
    if (c->stream) cudaStreamDestroy(c->stream);
    cudaSetDevice(prev);
    delete c;
}

extern "C" AION_API aion_status aion_free(aion_ctx* ctx) {
    ctx_destroy(ctx);
    return AION_OK;
}

extern "C" AION_API aion_status aion_get_config(const aion_ctx* ctx, aion_config* out) {
    if (!ctx || !out) return AION_ERR_ARG;
    *out = ctx->cfg;
    return AION_OK;
}

extern "C" AION_API const float* aion_logits_dev(const aion_ctx* ctx) { return ctx ? ctx->logits : nullptr; }

extern "C" AION_API int32_t aion_get_mode(const aion_ctx* ctx) {
    if (!ctx) return -1;
    return ctx->mode == MODE_F32 ? AION_MODE_F32 : ctx->mode == MODE_W4A8 ? AION_MODE_W4A8 : AION_MODE_W4A16;
}

extern "C" AION_API void* aion_stream(const aion_ctx* c) { return c ? (void*)c->stream : nullptr; }

// Byte size of an int4 checkpoint for a header, 64-bit.
static long long int4_file_bytes(const aion_config& c) {
    long long dim = c.dim, hid = c.hidden_dim, L = c.n_layers, nh = c.n_heads, nkv = c.n_kv_heads,
              vocab = c.vocab_size, seq = c.seq_len;
    long long hs = dim / nh, kv = dim * nkv / nh;
    auto qb = [](long long cnt) { return cnt / 32 * 4 + cnt / 2; };
    return 28 + qb(vocab * dim) + L * dim * 4 + qb(L * dim * dim) + 2 * qb(L * dim * kv) + qb(L * dim * dim) +
           L * dim * 4 + 3 * qb(L * dim * hid) + dim * 4 + 2 * seq * (hs / 2) * 4;
}

// ---------------------------------------------------------------------------
// Decode launches
// ---------------------------------------------------------------------------
template <int MODE>
static cudaError_t launch_decode_mode(aion_ctx* c, int steps) {
    DecodeArgs a;
    a.ops = c->ops;
    a.nops = c->nops;
    a.emb = c->emb;
    a.dim = (int)c->dim;
    a.hidden = (int)c->hid_l;
    a.n_layers = (int)c->L;
    a.n_heads = (int)c->nh_l;
    a.kv_mul = (int)c->kv_mul;
    a.head_size = (int)c->hs;
    a.kv_dim = (int)c->kv_l;
    a.vocab = (int)c->vocab;
    a.q_dim = (int)c->q_l;
    a.tp_n = c->tp_n;
    a.tp_rank = c->tp_rank;
    a.vocab_off = (int)c->vocab_off;
    a.tp_peers = c->peers_dev;
    a.tp_keys_off = c->xr_keys_off;
    a.tp_flags_off = c->xr_flags_off;
    a.max_pos = c->max_pos;
    a.rms_att = c->rms_att;
    a.rms_ffn = c->rms_ffn;
    a.rms_final = c->rms_final;
    a.freq_re = c->freq_re;
    a.freq_im = c->freq_im;
    a.x = c->x;
    a.q = c->q;
    a.att = c->att;
    a.hb = c->hb;
    a.logits = c->logits;
    a.kcache = c->kcache + (size_t)c->cur_seq * c->kv_seq;
    a.vcache = c->vcache + (size_t)c->cur_seq * c->kv_seq;
    a.attn_part = c->attn_part;
    a.attn_cnt = c->attn_cnt;
    a.max_chunks = c->max_chunks;
    a.split_part = c->split_part;
    a.step = c->step;
    a.argmax = c->argmax;
    a.history = c->history;
    a.steps = steps;
    a.P = c->plan.P;
    a.slot_bytes = c->plan.slot_bytes;
    a.xbytes = c->plan.ring_off;
    a.xs_off = c->plan.xs_off;
    a.ops_off = c->plan.xbytes;
    a.exp_host.x = c->exp_tab;
    a.exp_host.n = c->exp_n;
    a.exp_host.delta = c->exp_delta;
    a.cr_exp = MODE != MODE_W4A16;
    a.wait_ns = (unsigned long long)(c->opts.wait_ms > 0 ? c->opts.wait_ms : 2000) * 1000000ull;
    a.samp = c->samp;
    a.sampling = c->sampling;
    // The grid-barrier counter starts from zero in every launch.
    cudaError_t e = cudaMemsetAsync(&c->step->barrier, 0, sizeof(uint32_t), c->stream);
    if (e != cudaSuccess) return e;
    return launch_ex(k_decode<MODE>, dim3(c->grid), dim3(kDecodeThreads), (size_t)c->plan.total, c->stream, false, true, a);
}

static cudaError_t launch_decode(aion_ctx* c, int steps) {
    if (c->mode == MODE_F32) return launch_decode_mode<MODE_F32>(c, steps);
    return c->mode == MODE_W4A8 ? launch_decode_mode<MODE_W4A8>(c, steps) : launch_decode_mode<MODE_W4A16>(c, steps);
}

static aion_status build_graph(aion_ctx* c) {
    if (c->gexec) return AION_OK;
    CK_RET(&c->err, cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    cudaError_t e = launch_decode(c, 1);
    cudaGraph_t g = nullptr;
    cudaError_t e2 = cudaStreamEndCapture(c->stream, &g);
    if (e != cudaSuccess || e2 != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        set_err(&c->err, "graph capture failed: %s / %s", cudaGetErrorString(e), cudaGetErrorString(e2));
        return AION_ERR_CUDA;
    }
    c->graph = g;
    CK_RET(&c->err, cudaGraphInstantiate(&c->gexec, g, 0));
    return AION_OK;
}

// Enqueues `steps` decode steps: one graph replay when steps == 1 and graphs
// are on, else one launch that runs all steps.
static aion_status tp_ready(aion_ctx* c);

static aion_status enqueue_steps(aion_ctx* c, int steps) {
    if (steps <= 0) return AION_OK;
    const aion_status ready = tp_ready(c);
    if (ready != AION_OK) return ready;
    if (steps == 1 && c->opts.use_graph) {
        aion_status s = build_graph(c);
        if (s != AION_OK) return s;
        CK_RET(&c->err, cudaGraphLaunch(c->gexec, c->stream));
        return AION_OK;
    }
    CK_RET(&c->err, launch_decode(c, steps));
    return AION_OK;
}

// The step state's error word, read from the copy in c->h_step.
static aion_status decode_device_error(aion_ctx* c) {
    switch (c->h_step->error) {
    case DEV_OK: return AION_OK;
    case DEV_BAD_INPUT:
        set_err(&c->err, "a decode step rejected its token or position");
        return AION_ERR_STATE;
    default:
        set_err(&c->err, "a bounded device wait gave up (code %d); call aion_reset", c->h_step->error);
        return AION_ERR_TIMEOUT;
    }
}
static aion_status check_device_error(aion_ctx* c) {
    CK_RET(&c->err, cudaMemcpy(c->h_step, c->step, sizeof(StepState), cudaMemcpyDeviceToHost));
    return decode_device_error(c);
}

// ---------------------------------------------------------------------------
// Loading
// ---------------------------------------------------------------------------
static aion_status validate_config(const aion_config& c, std::string* err) {
    if (c.dim <= 0 || c.hidden_dim <= 0 || c.n_layers <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 || c.vocab_size <= 0 ||
        c.seq_len <= 0) {
        set_err(err, "header has a non-positive field");
        return AION_ERR_FORMAT;
    }
    if (c.dim % c.n_heads || c.n_heads % c.n_kv_heads) {
        set_err(err, "dim %% n_heads or n_heads %% n_kv_heads is not zero");
        return AION_ERR_SHAPE;
    }
    const long long hs = c.dim / c.n_heads, kv = (long long)c.dim * c.n_kv_heads / c.n_heads;
    if (hs % 16 || hs > kMaxHead || c.dim % 32 || c.hidden_dim % 32 || kv % 32 ||
        c.dim > kMaxNormVec * 4 * kThreads || c.hidden_dim > kMaxVec * 4 * kThreads) {
        set_err(err,
                "unsupported shape: head_size %lld, dim %d, hidden %d, kv_dim %lld (need head_size a multiple of 16, "
                "<= %d; dim, hidden, kv_dim multiples of 32, dim <= %d, hidden <= %d)",
                hs, c.dim, c.hidden_dim, kv, kMaxHead, kMaxNormVec * 4 * kThreads, kMaxVec * 4 * kThreads);
        return AION_ERR_SHAPE;
    }
    return AION_OK;
}

// Reads and validates the 28-byte header and the file size (64-bit) before
// any device work: a truncated or inconsistent file fails here.
// Byte size of an fp32 llama2.c file (src/kernel_simd.c:906-936) for a
// header, 64-bit; a negative vocab_size announces a separate classifier
// after the RoPE tables, which the reference never reads.
static long long f32_file_bytes(const aion_config& c, bool wcls) {
    long long dim = c.dim, hid = c.hidden_dim, L = c.n_layers, nh = c.n_heads, nkv = c.n_kv_heads,
              vocab = c.vocab_size, seq = c.seq_len;
    long long hs = dim / nh, kv = dim * nkv / nh;
    long long f = vocab * dim + L * dim + L * dim * dim + 2 * L * dim * kv + L * dim * dim + L * dim + 3 * L * dim * hid +
                  dim + 2 * seq * (hs / 2) + (wcls ? vocab * dim : 0);
    return 28 + 4 * f;
}

static aion_status read_header(const char* path, aion_config* cfg, std::string* err, bool* f32 = nullptr) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) {
        set_err(err, "cannot open %s: %s", path, strerror(errno));
        return AION_ERR_IO;
    }
    struct stat st;
    int32_t hdr[7];
    aion_status s = AION_OK;
    if (fstat(fd, &st) != 0 || st.st_size < 28 || pread(fd, hdr, 28, 0) != 28) {
        set_err(err, "%s: file shorter than the 28-byte header", path);
        s = AION_ERR_FORMAT;
    } else {
        memcpy(cfg, hdr, 28);
        const bool wcls = cfg->vocab_size < 0;
        if (cfg->vocab_size < 0) cfg->vocab_size = -cfg->vocab_size;  // src/kernel_simd.c:945
        s = validate_config(*cfg, err);
        if (f32) *f32 = false;
        if (s == AION_OK) {
            const long long want = int4_file_bytes(*cfg), want_f = f32_file_bytes(*cfg, wcls);
            if (f32 && want_f == (long long)st.st_size && want != want_f) {
                *f32 = true;   // the reference's fp32 path (its CLI without "int4")
            } else if (want != (long long)st.st_size) {
                set_err(err, "%s: header implies %lld bytes for an int4 file (%lld for fp32), file has %lld", path,
                        want, want_f, (long long)st.st_size);
                s = AION_ERR_FORMAT;
            }
        }
    }
    close(fd);
    return s;
}

static aion_status upload_range(aion_ctx* c, int fd, long long off, long long bytes, uint8_t* dst, uint8_t* pinned[2],
                                cudaEvent_t ev[2], size_t chunk) {
    long long done = 0;
    int i = 0;
    while (done < bytes) {
        size_t n = (size_t)std::min<long long>(bytes - done, (long long)chunk);
        CK_RET(&c->err, cudaEventSynchronize(ev[i]));
        size_t got = 0;
        while (got < n) {
            ssize_t r = pread(fd, pinned[i] + got, n - got, (off_t)(off + done + (long long)got));
            if (r < 0 && errno == EINTR) continue;
            if (r <= 0) {
                set_err(&c->err, "read failed at offset %lld: %s", off + done, r < 0 ? strerror(errno) : "end of file");
                return AION_ERR_IO;
            }
            got += (size_t)r;
        }
        CK_RET(&c->err, cudaMemcpyAsync(dst + done, pinned[i], n, cudaMemcpyHostToDevice, c->stream));
        CK_RET(&c->err, cudaEventRecord(ev[i], c->stream));
        done += (long long)n;
        i ^= 1;
    }
    return AION_OK;
}

template <int MODE>
static aion_status setup_decode_kernel(aion_ctx* c, int max_n, int max_chunk) {
    const DevInfo& di = dev_info(c->dev);
    cudaFuncAttributes fa;
    CK_RET(&c->err, cudaFuncGetAttributes(&fa, k_decode<MODE>));
    // W4A8 stages the RMSNorm input (dim floats) and the reference-order
    // attention scores (max_pos floats) in the digit area; the sampler uses
    // it as scratch between steps.
    const int stage = MODE == MODE_W4A8 ? std::max(c->max_pos, (int)c->dim) * 4 : 0;
    c->plan = plan_smem(max_n, max_chunk, di.smem_optin, (int)fa.sharedSizeBytes, std::max(stage, kSampleScratch),
                        (int)(c->nops * sizeof(OpDesc)));
    if (c->plan.P < 2) {
        set_err(&c->err, "shared memory too small for the decode rings (P = %d)", c->plan.P);
        return AION_ERR_SHAPE;
    }
    CK_RET(&c->err, cudaFuncSetAttribute(k_decode<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, c->plan.total));
    int nb = 0;
    CK_RET(&c->err, cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, k_decode<MODE>, kDecodeThreads, c->plan.total));
    if (nb < 1) {
        set_err(&c->err, "decode kernel cannot be resident (smem %d)", c->plan.total);
        return AION_ERR_CUDA;
    }
    c->grid = di.sms;
    return AION_OK;
}

static aion_status load_impl(aion_ctx* c, const char* path) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) {
        set_err(&c->err, "cannot open %s: %s", path, strerror(errno));
        return AION_ERR_IO;
    }
    aion_status s = AION_OK;
    uint8_t* pinned[2] = {nullptr, nullptr};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    uint8_t* staging = nullptr;
    const size_t chunk = 32u << 20;
    do {
        c->dim = c->cfg.dim; c->hidden = c->cfg.hidden_dim; c->L = c->cfg.n_layers; c->nh = c->cfg.n_heads;
        c->nkv = c->cfg.n_kv_heads; c->vocab = c->cfg.vocab_size; c->seq = c->cfg.seq_len;
        c->hs = c->dim / c->nh; c->kv_dim = c->dim * c->nkv / c->nh; c->kv_mul = c->nh / c->nkv;
        c->max_pos = c->opts.max_pos > 0 ? c->opts.max_pos : (int)c->seq;
        if (c->max_pos > c->seq) {
            set_err(&c->err, "max_pos %d exceeds the header seq_len %lld (RoPE tables end there)", c->max_pos, c->seq);
            s = AION_ERR_ARG;
            break;
        }
        c->max_chunks = (c->max_pos + kAttnUnit - 1) / kAttnUnit;
        const long long dim = c->dim, hid = c->hidden, L = c->L, kv = c->kv_dim;
        const long long R = c->tp_rank;
        int64_t plan[AION_TP_PLAN_FIELDS];
        if (aion_tp_plan(&c->cfg, c->tp_n, c->tp_rank, plan) != AION_OK) {
            set_err(&c->err,
                    "tensor parallelism over %d ranks needs n_heads, n_kv_heads divisible by it, dim/%d and "
                    "hidden/%d multiples of 32 and vocab a multiple of %d", c->tp_n, c->tp_n, c->tp_n, c->tp_n * kTR);
            s = AION_ERR_SHAPE;
            break;
        }
        c->q_l = plan[1];
        c->kv_l = plan[3];
        c->hid_l = plan[5];
        c->vocab_off = plan[6];
        c->vocab_l = plan[7];
        c->nh_l = plan[8];
        const long long ql = c->q_l, kvl = c->kv_l, hl = c->hid_l;

        // Matrix layouts (pointers filled below).  Under tensor parallelism
        // this rank holds wq/wk/wv/w1/w3 rows [R/N, (R+1)/N) of each and
        // wo/w2 columns [R/N, (R+1)/N) (partial sums, summed across ranks).
        const int gb = c->mode == MODE_F32 ? kGBF : kGB;   // bytes per (tile, group)
        c->emb = make_desc(nullptr, c->vocab, (int)dim, gb);
        MatDesc dq = make_desc(nullptr, ql + 2 * kvl, (int)dim, gb), dwo = make_desc(nullptr, dim, (int)ql, gb);
        MatDesc d13 = make_desc(nullptr, 2 * hl, (int)dim, gb), d2 = make_desc(nullptr, dim, (int)hl, gb);

        size_t bytes = align256(desc_bytes(c->emb));
        bytes += L * (align256(desc_bytes(dq)) + align256(desc_bytes(dwo)) + align256(desc_bytes(d13)) +
                      align256(desc_bytes(d2)));
        bytes += align256(L * dim * 4) * 2 + align256(dim * 4) + 2 * align256(c->seq * (c->hs / 2) * 4);
        bytes += 2 * align256((size_t)c->nseq * L * c->max_pos * kvl * 4);
        bytes += 3 * align256(dim * 4) + align256(hl * 4) + align256(c->vocab_l * 4);
        bytes += align256((size_t)c->nh_l * c->max_chunks * (c->hs + 4) * 4) + align256(c->nh_l * 4);
        bytes += align256(sizeof(StepState)) + align256(8) + align256((size_t)c->max_pos * 4);
        bytes += align256((size_t)(4 * L + 1) * sizeof(OpDesc));
        c->max_tiles = std::max({c->emb.ntiles, dq.ntiles, dwo.ntiles, d13.ntiles, d2.ntiles});
        bytes += align256((size_t)c->max_tiles * kTR * 8);
        c->arena_bytes = bytes + 4096;
        CK_RET(&c->err, cudaMalloc(&c->arena, c->arena_bytes));
        CK_RET(&c->err, cudaMemsetAsync(c->arena, 0, c->arena_bytes, c->stream));

        c->emb.w = arena_take(c, desc_bytes(c->emb));
        // Classifier rows of this rank: tiles [vocab_off / 16, ...) of the embedding.
        c->cls = make_desc(c->emb.w + (size_t)(c->vocab_off / kTR) * c->emb.tile_bytes, c->vocab_l, (int)dim, gb);
        // The decode kernel's grid is one CTA per SM (setup_decode_kernel).
        for (MatDesc* d : {&dq, &dwo, &d13, &d2, &c->cls}) tune_chunks(*d, c->mode, dev_info(c->dev).sms);
        c->qkv.assign(L, dq); c->wo.assign(L, dwo); c->w13.assign(L, d13); c->w2.assign(L, d2);
        for (long long l = 0; l < L; l++) {
            c->qkv[l].w = arena_take(c, desc_bytes(dq));
            c->wo[l].w = arena_take(c, desc_bytes(dwo));
            c->w13[l].w = arena_take(c, desc_bytes(d13));
            c->w2[l].w = arena_take(c, desc_bytes(d2));
        }
        c->rms_att = (float*)arena_take(c, L * dim * 4);
        c->rms_ffn = (float*)arena_take(c, L * dim * 4);
        c->rms_final = (float*)arena_take(c, dim * 4);
        c->freq_re = (float*)arena_take(c, c->seq * (c->hs / 2) * 4);
        c->freq_im = (float*)arena_take(c, c->seq * (c->hs / 2) * 4);
        c->kv_seq = (size_t)L * c->max_pos * kvl;
        c->kcache = (float*)arena_take(c, (size_t)c->nseq * c->kv_seq * 4);
        c->vcache = (float*)arena_take(c, (size_t)c->nseq * c->kv_seq * 4);
        c->x = (float*)arena_take(c, dim * 4);
        c->q = (float*)arena_take(c, dim * 4);
        c->att = (float*)arena_take(c, dim * 4);
        c->hb = (float*)arena_take(c, hl * 4);
        c->logits = (float*)arena_take(c, c->vocab_l * 4);
        c->attn_part = (float*)arena_take(c, (size_t)c->nh_l * c->max_chunks * (c->hs + 4) * 4);
        c->attn_cnt = (int*)arena_take(c, c->nh_l * 4);
        c->step = (StepState*)arena_take(c, sizeof(StepState));
        c->argmax = (unsigned long long*)arena_take(c, 8);
        c->history = (int32_t*)arena_take(c, (size_t)c->max_pos * 4);
        c->ops = (OpDesc*)arena_take(c, (size_t)(4 * L + 1) * sizeof(OpDesc));
        c->split_part = (uint64_t*)arena_take(c, (size_t)c->max_tiles * kTR * 8);
        if (!c->split_part) {
            set_err(&c->err, "internal: arena too small");
            s = AION_ERR_OOM;
            break;
        }

        auto qb = [](long long cnt) { return cnt / 32 * 4 + cnt / 2; };
        long long stage = std::max({qb(c->vocab * dim), qb(L * dim * hid), qb(L * dim * dim)}) + 256;
        if (c->mode == MODE_F32) stage = std::max(c->vocab, hid) * dim * 4 + 256;   // one fp32 matrix at a time
        CK_RET(&c->err, cudaMalloc(&staging, (size_t)stage));
        CK_RET(&c->err, cudaHostAlloc(&pinned[0], chunk, cudaHostAllocDefault));
        CK_RET(&c->err, cudaHostAlloc(&pinned[1], chunk, cudaHostAllocDefault));
        CK_RET(&c->err, cudaEventCreateWithFlags(&ev[0], cudaEventDisableTiming));
        CK_RET(&c->err, cudaEventCreateWithFlags(&ev[1], cudaEventDisableTiming));
        CK_RET(&c->err, cudaEventRecord(ev[0], c->stream));
        CK_RET(&c->err, cudaEventRecord(ev[1], c->stream));

        long long off = 28;
        // Walks the file in the order of quantize.c:192-229 /
        // src/kernel_simd.c:970-986; `fn` re-tiles each quantized tensor.
        auto qtensor = [&](long long count, auto fn) -> aion_status {
            // Scales, then the packed bytes on a 256-byte boundary (the file
            // places them right after the scales, at any 4-byte offset).
            const long long sb = count / 32 * 4, po = (long long)align256((size_t)sb);
            aion_status r = upload_range(c, fd, off, sb, staging, pinned, ev, chunk);
            if (r == AION_OK) r = upload_range(c, fd, off + sb, count / 2, staging + po, pinned, ev, chunk);
            if (r != AION_OK) return r;
            const long long b = qb(count);
            cudaError_t e = fn((const float*)staging, staging + po);
            if (e != cudaSuccess) {
                set_err(&c->err, "re-tile failed: %s", cudaGetErrorString(e));
                return AION_ERR_CUDA;
            }
            off += b;
            return AION_OK;
        };
        auto ftensor = [&](long long count, float* dst) -> aion_status {
            aion_status r = upload_range(c, fd, off, count * 4, (uint8_t*)dst, pinned, ev, chunk);
            off += count * 4;
            return r;
        };
        // Layer l's matrix in the file is [rows][n]; the tiles take rows
        // [r0, r0 + take) and column groups [g0, g0 + tiles' width).
        auto per_layer = [&](long long rows, long long n, long long r0, long long take, long long g0,
                             std::vector<MatDesc>* dst, int row_offset, int interleave, int slot) {
            return [c, L, rows, n, r0, take, g0, dst, row_offset, interleave, slot](const float* sc,
                                                                                  const uint8_t* pk) -> cudaError_t {
                for (long long l = 0; l < L; l++) {
                    const long long e0 = l * rows * n + r0 * n;
                    cudaError_t e = retile((*dst)[l], sc + e0 / 32, pk + e0 / 2, take, row_offset, interleave, slot, 0,
                                           c->stream, (int)(n / 32), (int)g0);
                    if (e != cudaSuccess) return e;
                }
                return cudaSuccess;
            };
        };
        if (c->mode == MODE_F32) {
            // The fp32 file (src/kernel_simd.c:924-936): each matrix of each
            // layer goes through the staging buffer into fp32 tiles; the
            // classifier stays tied to the embedding, as in the reference.
            auto fmat = [&](long long rows, long long n, long long r0, long long take, long long g0, const MatDesc& dst,
                            int row_offset, int interleave, int slot) -> aion_status {
                aion_status r = upload_range(c, fd, off, rows * n * 4, staging, pinned, ev, chunk);
                if (r != AION_OK) return r;
                cudaError_t e = retile_f32(dst, (const float*)staging + r0 * n, take, row_offset, interleave, slot,
                                           (int)n, (int)g0, c->stream);
                if (e != cudaSuccess) {
                    set_err(&c->err, "re-tile failed: %s", cudaGetErrorString(e));
                    return AION_ERR_CUDA;
                }
                off += rows * n * 4;
                return AION_OK;
            };
            auto flayers = [&](long long rows, long long n, long long r0, long long take, long long g0,
                               std::vector<MatDesc>& dst, int row_offset, int interleave, int slot) -> aion_status {
                for (long long l = 0; l < L; l++) {
                    aion_status r = fmat(rows, n, r0, take, g0, dst[l], row_offset, interleave, slot);
                    if (r != AION_OK) return r;
                }
                return AION_OK;
            };
            if ((s = fmat(c->vocab, dim, 0, c->vocab, 0, c->emb, 0, 0, 0)) != AION_OK) break;
            if ((s = ftensor(L * dim, c->rms_att)) != AION_OK) break;
            if ((s = flayers(dim, dim, 0, ql, 0, c->qkv, 0, 0, 0)) != AION_OK) break;
            if ((s = flayers(kv, dim, 0, kvl, 0, c->qkv, (int)ql, 0, 0)) != AION_OK) break;
            if ((s = flayers(kv, dim, 0, kvl, 0, c->qkv, (int)(ql + kvl), 0, 0)) != AION_OK) break;
            if ((s = flayers(dim, dim, 0, dim, 0, c->wo, 0, 0, 0)) != AION_OK) break;
            if ((s = ftensor(L * dim, c->rms_ffn)) != AION_OK) break;
            if ((s = flayers(hid, dim, 0, hl, 0, c->w13, 0, 1, 0)) != AION_OK) break;
            if ((s = flayers(dim, hid, 0, dim, 0, c->w2, 0, 0, 0)) != AION_OK) break;
            if ((s = flayers(hid, dim, 0, hl, 0, c->w13, 0, 1, 1)) != AION_OK) break;
            if ((s = ftensor(dim, c->rms_final)) != AION_OK) break;
            if ((s = ftensor(c->seq * (c->hs / 2), c->freq_re)) != AION_OK) break;
            if ((s = ftensor(c->seq * (c->hs / 2), c->freq_im)) != AION_OK) break;
        } else {
        if ((s = qtensor(c->vocab * dim, [&](const float* sc, const uint8_t* pk) {
                 cudaError_t e = retile(c->emb, sc, pk, c->vocab, 0, 0, 0, 0, c->stream);
                 return e != cudaSuccess ? e : fill_pad(c->emb, c->stream);
             })) != AION_OK) break;
        if ((s = ftensor(L * dim, c->rms_att)) != AION_OK) break;
        if ((s = qtensor(L * dim * dim, per_layer(dim, dim, R * ql, ql, 0, &c->qkv, 0, 0, 0))) != AION_OK) break;
        if ((s = qtensor(L * dim * kv, per_layer(kv, dim, R * kvl, kvl, 0, &c->qkv, (int)ql, 0, 0))) != AION_OK)
            break;
        if ((s = qtensor(L * dim * kv, per_layer(kv, dim, R * kvl, kvl, 0, &c->qkv, (int)(ql + kvl), 0, 0))) !=
            AION_OK)
            break;
        if ((s = qtensor(L * dim * dim, per_layer(dim, dim, 0, dim, R * ql / 32, &c->wo, 0, 0, 0))) != AION_OK) break;
        if ((s = ftensor(L * dim, c->rms_ffn)) != AION_OK) break;
        if ((s = qtensor(L * dim * hid, per_layer(hid, dim, R * hl, hl, 0, &c->w13, 0, 1, 0))) != AION_OK) break;
        if ((s = qtensor(L * hid * dim, per_layer(dim, hid, 0, dim, R * hl / 32, &c->w2, 0, 0, 0))) != AION_OK) break;
        if ((s = qtensor(L * dim * hid, per_layer(hid, dim, R * hl, hl, 0, &c->w13, 0, 1, 1))) != AION_OK) break;
        if ((s = ftensor(dim, c->rms_final)) != AION_OK) break;
        if ((s = ftensor(c->seq * (c->hs / 2), c->freq_re)) != AION_OK) break;
        if ((s = ftensor(c->seq * (c->hs / 2), c->freq_im)) != AION_OK) break;
        for (long long l = 0; l < L; l++) {
            cudaError_t e = fill_pad(c->qkv[l], c->stream);
            if (e == cudaSuccess) e = fill_pad(c->wo[l], c->stream);
            if (e == cudaSuccess) e = fill_pad(c->w2[l], c->stream);
            CK_RET(&c->err, e);
        }
        }   // int4 file

        // Op table of one token.
        std::vector<OpDesc> ops;
        int max_chunk = 0;
        for (long long l = 0; l < L; l++) {
            ops.push_back({c->qkv[l], OP_QKV, (int)l});
            ops.push_back({c->wo[l], OP_WO, (int)l});
            ops.push_back({c->w13[l], OP_W13, (int)l});
            ops.push_back({c->w2[l], OP_W2, (int)l});
        }
        ops.push_back({c->cls, OP_CLS, 0});
        for (const OpDesc& o : ops) max_chunk = std::max(max_chunk, max_chunk_bytes(o.m));
        c->nops = (int)ops.size();
        CK_RET(&c->err, cudaMemcpyAsync(c->ops, ops.data(), ops.size() * sizeof(OpDesc), cudaMemcpyHostToDevice,
                                        c->stream));
        const int max_n = (int)std::max(dim, hid);
        s = c->mode == MODE_W4A8  ? setup_decode_kernel<MODE_W4A8>(c, max_n, max_chunk)
            : c->mode == MODE_F32 ? setup_decode_kernel<MODE_F32>(c, max_n, max_chunk)
                                  : setup_decode_kernel<MODE_W4A16>(c, max_n, max_chunk);
        if (s != AION_OK) break;
        if (c->mode == MODE_W4A8) {   // the bit-exact mode follows the host expf
            const HostExpTable& t = host_exp_table();
            if (t.usable && !t.x.empty()) {
                CK_RET(&c->err, cudaMalloc(&c->exp_tab, t.x.size() * 4));
                CK_RET(&c->err, cudaMemcpyAsync(c->exp_tab, t.x.data(), t.x.size() * 4, cudaMemcpyHostToDevice,
                                                c->stream));
                c->exp_n = (int)t.x.size();
                c->exp_delta = t.delta;
            }
        }

        // Step state: pos 0, no forced token, argmax key at its initial value.
        StepState init = {};
        init.forced_token = -1;
        const unsigned long long key0 = argmax_key(-1e9f, 0);
        CK_RET(&c->err, cudaMemcpyAsync(c->step, &init, sizeof(init), cudaMemcpyHostToDevice, c->stream));
        CK_RET(&c->err, cudaMemcpyAsync(c->argmax, &key0, 8, cudaMemcpyHostToDevice, c->stream));
        CK_RET(&c->err, cudaStreamSynchronize(c->stream));
    } while (0);
    close(fd);
    if (staging) cudaFree(staging);
    if (pinned[0]) cudaFreeHost(pinned[0]);
    if (pinned[1]) cudaFreeHost(pinned[1]);
    if (ev[0]) cudaEventDestroy(ev[0]);
    if (ev[1]) cudaEventDestroy(ev[1]);
    return s;
}

extern "C" AION_API aion_status aion_load(const char* path, const aion_opts* opts, aion_ctx** out) {
    if (!path || !out) {
        set_err(nullptr, "aion_load: null argument");
        return AION_ERR_ARG;
    }
    *out = nullptr;
    aion_ctx* c = new aion_ctx();
    if (opts) c->opts = *opts; else aion_default_opts(&c->opts);
    if (c->opts.mode != AION_MODE_W4A16 && c->opts.mode != AION_MODE_W4A8) {
        set_err(&c->err, "unknown mode %d", c->opts.mode);
        delete c;
        return AION_ERR_ARG;
    }
    if (c->opts.tp_size < 1 || c->opts.tp_size > kMaxTpRanks || c->opts.tp_rank < 0 ||
        c->opts.tp_rank >= c->opts.tp_size) {
        set_err(&c->err, "tp_size %d / tp_rank %d out of range (1 <= tp_size <= %d: the GPUs of one NVLink node)",
                c->opts.tp_size, c->opts.tp_rank, kMaxTpRanks);
        delete c;
        return AION_ERR_ARG;
    }
    c->tp_n = c->opts.tp_size;
    c->tp_rank = c->opts.tp_rank;
    if (c->opts.max_batch < 1 || c->opts.max_batch > 1024) {
        set_err(&c->err, "max_batch %d out of range [1, 1024]", c->opts.max_batch);
        delete c;
        return AION_ERR_ARG;
    }
    c->nseq = c->opts.max_batch;
    c->mode = c->opts.mode == AION_MODE_W4A8 ? MODE_W4A8 : MODE_W4A16;
    c->dev = c->opts.device;
    bool f32 = false;
    aion_status hs = read_header(path, &c->cfg, &c->err, &f32);
    if (hs != AION_OK) {
        delete c;
        return hs;
    }
    if (f32) {
        if (c->mode == MODE_W4A8 || c->tp_n > 1) {
            set_err(&c->err, "%s is an fp32 file: it runs the fp32 path on one GPU (no W4A8, no tensor parallelism)",
                    path);
            delete c;
            return AION_ERR_ARG;
        }
        c->mode = MODE_F32;
    }
    cudaError_t e = cudaSetDevice(c->dev);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaHostAlloc(&c->h_step, sizeof(StepState), cudaHostAllocDefault);
    if (e != cudaSuccess) {
        set_err(&c->err, "CUDA init failed: %s", cudaGetErrorString(e));
        ctx_destroy(c);
        return AION_ERR_CUDA;
    }
    aion_status s = load_impl(c, path);
    if (s == AION_OK && c->tp_n > 1) {
        // Exchange region: tagged receive rows [2][tp_n][dim] u64, keys [tp_n] u64,
        // flags [tp_n] u32; then the batched decode's receive rows
        // [2][tp_n][nbmax][dim] u64 (nbmax = min(max_batch, 32)) and keys
        // [tp_n][32] u64.
        // Shared with the other ranks by aion_tp_connect.
        const size_t recv = align256((size_t)2 * c->tp_n * c->dim * 8), keys = align256((size_t)c->tp_n * 8);
        const size_t flags = align256((size_t)c->tp_n * 4);
        c->xr_nbmax = std::min(c->nseq, kBMaxSeq);
        const size_t brecv = align256((size_t)2 * c->tp_n * c->xr_nbmax * c->dim * 8);
        const size_t bkeys = align256((size_t)c->tp_n * kBMaxSeq * 8);
        c->xr_keys_off = (int)recv;
        c->xr_flags_off = (int)(recv + keys);
        c->xr_brecv_off = (long long)(recv + keys + flags);
        c->xr_bkeys_off = c->xr_brecv_off + (long long)brecv;
        c->xr_bytes = recv + keys + flags + brecv + bkeys;
        cudaError_t e2 = cudaMalloc(&c->xr, c->xr_bytes);
        if (e2 == cudaSuccess) e2 = cudaMemset(c->xr, 0, c->xr_bytes);
        if (e2 == cudaSuccess) e2 = cudaMalloc(&c->peers_dev, (size_t)c->tp_n * sizeof(unsigned char*));
        if (e2 != cudaSuccess) {
            set_err(&c->err, "exchange region: %s", cudaGetErrorString(e2));
            s = cuda_status(e2);
        }
        c->peers.assign(c->tp_n, nullptr);
        c->peers[c->tp_rank] = c->xr;
    }
    if (s != AION_OK) {
        g_thread_err = c->err;
        ctx_destroy(c);
        return s;
    }
    *out = c;
    return AION_OK;
}

// ---------------------------------------------------------------------------
// Tensor parallelism: the shard plan, and sharing the exchange regions
// between the ranks' processes (no counterpart in the reference).
// ---------------------------------------------------------------------------
extern "C" AION_API aion_status aion_tp_plan(const aion_config* cfg, int32_t tp_size, int32_t tp_rank, int64_t* out) {
    if (!cfg || !out || tp_size < 1 || tp_rank < 0 || tp_rank >= tp_size || cfg->n_heads <= 0 || cfg->n_kv_heads <= 0)
        return AION_ERR_ARG;
    const long long N = tp_size, R = tp_rank, dim = cfg->dim, hid = cfg->hidden_dim, nh = cfg->n_heads,
                    nkv = cfg->n_kv_heads, vocab = cfg->vocab_size < 0 ? -(long long)cfg->vocab_size : cfg->vocab_size;
    const long long kv = dim * nkv / nh;
    if (N > 1 && (nh % N || nkv % N || (dim / N) % 32 || dim % N || (hid / N) % 32 || hid % N || vocab % (N * kTR)))
        return AION_ERR_SHAPE;
    const long long ql = dim / N, kvl = kv / N, hl = hid / N, vl = vocab / N;
    const int64_t v[AION_TP_PLAN_FIELDS] = {R * ql, ql, R * kvl, kvl, R * hl, hl, R * vl, vl, nh / N};
    memcpy(out, v, sizeof(v));
    return AION_OK;
}
extern "C" AION_API aion_status aion_tp_handle(const aion_ctx* c, void* handle_out) {
    if (!c || !handle_out || c->tp_n < 2) return AION_ERR_ARG;
    cudaIpcMemHandle_t h;
    CK_RET(nullptr, cudaSetDevice(c->dev));
    CK_RET(nullptr, cudaIpcGetMemHandle(&h, c->xr));
    static_assert(sizeof(h) == AION_TP_HANDLE_BYTES, "IPC handle size");
    memcpy(handle_out, &h, sizeof(h));
    return AION_OK;
}

extern "C" AION_API aion_status aion_tp_connect(aion_ctx* c, const void* handles) {
    if (!c || !handles || c->tp_n < 2) return AION_ERR_ARG;
    if (c->tp_connected) return AION_OK;
    CK_RET(&c->err, cudaSetDevice(c->dev));
    for (int j = 0; j < c->tp_n; j++) {
        if (j == c->tp_rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const unsigned char*>(handles) + (size_t)j * AION_TP_HANDLE_BYTES, sizeof(h));
        void* p = nullptr;
        CK_RET(&c->err, cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
        c->peers[j] = static_cast<unsigned char*>(p);
    }
    CK_RET(&c->err, cudaMemcpy(c->peers_dev, c->peers.data(), (size_t)c->tp_n * sizeof(unsigned char*),
                               cudaMemcpyHostToDevice));
    c->tp_connected = true;
    return AION_OK;
}

static aion_status tp_ready(aion_ctx* c) {
    if (c->tp_n > 1 && !c->tp_connected) {
        set_err(&c->err, "tensor-parallel context not connected (aion_tp_connect)");
        return AION_ERR_STATE;
    }
    return AION_OK;
}

// Writes the next step's token and position (and clears the error word).
// The barrier and exchange counters stay (they only ever grow).  The
// pinned host buffer is reused, so with sync == false the caller must
// synchronise the stream before the host touches c->h_step again.
static aion_status set_step(aion_ctx* c, int32_t token, int32_t pos, bool sync = true) {
    memset(c->h_step, 0, sizeof(StepState));
    c->h_step->pos_next = pos;
    c->h_step->forced_token = token;
    CK_RET(&c->err, cudaMemcpyAsync(c->step, c->h_step, offsetof(StepState, barrier), cudaMemcpyHostToDevice,
                                    c->stream));
    if (sync) CK_RET(&c->err, cudaStreamSynchronize(c->stream));
    return AION_OK;
}

extern "C" AION_API aion_status aion_forward(aion_ctx* c, int32_t token, int32_t pos, float* logits_host) {
    if (!c) return AION_ERR_ARG;
    if (token < 0 || token >= c->vocab || pos < 0 || pos >= c->max_pos) {
        set_err(&c->err, "aion_forward: token %d or pos %d out of range (vocab %lld, max_pos %d)", token, pos, c->vocab,
                c->max_pos);
        return AION_ERR_ARG;
    }
    CK_RET(&c->err, cudaSetDevice(c->dev));
    // One host round trip a token: the step state goes in, the logits and
    // the step state (its error word) come back, all ordered on the stream.
    aion_status s = set_step(c, token, pos, false);
    if (s == AION_OK) s = enqueue_steps(c, 1);
    if (s != AION_OK) {
        cudaStreamSynchronize(c->stream);   // the pinned step buffer may still be in flight
        return s;
    }
    if (logits_host)
        CK_RET(&c->err, cudaMemcpyAsync(logits_host, c->logits, c->vocab_l * 4, cudaMemcpyDeviceToHost, c->stream));
    CK_RET(&c->err, cudaMemcpyAsync(c->h_step, c->step, sizeof(StepState), cudaMemcpyDeviceToHost, c->stream));
    CK_RET(&c->err, cudaStreamSynchronize(c->stream));
    return decode_device_error(c);
}

extern "C" AION_API aion_status aion_generate(aion_ctx* c, int32_t bos, int32_t steps, int32_t* tokens_out,
                                              double* seconds) {
    if (!c) return AION_ERR_ARG;
    if (bos < 0 || bos >= c->vocab || steps < 0 || steps > c->max_pos) {
        set_err(&c->err, "aion_generate: bos %d or steps %d out of range (vocab %lld, max_pos %d)", bos, steps, c->vocab,
                c->max_pos);
        return AION_ERR_ARG;
    }
    CK_RET(&c->err, cudaSetDevice(c->dev));
    aion_status s = set_step(c, bos, 0);
    if (s != AION_OK) return s;
    struct timespec t0, t1;
    clock_gettime(CLOCK_MONOTONIC, &t0);
    s = enqueue_steps(c, steps);
    if (s != AION_OK) return s;
    CK_RET(&c->err, cudaStreamSynchronize(c->stream));
    clock_gettime(CLOCK_MONOTONIC, &t1);
    if (seconds) *seconds = (double)(t1.tv_sec - t0.tv_sec) + 1e-9 * (double)(t1.tv_nsec - t0.tv_nsec);
    if (tokens_out && steps > 0)
        CK_RET(&c->err, cudaMemcpy(tokens_out, c->history, (size_t)steps * 4, cudaMemcpyDeviceToHost));
    return check_device_error(c);
}

extern "C" AION_API aion_status aion_decode_async(aion_ctx* c, int32_t token, int32_t pos, int32_t steps) {
    if (!c || steps < 0) return AION_ERR_ARG;
    if (token >= c->vocab || pos >= c->max_pos) {
        set_err(&c->err, "aion_decode_async: token %d or pos %d out of range", token, pos);
        return AION_ERR_ARG;
    }
    CK_RET(&c->err, cudaSetDevice(c->dev));
    if (token >= 0 || pos >= 0) {
        k_set_step<<<1, 32, 0, c->stream>>>(c->step, pos, token);
        CK_RET(&c->err, cudaGetLastError());
    }
    return enqueue_steps(c, steps);
}

extern "C" AION_API aion_status aion_tokens(aion_ctx* c, int32_t* out, int32_t n) {
    if (!c || !out || n < 0 || n > c->max_pos) return AION_ERR_ARG;
    CK_RET(&c->err, cudaSetDevice(c->dev));
    CK_RET(&c->err, cudaStreamSynchronize(c->stream));
    if (n) CK_RET(&c->err, cudaMemcpy(out, c->history, (size_t)n * 4, cudaMemcpyDeviceToHost));
    return check_device_error(c);
}

extern "C" AION_API aion_status aion_reset(aion_ctx* c) {
    if (!c) return AION_ERR_ARG;
    CK_RET(&c->err, cudaSetDevice(c->dev));
    const size_t kvb = c->kv_seq * 4;
    CK_RET(&c->err, cudaMemsetAsync(c->kcache + (size_t)c->cur_seq * c->kv_seq, 0, kvb, c->stream));
    CK_RET(&c->err, cudaMemsetAsync(c->vcache + (size_t)c->cur_seq * c->kv_seq, 0, kvb, c->stream));
    CK_RET(&c->err, cudaMemsetAsync(&c->step->error, 0, sizeof(int32_t), c->stream));
    CK_RET(&c->err, cudaMemsetAsync(c->attn_cnt, 0, c->nh * 4, c->stream));
    CK_RET(&c->err, cudaMemsetAsync(c->split_part, 0, (size_t)c->max_tiles * kTR * 8, c->stream));
    CK_RET(&c->err, cudaStreamSynchronize(c->stream));
    return AION_OK;
}

// ---------------------------------------------------------------------------
// Sequences and batched prefill (no counterpart in the reference, whose
// transformer() takes one token of one sequence)
// ---------------------------------------------------------------------------
extern "C" AION_API aion_status aion_set_sequence(aion_ctx* c, int32_t seq) {
    if (!c) return AION_ERR_ARG;
    if (seq < 0 || seq >= c->nseq) {
        set_err(&c->err, "aion_set_sequence: sequence %d out of range [0, %d)", seq, c->nseq);
        return AION_ERR_ARG;
    }
    if (seq == c->cur_seq) return AION_OK;
    CK_RET(&c->err, cudaSetDevice(c->dev));
    CK_RET(&c->err, cudaStreamSynchronize(c->stream));
    c->cur_seq = seq;
    // The per-token graph holds the previous sequence's cache pointers.
    if (c->gexec) {
        cudaGraphExecDestroy(c->gexec);
        c->gexec = nullptr;
    }
    if (c->graph) {
        cudaGraphDestroy(c->graph);
        c->graph = nullptr;
    }
    return AION_OK;
}

static aion_status launch_gemm_bf16(const void* a, const void* b, float* c, int64_t m, int64_t n, int64_t k,
                                    int64_t ldc, int dev, cudaStream_t st, int* err_dev, std::string* err);

// Grows a prefill buffer to at least `bytes`.
static cudaError_t pf_grow(void** p, size_t* cap, size_t bytes) {
    if (*cap >= bytes) return cudaSuccess;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    cudaError_t e = cudaMalloc(p, bytes);
    if (e == cudaSuccess) *cap = bytes;
    return e;
}

static inline long long round_up(long long v, long long m) { return (v + m - 1) / m * m; }

// One int4 matrix product of the prefill: C[mpad][np] = A(3*kp) * B(matrix)^T.
static aion_status pf_matmul(aion_ctx* c, const MatDesc& w, long long mpad, long long kp, long long* np_out) {
    const long long np = round_up(w.d, kGemmBN);
    const long long tasks = np * (kp / 8);
    const int blocks = (int)std::min<long long>((tasks + 255) / 256, 148LL * 32);
    k_pf_dequant<<<blocks, 256, 0, c->stream>>>(w, (int)np, (int)kp, c->pf.b);
    CK_RET(&c->err, cudaGetLastError());
    const aion_status s = launch_gemm_bf16(c->pf.a, c->pf.b, c->pf.c, mpad, np, 3 * kp, np, c->dev, c->stream,
                                           &c->step->error, &c->err);
    *np_out = np;
    return s;
}

extern "C" AION_API aion_status aion_prefill(aion_ctx* c, const int32_t* tokens, int32_t n_seq, int32_t n_tok,
                                             float* logits_host) {
    if (!c || !tokens || n_seq < 1 || n_tok < 1) return AION_ERR_ARG;
    if (c->tp_n > 1 || c->mode == MODE_F32) {
        set_err(&c->err, "aion_prefill needs an int4 file on one GPU");
        return AION_ERR_STATE;
    }
    if (n_seq > c->nseq || n_tok > c->max_pos) {
        set_err(&c->err, "aion_prefill: %d sequences x %d tokens exceed the context (%d sequences, %d positions)",
                n_seq, n_tok, c->nseq, c->max_pos);
        return AION_ERR_ARG;
    }
    for (long long i = 0; i < (long long)n_seq * n_tok; i++)
        if (tokens[i] < 0 || tokens[i] >= c->vocab) {
            set_err(&c->err, "aion_prefill: token %d at %lld out of range", tokens[i], i);
            return AION_ERR_ARG;
        }
    CK_RET(&c->err, cudaSetDevice(c->dev));
    const long long dim = c->dim, hid = c->hidden, kv = c->kv_dim, L = c->L;
    const long long mrows = (long long)n_seq * n_tok, mpad = round_up(mrows, kGemmBM);
    const long long kpd = round_up(dim, kGemmBK), kph = round_up(hid, kGemmBK);
    const long long np_max = std::max({round_up(dim + 2 * kv, kGemmBN), round_up(2 * hid, kGemmBN),
                                       round_up(dim, kGemmBN)});
    const long long np_cls = round_up(c->vocab, kGemmBN), mcls = round_up(n_seq, kGemmBM);
    const long long kmax = std::max(kpd, kph);
    const size_t a_bytes = (size_t)std::max(mpad, mcls) * 3 * kmax * 2;
    const size_t b_bytes = (size_t)std::max({np_max * 3 * kpd, round_up(dim, kGemmBN) * 3 * kph, np_cls * 3 * kpd}) * 2;
    const size_t c_bytes = (size_t)std::max(mpad * np_max, mcls * np_cls) * 4;
    auto& pf = c->pf;
    CK_RET(&c->err, pf_grow((void**)&pf.a, &pf.a_cap, a_bytes));
    CK_RET(&c->err, pf_grow((void**)&pf.b, &pf.b_cap, b_bytes));
    CK_RET(&c->err, pf_grow((void**)&pf.c, &pf.c_cap, c_bytes));
    CK_RET(&c->err, pf_grow((void**)&pf.x, &pf.x_cap, (size_t)mrows * dim * 4));
    CK_RET(&c->err, pf_grow((void**)&pf.q, &pf.q_cap, (size_t)mrows * dim * 4));
    CK_RET(&c->err, pf_grow((void**)&pf.tok, &pf.tok_cap, (size_t)mrows * 4));
    CK_RET(&c->err, pf_grow((void**)&pf.map, &pf.map_cap, (size_t)mcls * 4));
    CK_RET(&c->err, cudaMemcpyAsync(pf.tok, tokens, (size_t)mrows * 4, cudaMemcpyHostToDevice, c->stream));
    std::vector<int> map(n_seq);
    for (int s = 0; s < n_seq; s++) map[s] = s * n_tok + n_tok - 1;
    CK_RET(&c->err, cudaMemcpyAsync(pf.map, map.data(), n_seq * 4, cudaMemcpyHostToDevice, c->stream));
    CK_RET(&c->err, cudaFuncSetAttribute(k_pf_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, kPfAttnSmem));

    k_pf_embed<<<(unsigned)mrows, 256, 0, c->stream>>>(pf.tok, (int)mrows, c->emb, (int)dim, pf.x);
    CK_RET(&c->err, cudaGetLastError());
    for (long long l = 0; l < L; l++) {
        long long np = 0;
        // attention block
        k_pf_norm_split<<<(unsigned)mpad, 256, 0, c->stream>>>(pf.x, nullptr, (int)mrows, (int)dim, (int)kpd,
                                                                c->rms_att + l * dim, pf.a);
        aion_status st = pf_matmul(c, c->qkv[l], mpad, kpd, &np);
        if (st != AION_OK) return st;
        PfRopeArgs ra;
        ra.c = pf.c;
        ra.ldc = (int)np;
        ra.mrows = (int)mrows;
        ra.T = n_tok;
        ra.dim = (int)dim;
        ra.kv_dim = (int)kv;
        ra.hs = (int)c->hs;
        ra.freq_re = c->freq_re;
        ra.freq_im = c->freq_im;
        ra.q = pf.q;
        ra.kcache = c->kcache + (size_t)l * c->max_pos * kv;
        ra.vcache = c->vcache + (size_t)l * c->max_pos * kv;
        ra.seq_stride = c->kv_seq;
        k_pf_rope_kv<<<(unsigned)mrows, 256, 0, c->stream>>>(ra);
        PfAttnArgs aa;
        aa.q = pf.q;
        aa.kcache = ra.kcache;
        aa.vcache = ra.vcache;
        aa.seq_stride = c->kv_seq;
        aa.T = n_tok;
        aa.dim = (int)dim;
        aa.kv_dim = (int)kv;
        aa.hs = (int)c->hs;
        aa.kv_mul = (int)c->kv_mul;
        aa.kp = (int)kpd;
        aa.out = pf.a;
        k_pf_attention<<<dim3((unsigned)((n_tok + kPfTQ - 1) / kPfTQ), (unsigned)c->nh, (unsigned)n_seq), kPfAttnThreads,
                         kPfAttnSmem, c->stream>>>(aa);
        CK_RET(&c->err, cudaGetLastError());
        st = pf_matmul(c, c->wo[l], mpad, kpd, &np);
        if (st != AION_OK) return st;
        k_pf_residual<<<(unsigned)mrows, 256, 0, c->stream>>>(pf.x, pf.c, (int)np, (int)mrows, (int)dim);
        // feed-forward block
        k_pf_norm_split<<<(unsigned)mpad, 256, 0, c->stream>>>(pf.x, nullptr, (int)mrows, (int)dim, (int)kpd,
                                                                c->rms_ffn + l * dim, pf.a);
        st = pf_matmul(c, c->w13[l], mpad, kpd, &np);
        if (st != AION_OK) return st;
        k_pf_swiglu_split<<<(unsigned)mpad, 256, 0, c->stream>>>(pf.c, (int)np, (int)mrows, (int)hid, (int)kph,
                                                                  pf.a);
        st = pf_matmul(c, c->w2[l], mpad, kph, &np);
        if (st != AION_OK) return st;
        k_pf_residual<<<(unsigned)mrows, 256, 0, c->stream>>>(pf.x, pf.c, (int)np, (int)mrows, (int)dim);
        CK_RET(&c->err, cudaGetLastError());
    }
    // Logits of each sequence's last position.
    k_pf_norm_split<<<(unsigned)mcls, 256, 0, c->stream>>>(pf.x, pf.map, n_seq, (int)dim, (int)kpd, c->rms_final,
                                                            pf.a);
    long long np = 0;
    aion_status st = pf_matmul(c, c->emb, mcls, kpd, &np);
    if (st != AION_OK) return st;
    if (logits_host)
        CK_RET(&c->err, cudaMemcpy2DAsync(logits_host, (size_t)c->vocab * 4, pf.c, (size_t)np * 4,
                                          (size_t)c->vocab * 4, (size_t)n_seq, cudaMemcpyDeviceToHost, c->stream));
    CK_RET(&c->err, cudaStreamSynchronize(c->stream));
    return check_device_error(c);
}

// ---------------------------------------------------------------------------
// Kernel-level API
// ---------------------------------------------------------------------------
// Cut-tile flag tag of the next standalone call: 1 .. 0x7FFFFFFF, cycling.
static uint32_t next_epoch(std::atomic<uint32_t>& counter) { return counter.fetch_add(1) % 0x7FFFFFFFu + 1u; }

struct aion_qmatrix {
    std::atomic<uint32_t> epoch{0};
    int device;
    MatDesc m;
    Scratch sc;
    uint8_t* scratch_mem;
};

extern "C" AION_API aion_status aion_qmatrix_upload(const float* scales, const uint8_t* packed, int64_t rows,
                                                    int64_t cols, int32_t device, aion_qmatrix** out) {
    if (!scales || !packed || !out || rows <= 0 || cols <= 0 || cols % 32 || cols > (1 << 24) || rows > (1 << 28)) {
        set_err(nullptr, "aion_qmatrix_upload: invalid arguments (rows %lld, cols %lld; cols must be a multiple of 32)",
                (long long)rows, (long long)cols);
        return AION_ERR_ARG;
    }
    *out = nullptr;
    CK_RET(nullptr, cudaSetDevice(device));
    MatDesc m = make_desc(nullptr, rows, (int)cols);
    tune_chunks(m, MODE_W4A16, dev_info(device).sms);
    uint8_t* w = nullptr;
    cudaError_t e = cudaMalloc(&w, (size_t)desc_bytes(m));
    if (e != cudaSuccess) {
        set_err(nullptr, "cudaMalloc failed: %s", cudaGetErrorString(e));
        return cuda_status(e);
    }
    m.w = w;
    // Packed bytes start on a 256-byte boundary of the staging buffer: the
    // re-tile moves them as 16-byte vectors.
    const size_t sb = (size_t)(rows * cols / 32 * 4), pb = (size_t)(rows * cols / 2), po = align256(sb);
    uint8_t* stage = nullptr;
    e = cudaMalloc(&stage, po + pb);
    if (e == cudaSuccess) e = cudaMemcpy(stage, scales, sb, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(stage + po, packed, pb, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = retile(m, (const float*)stage, stage + po, rows, 0, 0, 0, 0, 0);
    if (e == cudaSuccess) e = fill_pad(m, 0);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (stage) cudaFree(stage);
    if (e != cudaSuccess) {
        cudaFree(w);
        set_err(nullptr, "aion_qmatrix_upload: %s", cudaGetErrorString(e));
        return cuda_status(e);
    }
    // Scratch of the split-tile combine: tagged partial rows (zero: tag 0
    // is never used) and the error word.
    const size_t pbytes = align256((size_t)m.ntiles * kTR * 8);
    uint8_t* scr = nullptr;
    e = cudaMalloc(&scr, pbytes + 256);
    if (e == cudaSuccess) e = cudaMemset(scr, 0, pbytes + 256);
    if (e != cudaSuccess) {
        cudaFree(w);
        if (scr) cudaFree(scr);
        set_err(nullptr, "aion_qmatrix_upload: %s", cudaGetErrorString(e));
        return cuda_status(e);
    }
    aion_qmatrix* q = new aion_qmatrix();
    q->device = device;
    q->m = m;
    q->scratch_mem = scr;
    q->sc.split_part = (uint64_t*)scr;
    q->sc.error = (int*)(scr + pbytes);
    *out = q;
    return AION_OK;
}

extern "C" AION_API aion_status aion_qmatrix_download(const aion_qmatrix* q, float* scales, uint8_t* packed) {
    if (!q || !scales || !packed) return AION_ERR_ARG;
    CK_RET(nullptr, cudaSetDevice(q->device));
    const long long rows = q->m.d, cols = q->m.n;
    const size_t sb = (size_t)(rows * cols / 32 * 4), pb = (size_t)(rows * cols / 2), po = align256(sb);
    uint8_t* stage = nullptr;
    cudaError_t e = cudaMalloc(&stage, po + pb);
    if (e == cudaSuccess) e = retile(q->m, (const float*)stage, stage + po, rows, 0, 0, 0, 1, 0);
    if (e == cudaSuccess) e = cudaMemcpy(scales, stage, sb, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(packed, stage + po, pb, cudaMemcpyDeviceToHost);
    if (stage) cudaFree(stage);
    if (e != cudaSuccess) {
        set_err(nullptr, "aion_qmatrix_download: %s", cudaGetErrorString(e));
        return cuda_status(e);
    }
    return AION_OK;
}

extern "C" AION_API aion_status aion_qmatrix_free(aion_qmatrix* q) {
    if (!q) return AION_OK;
    cudaSetDevice(q->device);
    cudaFree((void*)q->m.w);
    cudaFree(q->scratch_mem);
    delete q;
    return AION_OK;
}

static aion_status matvec_api(int mode, const aion_qmatrix* q, const float* x, float* y, void* stream) {
    if (!q || !x || !y) {
        set_err(nullptr, "matvec: null argument");
        return AION_ERR_ARG;
    }
    if (((uintptr_t)x & 15) || ((uintptr_t)y & 3)) {
        set_err(nullptr, "matvec: x must be 16-byte aligned, y 4-byte aligned");
        return AION_ERR_ARG;
    }
    CK_RET(nullptr, cudaSetDevice(q->device));
    aion_qmatrix* qm = const_cast<aion_qmatrix*>(q);
    const uint32_t ep = next_epoch(qm->epoch);
    cudaError_t e = mode == MODE_W4A8
                        ? launch_standalone<MODE_W4A8>(q->m, q->sc, x, y, q->device, (cudaStream_t)stream, ep)
                        : launch_standalone<MODE_W4A16>(q->m, q->sc, x, y, q->device, (cudaStream_t)stream, ep);
    CK_RET(nullptr, e);
    return AION_OK;
}

extern "C" AION_API aion_status aion_matvec_w4a16(const aion_qmatrix* w, const float* x_dev, float* y_dev, void* stream) {
    return matvec_api(MODE_W4A16, w, x_dev, y_dev, stream);
}

extern "C" AION_API aion_status aion_matvec_w4a8(const aion_qmatrix* w, const float* x_dev, float* y_dev, void* stream) {
    return matvec_api(MODE_W4A8, w, x_dev, y_dev, stream);
}

// ---------------------------------------------------------------------------
// W4A16 matvec on scratch that exists from module load (no counterpart in
// the reference).  aion_matvec_w4a16 uses the scratch aion_qmatrix_upload
// allocated next to the weights.  This variant runs the same kernel on a
// fixed file-scope device array instead, and calls no allocating function.
// It is for callers that cannot allocate device memory on the call path:
// a serving loop that has budgeted all device memory at start-up and treats
// any later allocation as an error, or code that must not trigger the
// implicit device-wide synchronisation that cudaMalloc / cudaFree can cause
// while other streams are busy.
//
// Limits: matrices of at most kStaticScratchTiles * 16 = 32768 rows (larger
// ones are rejected with AION_ERR_SHAPE).  The scratch is one array per
// device shared by every call, so calls that overlap in time (on different
// streams or threads) race on it and must be serialised by the caller.  The
// first call on a device looks the array's address up (cudaGetSymbolAddress);
// make that first call before any stream capture on that device.
// ---------------------------------------------------------------------------
constexpr int kStaticScratchTiles = 2048;
constexpr size_t kStaticPartBytes = (size_t)kStaticScratchTiles * kTR * 8;   // tagged second parts of cut tiles
constexpr size_t kStaticScratchBytes = kStaticPartBytes + 256;               // + error word: starts at zero
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

constexpr int kMaxStaticDevices = 64;
static std::mutex g_static_mu;
static unsigned char* g_static_addr[kMaxStaticDevices];
static std::atomic<uint32_t> g_static_epoch[kMaxStaticDevices];

// Address of this device's g_static_scratch; the device must be current.
static aion_status static_scratch_addr(int dev, unsigned char** out) {
    if (dev < 0 || dev >= kMaxStaticDevices) {
        set_err(nullptr, "aion_matvec_w4a16_static: device %d out of range", dev);
        return AION_ERR_ARG;
    }
    std::lock_guard<std::mutex> lock(g_static_mu);
    if (!g_static_addr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess) {
            set_err(nullptr, "aion_matvec_w4a16_static: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
            return cuda_status(e);
        }
        g_static_addr[dev] = static_cast<unsigned char*>(p);
    }
    *out = g_static_addr[dev];
    return AION_OK;
}

extern "C" AION_API aion_status aion_matvec_w4a16_static(const aion_qmatrix* w, const float* x_dev, float* y_dev,
                                                         void* stream) {
    if (!w || !x_dev || !y_dev) {
        set_err(nullptr, "aion_matvec_w4a16_static: null argument");
        return AION_ERR_ARG;
    }
    if (((uintptr_t)x_dev & 15) || ((uintptr_t)y_dev & 3)) {
        set_err(nullptr, "aion_matvec_w4a16_static: x must be 16-byte aligned, y 4-byte aligned");
        return AION_ERR_ARG;
    }
    if (w->m.ntiles > kStaticScratchTiles) {
        set_err(nullptr, "aion_matvec_w4a16_static: %d rows exceed the static scratch limit of %d rows", w->m.d,
                kStaticScratchTiles * kTR);
        return AION_ERR_SHAPE;
    }
    CK_RET(nullptr, cudaSetDevice(w->device));
    unsigned char* base = nullptr;
    const aion_status st = static_scratch_addr(w->device, &base);
    if (st != AION_OK) return st;
    Scratch sc;
    sc.split_part = reinterpret_cast<uint64_t*>(base);
    sc.error = reinterpret_cast<int*>(base + kStaticPartBytes);
    // Cut-tile parts carry this call's tag, so parts left by an earlier call
    // need no clearing (the array starts at zero, and tag 0 is never used).
    // The error word starts at zero and aion_matvec_status reads and clears
    // it.
    CK_RET(nullptr, launch_standalone<MODE_W4A16>(w->m, sc, x_dev, y_dev, w->device, (cudaStream_t)stream,
                                                  next_epoch(g_static_epoch[w->device])));
    return AION_OK;
}

// Reads and clears one device error word (the stream has been waited for).
static aion_status take_error_word(int* word, const char* what) {
    int v = 0;
    CK_RET(nullptr, cudaMemcpy(&v, word, sizeof(int), cudaMemcpyDeviceToHost));
    if (v == 0) return AION_OK;
    CK_RET(nullptr, cudaMemset(word, 0, sizeof(int)));
    set_err(nullptr, "%s: a bounded wait inside the matvec gave up (code %d); its y is invalid", what, v);
    return AION_ERR_TIMEOUT;
}

extern "C" AION_API aion_status aion_matvec_status(const aion_qmatrix* w, void* stream) {
    if (!w) {
        set_err(nullptr, "aion_matvec_status: null matrix");
        return AION_ERR_ARG;
    }
    CK_RET(nullptr, cudaSetDevice(w->device));
    CK_RET(nullptr, cudaStreamSynchronize((cudaStream_t)stream));
    aion_status st = take_error_word(w->sc.error, "aion_matvec_w4a16/_w4a8");
    unsigned char* base = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_static_mu);
        if (w->device >= 0 && w->device < kMaxStaticDevices) base = g_static_addr[w->device];
    }
    if (base) {
        const aion_status s2 =
            take_error_word(reinterpret_cast<int*>(base + kStaticPartBytes), "aion_matvec_w4a16_static");
        if (st == AION_OK) st = s2;
    }
    return st;
}

extern "C" AION_API aion_status aion_matvec_inject_timeout(const aion_qmatrix* w) {
    if (!w) {
        set_err(nullptr, "aion_matvec_inject_timeout: null matrix");
        return AION_ERR_ARG;
    }
    CK_RET(nullptr, cudaSetDevice(w->device));
    const int code = DEV_COPY_TIMEOUT;
    CK_RET(nullptr, cudaMemcpy(w->sc.error, &code, sizeof(int), cudaMemcpyHostToDevice));
    return AION_OK;
}

// ---------------------------------------------------------------------------
// Sampling beyond greedy (no counterpart in the reference, whose loop takes
// the argmax): the decode kernels draw each next token on the device.
// ---------------------------------------------------------------------------
// Copies the logits of the last decoded step (aion_decode_async /
// aion_generate) to the host.
extern "C" AION_API aion_status aion_read_logits(aion_ctx* c, float* host) {
    if (!c || !host) return AION_ERR_ARG;
    CK_RET(&c->err, cudaSetDevice(c->dev));
    CK_RET(&c->err, cudaStreamSynchronize(c->stream));
    CK_RET(&c->err, cudaMemcpy(host, c->logits, (size_t)c->vocab_l * 4, cudaMemcpyDeviceToHost));
    return AION_OK;
}

extern "C" AION_API aion_status aion_set_sampler(aion_ctx* c, const aion_sampler* s) {
    if (!c) return AION_ERR_ARG;
    if (s && s->temperature > 0.0f) {
        if (!std::isfinite(s->temperature) || !(s->top_p > 0.0f && s->top_p <= 1.0f) || s->top_k < 0) {
            set_err(&c->err, "aion_set_sampler: temperature %g, top_p %g, top_k %d out of range", s->temperature,
                    s->top_p, s->top_k);
            return AION_ERR_ARG;
        }
        if (c->tp_n > 1) {
            set_err(&c->err, "aion_set_sampler: sampling needs the whole vocabulary on one GPU (tp_size 1)");
            return AION_ERR_STATE;
        }
    }
    CK_RET(&c->err, cudaSetDevice(c->dev));
    CK_RET(&c->err, cudaStreamSynchronize(c->stream));
    c->sampling = (s && s->temperature > 0.0f) ? 1 : 0;
    c->samp = SamplerParams{};
    if (c->sampling) {
        c->samp.temperature = s->temperature;
        c->samp.top_p = s->top_p;
        c->samp.top_k = s->top_k;
        c->samp.seed = s->seed;
    }
    // The single-step graph captured the old parameters.
    if (c->gexec) cudaGraphExecDestroy(c->gexec);
    if (c->graph) cudaGraphDestroy(c->graph);
    c->gexec = nullptr;
    c->graph = nullptr;
    return AION_OK;
}

// ---------------------------------------------------------------------------
// Lock-step batched decode (no counterpart in the reference, which decodes
// one sequence): sequences 0..n_seq-1, each on its own KV cache.
// ---------------------------------------------------------------------------
// K slices of a matvec for NBLK blocks of 8 sequences: enough that one
// slice's digits fit kBDigitBudget, and enough (tile, slice) units for about
// two per warp; at most one slice per group and per CTA.
static int batch_slices(const MatDesc& m, int nblk, int grid) {
    const int gs_max = std::max(1, kBDigitBudget / (nblk * kBGroupBytes));
    int S = (m.G + gs_max - 1) / gs_max;
    S = std::max(S, (2 * kWarps * grid + m.ntiles - 1) / m.ntiles);
    return std::min(S, std::min(m.G, grid));
}

template <int NBLK>
static aion_status batch_plan(aion_ctx* c) {
    auto& pl = c->bt.plan[NBLK];
    if (pl.ops) return AION_OK;
    const DevInfo& di = dev_info(c->dev);
    const int grid = di.sms;
    std::vector<BOpDesc> ops;
    auto add = [&](const MatDesc& m, int kind, int layer) {
        BOpDesc o;
        o.m = m;
        o.kind = kind;
        o.layer = layer;
        o.S = batch_slices(m, NBLK, grid);
        o.pad = 0;
        ops.push_back(o);
    };
    for (long long l = 0; l < c->L; l++) {
        add(c->qkv[l], OP_QKV, (int)l);
        add(c->wo[l], OP_WO, (int)l);
        add(c->w13[l], OP_W13, (int)l);
        add(c->w2[l], OP_W2, (int)l);
    }
    add(c->cls, OP_CLS, 0);
    int gs = 1;
    size_t part = 0;
    for (const BOpDesc& o : ops) {
        for (int cta = 0; cta < grid; cta++) {
            const BSlice sl = bslice(o, cta, grid);
            gs = std::max(gs, sl.gb - sl.ga);
        }
        part = std::max(part, (size_t)o.S * o.m.ntiles * 8 * NBLK * kTR);
    }
    if ((long long)gs * NBLK * kBGroupBytes > kBDigitBudget + NBLK * kBGroupBytes * 8) {
        set_err(&c->err, "batched decode: a K slice of %d groups does not fit shared memory", gs);
        return AION_ERR_SHAPE;
    }
    cudaFuncAttributes fa;
    CK_RET(&c->err, cudaFuncGetAttributes(&fa, k_decode_batch<NBLK>));
    const int digits = (int)align256(std::max((size_t)gs * NBLK * kBGroupBytes, (size_t)kBAttnScratch));
    if ((size_t)grid * kBMaxSeq * sizeof(float) > (size_t)digits) {   // the norm factors' staging area
        set_err(&c->err, "batched decode: %d CTAs' norm partial sums do not fit the digit buffer", grid);
        return AION_ERR_SHAPE;
    }
    const int opsb = (int)align256(ops.size() * sizeof(BOpDesc));
    const int avail = di.smem_optin - (int)fa.sharedSizeBytes - digits - opsb - 1024;
    const int P = std::min(8, avail / (kWarps * kBChunkBytes));
    if (P < 2) {
        set_err(&c->err, "batched decode: shared memory too small for the rings (P = %d)", P);
        return AION_ERR_SHAPE;
    }
    pl.ring_off = digits;
    pl.ops_off = pl.ring_off + P * kWarps * kBChunkBytes;
    pl.total = pl.ops_off + opsb;
    pl.P = P;
    pl.part_floats = part;
    CK_RET(&c->err, cudaFuncSetAttribute(k_decode_batch<NBLK>, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.total));
    int nb = 0;
    CK_RET(&c->err, cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, k_decode_batch<NBLK>, kDecodeThreads, pl.total));
    if (nb < 1) {
        set_err(&c->err, "batched decode kernel cannot be resident (smem %d)", pl.total);
        return AION_ERR_CUDA;
    }
    CK_RET(&c->err, cudaMalloc(&pl.ops, ops.size() * sizeof(BOpDesc)));
    CK_RET(&c->err, cudaMemcpy(pl.ops, ops.data(), ops.size() * sizeof(BOpDesc), cudaMemcpyHostToDevice));
    return AION_OK;
}

template <int NBLK>
static aion_status batch_launch(aion_ctx* c, int nb, int steps) {
    aion_status s = batch_plan<NBLK>(c);
    if (s != AION_OK) return s;
    auto& bt = c->bt;
    auto& pl = bt.plan[NBLK];
    CK_RET(&c->err, pf_grow((void**)&bt.part, &bt.part_cap, pl.part_floats * 4));
    BatchArgs a;
    a.ops = pl.ops;
    a.nops = c->nops;
    a.emb = c->emb;
    a.dim = (int)c->dim;
    a.hidden = (int)c->hid_l;
    a.n_layers = (int)c->L;
    a.n_heads = (int)c->nh_l;
    a.kv_mul = (int)c->kv_mul;
    a.head_size = (int)c->hs;
    a.kv_dim = (int)c->kv_l;
    a.q_dim = (int)c->q_l;
    a.vocab = (int)c->vocab;
    a.max_pos = c->max_pos;
    a.rms_att = c->rms_att;
    a.rms_ffn = c->rms_ffn;
    a.rms_final = c->rms_final;
    a.freq_re = c->freq_re;
    a.freq_im = c->freq_im;
    a.nb = nb;
    a.x = bt.x;
    a.q = bt.q;
    a.att = bt.att;
    a.dg = bt.dg;
    a.logits = bt.logits;
    a.kcache = c->kcache;
    a.vcache = c->vcache;
    a.kv_seq = c->kv_seq;
    a.part = bt.part;
    a.ssq = bt.ssq;
    a.step = c->step;
    a.argmax = bt.argmax;
    a.first = bt.first;
    a.pos0 = bt.pos0;
    a.tokens = bt.tokens;
    a.steps = steps;
    a.P = pl.P;
    a.ring_off = pl.ring_off;
    a.ops_off = pl.ops_off;
    a.samp = c->samp;
    a.sampling = c->sampling;
    a.vocab_rows = (int)c->vocab_l;
    a.vocab_off = (int)c->vocab_off;
    a.tp_n = c->tp_n;
    a.tp_rank = c->tp_rank;
    a.tp_nbmax = c->xr_nbmax;
    a.tp_peers = c->peers_dev;
    a.tp_brecv_off = c->xr_brecv_off;
    a.tp_bkeys_off = c->xr_bkeys_off;
    a.tp_flags_off = c->xr_flags_off;
    CK_RET(&c->err, cudaMemsetAsync(&c->step->barrier, 0, sizeof(uint32_t), c->stream));
    CK_RET(&c->err, launch_ex(k_decode_batch<NBLK>, dim3(dev_info(c->dev).sms), dim3(kDecodeThreads), (size_t)pl.total,
                              c->stream, false, true, a));
    return AION_OK;
}

extern "C" AION_API aion_status aion_decode_batch(aion_ctx* c, int32_t n_seq, int32_t steps, const int32_t* first_tokens,
                                                  const int32_t* pos0, int32_t* tokens, float* logits) {
    if (!c || !first_tokens || !pos0 || !tokens) return AION_ERR_ARG;
    if (c->mode != MODE_W4A16) {
        set_err(&c->err, "aion_decode_batch runs the W4A16 mode (an int4 file)");
        return AION_ERR_STATE;
    }
    {
        const aion_status ready = tp_ready(c);
        if (ready != AION_OK) return ready;
    }
    const int cap = std::min(c->nseq, kBMaxSeq);
    if (n_seq < 1 || n_seq > cap || steps < 1) {
        set_err(&c->err, "aion_decode_batch: %d sequences (1..%d held) x %d steps", n_seq, cap, steps);
        return AION_ERR_ARG;
    }
    for (int b = 0; b < n_seq; b++)
        if (first_tokens[b] < 0 || first_tokens[b] >= c->vocab || pos0[b] < 0 ||
            (long long)pos0[b] + steps > c->max_pos) {
            set_err(&c->err, "aion_decode_batch: sequence %d: token %d at position %d for %d steps is out of range", b,
                    first_tokens[b], pos0[b], steps);
            return AION_ERR_ARG;
        }
    if ((c->dim / 32 + dev_info(c->dev).sms - 1) / dev_info(c->dev).sms > kBMaxResGroups || c->vocab_l % 4) {
        set_err(&c->err, "aion_decode_batch: dim %lld or vocab %lld unsupported", c->dim, c->vocab);
        return AION_ERR_SHAPE;
    }
    CK_RET(&c->err, cudaSetDevice(c->dev));
    auto& bt = c->bt;
    if (!bt.x) {
        const size_t nb = (size_t)cap, grid = (size_t)dev_info(c->dev).sms;
        CK_RET(&c->err, cudaMalloc(&bt.x, nb * c->dim * 4));
        CK_RET(&c->err, cudaMalloc(&bt.q, nb * c->q_l * 4));
        CK_RET(&c->err, cudaMalloc(&bt.att, nb * c->q_l * 4));
        const size_t gmax = (size_t)std::max(c->dim, c->hid_l) / 32;
        CK_RET(&c->err, cudaMalloc(&bt.dg, gmax * (kBMaxSeq / 8) * kBGroupBytes));
        CK_RET(&c->err, cudaMalloc(&bt.logits, nb * c->vocab * 4));
        CK_RET(&c->err, cudaMalloc(&bt.ssq, grid * nb * 4));
        CK_RET(&c->err, cudaMalloc(&bt.argmax, 2 * kBMaxSeq * 8));
        CK_RET(&c->err, cudaMalloc(&bt.first, kBMaxSeq * 4));
        CK_RET(&c->err, cudaMalloc(&bt.pos0, kBMaxSeq * 4));
        bt.nb = cap;
    }
    CK_RET(&c->err, pf_grow((void**)&bt.tokens, &bt.tok_cap, ((size_t)steps + 1) * n_seq * 4));
    CK_RET(&c->err, cudaMemcpyAsync(bt.first, first_tokens, n_seq * 4, cudaMemcpyHostToDevice, c->stream));
    CK_RET(&c->err, cudaMemcpyAsync(bt.pos0, pos0, n_seq * 4, cudaMemcpyHostToDevice, c->stream));
    aion_status s;
    switch ((n_seq + 7) / 8) {
    case 1: s = batch_launch<1>(c, n_seq, steps); break;
    case 2: s = batch_launch<2>(c, n_seq, steps); break;
    case 3: s = batch_launch<3>(c, n_seq, steps); break;
    default: s = batch_launch<4>(c, n_seq, steps); break;
    }
    if (s != AION_OK) return s;
    CK_RET(&c->err, cudaMemcpyAsync(tokens, bt.tokens, ((size_t)steps + 1) * n_seq * 4, cudaMemcpyDeviceToHost,
                                    c->stream));
    if (logits)
        CK_RET(&c->err, cudaMemcpyAsync(logits, bt.logits, (size_t)n_seq * c->vocab_l * 4, cudaMemcpyDeviceToHost,
                                        c->stream));
    CK_RET(&c->err, cudaStreamSynchronize(c->stream));
    return check_device_error(c);
}

// ---------------------------------------------------------------------------
// tcgen05 bf16 GEMM (prefill building block)
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 2-D tensor map of a row-major bf16 [rows][cols] matrix, box (64 cols x
// box_rows rows), 128-byte swizzle (the UMMA K-major canonical layout).
static bool bf16_tensor_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int box_rows) {
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kGemmBK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int* g_gemm_err_dev[kMaxStaticDevices];
static __device__ int g_gemm_err_word;

// C[M][ldc] (fp32) = A[M][K] * B[N][K]^T, bf16 A and B with K contiguous.
static aion_status launch_gemm_bf16(const void* a, const void* b, float* c, int64_t m, int64_t n, int64_t k,
                                    int64_t ldc, int dev, cudaStream_t st, int* err_dev, std::string* err) {
    if (m <= 0 || n <= 0 || k <= 0 || m % kGemmBM || n % kGemmBN || k % kGemmBK || ldc < n || ldc % 4 ||
        (m / kGemmBM) * (n / kGemmBN) > 0x7FFFFFFF) {
        set_err(err, "gemm: M, N, K must be positive multiples of %d, %d, %d (got %lld, %lld, %lld)", kGemmBM,
                kGemmBN, kGemmBK, (long long)m, (long long)n, (long long)k);
        return AION_ERR_SHAPE;
    }
    if (((uintptr_t)a & 15) || ((uintptr_t)b & 15) || ((uintptr_t)c & 15)) {
        set_err(err, "gemm: A, B and C must be 16-byte aligned");
        return AION_ERR_ARG;
    }
    CUtensorMap ma, mb;
    if (!bf16_tensor_map(&ma, a, m, k, kGemmBM) || !bf16_tensor_map(&mb, b, n, k, kGemmBN)) {
        set_err(err, "gemm: cuTensorMapEncodeTiled is unavailable or rejected the operands");
        return AION_ERR_CUDA;
    }
    CK_RET(err, ensure_smem_attr((const void*)k_gemm_bf16_tn, ATTR_GEMM, dev, kGemmSmem));
    GemmArgs g;
    g.C = c;
    g.M = (int)m;
    g.N = (int)n;
    g.K = (int)k;
    g.ldc = (int)ldc;
    g.err = err_dev;
    const long long tiles = (m / kGemmBM) * (n / kGemmBN);
    const int grid = (int)std::min<long long>(tiles, dev_info(dev).sms);   // persistent: one CTA per SM
    k_gemm_bf16_tn<<<(unsigned)grid, kGemmThreads, kGemmSmem, st>>>(ma, mb, g);
    CK_RET(err, cudaGetLastError());
    return AION_OK;
}

extern "C" AION_API aion_status aion_gemm_bf16_tn(const void* a_dev, const void* b_dev, float* c_dev, int64_t m,
                                                  int64_t n, int64_t k, void* stream) {
    if (!a_dev || !b_dev || !c_dev) {
        set_err(nullptr, "aion_gemm_bf16_tn: null argument");
        return AION_ERR_ARG;
    }
    int dev = 0;
    CK_RET(nullptr, cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxStaticDevices) {
        set_err(nullptr, "aion_gemm_bf16_tn: device %d beyond the %d devices this library supports", dev,
                kMaxStaticDevices);
        return AION_ERR_ARG;
    }
    if (!g_gemm_err_dev[dev]) {
        void* p = nullptr;
        CK_RET(nullptr, cudaGetSymbolAddress(&p, g_gemm_err_word));
        g_gemm_err_dev[dev] = static_cast<int*>(p);
    }
    std::string err;
    const aion_status s = launch_gemm_bf16(a_dev, b_dev, c_dev, m, n, k, n, dev, (cudaStream_t)stream,
                                           g_gemm_err_dev[dev], &err);
    if (s != AION_OK) set_err(nullptr, "%s", err.c_str());
    return s;
}

extern "C" AION_API aion_status aion_quantize_buffer_dev(const float* in_dev, uint8_t* packed_dev, float* scales_dev,
                                                         int64_t n, void* stream) {
    if (!in_dev || !packed_dev || !scales_dev || n < 0 || n % 32) {
        set_err(nullptr, "aion_quantize_buffer_dev: null pointer, or n not a multiple of 32");
        return AION_ERR_ARG;
    }
    if (((uintptr_t)in_dev & 15) || ((uintptr_t)packed_dev & 15) || ((uintptr_t)scales_dev & 3)) {
        set_err(nullptr, "aion_quantize_buffer_dev: in and packed must be 16-byte aligned, scales 4-byte aligned");
        return AION_ERR_ARG;
    }
    if (n == 0) return AION_OK;
    const long long groups = n / 32;
    const int grid = (int)std::min<long long>((groups + 255) / 256, 148LL * 16);
    k_quantize_groups<<<grid, 256, 0, (cudaStream_t)stream>>>(in_dev, packed_dev, scales_dev, groups);
    CK_RET(nullptr, cudaGetLastError());
    return AION_OK;
}

extern "C" AION_API aion_status aion_quantize_activations(const float* x, int8_t* qx, float* xs, int64_t n, void* stream) {
    if (!x || !qx || !xs || n <= 0 || n % 32) {
        set_err(nullptr, "aion_quantize_activations: invalid arguments (n must be a positive multiple of 32)");
        return AION_ERR_ARG;
    }
    int grid = (int)std::min<long long>((n / 32 + 255) / 256, 4096);
    k_quantize_act<<<grid, 256, 0, (cudaStream_t)stream>>>(x, qx, xs, n);
    CK_RET(nullptr, cudaGetLastError());
    return AION_OK;
}

#ifdef AION_PHASE_TIMING
extern "C" AION_API aion_status aion_phase_clear() {
    const size_t tw = (size_t)kPhaseSteps * kPhaseOps * kPhaseCtas * 8;
    void* p = nullptr;
    CK_RET(nullptr, cudaGetSymbolAddress(&p, g_phase_w));
    CK_RET(nullptr, cudaMemset(p, 0, tw * sizeof(unsigned long long)));
    return AION_OK;
}
// Profiling builds only: copies the phase timestamps of the last decode
// launch (layout [step][op][cta][slot], see common.cuh) into `host`.
extern "C" AION_API aion_status aion_phase_dump(unsigned long long* host, size_t n) {
    const size_t total = (size_t)kPhaseSteps * kPhaseOps * kPhaseCtas * kPhaseSlots;
    if (!host || n < total) return AION_ERR_ARG;
    CK_RET(nullptr, cudaMemcpyFromSymbol(host, g_phase, total * sizeof(unsigned long long)));
    const size_t tw = (size_t)kPhaseSteps * kPhaseOps * kPhaseCtas * 8;
    if (n >= total + tw) CK_RET(nullptr, cudaMemcpyFromSymbol(host + total, g_phase_w, tw * sizeof(unsigned long long)));
    return AION_OK;
}
#endif
