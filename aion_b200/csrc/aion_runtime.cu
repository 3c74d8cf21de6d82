// Host side of libaion: the C ABI declared in include/aion.h.
//
// Replaces the reference's loader, run state, thread pool and forward driver
// (src/kernel_simd.c:631-787, 906-1169): the int4 checkpoint is uploaded
// once and re-tiled in HBM, and one decode step is a fixed sequence of
// fused kernels on one stream, captured once as a CUDA graph and replayed
// per token.  No host thread spins; nothing here exits the process.
#include <cuda_runtime.h>
#include <errno.h>
#include <fcntl.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>
#include <sys/stat.h>
#include <time.h>
#include <unistd.h>

#include <string>
#include <vector>

#include "../../include/aion.h"
#include "decode_kernels.cuh"

using namespace aion;

// ---------------------------------------------------------------------------
// Errors
// ---------------------------------------------------------------------------
static thread_local std::string g_thread_err;

struct aion_ctx;
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
// Tiled device matrices
// ---------------------------------------------------------------------------
struct DevMatrix {
    uint8_t* w = nullptr;
    long long tile_bytes = 0;
    int n = 0;
    long long rows = 0;      // logical rows
    long long rows_pad = 0;  // multiple of kRB
    int ntiles = 0;
};

static long long tiled_bytes(long long rows, int n) {
    long long rp = (rows + kRB - 1) / kRB * kRB;
    return rp / kRB * ((long long)kRB * n / 32 * 4 + (long long)kRB * n / 2);
}

static void dev_matrix_init(DevMatrix* m, uint8_t* w, long long rows, int n) {
    m->w = w;
    m->n = n;
    m->rows = rows;
    m->rows_pad = (rows + kRB - 1) / kRB * kRB;
    m->tile_bytes = (long long)kRB * n / 32 * 4 + (long long)kRB * n / 2;
    m->ntiles = (int)(m->rows_pad / kRB);
}

static int g_num_sms[64];

static int num_sms(int dev) {
    if (dev < 0 || dev >= 64) return 148;
    if (!g_num_sms[dev]) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
        g_num_sms[dev] = v;
    }
    return g_num_sms[dev];
}

// Launch with the programmatic-stream-serialization attribute (PDL): the
// kernel may start while its predecessor drains; it synchronises on the
// predecessor with griddepcontrol.wait before touching its outputs.
template <typename... KArgs, typename... Args>
static cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                          Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

typedef void (*MatvecKernel)(MatvecArgs);

template <int MODE>
static MatvecKernel pick_matvec(int pro, int epi) {
    if (pro == PRO_PLAIN) {
        switch (epi) {
        case EPI_STORE: return k_matvec<MODE, PRO_PLAIN, EPI_STORE>;
        case EPI_RESIDUAL: return k_matvec<MODE, PRO_PLAIN, EPI_RESIDUAL>;
        default: return nullptr;
        }
    }
    switch (epi) {
    case EPI_QKV: return k_matvec<MODE, PRO_RMSNORM, EPI_QKV>;
    case EPI_SWIGLU: return k_matvec<MODE, PRO_RMSNORM, EPI_SWIGLU>;
    case EPI_LOGITS: return k_matvec<MODE, PRO_RMSNORM, EPI_LOGITS>;
    case EPI_STORE: return k_matvec<MODE, PRO_RMSNORM, EPI_STORE>;
    default: return nullptr;
    }
}

static MatvecKernel matvec_kernel(int mode, int pro, int epi) {
    return mode == MODE_W4A8 ? pick_matvec<MODE_W4A8>(pro, epi) : pick_matvec<MODE_W4A16>(pro, epi);
}

static cudaError_t raise_smem_limits() {
    static bool done = false;
    if (done) return cudaSuccess;
    const int pros[2] = {PRO_PLAIN, PRO_RMSNORM};
    const int epis[5] = {EPI_STORE, EPI_RESIDUAL, EPI_QKV, EPI_SWIGLU, EPI_LOGITS};
    for (int mode = 0; mode < 2; mode++)
        for (int p = 0; p < 2; p++)
            for (int e = 0; e < 5; e++) {
                MatvecKernel k = matvec_kernel(mode, pros[p], epis[e]);
                if (!k) continue;
                cudaError_t err = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
                if (err != cudaSuccess) return err;
            }
    done = true;
    return cudaSuccess;
}

static cudaError_t launch_matvec(int mode, int pro, int epi, const DevMatrix& m, MatvecArgs a, int dev, cudaStream_t st,
                                 bool pdl) {
    a.w = m.w;
    a.tile_bytes = m.tile_bytes;
    a.n = m.n;
    a.ntiles = m.ntiles;
    if (a.d == 0) a.d = (int)m.rows;
    a.prefetch_tiles = kMvWarps;
    const int sms = num_sms(dev);
    int grid = (m.ntiles + kMvWarps - 1) / kMvWarps;
    if (grid > 2 * sms) grid = 2 * sms;
    if (grid < 1) grid = 1;
    return launch(matvec_kernel(mode, pro, epi), dim3(grid), dim3(kMvThreads), (size_t)matvec_smem_bytes(m.n, mode),
                  st, pdl, a);
}

static cudaError_t retile(const DevMatrix& m, const float* scales, const uint8_t* packed, long long rows,
                          int row_offset, int interleave, int slot, int inverse, cudaStream_t st) {
    RetileArgs a;
    a.src_scales = scales;
    a.src_packed = packed;
    a.dst = m.w;
    a.tile_bytes = m.tile_bytes;
    a.rows = rows;
    a.n = m.n;
    a.row_offset = row_offset;
    a.interleave = interleave;
    a.slot = slot;
    a.inverse = inverse;
    long long total = rows * (m.n / 32);
    int grid = (int)((total + 255) / 256);
    if (grid > 65535) grid = 65535;
    if (grid < 1) grid = 1;
    k_retile<<<grid, 256, 0, st>>>(a);
    return cudaGetLastError();
}

static cudaError_t fill_pad(const DevMatrix& m, cudaStream_t st) {
    if (m.rows_pad == m.rows) return cudaSuccess;
    k_fill_pad<<<8, 256, 0, st>>>(m.w, m.tile_bytes, m.rows, m.rows_pad, m.n);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Context
// ---------------------------------------------------------------------------
struct aion_ctx {
    std::string err;
    aion_opts opts;
    aion_config cfg;
    int dev = 0, mode = 0;
    long long dim = 0, hidden = 0, L = 0, nh = 0, nkv = 0, vocab = 0, seq = 0, hs = 0, kv_dim = 0, kv_mul = 0;
    int max_pos = 0;
    cudaStream_t stream = nullptr;
    uint8_t* arena = nullptr;
    size_t arena_bytes = 0, arena_used = 0;
    DevMatrix emb;
    std::vector<DevMatrix> qkv, wo, w13, w2;
    float *rms_att = nullptr, *rms_ffn = nullptr, *rms_final = nullptr, *freq_re = nullptr, *freq_im = nullptr;
    float *kcache = nullptr, *vcache = nullptr;
    float *x = nullptr, *q = nullptr, *att = nullptr, *hb = nullptr, *logits = nullptr;
    float* attn_partial = nullptr;
    int* attn_counters = nullptr;
    int split_len = 64, n_splits = 1;
    StepState* step = nullptr;
    unsigned long long* argmax = nullptr;
    int32_t* history = nullptr;
    StepState* h_step = nullptr;   // pinned
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t gexec = nullptr;
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
    o->device = 0;
    o->mode = AION_MODE_W4A16;
    o->max_batch = 1;
    o->max_pos = 0;
    o->tp_size = 1;
    o->tp_rank = 0;
    o->nccl_id = nullptr;
    o->use_graph = 1;
}

extern "C" AION_API const char* aion_last_error(const aion_ctx* ctx) {
    if (ctx) return ctx->err.c_str();
    return g_thread_err.c_str();
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
// One decode step: the kernel sequence of transformer() (src/kernel_simd.c:
// 1014-1169) with the matvecs fused to their neighbours:
//   embed | per layer: [rmsnorm + QKV + RoPE + KV append] [attention]
//   [wo + residual] [rmsnorm + w1/w3 + SwiGLU] [w2 + residual]
//   | [final rmsnorm + classifier + argmax]
// ---------------------------------------------------------------------------
static cudaError_t enqueue_step(aion_ctx* c) {
    cudaError_t e;
    cudaStream_t st = c->stream;
    EmbedArgs ea;
    ea.emb = c->emb.w;
    ea.tile_bytes = c->emb.tile_bytes;
    ea.dim = (int)c->dim;
    ea.vocab = (int)c->vocab;
    ea.max_pos = c->max_pos;
    ea.x = c->x;
    ea.step = c->step;
    ea.argmax = c->argmax;
    ea.history = c->history;
    if ((e = launch(k_embed, dim3(1), dim3(256), 0, st, true, ea)) != cudaSuccess) return e;

    const size_t layer_kv = (size_t)c->max_pos * c->kv_dim;
    for (long long l = 0; l < c->L; l++) {
        MatvecArgs a = {};
        a.x = c->x;
        a.norm_w = c->rms_att + l * c->dim;
        a.q_out = c->q;
        a.kcache = c->kcache + l * layer_kv;
        a.vcache = c->vcache + l * layer_kv;
        a.freq_re = c->freq_re;
        a.freq_im = c->freq_im;
        a.dim = (int)c->dim;
        a.kv_dim = (int)c->kv_dim;
        a.head_size = (int)c->hs;
        a.step = c->step;
        if ((e = launch_matvec(c->mode, PRO_RMSNORM, EPI_QKV, c->qkv[l], a, c->dev, st, true)) != cudaSuccess) return e;

        AttnArgs aa;
        aa.q = c->q;
        aa.kcache = c->kcache + l * layer_kv;
        aa.vcache = c->vcache + l * layer_kv;
        aa.out = c->att;
        aa.partial = c->attn_partial;
        aa.counters = c->attn_counters;
        aa.step = c->step;
        aa.n_heads = (int)c->nh;
        aa.kv_mul = (int)c->kv_mul;
        aa.head_size = (int)c->hs;
        aa.kv_dim = (int)c->kv_dim;
        aa.split_len = c->split_len;
        aa.n_splits = c->n_splits;
        if ((e = launch(k_attention, dim3((unsigned)c->nh, (unsigned)c->n_splits), dim3(kAttnThreads), 0, st, true, aa)) !=
            cudaSuccess)
            return e;

        MatvecArgs o = {};
        o.x = c->att;
        o.y = c->x;
        if ((e = launch_matvec(c->mode, PRO_PLAIN, EPI_RESIDUAL, c->wo[l], o, c->dev, st, true)) != cudaSuccess) return e;

        MatvecArgs f = {};
        f.x = c->x;
        f.norm_w = c->rms_ffn + l * c->dim;
        f.y = c->hb;
        f.d = (int)c->hidden;
        if ((e = launch_matvec(c->mode, PRO_RMSNORM, EPI_SWIGLU, c->w13[l], f, c->dev, st, true)) != cudaSuccess) return e;

        MatvecArgs d = {};
        d.x = c->hb;
        d.y = c->x;
        if ((e = launch_matvec(c->mode, PRO_PLAIN, EPI_RESIDUAL, c->w2[l], d, c->dev, st, true)) != cudaSuccess) return e;
    }
    MatvecArgs z = {};
    z.x = c->x;
    z.norm_w = c->rms_final;
    z.y = c->logits;
    z.argmax = c->argmax;
    z.step = c->step;
    return launch_matvec(c->mode, PRO_RMSNORM, EPI_LOGITS, c->emb, z, c->dev, st, true);
}

static aion_status build_graph(aion_ctx* c) {
    if (c->gexec) return AION_OK;
    CK_RET(&c->err, cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    cudaError_t e = enqueue_step(c);
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

static aion_status run_step(aion_ctx* c) {
    if (c->opts.use_graph) {
        aion_status s = build_graph(c);
        if (s != AION_OK) return s;
        CK_RET(&c->err, cudaGraphLaunch(c->gexec, c->stream));
    } else {
        CK_RET(&c->err, enqueue_step(c));
    }
    return AION_OK;
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
    if (hs % 2 || hs > kMaxHeadSize || c.dim % 32 || c.hidden_dim % 32 || kv % 32) {
        set_err(err, "unsupported shape: head_size %lld, dim %d, hidden %d, kv_dim %lld (need even head_size <= %d, "
                     "multiples of 32)", hs, c.dim, c.hidden_dim, kv, kMaxHeadSize);
        return AION_ERR_SHAPE;
    }
    return AION_OK;
}

static aion_status upload_range(aion_ctx* c, int fd, long long off, long long bytes, uint8_t* dst, uint8_t* pinned[2],
                                cudaEvent_t ev[2], size_t chunk) {
    long long done = 0;
    int i = 0;
    while (done < bytes) {
        size_t n = (size_t)((bytes - done) < (long long)chunk ? (bytes - done) : (long long)chunk);
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

// Reads and validates the 28-byte header and the file size (64-bit) before
// any device work: a truncated or inconsistent file fails here.
static aion_status read_header(const char* path, aion_config* cfg, std::string* err) {
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
        if (cfg->vocab_size < 0) cfg->vocab_size = -cfg->vocab_size;  // src/kernel_simd.c:945
        s = validate_config(*cfg, err);
        if (s == AION_OK) {
            const long long want = int4_file_bytes(*cfg);
            if (want != (long long)st.st_size) {
                set_err(err, "%s: header implies %lld bytes for an int4 file, file has %lld", path, want,
                        (long long)st.st_size);
                s = AION_ERR_FORMAT;
            }
        }
    }
    close(fd);
    return s;
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
        c->split_len = 64;
        c->n_splits = (c->max_pos + c->split_len - 1) / c->split_len;

        // Arena: weights + fp32 tensors + KV cache + activations + scratch.
        const long long dim = c->dim, hid = c->hidden, L = c->L, kv = c->kv_dim;
        size_t bytes = align256(tiled_bytes(c->vocab, (int)dim));
        bytes += L * (align256(tiled_bytes(dim + 2 * kv, (int)dim)) + align256(tiled_bytes(dim, (int)dim)) +
                      align256(tiled_bytes(2 * hid, (int)dim)) + align256(tiled_bytes(dim, (int)hid)));
        bytes += align256(L * dim * 4) * 2 + align256(dim * 4) + 2 * align256(c->seq * (c->hs / 2) * 4);
        bytes += 2 * align256((size_t)L * c->max_pos * kv * 4);
        bytes += 3 * align256(dim * 4) + align256(hid * 4) + align256(c->vocab * 4);
        bytes += align256((size_t)c->nh * c->n_splits * (c->hs + 2) * 4) + align256(c->nh * 4);
        bytes += align256(sizeof(StepState)) + align256(8) + align256((size_t)c->max_pos * 4);
        c->arena_bytes = bytes + 4096;
        CK_RET(&c->err, cudaMalloc(&c->arena, c->arena_bytes));
        CK_RET(&c->err, cudaMemsetAsync(c->arena, 0, c->arena_bytes, c->stream));

        dev_matrix_init(&c->emb, arena_take(c, tiled_bytes(c->vocab, (int)dim)), c->vocab, (int)dim);
        c->qkv.resize(L); c->wo.resize(L); c->w13.resize(L); c->w2.resize(L);
        for (long long l = 0; l < L; l++) {
            dev_matrix_init(&c->qkv[l], arena_take(c, tiled_bytes(dim + 2 * kv, (int)dim)), dim + 2 * kv, (int)dim);
            dev_matrix_init(&c->wo[l], arena_take(c, tiled_bytes(dim, (int)dim)), dim, (int)dim);
            dev_matrix_init(&c->w13[l], arena_take(c, tiled_bytes(2 * hid, (int)dim)), 2 * hid, (int)dim);
            dev_matrix_init(&c->w2[l], arena_take(c, tiled_bytes(dim, (int)hid)), dim, (int)hid);
        }
        c->rms_att = (float*)arena_take(c, L * dim * 4);
        c->rms_ffn = (float*)arena_take(c, L * dim * 4);
        c->rms_final = (float*)arena_take(c, dim * 4);
        c->freq_re = (float*)arena_take(c, c->seq * (c->hs / 2) * 4);
        c->freq_im = (float*)arena_take(c, c->seq * (c->hs / 2) * 4);
        c->kcache = (float*)arena_take(c, (size_t)L * c->max_pos * kv * 4);
        c->vcache = (float*)arena_take(c, (size_t)L * c->max_pos * kv * 4);
        c->x = (float*)arena_take(c, dim * 4);
        c->q = (float*)arena_take(c, dim * 4);
        c->att = (float*)arena_take(c, dim * 4);
        c->hb = (float*)arena_take(c, hid * 4);
        c->logits = (float*)arena_take(c, c->vocab * 4);
        c->attn_partial = (float*)arena_take(c, (size_t)c->nh * c->n_splits * (c->hs + 2) * 4);
        c->attn_counters = (int*)arena_take(c, c->nh * 4);
        c->step = (StepState*)arena_take(c, sizeof(StepState));
        c->argmax = (unsigned long long*)arena_take(c, 8);
        c->history = (int32_t*)arena_take(c, (size_t)c->max_pos * 4);
        if (!c->history) {
            set_err(&c->err, "internal: arena too small");
            s = AION_ERR_OOM;
            break;
        }

        // Largest quantized stacked tensor: the staging area for re-tiling.
        auto qb = [](long long cnt) { return cnt / 32 * 4 + cnt / 2; };
        long long stage = qb(c->vocab * dim);
        stage = std::max(stage, qb(L * dim * hid));
        stage = std::max(stage, qb(L * dim * dim));
        stage = std::max(stage, L * dim * 4);
        CK_RET(&c->err, cudaMalloc(&staging, (size_t)stage));
        CK_RET(&c->err, cudaHostAlloc(&pinned[0], chunk, cudaHostAllocDefault));
        CK_RET(&c->err, cudaHostAlloc(&pinned[1], chunk, cudaHostAllocDefault));
        CK_RET(&c->err, cudaEventCreateWithFlags(&ev[0], cudaEventDisableTiming));
        CK_RET(&c->err, cudaEventCreateWithFlags(&ev[1], cudaEventDisableTiming));
        CK_RET(&c->err, cudaEventRecord(ev[0], c->stream));
        CK_RET(&c->err, cudaEventRecord(ev[1], c->stream));

        long long off = 28;
        // Walks the file in the order of quantize.c:192-229 /
        // src/kernel_simd.c:970-986; `fn` re-tiles or copies each tensor.
        auto qtensor = [&](long long count, auto fn) -> aion_status {
            long long b = qb(count);
            aion_status r = upload_range(c, fd, off, b, staging, pinned, ev, chunk);
            if (r != AION_OK) return r;
            const float* sc = (const float*)staging;
            const uint8_t* pk = staging + count / 32 * 4;
            cudaError_t e = fn(sc, pk);
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
        auto per_layer = [&](long long rows, long long n, std::vector<DevMatrix>& dst, int row_offset, int interleave,
                             int slot) {
            return [&, rows, n, row_offset, interleave, slot](const float* sc, const uint8_t* pk) -> cudaError_t {
                for (long long l = 0; l < L; l++) {
                    long long e0 = l * rows * n;
                    cudaError_t e = retile(dst[l], sc + e0 / 32, pk + e0 / 2, rows, row_offset, interleave, slot, 0,
                                           c->stream);
                    if (e != cudaSuccess) return e;
                }
                return cudaSuccess;
            };
        };
        if ((s = qtensor(c->vocab * dim, [&](const float* sc, const uint8_t* pk) {
                 cudaError_t e = retile(c->emb, sc, pk, c->vocab, 0, 0, 0, 0, c->stream);
                 return e != cudaSuccess ? e : fill_pad(c->emb, c->stream);
             })) != AION_OK) break;
        if ((s = ftensor(L * dim, c->rms_att)) != AION_OK) break;
        if ((s = qtensor(L * dim * dim, per_layer(dim, dim, c->qkv, 0, 0, 0))) != AION_OK) break;
        if ((s = qtensor(L * dim * kv, per_layer(kv, dim, c->qkv, (int)dim, 0, 0))) != AION_OK) break;
        if ((s = qtensor(L * dim * kv, per_layer(kv, dim, c->qkv, (int)(dim + kv), 0, 0))) != AION_OK) break;
        if ((s = qtensor(L * dim * dim, per_layer(dim, dim, c->wo, 0, 0, 0))) != AION_OK) break;
        if ((s = ftensor(L * dim, c->rms_ffn)) != AION_OK) break;
        if ((s = qtensor(L * dim * hid, per_layer(hid, dim, c->w13, 0, 1, 0))) != AION_OK) break;
        if ((s = qtensor(L * hid * dim, per_layer(dim, hid, c->w2, 0, 0, 0))) != AION_OK) break;
        if ((s = qtensor(L * dim * hid, per_layer(hid, dim, c->w13, 0, 1, 1))) != AION_OK) break;
        if ((s = ftensor(dim, c->rms_final)) != AION_OK) break;
        if ((s = ftensor(c->seq * (c->hs / 2), c->freq_re)) != AION_OK) break;
        if ((s = ftensor(c->seq * (c->hs / 2), c->freq_im)) != AION_OK) break;
        for (long long l = 0; l < L; l++) {
            cudaError_t e = fill_pad(c->qkv[l], c->stream);
            if (e == cudaSuccess) e = fill_pad(c->wo[l], c->stream);
            if (e == cudaSuccess) e = fill_pad(c->w2[l], c->stream);
            CK_RET(&c->err, e);
        }
        // Step state: pos 0, no forced token, argmax key at its initial value.
        StepState init = {};
        init.forced_token = -1;
        unsigned long long key0 = argmax_key(-1e9f, 0);
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
    if (c->opts.max_batch > 1 || c->opts.tp_size > 1) {
        set_err(&c->err, "max_batch > 1 and tp_size > 1 are not available in this build");
        delete c;
        return AION_ERR_ARG;
    }
    c->mode = c->opts.mode == AION_MODE_W4A8 ? MODE_W4A8 : MODE_W4A16;
    c->dev = c->opts.device;
    aion_status hs = read_header(path, &c->cfg, &c->err);
    if (hs != AION_OK) {
        delete c;
        return hs;
    }
    cudaError_t e = cudaSetDevice(c->dev);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = raise_smem_limits();
    if (e == cudaSuccess) e = cudaHostAlloc(&c->h_step, sizeof(StepState), cudaHostAllocDefault);
    if (e != cudaSuccess) {
        set_err(&c->err, "CUDA init failed: %s", cudaGetErrorString(e));
        ctx_destroy(c);
        return AION_ERR_CUDA;
    }
    aion_status s = load_impl(c, path);
    if (s != AION_OK) {
        g_thread_err = c->err;
        ctx_destroy(c);
        return s;
    }
    *out = c;
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
    memset(c->h_step, 0, sizeof(StepState));
    c->h_step->pos_next = pos;
    c->h_step->forced_token = token;
    CK_RET(&c->err, cudaMemcpyAsync(c->step, c->h_step, sizeof(StepState), cudaMemcpyHostToDevice, c->stream));
    aion_status s = run_step(c);
    if (s != AION_OK) return s;
    if (logits_host)
        CK_RET(&c->err, cudaMemcpyAsync(logits_host, c->logits, c->vocab * 4, cudaMemcpyDeviceToHost, c->stream));
    CK_RET(&c->err, cudaStreamSynchronize(c->stream));
    return AION_OK;
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
    memset(c->h_step, 0, sizeof(StepState));
    c->h_step->pos_next = 0;
    c->h_step->forced_token = bos;
    CK_RET(&c->err, cudaMemcpyAsync(c->step, c->h_step, sizeof(StepState), cudaMemcpyHostToDevice, c->stream));
    if (c->opts.use_graph) {
        aion_status s = build_graph(c);
        if (s != AION_OK) return s;
    }
    CK_RET(&c->err, cudaStreamSynchronize(c->stream));
    struct timespec t0, t1;
    clock_gettime(CLOCK_MONOTONIC, &t0);
    for (int i = 0; i < steps; i++) {
        aion_status s = run_step(c);
        if (s != AION_OK) return s;
    }
    CK_RET(&c->err, cudaStreamSynchronize(c->stream));
    clock_gettime(CLOCK_MONOTONIC, &t1);
    if (seconds) *seconds = (double)(t1.tv_sec - t0.tv_sec) + 1e-9 * (double)(t1.tv_nsec - t0.tv_nsec);
    if (tokens_out && steps > 0)
        CK_RET(&c->err, cudaMemcpy(tokens_out, c->history, (size_t)steps * 4, cudaMemcpyDeviceToHost));
    CK_RET(&c->err, cudaMemcpy(c->h_step, c->step, sizeof(StepState), cudaMemcpyDeviceToHost));
    if (c->h_step->error) {
        set_err(&c->err, "a decode step rejected its token or position");
        return AION_ERR_STATE;
    }
    return AION_OK;
}

extern "C" AION_API void* aion_stream(const aion_ctx* c) { return c ? (void*)c->stream : nullptr; }

extern "C" AION_API aion_status aion_step_async(aion_ctx* c, int32_t token, int32_t pos) {
    if (!c) return AION_ERR_ARG;
    if (token >= c->vocab || pos >= c->max_pos) {
        set_err(&c->err, "aion_step_async: token %d or pos %d out of range", token, pos);
        return AION_ERR_ARG;
    }
    CK_RET(&c->err, cudaSetDevice(c->dev));
    if (token >= 0 || pos >= 0) {
        k_set_step<<<1, 32, 0, c->stream>>>(c->step, pos, token);
        CK_RET(&c->err, cudaGetLastError());
    }
    return run_step(c);
}

extern "C" AION_API aion_status aion_tokens(aion_ctx* c, int32_t* out, int32_t n) {
    if (!c || !out || n < 0 || n > c->max_pos) return AION_ERR_ARG;
    CK_RET(&c->err, cudaSetDevice(c->dev));
    CK_RET(&c->err, cudaStreamSynchronize(c->stream));
    if (n) CK_RET(&c->err, cudaMemcpy(out, c->history, (size_t)n * 4, cudaMemcpyDeviceToHost));
    return AION_OK;
}

// Times each kernel class of the decode step in isolation on the context's
// stream: for every class the per-layer launches of all layers run back to
// back `reps` times between two events; out_ms[k] receives the mean time of
// one launch.  Classes: 0 rmsnorm+QKV+RoPE, 1 attention, 2 wo+residual,
// 3 rmsnorm+w1/w3+SwiGLU, 4 w2+residual, 5 rmsnorm+classifier+argmax,
// 6 embed.  Clobbers the activations and the KV cache row of the current
// position; call it between sequences.
extern "C" AION_API aion_status aion_time_kernels(aion_ctx* c, int32_t reps, float* out_ms) {
    if (!c || !out_ms || reps <= 0) return AION_ERR_ARG;
    CK_RET(&c->err, cudaSetDevice(c->dev));
    cudaEvent_t e0, e1;
    CK_RET(&c->err, cudaEventCreate(&e0));
    CK_RET(&c->err, cudaEventCreate(&e1));
    const size_t layer_kv = (size_t)c->max_pos * c->kv_dim;
    aion_status status = AION_OK;
    for (int k = 0; k < 7 && status == AION_OK; k++) {
        cudaError_t e = cudaEventRecord(e0, c->stream);
        int launches = 0;
        for (int r = 0; r < reps && e == cudaSuccess; r++) {
            const long long nl = (k == 5 || k == 6) ? 1 : c->L;
            for (long long l = 0; l < nl && e == cudaSuccess; l++) {
                launches++;
                if (k == 0) {
                    MatvecArgs a = {};
                    a.x = c->x; a.norm_w = c->rms_att + l * c->dim; a.q_out = c->q;
                    a.kcache = c->kcache + l * layer_kv; a.vcache = c->vcache + l * layer_kv;
                    a.freq_re = c->freq_re; a.freq_im = c->freq_im; a.dim = (int)c->dim; a.kv_dim = (int)c->kv_dim;
                    a.head_size = (int)c->hs; a.step = c->step;
                    e = launch_matvec(c->mode, PRO_RMSNORM, EPI_QKV, c->qkv[l], a, c->dev, c->stream, true);
                } else if (k == 1) {
                    AttnArgs aa;
                    aa.q = c->q; aa.kcache = c->kcache + l * layer_kv; aa.vcache = c->vcache + l * layer_kv;
                    aa.out = c->att; aa.partial = c->attn_partial; aa.counters = c->attn_counters; aa.step = c->step;
                    aa.n_heads = (int)c->nh; aa.kv_mul = (int)c->kv_mul; aa.head_size = (int)c->hs;
                    aa.kv_dim = (int)c->kv_dim; aa.split_len = c->split_len; aa.n_splits = c->n_splits;
                    e = launch(k_attention, dim3((unsigned)c->nh, (unsigned)c->n_splits), dim3(kAttnThreads), 0,
                               c->stream, true, aa);
                } else if (k == 2 || k == 4) {
                    MatvecArgs o = {};
                    o.x = k == 2 ? c->att : c->hb;
                    o.y = c->x;
                    e = launch_matvec(c->mode, PRO_PLAIN, EPI_RESIDUAL, k == 2 ? c->wo[l] : c->w2[l], o, c->dev,
                                      c->stream, true);
                } else if (k == 3) {
                    MatvecArgs f = {};
                    f.x = c->x; f.norm_w = c->rms_ffn + l * c->dim; f.y = c->hb; f.d = (int)c->hidden;
                    e = launch_matvec(c->mode, PRO_RMSNORM, EPI_SWIGLU, c->w13[l], f, c->dev, c->stream, true);
                } else if (k == 5) {
                    MatvecArgs z = {};
                    z.x = c->x; z.norm_w = c->rms_final; z.y = c->logits; z.argmax = c->argmax; z.step = c->step;
                    e = launch_matvec(c->mode, PRO_RMSNORM, EPI_LOGITS, c->emb, z, c->dev, c->stream, true);
                } else {
                    EmbedArgs ea;
                    ea.emb = c->emb.w; ea.tile_bytes = c->emb.tile_bytes; ea.dim = (int)c->dim;
                    ea.vocab = (int)c->vocab; ea.max_pos = c->max_pos; ea.x = c->x; ea.step = c->step;
                    ea.argmax = c->argmax; ea.history = c->history;
                    e = launch(k_embed, dim3(1), dim3(256), 0, c->stream, true, ea);
                }
            }
        }
        if (e == cudaSuccess) e = cudaEventRecord(e1, c->stream);
        if (e == cudaSuccess) e = cudaEventSynchronize(e1);
        float ms = 0.0f;
        if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
        if (e != cudaSuccess) {
            set_err(&c->err, "aion_time_kernels: %s", cudaGetErrorString(e));
            status = cuda_status(e);
        }
        out_ms[k] = ms / (float)launches;
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    return status;
}

extern "C" AION_API aion_status aion_reset(aion_ctx* c) {
    if (!c) return AION_ERR_ARG;
    CK_RET(&c->err, cudaSetDevice(c->dev));
    const size_t kvb = (size_t)c->L * c->max_pos * c->kv_dim * 4;
    CK_RET(&c->err, cudaMemsetAsync(c->kcache, 0, kvb, c->stream));
    CK_RET(&c->err, cudaMemsetAsync(c->vcache, 0, kvb, c->stream));
    CK_RET(&c->err, cudaStreamSynchronize(c->stream));
    return AION_OK;
}

// ---------------------------------------------------------------------------
// Kernel-level API
// ---------------------------------------------------------------------------
struct aion_qmatrix {
    int device;
    DevMatrix m;
};

extern "C" AION_API aion_status aion_qmatrix_upload(const float* scales, const uint8_t* packed, int64_t rows,
                                                    int64_t cols, int32_t device, aion_qmatrix** out) {
    if (!scales || !packed || !out || rows <= 0 || cols <= 0 || cols % 32 || cols > (1 << 30)) {
        set_err(nullptr, "aion_qmatrix_upload: invalid arguments (rows %lld, cols %lld; cols must be a multiple of 32)",
                (long long)rows, (long long)cols);
        return AION_ERR_ARG;
    }
    *out = nullptr;
    CK_RET(nullptr, cudaSetDevice(device));
    aion_qmatrix* q = new aion_qmatrix();
    q->device = device;
    uint8_t* w = nullptr;
    cudaError_t e = cudaMalloc(&w, (size_t)tiled_bytes(rows, (int)cols));
    if (e != cudaSuccess) {
        delete q;
        set_err(nullptr, "cudaMalloc failed: %s", cudaGetErrorString(e));
        return cuda_status(e);
    }
    dev_matrix_init(&q->m, w, rows, (int)cols);
    const size_t sb = (size_t)(rows * cols / 32 * 4), pb = (size_t)(rows * cols / 2);
    uint8_t* stage = nullptr;
    e = cudaMalloc(&stage, sb + pb);
    if (e == cudaSuccess) e = cudaMemcpy(stage, scales, sb, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(stage + sb, packed, pb, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = retile(q->m, (const float*)stage, stage + sb, rows, 0, 0, 0, 0, 0);
    if (e == cudaSuccess) e = fill_pad(q->m, 0);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (stage) cudaFree(stage);
    if (e != cudaSuccess) {
        cudaFree(w);
        delete q;
        set_err(nullptr, "aion_qmatrix_upload: %s", cudaGetErrorString(e));
        return cuda_status(e);
    }
    *out = q;
    return AION_OK;
}

extern "C" AION_API aion_status aion_qmatrix_download(const aion_qmatrix* q, float* scales, uint8_t* packed) {
    if (!q || !scales || !packed) return AION_ERR_ARG;
    CK_RET(nullptr, cudaSetDevice(q->device));
    const long long rows = q->m.rows, cols = q->m.n;
    const size_t sb = (size_t)(rows * cols / 32 * 4), pb = (size_t)(rows * cols / 2);
    uint8_t* stage = nullptr;
    cudaError_t e = cudaMalloc(&stage, sb + pb);
    if (e == cudaSuccess) e = retile(q->m, (const float*)stage, stage + sb, rows, 0, 0, 0, 1, 0);
    if (e == cudaSuccess) e = cudaMemcpy(scales, stage, sb, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(packed, stage + sb, pb, cudaMemcpyDeviceToHost);
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
    cudaFree(q->m.w);
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
    CK_RET(nullptr, raise_smem_limits());
    MatvecArgs a = {};
    a.x = x;
    a.y = y;
    CK_RET(nullptr, launch_matvec(mode, PRO_PLAIN, EPI_STORE, q->m, a, q->device, (cudaStream_t)stream, false));
    return AION_OK;
}

extern "C" AION_API aion_status aion_matvec_w4a16(const aion_qmatrix* w, const float* x_dev, float* y_dev, void* stream) {
    return matvec_api(MODE_W4A16, w, x_dev, y_dev, stream);
}

extern "C" AION_API aion_status aion_matvec_w4a8(const aion_qmatrix* w, const float* x_dev, float* y_dev, void* stream) {
    return matvec_api(MODE_W4A8, w, x_dev, y_dev, stream);
}

extern "C" AION_API aion_status aion_quantize_activations(const float* x, int8_t* qx, float* xs, int64_t n, void* stream) {
    if (!x || !qx || !xs || n <= 0 || n % 32) {
        set_err(nullptr, "aion_quantize_activations: invalid arguments (n must be a positive multiple of 32)");
        return AION_ERR_ARG;
    }
    int grid = (int)((n / 32 + 255) / 256);
    if (grid > 4096) grid = 4096;
    k_quantize_act<<<grid, 256, 0, (cudaStream_t)stream>>>(x, qx, xs, n);
    CK_RET(nullptr, cudaGetLastError());
    return AION_OK;
}
