/*
 * AION int4 decode oracle -- TEST INFRASTRUCTURE, not part of the product.
 *
 * A plain C11 restatement of the reference's int4 Llama-2 decode path, used
 * only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg as
 * the checker.  Every function follows the reference's operation order so
 * that it reproduces the reference bit for bit where the reference is
 * deterministic C (pinned against the reference binaries built by
 * oracle/Makefile and against tests/golden/).  Differences from the
 * reference are deliberate and listed here:
 *   - all element offsets use size_t / int64 (the reference overflows int at
 *     the 13B shape: quantize.c:174-175, src/kernel_simd.c:1132-1144);
 *   - the row loop of a matvec may be split across pthreads; each row is
 *     still computed by one thread in the reference order, so results do not
 *     depend on the thread count (as in src/kernel_simd.c:660-674);
 *   - the W4A8 forward wires quantize_activations + matmul_w4a8 into every
 *     matvec, which the reference CLI never does (src/kernel_simd.c:1193).
 *
 * Citations are to files of the reference project (farukalpay/AION).
 */
#define _GNU_SOURCE
#include <errno.h>
#include <fcntl.h>
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#define ORC_GROUP 32
#define ORC_EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------------- */
/* Threading: rows of a matvec are split into contiguous chunks.              */
/* ------------------------------------------------------------------------- */

static int g_threads = 1;

ORC_EXPORT void orc_set_threads(int n) { g_threads = n < 1 ? 1 : (n > 256 ? 256 : n); }
ORC_EXPORT int orc_get_threads(void) { return g_threads; }

typedef void (*orc_rows_fn)(void* arg, int64_t r0, int64_t r1);
typedef struct { orc_rows_fn fn; void* arg; int64_t r0, r1; } orc_job;

static void* orc_job_main(void* p) {
    orc_job* j = (orc_job*)p;
    if (j->r0 < j->r1) j->fn(j->arg, j->r0, j->r1);
    return NULL;
}

static void orc_parallel_rows(orc_rows_fn fn, void* arg, int64_t d) {
    int t = g_threads;
    if (t <= 1 || d < 64) { fn(arg, 0, d); return; }
    if (t > d) t = (int)d;
    pthread_t th[256];
    orc_job jobs[256];
    int64_t chunk = (d + t - 1) / t;
    for (int i = 0; i < t; i++) {
        jobs[i].fn = fn; jobs[i].arg = arg;
        jobs[i].r0 = (int64_t)i * chunk;
        jobs[i].r1 = jobs[i].r0 + chunk > d ? d : jobs[i].r0 + chunk;
    }
    for (int i = 1; i < t; i++) pthread_create(&th[i], NULL, orc_job_main, &jobs[i]);
    orc_job_main(&jobs[0]);
    for (int i = 1; i < t; i++) pthread_join(th[i], NULL);
}

/* ------------------------------------------------------------------------- */
/* C1: group-32 symmetric int4 quantizer (quantize.c:59-109).                 */
/* ------------------------------------------------------------------------- */

ORC_EXPORT void orc_quantize_buffer(const float* in, uint8_t* packed, float* scales, int64_t n) {
    int64_t ng = n / ORC_GROUP;
    for (int64_t g = 0; g < ng; g++) {
        const float* w = in + g * ORC_GROUP;
        float amax = 0.0f;
        for (int i = 0; i < ORC_GROUP; i++) {
            float a = fabsf(w[i]);
            if (a > amax) amax = a;
        }
        float scale = amax / 7.0f;
        if (scale == 0.0f) scale = 1.0f;
        scales[g] = scale;
        float inv = 1.0f / scale;
        for (int i = 0; i < ORC_GROUP; i += 2) {
            int8_t q0 = (int8_t)roundf(w[i] * inv);
            int8_t q1 = (int8_t)roundf(w[i + 1] * inv);
            if (q0 < -7) q0 = -7;
            if (q0 > 7) q0 = 7;
            if (q1 < -7) q1 = -7;
            if (q1 > 7) q1 = 7;
            uint8_t lo = (uint8_t)(q0 + 8), hi = (uint8_t)(q1 + 8);
            packed[(g * ORC_GROUP + i) / 2] = (uint8_t)((lo & 0xF) | ((hi & 0xF) << 4));
        }
    }
}

/* Dequantize one contiguous span (the embedding-row lookup of
 * src/kernel_simd.c:1032-1040): x[i] = (int8)(nibble - 8) * scale[i/32]. */
ORC_EXPORT void orc_dequant(float* out, const float* scales, const uint8_t* packed, int64_t n) {
    for (int64_t i = 0; i < n; i += 2) {
        uint8_t b = packed[i / 2];
        float s = scales[i / 32];
        int8_t v0 = (int8_t)((b & 0xF) - 8);
        int8_t v1 = (int8_t)((b >> 4) - 8);
        out[i] = v0 * s;
        out[i + 1] = v1 * s;
    }
}

/* ------------------------------------------------------------------------- */
/* C4: W4A16 matvec, scalar order (src/kernel_simd.c:341-363).                */
/* y[i] = sum over the row in element order of (q * scale) * x, one rounding   */
/* per multiply and per add (built with -ffp-contract=off).                   */
/* ------------------------------------------------------------------------- */

/* C10: the fp32 matvec of the reference's fp32 path, matmul_block_4x4
 * (src/kernel_simd.c:547-620) as run on one thread (rows 0.. in blocks of
 * 4): rows of a full block keep four lane sums, lane j adding w[k] * x[k]
 * for k = j mod 4 with a fused multiply-add (FMLA) over the 16-column
 * blocks, then (lane0 + lane1) + (lane2 + lane3) (FADDP), then the columns
 * past the last full 16 one by one; rows after the last full block of 4
 * sum w[k] * x[k] in order with separate multiply and add. */
typedef struct { float* y; const float* x; const float* w; int64_t n, d; } orc_f32_args;

static void orc_f32_rows(void* p, int64_t r0, int64_t r1) {
    orc_f32_args* a = (orc_f32_args*)p;
    const int64_t n = a->n, n16 = n / 16 * 16, d4 = a->d / 4 * 4;
    for (int64_t i = r0; i < r1; i++) {
        const float* w = a->w + i * n;
        float val;
        if (i < d4) {
            float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (int64_t k = 0; k < n16; k += 4)
                for (int j = 0; j < 4; j++) acc[j] = fmaf(w[k + j], a->x[k + j], acc[j]);
            val = (acc[0] + acc[1]) + (acc[2] + acc[3]);
            for (int64_t k = n16; k < n; k++) val += w[k] * a->x[k];
        } else {
            val = 0.0f;
            for (int64_t k = 0; k < n; k++) val += w[k] * a->x[k];
        }
        a->y[i] = val;
    }
}

ORC_EXPORT void orc_matvec_f32(float* y, const float* x, const float* w, int64_t n, int64_t d) {
    orc_f32_args a = {y, x, w, n, d};
    orc_parallel_rows(orc_f32_rows, &a, d);
}

typedef struct { float* y; const float* x; const float* scales; const uint8_t* packed; int64_t n; } orc_mv_args;

static void orc_matvec_rows(void* p, int64_t r0, int64_t r1) {
    orc_mv_args* a = (orc_mv_args*)p;
    int64_t n = a->n;
    for (int64_t i = r0; i < r1; i++) {
        float val = 0.0f;
        const uint8_t* rp = a->packed + i * (n / 2);
        const float* rs = a->scales + i * (n / 32);
        for (int64_t j = 0; j < n; j += 32) {
            float scale = rs[j / 32];
            for (int k = 0; k < 32; k += 2) {
                uint8_t b = rp[(j + k) / 2];
                int8_t w0 = (int8_t)((b & 0xF) - 8);
                int8_t w1 = (int8_t)((b >> 4) - 8);
                val += w0 * scale * a->x[j + k];
                val += w1 * scale * a->x[j + k + 1];
            }
        }
        a->y[i] = val;
    }
}

ORC_EXPORT void orc_matvec_w4a16(float* y, const float* x, const float* scales, const uint8_t* packed,
                                 int64_t n, int64_t d) {
    orc_mv_args a = { y, x, scales, packed, n };
    orc_parallel_rows(orc_matvec_rows, &a, d);
}

/* ------------------------------------------------------------------------- */
/* C5: W4A8 (src/kernel_simd.c:186-227 and :244-337).                        */
/* ------------------------------------------------------------------------- */

ORC_EXPORT void orc_quantize_activations(int8_t* qx, float* xs, const float* x, int64_t n) {
    for (int64_t i = 0; i < n; i += 32) {
        float amax = 0.0f;
        for (int k = 0; k < 32; k++) {
            float a = fabsf(x[i + k]);
            if (a > amax) amax = a;
        }
        float scale = (amax > 1e-9f) ? (127.0f / amax) : 1.0f;
        xs[i / 32] = (amax > 1e-9f) ? (amax / 127.0f) : 1.0f;
        for (int k = 0; k < 32; k++) {
            float qf = x[i + k] * scale;
            float r = roundf(qf);             /* ties away from zero */
            int32_t qi = (int32_t)r;
            qx[i + k] = (int8_t)qi;
        }
    }
}

typedef struct { float* y; const int8_t* qx; const float* xs; const float* scales; const uint8_t* packed; int64_t n; } orc_w8_args;

static void orc_w4a8_rows(void* p, int64_t r0, int64_t r1) {
    orc_w8_args* a = (orc_w8_args*)p;
    int64_t n = a->n;
    for (int64_t i = r0; i < r1; i++) {
        float row = 0.0f;
        const uint8_t* rp = a->packed + i * (n / 2);
        const float* rs = a->scales + i * (n / 32);
        for (int64_t j = 0; j < n; j += 32) {
            float combined = rs[j / 32] * a->xs[j / 32];
            int32_t acc = 0;
            for (int k = 0; k < 32; k += 2) {
                uint8_t b = rp[(j + k) / 2];
                acc += ((int32_t)(b & 0xF) - 8) * (int32_t)a->qx[j + k];
                acc += ((int32_t)(b >> 4) - 8) * (int32_t)a->qx[j + k + 1];
            }
            row += (float)acc * combined;
        }
        a->y[i] = row;
    }
}

ORC_EXPORT void orc_matvec_w4a8(float* y, const int8_t* qx, const float* xs, const float* scales,
                                const uint8_t* packed, int64_t n, int64_t d) {
    orc_w8_args a = { y, qx, xs, scales, packed, n };
    orc_parallel_rows(orc_w4a8_rows, &a, d);
}

/* Integer dot of every group of a matrix with quantized activations:
 * out[row * (n/32) + g] = sum_k (nib - 8) * qx (the exact int32 group dot of
 * src/kernel_simd.c:319-331). */
ORC_EXPORT void orc_group_dots(int32_t* out, const int8_t* qx, const uint8_t* packed, int64_t n, int64_t d) {
    for (int64_t i = 0; i < d; i++)
        for (int64_t j = 0; j < n; j += 32) {
            int32_t acc = 0;
            for (int k = 0; k < 32; k += 2) {
                uint8_t b = packed[i * (n / 2) + (j + k) / 2];
                acc += ((int32_t)(b & 0xF) - 8) * (int32_t)qx[j + k];
                acc += ((int32_t)(b >> 4) - 8) * (int32_t)qx[j + k + 1];
            }
            out[i * (n / 32) + j / 32] = acc;
        }
}

/* ------------------------------------------------------------------------- */
/* C6: per-token elementwise ops (src/kernel_simd.c:793-849).                 */
/* ------------------------------------------------------------------------- */

/* rmsnorm with four lane partial sums, pairwise lane reduction, scalar tail. */
ORC_EXPORT void orc_rmsnorm(float* o, const float* x, const float* w, int64_t size) {
    float lane[4] = { 0.0f, 0.0f, 0.0f, 0.0f };
    int64_t i = 0;
    for (; i <= size - 4; i += 4)
        for (int l = 0; l < 4; l++) { float p = x[i + l] * x[i + l]; lane[l] = lane[l] + p; }
    float lo = lane[0] + lane[1], hi = lane[2] + lane[3];
    float sum = lo + hi;
    for (; i < size; i++) sum += x[i] * x[i];
    sum /= (float)size;
    float ss = 1.0f / sqrtf(sum + 1e-5f);
    for (i = 0; i < size; i++) { float t = x[i] * ss; o[i] = t * w[i]; }
}

ORC_EXPORT void orc_softmax(float* x, int64_t size) {
    float m = x[0];
    for (int64_t i = 1; i < size; i++) if (x[i] > m) m = x[i];
    float sum = 0.0f;
    for (int64_t i = 0; i < size; i++) { x[i] = expf(x[i] - m); sum += x[i]; }
    float scale = 1.0f / sum;
    for (int64_t i = 0; i < size; i++) x[i] *= scale;
}

/* SwiGLU: the four-wide body evaluates v / (1 + e^-v); the tail evaluates
 * v * (1 / (1 + e^-v)); the two round differently (src/kernel_simd.c:828-849). */
ORC_EXPORT void orc_swiglu(float* hb, const float* hb2, int64_t size) {
    int64_t i = 0;
    for (; i <= size - 4; i += 4)
        for (int l = 0; l < 4; l++) {
            float v = hb[i + l];
            float s = v / (1.0f + expf(-v));
            hb[i + l] = s * hb2[i + l];
        }
    for (; i < size; i++) {
        float v = hb[i] * (1.0f / (1.0f + expf(-hb[i])));
        hb[i] = v * hb2[i];
    }
}

/* ------------------------------------------------------------------------- */
/* Checkpoint (C1 format, read by src/kernel_simd.c:941-989).                 */
/* ------------------------------------------------------------------------- */

typedef struct { int32_t dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len; } orc_config;
/* A weight tensor: int4 (scales + packed) or, for fp32 files, plain floats. */
typedef struct { const float* scales; const uint8_t* packed; const float* f; } orc_qw;

typedef struct orc_model {
    orc_config c;
    int64_t kv_dim, head_size;
    void* map; size_t map_size;
    orc_qw emb, wq, wk, wv, wo, w1, w2, w3;
    const float *rms_att, *rms_ffn, *rms_final, *freq_re, *freq_im;
    /* run state */
    float *x, *xb, *xb2, *hb, *hb2, *q, *k, *v, *att, *logits, *kcache, *vcache;
    int8_t* qx; float* xs;
    int f32;                       /* fp32 llama2.c file (the reference's fp32 path) */
} orc_model;

static orc_qw qw_at(orc_qw w, int64_t elems) {
    orc_qw r = { NULL, NULL, NULL };
    if (w.f) r.f = w.f + elems;
    else { r.scales = w.scales + elems / 32; r.packed = w.packed + elems / 2; }
    return r;
}

/* Expected byte size of an fp32 llama2.c file (src/kernel_simd.c:906-936),
 * plus the separate classifier that a negative vocab_size announces (which
 * the reference never reads). */
ORC_EXPORT int64_t orc_f32_file_size(const int32_t* cfg7) {
    int64_t dim = cfg7[0], hid = cfg7[1], L = cfg7[2], nh = cfg7[3], nkv = cfg7[4];
    int64_t vocab = cfg7[5] < 0 ? -(int64_t)cfg7[5] : cfg7[5], seq = cfg7[6];
    if (dim <= 0 || hid <= 0 || L <= 0 || nh <= 0 || nkv <= 0 || vocab <= 0 || seq <= 0) return -1;
    int64_t hs = dim / nh, kv = dim * nkv / nh;
    int64_t f = vocab * dim + L * dim + L * dim * dim + 2 * L * dim * kv + L * dim * dim + L * dim + 3 * L * dim * hid +
                dim + 2 * seq * (hs / 2);
    if (cfg7[5] < 0) f += vocab * dim;
    return 28 + 4 * f;
}

/* Expected byte size of an int4 file for a header (size_t arithmetic). */
ORC_EXPORT int64_t orc_int4_file_size(const int32_t* cfg7) {
    int64_t dim = cfg7[0], hid = cfg7[1], L = cfg7[2], nh = cfg7[3], nkv = cfg7[4];
    int64_t vocab = cfg7[5] < 0 ? -(int64_t)cfg7[5] : cfg7[5], seq = cfg7[6];
    if (dim <= 0 || hid <= 0 || L <= 0 || nh <= 0 || nkv <= 0 || vocab <= 0 || seq <= 0) return -1;
    int64_t hs = dim / nh, kv = dim * nkv / nh;
    int64_t q = 0;
#define QB(cnt) (((cnt) / 32) * 4 + (cnt) / 2)
    q += QB(vocab * dim) + L * dim * 4 + QB(L * dim * dim) + 2 * QB(L * dim * kv) + QB(L * dim * dim);
    q += L * dim * 4 + 3 * QB(L * dim * hid) + dim * 4 + 2 * seq * (hs / 2) * 4;
#undef QB
    return 28 + q;
}

ORC_EXPORT void orc_close(orc_model* m) {
    if (!m) return;
    if (m->map) munmap(m->map, m->map_size);
    free(m->x); free(m->xb); free(m->xb2); free(m->hb); free(m->hb2); free(m->q); free(m->k); free(m->v);
    free(m->att); free(m->logits); free(m->kcache); free(m->vcache); free(m->qx); free(m->xs);
    free(m);
}

ORC_EXPORT orc_model* orc_open(const char* path, char* err, int errlen) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) { snprintf(err, errlen, "open %s: %s", path, strerror(errno)); return NULL; }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 28) { snprintf(err, errlen, "short file"); close(fd); return NULL; }
    void* map = mmap(NULL, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) { snprintf(err, errlen, "mmap failed"); return NULL; }
    orc_model* m = calloc(1, sizeof(*m));
    m->map = map; m->map_size = (size_t)st.st_size;
    memcpy(&m->c, map, 28);
    int64_t want = orc_int4_file_size(&m->c.dim), want_f = orc_f32_file_size(&m->c.dim);
    if (m->c.vocab_size < 0) m->c.vocab_size = -m->c.vocab_size;
    if (want_f == (int64_t)st.st_size && want != want_f) m->f32 = 1;
    else if (want < 0 || want != (int64_t)st.st_size) {
        snprintf(err, errlen, "size mismatch: header implies %lld (int4) or %lld (fp32) bytes, file has %lld",
                 (long long)want, (long long)want_f, (long long)st.st_size);
        orc_close(m); return NULL;
    }
    int64_t dim = m->c.dim, hid = m->c.hidden_dim, L = m->c.n_layers, vocab = m->c.vocab_size, seq = m->c.seq_len;
    m->head_size = dim / m->c.n_heads;
    m->kv_dim = dim * m->c.n_kv_heads / m->c.n_heads;
    const char* p = (const char*)map + 28;
#define MAPQ(w, cnt) do { int64_t n_ = (cnt); if (m->f32) { (w).f = (const float*)p; p += n_ * 4; } else { (w).scales = (const float*)p; p += (n_ / 32) * 4; (w).packed = (const uint8_t*)p; p += n_ / 2; } } while (0)
#define MAPF(w, cnt) do { (w) = (const float*)p; p += (int64_t)(cnt) * 4; } while (0)
    MAPQ(m->emb, vocab * dim);
    MAPF(m->rms_att, L * dim);
    MAPQ(m->wq, L * dim * dim);
    MAPQ(m->wk, L * dim * m->kv_dim);
    MAPQ(m->wv, L * dim * m->kv_dim);
    MAPQ(m->wo, L * dim * dim);
    MAPF(m->rms_ffn, L * dim);
    MAPQ(m->w1, L * dim * hid);
    MAPQ(m->w2, L * hid * dim);
    MAPQ(m->w3, L * dim * hid);
    MAPF(m->rms_final, dim);
    MAPF(m->freq_re, seq * (m->head_size / 2));
    MAPF(m->freq_im, seq * (m->head_size / 2));
#undef MAPQ
#undef MAPF
    int64_t big = dim > hid ? dim : hid;
    m->x = calloc(dim, 4); m->xb = calloc(dim, 4); m->xb2 = calloc(dim, 4);
    m->hb = calloc(hid, 4); m->hb2 = calloc(hid, 4); m->q = calloc(dim, 4);
    m->k = calloc(m->kv_dim, 4); m->v = calloc(m->kv_dim, 4);
    m->att = calloc((size_t)m->c.n_heads * seq, 4); m->logits = calloc(vocab, 4);
    m->kcache = calloc((size_t)(L * seq * m->kv_dim), 4); m->vcache = calloc((size_t)(L * seq * m->kv_dim), 4);
    m->qx = calloc(big, 1); m->xs = calloc(big / 32 + 1, 4);
    if (!m->x || !m->kcache || !m->vcache || !m->att || !m->qx) { snprintf(err, errlen, "out of memory"); orc_close(m); return NULL; }
    return m;
}

ORC_EXPORT void orc_config_of(const orc_model* m, int32_t* out7) { memcpy(out7, &m->c, 28); }
ORC_EXPORT float* orc_logits(orc_model* m) { return m->logits; }

ORC_EXPORT void orc_reset(orc_model* m) {
    size_t kvn = (size_t)m->c.n_layers * m->c.seq_len * m->kv_dim;
    memset(m->kcache, 0, kvn * 4);
    memset(m->vcache, 0, kvn * 4);
}

/* Raw views of a stacked tensor, for tests that slice one layer.
 * which: 0 emb, 1 wq, 2 wk, 3 wv, 4 wo, 5 w1, 6 w2, 7 w3. */
ORC_EXPORT int orc_tensor(const orc_model* m, int which, const float** scales, const uint8_t** packed) {
    const orc_qw* t[8] = { &m->emb, &m->wq, &m->wk, &m->wv, &m->wo, &m->w1, &m->w2, &m->w3 };
    if (which < 0 || which > 7) return -1;
    *scales = t[which]->scales; *packed = t[which]->packed;
    return 0;
}

ORC_EXPORT const float* orc_fp32_tensor(const orc_model* m, int which) {
    switch (which) {
    case 0: return m->rms_att; case 1: return m->rms_ffn; case 2: return m->rms_final;
    case 3: return m->freq_re; case 4: return m->freq_im; default: return NULL;
    }
}

/* One matvec of the forward in the selected mode: W4A16 uses the scalar
 * int4 kernel; W4A8 quantizes the input per 32 and runs the integer kernel. */
static void orc_mm(orc_model* m, int mode, float* y, const float* x, orc_qw w, int64_t n, int64_t d) {
    if (w.f) {
        orc_matvec_f32(y, x, w.f, n, d);
    } else if (mode == 1) {
        orc_quantize_activations(m->qx, m->xs, x, n);
        orc_matvec_w4a8(y, m->qx, m->xs, w.scales, w.packed, n, d);
    } else {
        orc_matvec_w4a16(y, x, w.scales, w.packed, n, d);
    }
}

/* C7: one token through the model (src/kernel_simd.c:1014-1169, int4 branch). */
ORC_EXPORT int orc_forward(orc_model* m, int token, int pos, int mode) {
    const orc_config* p = &m->c;
    if (token < 0 || token >= p->vocab_size || pos < 0 || pos >= p->seq_len) return -1;
    int64_t dim = p->dim, kv_dim = m->kv_dim, hid = p->hidden_dim, hs = m->head_size, seq = p->seq_len;
    int64_t kv_mul = p->n_heads / p->n_kv_heads;
    float* x = m->x;

    orc_qw row = qw_at(m->emb, (int64_t)token * dim);
    if (row.f) memcpy(x, row.f, (size_t)dim * 4);   /* fp32 path: src/kernel_simd.c:1041-1043 */
    else orc_dequant(x, row.scales, row.packed, dim);

    for (int64_t l = 0; l < p->n_layers; l++) {
        orc_rmsnorm(m->xb, x, m->rms_att + l * dim, dim);
        /* W4A8 quantizes xb once per matvec; the result is identical for the
         * three projections because they share the input. */
        orc_mm(m, mode, m->q, m->xb, qw_at(m->wq, l * dim * dim), dim, dim);
        orc_mm(m, mode, m->k, m->xb, qw_at(m->wk, l * dim * kv_dim), dim, kv_dim);
        orc_mm(m, mode, m->v, m->xb, qw_at(m->wv, l * dim * kv_dim), dim, kv_dim);

        for (int64_t i = 0; i < dim; i += 2) {
            int64_t hd = i % hs;
            float fr = m->freq_re[pos * (hs / 2) + hd / 2], fi = m->freq_im[pos * (hs / 2) + hd / 2];
            float q0 = m->q[i], q1 = m->q[i + 1];
            m->q[i] = q0 * fr - q1 * fi;
            m->q[i + 1] = q0 * fi + q1 * fr;
        }
        for (int64_t i = 0; i < kv_dim; i += 2) {
            int64_t hd = i % hs;
            float fr = m->freq_re[pos * (hs / 2) + hd / 2], fi = m->freq_im[pos * (hs / 2) + hd / 2];
            float k0 = m->k[i], k1 = m->k[i + 1];
            m->k[i] = k0 * fr - k1 * fi;
            m->k[i + 1] = k0 * fi + k1 * fr;
        }
        int64_t loff = l * seq * kv_dim;
        memcpy(m->kcache + loff + pos * kv_dim, m->k, kv_dim * 4);
        memcpy(m->vcache + loff + pos * kv_dim, m->v, kv_dim * 4);

        for (int64_t h = 0; h < p->n_heads; h++) {
            const float* q = m->q + h * hs;
            float* att = m->att + h * seq;
            for (int64_t t = 0; t <= pos; t++) {
                const float* k = m->kcache + loff + t * kv_dim + (h / kv_mul) * hs;
                float score = 0.0f;
                for (int64_t j = 0; j < hs; j++) score += q[j] * k[j];
                score /= sqrtf((float)hs);
                att[t] = score;
            }
            orc_softmax(att, pos + 1);
            float* xb = m->xb + h * hs;
            memset(xb, 0, hs * 4);
            for (int64_t t = 0; t <= pos; t++) {
                const float* v = m->vcache + loff + t * kv_dim + (h / kv_mul) * hs;
                float a = att[t];
                for (int64_t j = 0; j < hs; j++) xb[j] += a * v[j];
            }
        }
        orc_mm(m, mode, m->xb2, m->xb, qw_at(m->wo, l * dim * dim), dim, dim);
        for (int64_t i = 0; i < dim; i++) x[i] += m->xb2[i];

        orc_rmsnorm(m->xb, x, m->rms_ffn + l * dim, dim);
        orc_mm(m, mode, m->hb, m->xb, qw_at(m->w1, l * dim * hid), dim, hid);
        orc_mm(m, mode, m->hb2, m->xb, qw_at(m->w3, l * dim * hid), dim, hid);
        orc_swiglu(m->hb, m->hb2, hid);
        orc_mm(m, mode, m->xb, m->hb, qw_at(m->w2, l * hid * dim), hid, dim);
        for (int64_t i = 0; i < dim; i++) x[i] += m->xb[i];
    }
    orc_rmsnorm(x, x, m->rms_final, dim);
    orc_mm(m, mode, m->logits, x, m->emb, dim, p->vocab_size);
    return 0;
}

/* Greedy pick: first index of the maximum, strict '>' from -1e9
 * (src/kernel_simd.c:1236-1243).  *gap receives top1 - top2. */
ORC_EXPORT int orc_argmax(const float* logits, int64_t n, float* gap) {
    float best = -1e9f, second = -INFINITY;
    int idx = 0;
    for (int64_t i = 0; i < n; i++) {
        if (logits[i] > best) { second = best; best = logits[i]; idx = (int)i; }
        else if (logits[i] > second) second = logits[i];
    }
    if (gap) *gap = best - second;
    return idx;
}

/* C9: greedy generate from `bos` for `steps` positions (src/kernel_simd.c:
 * 1223-1250).  tokens[pos] receives the INPUT token of step pos, as the
 * reference prints it; gaps/logits_dump are optional per-step outputs. */
ORC_EXPORT int orc_generate(orc_model* m, int bos, int steps, int mode, int32_t* tokens, float* gaps,
                            float* logits_dump) {
    int token = bos;
    orc_reset(m);
    for (int pos = 0; pos < steps; pos++) {
        if (orc_forward(m, token, pos, mode) != 0) return -1;
        float gap = 0.0f;
        int next = orc_argmax(m->logits, m->c.vocab_size, &gap);
        tokens[pos] = token;
        if (gaps) gaps[pos] = gap;
        if (logits_dump) memcpy(logits_dump + (size_t)pos * m->c.vocab_size, m->logits, (size_t)m->c.vocab_size * 4);
        token = next;
    }
    return token;
}
