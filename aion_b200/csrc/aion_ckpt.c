/*
 * Checkpoint tools for the int4 decode path (host C11, part of libaion).
 *
 *  - aion_quantize_buffer: the group-32 symmetric int4 quantizer with the
 *    arithmetic of the reference converter (quantize.c:59-109): scale =
 *    max|w| / 7 (a zero scale becomes 1.0), q = clamp(roundf(w * (1/scale)),
 *    -7, 7) stored as q + 8, the even element in the low nibble.  Element
 *    counts are 64-bit here; the reference converter uses int and cannot
 *    write a 13B-shape file (quantize.c:174-175, 199-220).
 *  - aion_quantize_file: fp32 llama2.c legacy file -> int4 file, tensor order
 *    and "all scales, then all packed bytes" per tensor as quantize.c:192-229.
 *  - aion_synth_checkpoint: writes a seeded random-init checkpoint (matrices
 *    N(0, 0.02), RMSNorm weights 1.0, RoPE tables) directly in the fp32 or
 *    the int4 format, in parallel, without materialising the fp32 model.
 *
 * Build with -ffp-contract=off: the quantizer's products must round as in
 * the reference converter.
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

#include "../../include/aion.h"

#define GROUP 32

AION_API void aion_quantize_buffer(const float* in, uint8_t* packed, float* scales, int64_t n) {
    for (int64_t g = 0; g < n / GROUP; g++) {
        const float* w = in + g * GROUP;
        float amax = 0.0f;
        for (int i = 0; i < GROUP; i++) {
            float a = fabsf(w[i]);
            if (a > amax) amax = a;
        }
        float scale = amax / 7.0f;
        if (scale == 0.0f) scale = 1.0f;
        scales[g] = scale;
        float inv = 1.0f / scale;
        uint8_t* out = packed + g * (GROUP / 2);
        for (int i = 0; i < GROUP; i += 2) {
            int q0 = (int8_t)roundf(w[i] * inv);
            int q1 = (int8_t)roundf(w[i + 1] * inv);
            q0 = q0 < -7 ? -7 : (q0 > 7 ? 7 : q0);
            q1 = q1 < -7 ? -7 : (q1 > 7 ? 7 : q1);
            out[i / 2] = (uint8_t)(((q0 + 8) & 0xF) | (((q1 + 8) & 0xF) << 4));
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Tensor table of the llama2.c legacy layout (src/kernel_simd.c:924-936).   */
/* ------------------------------------------------------------------------ */

typedef struct { int64_t count; int quantized; int kind; } tensor_desc;
enum { K_MATRIX = 0, K_ONES = 1, K_FREQ_RE = 2, K_FREQ_IM = 3 };

static int describe(const int32_t* c, tensor_desc t[13]) {
    int64_t dim = c[0], hid = c[1], L = c[2], nh = c[3], nkv = c[4];
    int64_t vocab = c[5] < 0 ? -(int64_t)c[5] : c[5], seq = c[6];
    if (dim <= 0 || hid <= 0 || L <= 0 || nh <= 0 || nkv <= 0 || vocab <= 0 || seq <= 0) return -1;
    if (dim % nh || nh % nkv || (dim / nh) % 2 || dim % GROUP || hid % GROUP) return -1;
    int64_t kv = dim * nkv / nh, hs = dim / nh;
    tensor_desc d[13] = {
        { vocab * dim, 1, K_MATRIX }, { L * dim, 0, K_ONES },  { L * dim * dim, 1, K_MATRIX },
        { L * dim * kv, 1, K_MATRIX }, { L * dim * kv, 1, K_MATRIX }, { L * dim * dim, 1, K_MATRIX },
        { L * dim, 0, K_ONES }, { L * dim * hid, 1, K_MATRIX }, { L * hid * dim, 1, K_MATRIX },
        { L * dim * hid, 1, K_MATRIX }, { dim, 0, K_ONES },
        { seq * (hs / 2), 0, K_FREQ_RE }, { seq * (hs / 2), 0, K_FREQ_IM },
    };
    memcpy(t, d, sizeof(d));
    return 0;
}

static int64_t tensor_bytes(const tensor_desc* t, int int4) {
    return (int4 && t->quantized) ? (t->count / GROUP) * 4 + t->count / 2 : t->count * 4;
}

AION_API int64_t aion_checkpoint_bytes(const int32_t* cfg7, int int4) {
    tensor_desc t[13];
    if (describe(cfg7, t) != 0) return -1;
    int64_t total = 28;
    for (int i = 0; i < 13; i++) total += tensor_bytes(&t[i], int4);
    return total;
}

/* ------------------------------------------------------------------------ */
/* Seeded normal generator: counter-based, so any chunk is reproducible      */
/* independently of the thread that makes it.  SplitMix64 finaliser (Steele, */
/* Lea, Flood 2014) over (seed, tensor, pair index); Box-Muller on the two    */
/* 53-bit uniforms gives the pair (z0, z1) for elements 2j and 2j+1.          */
/* ------------------------------------------------------------------------ */

static inline uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

static void normal_fill(float* out, uint64_t seed, int tensor, int64_t first, int64_t count, float stddev) {
    const double two_pi = 6.283185307179586476925286766559;
    uint64_t key = mix64(seed * 0x9E3779B97F4A7C15ULL + (uint64_t)(tensor + 1) * 0xD1B54A32D192ED03ULL);
    for (int64_t i = first; i < first + count;) {
        int64_t j = i >> 1;
        uint64_t h1 = mix64(key ^ (uint64_t)j * 0x9E3779B97F4A7C15ULL);
        uint64_t h2 = mix64(h1 + 0x632BE59BD9B4E019ULL);
        double u1 = ((double)(h1 >> 11) + 0.5) * (1.0 / 9007199254740992.0);
        double u2 = (double)(h2 >> 11) * (1.0 / 9007199254740992.0);
        double r = sqrt(-2.0 * log(u1));
        double z0 = r * cos(two_pi * u2), z1 = r * sin(two_pi * u2);
        if ((i & 1) == 0) {
            out[i - first] = (float)(stddev * z0);
            if (i + 1 < first + count) out[i + 1 - first] = (float)(stddev * z1);
            i += 2;
        } else {
            out[i - first] = (float)(stddev * z1);
            i += 1;
        }
    }
}

/* RoPE tables: freq_i = 1 / 10000^(2i/hs) in float, angle = t * freq_i in
 * double, stored as cos / sin in float (the formula of the reference's
 * fp32 oracle, src/reference_oracle.py:18-23). */
static void freq_fill(float* out, int64_t first, int64_t count, int64_t hs, int imag) {
    int64_t half = hs / 2;
    for (int64_t e = first; e < first + count; e++) {
        int64_t t = e / half, i = e % half;
        float f = 1.0f / powf(10000.0f, (float)(2 * i) / (float)hs);
        double ang = (double)t * (double)f;
        out[e - first] = (float)(imag ? sin(ang) : cos(ang));
    }
}

/* ------------------------------------------------------------------------ */
/* Parallel chunked writer.                                                  */
/* ------------------------------------------------------------------------ */

#define CHUNK (1 << 20) /* elements per work item; multiple of GROUP */

typedef struct {
    int fd, int4;
    const tensor_desc* t;
    int64_t base;            /* byte offset of the tensor in the output file */
    int tensor_index;
    uint64_t seed;
    int64_t head_size;
    const float* src;        /* fp32 source for aion_quantize_file, or NULL */
    int64_t nchunks;
    int64_t next;            /* shared work counter */
    pthread_mutex_t mu;
    int failed;
} write_job;

static int pwrite_all(int fd, const void* buf, size_t n, int64_t off) {
    const char* p = (const char*)buf;
    while (n) {
        ssize_t w = pwrite(fd, p, n, (off_t)off);
        if (w <= 0) { if (w < 0 && errno == EINTR) continue; return -1; }
        p += w; n -= (size_t)w; off += w;
    }
    return 0;
}

static void* write_worker(void* arg) {
    write_job* j = (write_job*)arg;
    float* vals = malloc(CHUNK * sizeof(float));
    uint8_t* packed = malloc(CHUNK / 2);
    float* scales = malloc((CHUNK / GROUP) * sizeof(float));
    if (!vals || !packed || !scales) { j->failed = 1; goto out; }
    for (;;) {
        pthread_mutex_lock(&j->mu);
        int64_t c = j->next++;
        pthread_mutex_unlock(&j->mu);
        if (c >= j->nchunks || j->failed) break;
        int64_t e0 = c * CHUNK;
        int64_t cnt = j->t->count - e0 < CHUNK ? j->t->count - e0 : CHUNK;
        const float* v = vals;
        if (j->src) v = j->src + e0;
        else if (j->t->kind == K_MATRIX) normal_fill(vals, j->seed, j->tensor_index, e0, cnt, 0.02f);
        else if (j->t->kind == K_ONES) for (int64_t i = 0; i < cnt; i++) vals[i] = 1.0f;
        else freq_fill(vals, e0, cnt, j->head_size, j->t->kind == K_FREQ_IM);
        int rc;
        if (j->int4 && j->t->quantized) {
            aion_quantize_buffer(v, packed, scales, cnt);
            int64_t sbytes = (j->t->count / GROUP) * 4;
            rc = pwrite_all(j->fd, scales, (size_t)(cnt / GROUP) * 4, j->base + (e0 / GROUP) * 4);
            if (!rc) rc = pwrite_all(j->fd, packed, (size_t)cnt / 2, j->base + sbytes + e0 / 2);
        } else {
            rc = pwrite_all(j->fd, v, (size_t)cnt * 4, j->base + e0 * 4);
        }
        if (rc) { j->failed = 1; break; }
    }
out:
    free(vals); free(packed); free(scales);
    return NULL;
}

static int write_model(const char* path, const int32_t* cfg, int int4, uint64_t seed, const float* src_f32,
                       int threads, char* err, int errlen) {
    tensor_desc t[13];
    if (describe(cfg, t) != 0) { snprintf(err, errlen, "invalid config"); return AION_ERR_SHAPE; }
    for (int i = 0; i < 13; i++)
        if (t[i].quantized && t[i].count % GROUP) { snprintf(err, errlen, "tensor %d not a multiple of 32", i); return AION_ERR_SHAPE; }
    int fd = open(path, O_WRONLY | O_CREAT | O_TRUNC, 0644);
    if (fd < 0) { snprintf(err, errlen, "open %s: %s", path, strerror(errno)); return AION_ERR_IO; }
    int64_t total = aion_checkpoint_bytes(cfg, int4);
    int32_t hdr[7];
    memcpy(hdr, cfg, sizeof(hdr));
    if (ftruncate(fd, (off_t)total) != 0 || pwrite_all(fd, hdr, 28, 0) != 0) {
        snprintf(err, errlen, "write %s: %s", path, strerror(errno)); close(fd); return AION_ERR_IO;
    }
    if (threads < 1) threads = (int)sysconf(_SC_NPROCESSORS_ONLN);
    if (threads < 1) threads = 1;
    if (threads > 128) threads = 128;
    int64_t off = 28;
    const float* src = src_f32;
    for (int i = 0; i < 13; i++) {
        write_job j;
        memset(&j, 0, sizeof(j));
        j.fd = fd; j.int4 = int4; j.t = &t[i]; j.base = off; j.tensor_index = i; j.seed = seed;
        j.head_size = cfg[0] / cfg[3]; j.src = src;
        j.nchunks = (t[i].count + CHUNK - 1) / CHUNK;
        pthread_mutex_init(&j.mu, NULL);
        pthread_t th[128];
        int nt = threads < j.nchunks ? threads : (int)j.nchunks;
        for (int k = 1; k < nt; k++) pthread_create(&th[k], NULL, write_worker, &j);
        write_worker(&j);
        for (int k = 1; k < nt; k++) pthread_join(th[k], NULL);
        pthread_mutex_destroy(&j.mu);
        if (j.failed) { snprintf(err, errlen, "write failed at tensor %d", i); close(fd); return AION_ERR_IO; }
        off += tensor_bytes(&t[i], int4);
        if (src) src += t[i].count;
    }
    if (close(fd) != 0) { snprintf(err, errlen, "close: %s", strerror(errno)); return AION_ERR_IO; }
    return AION_OK;
}

AION_API int aion_synth_checkpoint(const char* path, const int32_t* cfg7, uint64_t seed, int int4, int threads,
                                   char* err, int errlen) {
    return write_model(path, cfg7, int4, seed, NULL, threads, err, errlen);
}

AION_API int aion_quantize_file(const char* in_path, const char* out_path, int threads, char* err, int errlen) {
    int fd = open(in_path, O_RDONLY);
    if (fd < 0) { snprintf(err, errlen, "open %s: %s", in_path, strerror(errno)); return AION_ERR_IO; }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 28) { close(fd); snprintf(err, errlen, "short file"); return AION_ERR_FORMAT; }
    void* map = mmap(NULL, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) { snprintf(err, errlen, "mmap failed"); return AION_ERR_IO; }
    int32_t cfg[7];
    memcpy(cfg, map, 28);
    int32_t cfg_abs[7];
    memcpy(cfg_abs, cfg, 28);
    if (cfg_abs[5] < 0) cfg_abs[5] = -cfg_abs[5];
    int64_t want = aion_checkpoint_bytes(cfg_abs, 0);
    int rc;
    if (want < 0 || want > st.st_size) {
        snprintf(err, errlen, "fp32 file too short for its header (%lld < %lld)", (long long)st.st_size, (long long)want);
        rc = AION_ERR_FORMAT;
    } else {
        /* The header is copied as read (sign of vocab kept), as quantize.c:141. */
        tensor_desc t[13];
        describe(cfg_abs, t);
        rc = write_model(out_path, cfg_abs, 1, 0, (const float*)((const char*)map + 28), threads, err, errlen);
        if (rc == AION_OK && cfg[5] < 0) {
            int ofd = open(out_path, O_WRONLY);
            if (ofd < 0 || pwrite_all(ofd, cfg, 28, 0) != 0) rc = AION_ERR_IO;
            if (ofd >= 0) close(ofd);
        }
    }
    munmap(map, (size_t)st.st_size);
    return rc;
}
