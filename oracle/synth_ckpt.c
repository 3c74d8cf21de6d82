/*
 * synth_ckpt -- seeded random-init int4 checkpoint writer for the reference
 * arm of bench.py -- TEST INFRASTRUCTURE ONLY.
 *
 *   synth_ckpt <out.int4> <dim> <hidden> <layers> <heads> <kv_heads> <vocab> <seq_len> <seed> [threads]
 *
 * Writes the llama2.c legacy layout in the quantize.c int4 format (per
 * tensor: all fp32 group scales, then all packed bytes; tensor order as
 * quantize.c:192-229) without materialising the fp32 model.  The int4
 * conversion is the reference's own quantize_buffer (quantize.c:59-109),
 * compiled in from the reference source (#included with its main()
 * renamed, as ref_quant_harness.c does), so the reference arm times the
 * reference on a file the reference's quantizer wrote and loads nothing of
 * the product library.
 *
 * Values: matrices N(0, 0.02) from a counter-based generator (SplitMix64
 * finaliser over (seed, tensor, pair index), Box-Muller on two 53-bit
 * uniforms), RMSNorm weights 1.0, RoPE tables cos / sin of t * 10000^(-2i/hs)
 * (the reference fp32 oracle's formula, src/reference_oracle.py:18-23).
 * The same generator feeds aion_synth_checkpoint; tests check that both
 * write identical bytes.  Build with -ffp-contract=off.
 */
#define main aion_reference_quantize_main
#include "quantize.c"
#undef main

#include <errno.h>
#include <fcntl.h>
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#define SYN_GROUP 32
#define SYN_CHUNK (1 << 20)

typedef struct {
    int64_t count;
    int quantized, kind;   /* kind: 0 matrix, 1 ones, 2 freq cos, 3 freq sin */
} syn_tensor;

static uint64_t syn_mix(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

/* Elements [first, first + count) of matrix `tensor`: element 2j and 2j + 1
 * are the Box-Muller pair of index j. */
static void syn_normal(float* out, uint64_t seed, int tensor, int64_t first, int64_t count) {
    const double two_pi = 6.283185307179586476925286766559;
    const float stddev = 0.02f;
    const uint64_t key = syn_mix(seed * 0x9E3779B97F4A7C15ULL + (uint64_t)(tensor + 1) * 0xD1B54A32D192ED03ULL);
    int64_t i = first;
    while (i < first + count) {
        const int64_t j = i >> 1;
        const uint64_t h1 = syn_mix(key ^ (uint64_t)j * 0x9E3779B97F4A7C15ULL);
        const uint64_t h2 = syn_mix(h1 + 0x632BE59BD9B4E019ULL);
        const double u1 = ((double)(h1 >> 11) + 0.5) * (1.0 / 9007199254740992.0);
        const double u2 = (double)(h2 >> 11) * (1.0 / 9007199254740992.0);
        const double r = sqrt(-2.0 * log(u1));
        const double z0 = r * cos(two_pi * u2), z1 = r * sin(two_pi * u2);
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

static void syn_freq(float* out, int64_t first, int64_t count, int64_t hs, int imag) {
    const int64_t half = hs / 2;
    for (int64_t e = first; e < first + count; e++) {
        const int64_t t = e / half, i = e % half;
        const float f = 1.0f / powf(10000.0f, (float)(2 * i) / (float)hs);
        const double ang = (double)t * (double)f;
        out[e - first] = (float)(imag ? sin(ang) : cos(ang));
    }
}

static int syn_pwrite(int fd, const void* buf, size_t n, int64_t off) {
    const char* p = (const char*)buf;
    while (n) {
        const ssize_t w = pwrite(fd, p, n, (off_t)off);
        if (w <= 0) {
            if (w < 0 && errno == EINTR) continue;
            return -1;
        }
        p += w;
        n -= (size_t)w;
        off += w;
    }
    return 0;
}

typedef struct {
    int fd, tensor;
    const syn_tensor* t;
    int64_t base, hs, nchunks, next;
    uint64_t seed;
    pthread_mutex_t mu;
    int failed;
} syn_job;

static void* syn_worker(void* arg) {
    syn_job* j = (syn_job*)arg;
    float* vals = malloc(SYN_CHUNK * sizeof(float));
    uint8_t* packed = malloc(SYN_CHUNK / 2);
    float* scales = malloc((SYN_CHUNK / SYN_GROUP) * sizeof(float));
    if (!vals || !packed || !scales) j->failed = 1;
    while (!j->failed) {
        pthread_mutex_lock(&j->mu);
        const int64_t c = j->next++;
        pthread_mutex_unlock(&j->mu);
        if (c >= j->nchunks) break;
        const int64_t e0 = c * SYN_CHUNK;
        const int64_t cnt = j->t->count - e0 < SYN_CHUNK ? j->t->count - e0 : SYN_CHUNK;
        if (j->t->kind == 0) syn_normal(vals, j->seed, j->tensor, e0, cnt);
        else if (j->t->kind == 1) for (int64_t i = 0; i < cnt; i++) vals[i] = 1.0f;
        else syn_freq(vals, e0, cnt, j->hs, j->t->kind == 3);
        int rc;
        if (j->t->quantized) {
            quantize_buffer(vals, packed, scales, (int)cnt);   /* the reference converter */
            const int64_t sbytes = (j->t->count / SYN_GROUP) * 4;
            rc = syn_pwrite(j->fd, scales, (size_t)(cnt / SYN_GROUP) * 4, j->base + (e0 / SYN_GROUP) * 4);
            if (!rc) rc = syn_pwrite(j->fd, packed, (size_t)cnt / 2, j->base + sbytes + e0 / 2);
        } else {
            rc = syn_pwrite(j->fd, vals, (size_t)cnt * 4, j->base + e0 * 4);
        }
        if (rc) j->failed = 1;
    }
    free(vals);
    free(packed);
    free(scales);
    return NULL;
}

int main(int argc, char** argv) {
    if (argc < 10) {
        fprintf(stderr, "usage: %s out.int4 dim hidden layers heads kv_heads vocab seq_len seed [threads]\n", argv[0]);
        return 2;
    }
    int32_t cfg[7];
    for (int i = 0; i < 7; i++) cfg[i] = (int32_t)atol(argv[2 + i]);
    const uint64_t seed = strtoull(argv[9], NULL, 10);
    int threads = argc > 10 ? atoi(argv[10]) : (int)sysconf(_SC_NPROCESSORS_ONLN);
    if (threads < 1) threads = 1;
    if (threads > 128) threads = 128;
    const int64_t dim = cfg[0], hid = cfg[1], L = cfg[2], nh = cfg[3], nkv = cfg[4], vocab = cfg[5], seq = cfg[6];
    if (dim <= 0 || hid <= 0 || L <= 0 || nh <= 0 || nkv <= 0 || vocab <= 0 || seq <= 0 || dim % nh || nh % nkv ||
        (dim / nh) % 2 || dim % SYN_GROUP || hid % SYN_GROUP) {
        fprintf(stderr, "invalid config\n");
        return 2;
    }
    const int64_t kv = dim * nkv / nh, hs = dim / nh;
    const syn_tensor t[13] = {
        {vocab * dim, 1, 0}, {L * dim, 0, 1},       {L * dim * dim, 1, 0}, {L * dim * kv, 1, 0}, {L * dim * kv, 1, 0},
        {L * dim * dim, 1, 0}, {L * dim, 0, 1},     {L * dim * hid, 1, 0}, {L * hid * dim, 1, 0},
        {L * dim * hid, 1, 0}, {dim, 0, 1},         {seq * (hs / 2), 0, 2}, {seq * (hs / 2), 0, 3},
    };
    int64_t total = 28;
    for (int i = 0; i < 13; i++) total += t[i].quantized ? (t[i].count / SYN_GROUP) * 4 + t[i].count / 2 : t[i].count * 4;
    const int fd = open(argv[1], O_WRONLY | O_CREAT | O_TRUNC, 0644);
    if (fd < 0 || ftruncate(fd, (off_t)total) != 0 || syn_pwrite(fd, cfg, 28, 0) != 0) {
        fprintf(stderr, "cannot write %s: %s\n", argv[1], strerror(errno));
        return 1;
    }
    int64_t off = 28;
    for (int i = 0; i < 13; i++) {
        syn_job j;
        memset(&j, 0, sizeof(j));
        j.fd = fd;
        j.tensor = i;
        j.t = &t[i];
        j.base = off;
        j.hs = hs;
        j.seed = seed;
        j.nchunks = (t[i].count + SYN_CHUNK - 1) / SYN_CHUNK;
        pthread_mutex_init(&j.mu, NULL);
        pthread_t th[128];
        const int nt = threads < j.nchunks ? threads : (int)j.nchunks;
        for (int k = 1; k < nt; k++) pthread_create(&th[k], NULL, syn_worker, &j);
        syn_worker(&j);
        for (int k = 1; k < nt; k++) pthread_join(th[k], NULL);
        pthread_mutex_destroy(&j.mu);
        if (j.failed) {
            fprintf(stderr, "write failed at tensor %d\n", i);
            close(fd);
            return 1;
        }
        off += t[i].quantized ? (t[i].count / SYN_GROUP) * 4 + t[i].count / 2 : t[i].count * 4;
    }
    return close(fd) == 0 ? 0 : 1;
}
