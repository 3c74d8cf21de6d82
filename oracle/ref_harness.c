/*
 * Harness around the reference engine -- TEST INFRASTRUCTURE ONLY.
 *
 * Built by oracle/Makefile as oracle/_ref/libaionref.so from the reference's
 * own src/kernel_simd.c, included unmodified (its main() renamed by the
 * preprocessor) and compiled through the scalar <arm_neon.h> stand-in in
 * oracle/shim/.  It exposes the reference functions to the tests and adds
 * what the reference CLI lacks:
 *   - per-step logits (the CLI prints tokens only, src/kernel_simd.c:1245);
 *   - a W4A8 forward: the reference's transformer() sequence with
 *     quantize_activations_neon + dispatch_matmul_w4a8 in place of every
 *     dispatch_matmul_int4 (the CLI's "w4a8" flag never does this,
 *     src/kernel_simd.c:1193 vs :1054-1165);
 *   - the fp32 path (the CLI without "int4"): load_checkpoint +
 *     transformer() with TransformerWeights, unchanged.
 * The reference sources are read from the reference tree at build time and
 * never copied into this repository.
 */
#define main aion_reference_cli_main
#include "kernel_simd.c"
#undef main

#define REF_EXPORT __attribute__((visibility("default")))

static Config g_cfg;
static QuantizedTransformerWeights g_qw;
static TransformerWeights g_w;
static int g_f32 = 0;
static RunState g_rs;
static int g_fd = -1;
static float* g_data = NULL;
static size_t g_size = 0;
static int g_pool = 0;
static QActivations g_qa;

REF_EXPORT int ref_open(const char* path, int n_threads, int scalar) {
    g_f32 = 0;
    load_checkpoint_int4(path, &g_cfg, &g_qw, &g_fd, &g_data, &g_size);
    malloc_run_state(&g_rs, &g_cfg);
    int big = g_cfg.dim > g_cfg.hidden_dim ? g_cfg.dim : g_cfg.hidden_dim;
    g_qa.qx = calloc((size_t)big, 1);
    g_qa.scales = calloc((size_t)big / 32 + 1, sizeof(float));
    USE_SCALAR_INT4 = scalar;
    if (!g_pool) { init_thread_pool(n_threads); g_pool = 1; }
    return 0;
}

/* The fp32 path: src/kernel_simd.c:906-936 (load_checkpoint) and the fp32
 * branch of transformer(). */
REF_EXPORT int ref_open_f32(const char* path, int n_threads) {
    load_checkpoint(path, &g_cfg, &g_w, &g_fd, &g_data, &g_size);
    malloc_run_state(&g_rs, &g_cfg);
    g_f32 = 1;
    if (!g_pool) { init_thread_pool(n_threads); g_pool = 1; }
    return 0;
}
REF_EXPORT void ref_forward_f32(int token, int pos) { transformer(token, pos, &g_cfg, &g_rs, &g_w, NULL); }

REF_EXPORT void ref_config(int* out7) { memcpy(out7, &g_cfg, sizeof(Config)); }
REF_EXPORT float* ref_logits(void) { return g_rs.logits; }

REF_EXPORT void ref_reset(void) {
    int kv_dim = (g_cfg.dim * g_cfg.n_kv_heads) / g_cfg.n_heads;
    size_t n = (size_t)g_cfg.n_layers * g_cfg.seq_len * kv_dim;
    memset(g_rs.key_cache, 0, n * sizeof(float));
    memset(g_rs.value_cache, 0, n * sizeof(float));
}

/* W4A16: the reference's own transformer(), int4 branch. */
REF_EXPORT void ref_forward(int token, int pos) { transformer(token, pos, &g_cfg, &g_rs, NULL, &g_qw); }

static void ref_mm_w4a8(float* out, float* x, QWeight* w, int n, int d) {
    quantize_activations_neon(&g_qa, x, n);
    dispatch_matmul_w4a8(out, &g_qa, w, n, d);
}

/* W4A8: transformer()'s int4 branch with every matvec replaced by
 * activation quantization + the reference W4A8 kernel. */
REF_EXPORT void ref_forward_w4a8(int token, int pos) {
    Config* p = &g_cfg;
    RunState* s = &g_rs;
    QuantizedTransformerWeights* qw = &g_qw;
    float* x = s->x;
    int dim = p->dim;
    int kv_dim = (p->dim * p->n_kv_heads) / p->n_heads;
    int kv_mul = p->n_heads / p->n_kv_heads;
    int hidden_dim = p->hidden_dim;
    int head_size = dim / p->n_heads;

    QWeight row = qw_offset(qw->token_embedding_table, token * dim);
    for (int i = 0; i < dim; i += 2) {
        uint8_t b = row.packed[i / 2];
        float sc = row.scales[i / 32];
        x[i] = (int8_t)((b & 0xF) - 8) * sc;
        x[i + 1] = (int8_t)((b >> 4) - 8) * sc;
    }
    for (int l = 0; l < p->n_layers; l++) {
        rmsnorm(s->xb, x, qw->rms_att_weight + l * dim, dim);
        QWeight wq = qw_offset(qw->wq, l * dim * dim);
        QWeight wk = qw_offset(qw->wk, l * dim * kv_dim);
        QWeight wv = qw_offset(qw->wv, l * dim * kv_dim);
        ref_mm_w4a8(s->q, s->xb, &wq, dim, dim);
        ref_mm_w4a8(s->k, s->xb, &wk, dim, kv_dim);
        ref_mm_w4a8(s->v, s->xb, &wv, dim, kv_dim);
        float* fr = qw->freq_cis_real;
        float* fi = qw->freq_cis_imag;
        for (int i = 0; i < dim; i += 2) {
            int hd = i % head_size;
            float c = fr[pos * (head_size / 2) + hd / 2], sn = fi[pos * (head_size / 2) + hd / 2];
            float a0 = s->q[i], a1 = s->q[i + 1];
            s->q[i] = a0 * c - a1 * sn;
            s->q[i + 1] = a0 * sn + a1 * c;
        }
        for (int i = 0; i < kv_dim; i += 2) {
            int hd = i % head_size;
            float c = fr[pos * (head_size / 2) + hd / 2], sn = fi[pos * (head_size / 2) + hd / 2];
            float a0 = s->k[i], a1 = s->k[i + 1];
            s->k[i] = a0 * c - a1 * sn;
            s->k[i + 1] = a0 * sn + a1 * c;
        }
        int loff = l * p->seq_len * kv_dim;
        memcpy(s->key_cache + loff + pos * kv_dim, s->k, kv_dim * sizeof(float));
        memcpy(s->value_cache + loff + pos * kv_dim, s->v, kv_dim * sizeof(float));
        for (int h = 0; h < p->n_heads; h++) {
            float* q = s->q + h * head_size;
            float* att = s->att + h * p->seq_len;
            for (int t = 0; t <= pos; t++) {
                float* k = s->key_cache + loff + t * kv_dim + (h / kv_mul) * head_size;
                float score = 0.0f;
                for (int j = 0; j < head_size; j++) score += q[j] * k[j];
                score /= sqrtf(head_size);
                att[t] = score;
            }
            softmax(att, pos + 1);
            float* xb = s->xb + h * head_size;
            memset(xb, 0, head_size * sizeof(float));
            for (int t = 0; t <= pos; t++) {
                float* v = s->value_cache + loff + t * kv_dim + (h / kv_mul) * head_size;
                float a = att[t];
                for (int j = 0; j < head_size; j++) xb[j] += a * v[j];
            }
        }
        QWeight wo = qw_offset(qw->wo, l * dim * dim);
        ref_mm_w4a8(s->xb2, s->xb, &wo, dim, dim);
        for (int i = 0; i < dim; i++) x[i] += s->xb2[i];
        rmsnorm(s->xb, x, qw->rms_ffn_weight + l * dim, dim);
        QWeight w1 = qw_offset(qw->w1, l * dim * hidden_dim);
        QWeight w3 = qw_offset(qw->w3, l * dim * hidden_dim);
        ref_mm_w4a8(s->hb, s->xb, &w1, dim, hidden_dim);
        ref_mm_w4a8(s->hb2, s->xb, &w3, dim, hidden_dim);
        swiglu(s->hb, s->hb2, hidden_dim);
        QWeight w2 = qw_offset(qw->w2, l * hidden_dim * dim);
        ref_mm_w4a8(s->xb, s->hb, &w2, hidden_dim, dim);
        for (int i = 0; i < dim; i++) x[i] += s->xb[i];
    }
    rmsnorm(x, x, qw->rms_final_weight, dim);
    QWeight emb = qw->token_embedding_table;
    ref_mm_w4a8(s->logits, x, &emb, dim, p->vocab_size);
}

/* Greedy loop of src/kernel_simd.c:1223-1250 with optional per-step dumps.
 * tokens[pos] = input token of step pos (what the CLI prints). */
REF_EXPORT int ref_generate(int bos, int steps, int w4a8, int* tokens, float* gaps, float* logits_dump) {
    int token = bos;
    ref_reset();
    for (int pos = 0; pos < steps; pos++) {
        if (g_f32) ref_forward_f32(token, pos);
        else if (w4a8) ref_forward_w4a8(token, pos);
        else ref_forward(token, pos);
        float max_p = -1e9f, second = -INFINITY;
        int next = 0;
        for (int i = 0; i < g_cfg.vocab_size; i++) {
            if (g_rs.logits[i] > max_p) { second = max_p; max_p = g_rs.logits[i]; next = i; }
            else if (g_rs.logits[i] > second) second = g_rs.logits[i];
        }
        tokens[pos] = token;
        if (gaps) gaps[pos] = max_p - second;
        if (logits_dump) memcpy(logits_dump + (size_t)pos * g_cfg.vocab_size, g_rs.logits, (size_t)g_cfg.vocab_size * sizeof(float));
        token = next;
    }
    return token;
}

/* Kernel-level entry points (row range = all rows). */
REF_EXPORT void ref_matmul_int4_scalar(float* y, const float* x, const float* scales, const uint8_t* packed, int n, int d) {
    QWeight w = { (float*)scales, (uint8_t*)packed };
    matmul_int4_scalar(y, x, &w, n, 0, d, d);
}
REF_EXPORT void ref_matmul_int4_neon(float* y, const float* x, const float* scales, const uint8_t* packed, int n, int d) {
    QWeight w = { (float*)scales, (uint8_t*)packed };
    matmul_int4_neon(y, x, &w, n, 0, d, d);
}
REF_EXPORT void ref_quantize_activations(int8_t* qx, float* xs, const float* x, int n) {
    QActivations a = { qx, xs };
    quantize_activations_neon(&a, x, n);
}
REF_EXPORT void ref_matmul_w4a8(float* y, const int8_t* qx, const float* xs, const float* scales, const uint8_t* packed, int n, int d) {
    QActivations a = { (int8_t*)qx, (float*)xs };
    QWeight w = { (float*)scales, (uint8_t*)packed };
    matmul_w4a8_neon(y, &a, &w, n, 0, d, d);
}
REF_EXPORT void ref_rmsnorm(float* o, float* x, float* w, int n) { rmsnorm(o, x, w, n); }
REF_EXPORT void ref_softmax(float* x, int n) { softmax(x, n); }
REF_EXPORT void ref_swiglu(float* hb, float* hb2, int n) { swiglu(hb, hb2, n); }
