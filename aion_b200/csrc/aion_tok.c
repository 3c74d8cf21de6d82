/*
 * Text I/O for llama2.c-family checkpoints: the tokenizer.bin format and
 * its byte-pair encoding (no counterpart in the reference, which reads and
 * prints token ids only, src/kernel_simd.c:1245).
 *
 * tokenizer.bin: int32 max_token_length, then for each of vocab_size
 * tokens a float32 merge score, an int32 byte length and the bytes.
 *
 * Encoding (the published llama2.c procedure, restated):
 *   1. a non-empty text gets a leading " " token (the SentencePiece dummy
 *      prefix), when the vocabulary has one;
 *   2. each UTF-8 code point becomes its token if the vocabulary holds it,
 *      else one byte-fallback token per byte (id = byte + 3, the pieces
 *      "<0x00>".."<0xFF>" after <unk>, <s>, </s>);
 *   3. while some adjacent pair concatenates to a vocabulary piece, the pair
 *      whose piece has the highest score (the leftmost on ties) merges;
 *   4. optional BOS (1) first and EOS (2) last.
 * Decoding returns a token's piece, without its leading space right after
 * BOS, and a byte-fallback piece as that single byte.
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../../include/aion.h"

#define TOK_BOS 1
#define TOK_EOS 2

typedef struct {
    const char* s;
    int32_t id;
} tok_entry;

struct aion_tokenizer {
    int32_t n, max_len;
    char** piece;           /* [n] NUL-terminated pieces */
    float* score;           /* [n] */
    tok_entry* sorted;      /* pieces sorted by bytes, for lookup */
    unsigned char bytes[256][2];   /* single-byte strings for byte-fallback decoding */
};

static int tok_cmp(const void* a, const void* b) {
    return strcmp(((const tok_entry*)a)->s, ((const tok_entry*)b)->s);
}

static int32_t tok_find(const aion_tokenizer* t, const char* s) {
    tok_entry key = {s, 0};
    const tok_entry* e = (const tok_entry*)bsearch(&key, t->sorted, (size_t)t->n, sizeof(tok_entry), tok_cmp);
    return e ? e->id : -1;
}

AION_API void aion_tokenizer_free(aion_tokenizer* t) {
    if (!t) return;
    if (t->piece)
        for (int32_t i = 0; i < t->n; i++) free(t->piece[i]);
    free(t->piece);
    free(t->score);
    free(t->sorted);
    free(t);
}

AION_API aion_status aion_tokenizer_load(const char* path, int32_t vocab_size, aion_tokenizer** out) {
    if (!path || !out || vocab_size <= 0) return AION_ERR_ARG;
    *out = NULL;
    FILE* f = fopen(path, "rb");
    if (!f) return AION_ERR_IO;
    aion_tokenizer* t = (aion_tokenizer*)calloc(1, sizeof(*t));
    aion_status st = AION_OK;
    if (!t) {
        fclose(f);
        return AION_ERR_OOM;
    }
    t->n = vocab_size;
    t->piece = (char**)calloc((size_t)vocab_size, sizeof(char*));
    t->score = (float*)calloc((size_t)vocab_size, sizeof(float));
    t->sorted = (tok_entry*)calloc((size_t)vocab_size, sizeof(tok_entry));
    if (!t->piece || !t->score || !t->sorted) st = AION_ERR_OOM;
    if (st == AION_OK && (fread(&t->max_len, 4, 1, f) != 1 || t->max_len <= 0)) st = AION_ERR_FORMAT;
    for (int32_t i = 0; st == AION_OK && i < vocab_size; i++) {
        int32_t len = 0;
        if (fread(&t->score[i], 4, 1, f) != 1 || fread(&len, 4, 1, f) != 1 || len < 0 || len > 4096) {
            st = AION_ERR_FORMAT;
            break;
        }
        t->piece[i] = (char*)malloc((size_t)len + 1);
        if (!t->piece[i]) {
            st = AION_ERR_OOM;
            break;
        }
        if (len > 0 && fread(t->piece[i], 1, (size_t)len, f) != (size_t)len) {
            st = AION_ERR_FORMAT;
            break;
        }
        t->piece[i][len] = '\0';
        t->sorted[i].s = t->piece[i];
        t->sorted[i].id = i;
    }
    fclose(f);
    if (st != AION_OK) {
        aion_tokenizer_free(t);
        return st;
    }
    qsort(t->sorted, (size_t)vocab_size, sizeof(tok_entry), tok_cmp);
    for (int b = 0; b < 256; b++) {
        t->bytes[b][0] = (unsigned char)b;
        t->bytes[b][1] = 0;
    }
    *out = t;
    return AION_OK;
}

AION_API aion_status aion_encode(const aion_tokenizer* t, const char* text, int32_t bos, int32_t eos, int32_t* tokens,
                                 int32_t capacity, int32_t* n_out) {
    if (!t || !text || !tokens || !n_out) return AION_ERR_ARG;
    const size_t tl = strlen(text);
    if ((size_t)capacity < tl + 3) return AION_ERR_ARG;   /* worst case: every byte a token, plus prefix, BOS, EOS */
    /* room for merging two pieces: 2 * max_len bytes + NUL */
    char* buf = (char*)malloc((size_t)t->max_len * 2 + 8);
    if (!buf) return AION_ERR_OOM;
    int32_t n = 0;
    if (bos) tokens[n++] = TOK_BOS;
    if (tl > 0) {
        const int32_t sp = tok_find(t, " ");
        if (sp >= 0) tokens[n++] = sp;
    }
    size_t blen = 0;
    for (const unsigned char* c = (const unsigned char*)text; *c; c++) {
        if ((*c & 0xC0) != 0x80) blen = 0;   /* a new code point starts */
        buf[blen++] = (char)*c;
        buf[blen] = '\0';
        /* the code point continues if the next byte is a continuation byte (at most 4 bytes) */
        if ((c[1] & 0xC0) == 0x80 && blen < 4) continue;
        const int32_t id = tok_find(t, buf);
        if (id >= 0) {
            tokens[n++] = id;
        } else {
            for (size_t i = 0; i < blen; i++) tokens[n++] = (int32_t)(unsigned char)buf[i] + 3;
        }
        blen = 0;
    }
    /* merge the best-scoring adjacent pair until none forms a piece */
    for (;;) {
        float best = -1e10f;
        int32_t best_id = -1, best_i = -1;
        const int32_t first = bos ? 1 : 0;
        for (int32_t i = first; i + 1 < n; i++) {
            const char* a = t->piece[tokens[i]];
            const char* b = t->piece[tokens[i + 1]];
            const size_t la = strlen(a), lb = strlen(b);
            if (la + lb > (size_t)t->max_len * 2) continue;
            memcpy(buf, a, la);
            memcpy(buf + la, b, lb + 1);
            const int32_t id = tok_find(t, buf);
            if (id >= 0 && t->score[id] > best) {
                best = t->score[id];
                best_id = id;
                best_i = i;
            }
        }
        if (best_i < 0) break;
        tokens[best_i] = best_id;
        memmove(tokens + best_i + 1, tokens + best_i + 2, (size_t)(n - best_i - 2) * sizeof(int32_t));
        n--;
    }
    if (eos) tokens[n++] = TOK_EOS;
    free(buf);
    *n_out = n;
    return AION_OK;
}

AION_API const char* aion_decode(const aion_tokenizer* t, int32_t prev, int32_t token) {
    if (!t || token < 0 || token >= t->n) return NULL;
    const char* p = t->piece[token];
    if (prev == TOK_BOS && p[0] == ' ') p++;
    unsigned int byte = 0;
    char tail = 0;
    if (p[0] == '<' && sscanf(p, "<0x%02X>%c", &byte, &tail) == 1 && strlen(p) == 6)
        return (const char*)((aion_tokenizer*)t)->bytes[byte & 0xFF];
    return p;
}
