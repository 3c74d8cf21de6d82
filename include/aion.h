/*
 * aion.h -- C ABI of the B200 int4 Llama-2 decode library (libaion.so).
 *
 * Drop-in boundary for the int4 path of the reference engine
 * (farukalpay/AION, src/kernel_simd.c).  Plain C11, no CUDA or torch types:
 * device pointers are passed as plain pointers, CUDA streams as void*.
 * Every call returns an aion_status; no call exits or aborts the process.
 * The message of the last failure is available from aion_last_error().
 *
 * Threading: one aion_ctx is used by one host thread at a time; distinct
 * contexts are independent.  All work of a context runs on its own stream.
 */
#ifndef AION_H
#define AION_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define AION_API __attribute__((visibility("default")))
#else
#define AION_API
#endif

typedef enum aion_status {
    AION_OK = 0,
    AION_ERR_IO = 1,      /* open / read / write failed                       */
    AION_ERR_FORMAT = 2,  /* file size or header inconsistent with the format */
    AION_ERR_SHAPE = 3,   /* unsupported or inconsistent dimensions           */
    AION_ERR_OOM = 4,     /* device or host allocation failed                 */
    AION_ERR_CUDA = 5,    /* CUDA runtime error                               */
    AION_ERR_NCCL = 6,    /* NCCL error (tensor-parallel contexts)            */
    AION_ERR_TIMEOUT = 7, /* a bounded device-side wait gave up               */
    AION_ERR_ARG = 8,     /* invalid argument (token, position, pointer ...)  */
    AION_ERR_STATE = 9    /* call not valid in the context's current state    */
} aion_status;

/* The 28-byte packed checkpoint header, field for field
 * (src/kernel_simd.c:40-48, quantize.c:33-41). */
typedef struct aion_config {
    int32_t dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len;
} aion_config;

/* AION_MODE_F32: the reference's fp32 path (its CLI without "int4"); chosen
 * by aion_load when the file is an fp32 llama2.c checkpoint. */
enum { AION_MODE_W4A16 = 0, AION_MODE_W4A8 = 1, AION_MODE_F32 = 2 };

typedef struct aion_opts {
    int32_t device;     /* CUDA device ordinal                                        */
    int32_t mode;       /* AION_MODE_W4A16 (default) or AION_MODE_W4A8                */
    int32_t max_batch;  /* sequences (KV caches) held, for aion_prefill and
                           aion_decode_batch (default 1)                            */
    int32_t max_pos;    /* KV positions allocated (0 = header seq_len; <= seq_len)     */
    int32_t tp_size;    /* tensor-parallel ranks, one process per GPU of one node
                           (1 <= tp_size <= 8; default 1)                          */
    int32_t tp_rank;    /* this rank, 0 <= tp_rank < tp_size                           */
    const void* nccl_id;/* reserved (the ranks exchange IPC handles, see aion_tp_*)    */
    int32_t use_graph;  /* 1 (default): replay one CUDA graph per decode step          */
    int32_t wait_ms;    /* bound of each wait on another GPU inside the decode kernels,
                           in milliseconds (0: 2000).  A wait that runs out makes the
                           call return AION_ERR_TIMEOUT; aion_reset clears it.        */
    int32_t reserved[6];
} aion_opts;

typedef struct aion_ctx aion_ctx;

/* Fills *opts with the defaults listed above. */
AION_API void aion_default_opts(aion_opts* opts);

/* Text of the last failure of ctx, or of the calling thread's last
 * context-free call (load, kernel-level, tools) when ctx is NULL. */
AION_API const char* aion_last_error(const aion_ctx* ctx);

/* ---------------------------------------------------------------------------
 * Model level
 * ------------------------------------------------------------------------- */

/* Replaces load_checkpoint_int4 (src/kernel_simd.c:941-989) + malloc_run_state
 * (:991-1008).  Validates the file size against the header in 64-bit
 * arithmetic before any upload, uploads every tensor once to HBM re-tiled
 * for the decode kernels, allocates the KV cache and activations, and
 * unmaps the file.  The context owns all device memory.
 * An fp32 llama2.c file (load_checkpoint, :906-936; a negative vocab_size
 * adds a separate classifier that, as in the reference, is not read) runs
 * the fp32 path: fp32 weights and activations, the classifier tied to the
 * embedding.  It needs tp_size 1 and a mode other than W4A8; prefill and
 * batched decode need an int4 file. */
AION_API aion_status aion_load(const char* int4_path, const aion_opts* opts, aion_ctx** out);
AION_API aion_status aion_free(aion_ctx* ctx);
AION_API aion_status aion_get_config(const aion_ctx* ctx, aion_config* out);

/* Replaces transformer(token, pos, ...) (src/kernel_simd.c:1014-1169, int4
 * branch): writes the KV cache at `pos` and produces the logits of (token,
 * pos).  logits_host (vocab floats) may be NULL; the device copy stays
 * readable through aion_logits_dev().  Requires 0 <= pos < max_pos. */
AION_API aion_status aion_forward(aion_ctx* ctx, int32_t token, int32_t pos, float* logits_host);

/* Device pointer to the logits of the last decode step ([vocab] fp32). */
AION_API const float* aion_logits_dev(const aion_ctx* ctx);

/* The mode the context runs: AION_MODE_W4A16, AION_MODE_W4A8 or
 * AION_MODE_F32 (an fp32 file); -1 for NULL. */
AION_API int32_t aion_get_mode(const aion_ctx* ctx);

/* Replaces the greedy loop of main (src/kernel_simd.c:1223-1258): starts at
 * pos 0 from `bos`, runs `steps` forward steps, picks the first index of the
 * maximum logit (strict '>', from -1e9; :1236-1243) on the device, and
 * writes tokens_out[pos] = input token of step pos (what :1245 prints).
 * *seconds (may be NULL) receives the wall time of the loop. */
AION_API aion_status aion_generate(aion_ctx* ctx, int32_t bos, int32_t steps, int32_t* tokens_out,
                                   double* seconds);

/* The context's cudaStream_t (all of its work runs there). */
AION_API void* aion_stream(const aion_ctx* ctx);

/* Enqueues `steps` greedy decode steps on the context's stream without
 * waiting (the asynchronous form of aion_generate's loop; one persistent
 * kernel launch).  token >= 0 forces the input token of the first step,
 * token < 0 takes the previous step's argmax; pos >= 0 sets the first
 * position, pos < 0 continues at the next one. */
AION_API aion_status aion_decode_async(aion_ctx* ctx, int32_t token, int32_t pos, int32_t steps);

/* ---------------------------------------------------------------------------
 * Tensor parallelism (opts.tp_size > 1; one process per GPU of one node).
 * Rank r holds rows [r/N, (r+1)/N) of wq, wk, wv, w1, w3 and of the
 * classifier, and columns [r/N, (r+1)/N) of wo and w2; the decode kernel
 * sums the ranks' wo / w2 partial rows and picks the argmax across ranks
 * itself, over NVLink peer memory (the reference has no counterpart).
 * Before the first decode call every rank passes every rank's handle, in
 * rank order, to aion_tp_connect; the caller's launcher moves the handles
 * between processes (AION_TP_HANDLE_BYTES each).  aion_forward then writes
 * this rank's slice of the logits, vocab rows [r*vocab/N, (r+1)*vocab/N).
 * ------------------------------------------------------------------------- */
#define AION_TP_HANDLE_BYTES 64
/* The rows and columns rank tp_rank holds: out[0..8] = first query row /
 * query rows (of wq; also the columns of wo), first K/V row / K/V rows (of
 * wk, wv), first hidden row / hidden rows (of w1, w3; also the columns of
 * w2), first vocab row / vocab rows (of the classifier), heads.
 * AION_ERR_SHAPE when the shape does not shard over tp_size ranks. */
#define AION_TP_PLAN_FIELDS 9
AION_API aion_status aion_tp_plan(const aion_config* cfg, int32_t tp_size, int32_t tp_rank, int64_t* out);
AION_API aion_status aion_tp_handle(const aion_ctx* ctx, void* handle_out);
AION_API aion_status aion_tp_connect(aion_ctx* ctx, const void* handles);

/* Copies the input tokens of positions [0, n) recorded on the device. */
AION_API aion_status aion_tokens(aion_ctx* ctx, int32_t* out, int32_t n);

/* Clears the KV cache of the selected sequence (a new sequence). */
AION_API aion_status aion_reset(aion_ctx* ctx);

/* ---------------------------------------------------------------------------
 * Several sequences and batched prefill (no counterpart in the reference,
 * whose transformer() takes one token of one sequence).  A context holds
 * opts.max_batch sequences, each with its own KV cache.
 * ------------------------------------------------------------------------- */

/* Selects the sequence whose KV cache aion_forward / aion_decode_async /
 * aion_generate / aion_reset use (default 0).  The step state (position,
 * token history) is shared: set the position explicitly after switching. */
AION_API aion_status aion_set_sequence(aion_ctx* ctx, int32_t seq);

/* Runs tokens[n_seq][n_tok] (host memory, row-major) through the model at
 * positions 0..n_tok-1 of sequences 0..n_seq-1, all tokens at once: every
 * matrix product on the tensor cores (int4 weights dequantized to bf16,
 * operands split into two bf16 parts, fp32 accumulate), causal attention
 * per sequence and head.  Writes each sequence's KV cache at those
 * positions and the logits of each sequence's last position to
 * logits_host[n_seq][vocab] (may be NULL).  Equivalent to n_tok
 * transformer() calls per sequence.  n_seq <= max_batch, n_tok <= max_pos. */
AION_API aion_status aion_prefill(aion_ctx* ctx, const int32_t* tokens, int32_t n_seq, int32_t n_tok,
                                  float* logits_host);

/* Lock-step greedy decode of sequences 0..n_seq-1 (n_seq <= min(max_batch,
 * 32)), W4A16, one persistent launch; under tensor parallelism every rank
 * makes the same call (after aion_tp_connect).  Step i feeds sequence b
 * one token at position pos0[b] + i: first_tokens[b] at step 0, afterwards
 * the first maximum of its previous logits (src/kernel_simd.c:1236-1243).
 * Each step is transformer() (src/kernel_simd.c:1014) of every sequence:
 * it writes the sequence's KV cache at that position.  tokens[(steps + 1)
 * * n_seq] (host) receives row i = the inputs of step i and row steps = the
 * picks after the last step; logits[n_seq][vocab / tp_size] (host, may be
 * NULL) the last step's logits (this rank's vocab rows).  Each weight is read once per step for all sequences.
 * Activations enter the integer dot as 24-bit fixed point per group of 32
 * (relative error below 2^-22 of the group's largest value), fp32
 * accumulate.  Needs pos0[b] + steps <= max_pos. */
AION_API aion_status aion_decode_batch(aion_ctx* ctx, int32_t n_seq, int32_t steps, const int32_t* first_tokens,
                                       const int32_t* pos0, int32_t* tokens, float* logits);

/* ---------------------------------------------------------------------------
 * Sampling beyond greedy (no counterpart in the reference, which takes the
 * argmax, src/kernel_simd.c:1236-1243).
 * ------------------------------------------------------------------------- */
typedef struct aion_sampler {
    float temperature;  /* <= 0: greedy (the reference's argmax)                   */
    float top_p;        /* keep the most likely tokens up to this mass; 1 = off     */
    int32_t top_k;      /* keep the top_k most likely tokens (ties kept); 0 = off   */
    int32_t reserved;
    uint64_t seed;      /* each draw is a function of (seed, sequence, position)    */
} aion_sampler;

/* Sets how aion_decode_async / aion_generate / aion_decode_batch pick the
 * next token (NULL: greedy).  With temperature T > 0 every step draws, on
 * the device, from the distribution e^((logit - max) / T) restricted to
 * the top_k largest logits and then to the smallest set of largest logits
 * whose mass reaches top_p: weights are floor(e^x * 2^32) integers,
 * thresholds exact, and the draw a SplitMix64 value of (seed, sequence,
 * position) scanned in index order, so a run is reproducible.  aion_forward
 * is unaffected (it returns logits).  Needs tp_size 1. */
AION_API aion_status aion_set_sampler(aion_ctx* ctx, const aion_sampler* sampler);

/* Copies the logits of the last step that aion_decode_async / aion_generate
 * ran (this rank's vocab rows) to host[vocab]; waits for the stream. */
AION_API aion_status aion_read_logits(aion_ctx* ctx, float* host);

/* ---------------------------------------------------------------------------
 * Text I/O (no counterpart in the reference, which reads and prints token
 * ids only, src/kernel_simd.c:1245): llama2.c tokenizer.bin files.
 * ------------------------------------------------------------------------- */
typedef struct aion_tokenizer aion_tokenizer;

/* Reads tokenizer.bin (int32 max_token_length, then per token: float score,
 * int32 length, the bytes) for vocab_size tokens. */
AION_API aion_status aion_tokenizer_load(const char* path, int32_t vocab_size, aion_tokenizer** out);
AION_API void aion_tokenizer_free(aion_tokenizer* tok);

/* Byte-pair encoding of UTF-8 text: a leading " " token (dummy prefix) for
 * non-empty text, one token per code point found in the vocabulary else
 * byte-fallback tokens (byte + 3), then repeated merges of the adjacent
 * pair whose concatenation has the highest score.  Optional BOS (1) first
 * and EOS (2) last.  capacity >= strlen(text) + 3. */
AION_API aion_status aion_encode(const aion_tokenizer* tok, const char* text, int32_t bos, int32_t eos,
                                 int32_t* tokens, int32_t capacity, int32_t* n_out);

/* The text of `token` following `prev`: its piece, without the leading
 * space right after BOS; a byte-fallback piece "<0xHH>" is that byte.
 * NULL for an id out of range.  The pointer lives as long as tok. */
AION_API const char* aion_decode(const aion_tokenizer* tok, int32_t prev, int32_t token);

/* ---------------------------------------------------------------------------
 * Kernel level (device pointers; stream = cudaStream_t or NULL)
 * ------------------------------------------------------------------------- */

typedef struct aion_qmatrix aion_qmatrix;

/* Uploads one int4 matrix [rows][cols] given in the quantize.c layout (the
 * QWeight view of src/kernel_simd.c:113-116: fp32 scales[rows*cols/32] and
 * packed bytes[rows*cols/2], host memory) and re-tiles it on the device.
 * cols must be a multiple of 32. */
AION_API aion_status aion_qmatrix_upload(const float* scales, const uint8_t* packed, int64_t rows, int64_t cols,
                                         int32_t device, aion_qmatrix** out);
/* Exact inverse of the re-tile: writes the quantize.c layout back to host
 * memory, byte for byte. */
AION_API aion_status aion_qmatrix_download(const aion_qmatrix* w, float* scales, uint8_t* packed);
AION_API aion_status aion_qmatrix_free(aion_qmatrix* w);

/* W4A16 matvec y[rows] = W x[cols] (fp32 in, fp32 accumulate, fp32 out).
 * Replaces matmul_int4_scalar / matmul_int4_neon (src/kernel_simd.c:341,377)
 * as dispatched by dispatch_matmul_int4 (:752) over all rows. */
AION_API aion_status aion_matvec_w4a16(const aion_qmatrix* w, const float* x_dev, float* y_dev, void* stream);

/* W4A8 matvec: per-32 dynamic int8 quantization of x fused with the int4 x
 * int8 group dot and the per-row sequential fp32 epilogue.  Replaces
 * quantize_activations_neon (:186) + matmul_w4a8_neon (:244) as
 * dispatch_matmul_w4a8 (:771) would run them.  Bit-exact with them. */
AION_API aion_status aion_matvec_w4a8(const aion_qmatrix* w, const float* x_dev, float* y_dev, void* stream);

/* The W4A16 matvec of aion_matvec_w4a16 with its scratch in a fixed device
 * array instead of the matrix's own scratch; it calls no allocating
 * function.  No counterpart in the reference.  At most 32768 rows
 * (AION_ERR_SHAPE beyond).  One scratch array per device is shared by all
 * calls: calls that overlap in time race and must be serialised by the
 * caller.  The first call on a device resolves the array's address; make it
 * before any stream capture on that device. */
AION_API aion_status aion_matvec_w4a16_static(const aion_qmatrix* w, const float* x_dev, float* y_dev, void* stream);

/* Waits for `stream`, then reports whether a matvec on `w` enqueued before
 * it (aion_matvec_w4a16 / _w4a8 on the matrix's scratch, or
 * aion_matvec_w4a16_static on this device's array) gave up one of its
 * bounded waits: AION_ERR_TIMEOUT means that call's y is invalid.  Clears
 * the record.  The reference's matmul has no failure mode (it spins in its
 * barrier, src/kernel_simd.c:93-106); this is the status-never-abort
 * contract's read-out for the asynchronous kernel-level calls.  Calls on
 * one matrix's scratch that overlap on the GPU (different streams) race, as
 * calls of the static variant do. */
AION_API aion_status aion_matvec_status(const aion_qmatrix* w, void* stream);

/* Diagnostic, for tests of the failure path: records in w's scratch the
 * same error a matvec on w records when one of its bounded waits gives up,
 * so that the next aion_matvec_status reports AION_ERR_TIMEOUT (and clears
 * it) without any wait being made to run out on the GPU. */
AION_API aion_status aion_matvec_inject_timeout(const aion_qmatrix* w);

/* Device resets: the static variant keeps its array's device address for
 * the life of the process, and matrices and contexts hold device memory, so
 * a cudaDeviceReset (or a recreated primary context) invalidates them; the
 * library does not support it while any of its objects or the static
 * variant is in use on that device. */

/* Dense GEMM on the tensor cores: C[m][n] (fp32) = A[m][k] * B[n][k]^T with
 * A and B bf16 (K contiguous), all device memory, on the current device.
 * The building block of the batched prefill, where B holds int4 weights
 * dequantized to bf16; no counterpart in the reference.  m, n, k must be
 * multiples of 128, 256 and 64; A, B and C 16-byte aligned. */
AION_API aion_status aion_gemm_bf16_tn(const void* a_dev, const void* b_dev, float* c_dev, int64_t m, int64_t n,
                                       int64_t k, void* stream);

/* Per-32 symmetric int8 activation quantization (quantize_activations_neon,
 * src/kernel_simd.c:186-227): qx[n] int8, xs[n/32] fp32.  Bit-exact. */
AION_API aion_status aion_quantize_activations(const float* x_dev, int8_t* qx_dev, float* xs_dev, int64_t n,
                                               void* stream);

/* ---------------------------------------------------------------------------
 * Checkpoint tools (host)
 * ------------------------------------------------------------------------- */

/* quantize_buffer (quantize.c:59-109) on the device, bit-exact with it:
 * in_dev[n] fp32 -> packed_dev[n/2], scales_dev[n/32] (device memory;
 * n a multiple of 32, in and packed 16-byte aligned). */
AION_API aion_status aion_quantize_buffer_dev(const float* in_dev, uint8_t* packed_dev, float* scales_dev, int64_t n,
                                              void* stream);
/* quantize_buffer (quantize.c:59-109) with 64-bit element counts. */
AION_API void aion_quantize_buffer(const float* in, uint8_t* packed, float* scales, int64_t n);
/* Byte size of a checkpoint for a 7-int header, fp32 (int4 = 0) or int4. */
AION_API int64_t aion_checkpoint_bytes(const int32_t* cfg7, int int4);
/* fp32 llama2.c legacy file -> int4 file in the quantize.c format
 * (quantize.c:119-238), 64-bit clean. */
AION_API int aion_quantize_file(const char* in_path, const char* out_path, int threads, char* err, int errlen);
/* Seeded random-init checkpoint: matrices N(0, 0.02), RMSNorm weights 1.0,
 * RoPE tables; written as fp32 (int4 = 0) or directly as int4. */
AION_API int aion_synth_checkpoint(const char* path, const int32_t* cfg7, uint64_t seed, int int4, int threads,
                                   char* err, int errlen);

#ifdef __cplusplus
}
#endif
#endif /* AION_H */
