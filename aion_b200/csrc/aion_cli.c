/*
 * aion -- command-line driver, a drop-in for the reference CLI
 * (src/kernel_simd.c:1175-1288):
 *
 *   aion <model> <steps> <gpus> [int4] [w4a8] [nograph]
 *
 * The file decides the path: an int4 file (quantize.c) runs the int4
 * path, an fp32 llama2.c file the fp32 path, as kernel_simd does with and
 * without "int4".
 *
 * Same argv order as `kernel_simd <model> <steps> <threads> [int4] ...`
 * with the thread count replaced by the GPU count.  Prints "pos token" per
 * step to stdout (the INPUT token of that step, as :1245 does), a banner
 * and the tok/s line to stderr, and appends a row to benchmarks.csv in the
 * reference's columns (Timestamp,Impl,Cores,Steps,Time,Tok/s; :1260-1281).
 * The whole greedy loop runs on the device; tokens are printed after it,
 * so the timed region excludes printing.
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "aion.h"

int main(int argc, char** argv) {
    if (argc < 4) {
        printf("Usage: %s <model_path> <steps> <gpus> [int4] [w4a8] [nograph]\n", argv[0]);
        return 1;
    }
    const char* path = argv[1];
    int steps = atoi(argv[2]);
    int gpus = atoi(argv[3]);
    aion_opts opts;
    aion_default_opts(&opts);
    for (int i = 4; i < argc; i++) {
        if (strcmp(argv[i], "w4a8") == 0) opts.mode = AION_MODE_W4A8;
        if (strcmp(argv[i], "nograph") == 0) opts.use_graph = 0;
    }
    if (gpus != 1) {
        fprintf(stderr, "[aion] only a single GPU per process is driven by this CLI build (gpus=%d)\n", gpus);
        return 1;
    }
    aion_ctx* ctx = NULL;
    aion_status s = aion_load(path, &opts, &ctx);
    if (s != AION_OK) {
        fprintf(stderr, "[aion] load failed (%d): %s\n", (int)s, aion_last_error(NULL));
        return 1;
    }
    aion_config cfg;
    aion_get_config(ctx, &cfg);
    if (steps > cfg.seq_len) steps = cfg.seq_len;
    const int mode = aion_get_mode(ctx);
    fprintf(stderr, "[aion] Mode: %s on B200. GPUs: %d. dim %d, layers %d, vocab %d.\n",
            mode == AION_MODE_W4A8 ? "W4A8" : mode == AION_MODE_F32 ? "Float32" : "Int4 (W4A16)", gpus, cfg.dim,
            cfg.n_layers, cfg.vocab_size);
    int* tokens = calloc(steps > 0 ? (size_t)steps : 1, sizeof(int));
    double secs = 0.0;
    s = aion_generate(ctx, 1, steps, tokens, &secs);
    if (s != AION_OK) {
        fprintf(stderr, "[aion] generate failed (%d): %s\n", (int)s, aion_last_error(ctx));
        aion_free(ctx);
        free(tokens);
        return 1;
    }
    for (int pos = 0; pos < steps; pos++) printf("%d %d\n", pos, tokens[pos]);
    fflush(stdout);
    double tps = secs > 0 ? steps / secs : 0.0;
    fprintf(stderr, "[aion] Finished %d steps in %.4f s (%.2f tok/s)\n", steps, secs, tps);
    FILE* csv = fopen("benchmarks.csv", "a");
    if (csv) {
        time_t now = time(NULL);
        char ts[26];
        ctime_r(&now, ts);
        ts[24] = '\0';
        fprintf(csv, "%s,%s,%d,%d,%.4f,%.2f\n", ts,
                mode == AION_MODE_W4A8 ? "B200_W4A8" : mode == AION_MODE_F32 ? "B200_F32" : "B200_Int4", gpus, steps,
                secs, tps);
        fclose(csv);
    }
    aion_free(ctx);
    free(tokens);
    return 0;
}
