/* ref_driver.c -- command-line driver around the REFERENCE engine's own C API.
 *
 * TEST INFRASTRUCTURE ONLY. This file is linked against the reference's
 * unmodified src/model.c, src/kv_cache.c, src/gemm/gemm_naive.c and
 * src/safetensors.c (see oracle/Makefile) to produce the binary oracle/_ref/
 * ref_gpt2. It is the checker the CUDA path is compared with and the CPU
 * baseline that bench.py times; nothing in the product links or runs it.
 *
 * What it runs is the reference's greedy loop on its cached path, the loop of
 * src/main.c:274-287 with --kv-cache: model_prefill over the prompt, the argmax
 * of the last row (model_argmax, model.c:920-925), then one
 * model_decode_step_cached per further token (model.c:870-896).
 *
 * usage: ref_gpt2 WEIGHTS INVENTORY CONFIG IDS.bin N_SEQ N_PROMPT N_NEW OUT.bin
 *                 [--first-seq S] [--cproj transposed] [--prefill-logits all|last|none]
 *                 [--step-logits] [--nocache] [--topk K] [--prefill-topk]
 *                 [--time-contexts C1,C2,... [--rounds R]]
 *
 * With --time-contexts the driver measures instead of generating: for the
 * first sequence it times model_prefill over the whole prompt (the cache is
 * written), then, R times over, one model_decode_step_cached at each listed
 * context C (the cache length set to C - 1 with model_kv_set_length, the ids
 * past the prompt filled with the prefill's greedy token). Decode cost is
 * affine in the context, so these samples give the cost of every step of a
 * generation ("none" times the prefill alone). Nothing is written to OUT.bin;
 * stdout gets one JSON line.
 *
 * IDS.bin holds N_SEQ x N_PROMPT int32 ids (row-major); sequences
 * [first-seq, first-seq + N_SEQ) of it are run. OUT.bin receives, per sequence:
 *   int32 ids[N_NEW]        the greedy tokens
 *   int32 kid[N_NEW][K]     the K largest logits' indices of the row each token
 *   float kval[N_NEW][K]    was chosen from, and their values (descending; ties by
 *                           lower index; K defaults to 2, so kval[.][0] - kval[.][1]
 *                           is the greedy margin)
 *   with --prefill-topk: int32 pid[N_PROMPT][K], float pval[N_PROMPT][K] for every
 *                           prefill position
 *   float prefill[...]      prefill logits: N_PROMPT x V (all), V (last) or nothing
 *   float steps[...]      with --step-logits: (N_NEW - 1) x V decode-step logits
 * One JSON line of CLOCK_MONOTONIC timings goes to stdout.
 */
#define _POSIX_C_SOURCE 200809L
#include "model.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

static double now_ms(void)
{
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec * 1e3 + (double)ts.tv_nsec * 1e-6;
}

/* The k largest entries of v (NaN skipped), descending, lower index first on
 * ties: k passes of a strict '>' scan that skips already-chosen indices. */
static void topk(const float *v, size_t n, int k, int32_t *ids, float *vals)
{
    for (int r = 0; r < k; ++r) {
        int32_t best = -1;
        for (size_t i = 0; i < n; ++i) {
            int taken = 0;
            for (int q = 0; q < r; ++q) if (ids[q] == (int32_t)i) { taken = 1; break; }
            if (taken || v[i] != v[i]) continue;
            if (best < 0 || v[i] > v[best]) best = (int32_t)i;
        }
        ids[r] = best;
        vals[r] = best >= 0 ? v[best] : 0.0f;
    }
}

int main(int argc, char **argv)
{
    if (argc < 9) {
        fprintf(stderr, "usage: %s WEIGHTS INVENTORY CONFIG IDS.bin N_SEQ N_PROMPT N_NEW OUT.bin "
                        "[--first-seq S] [--cproj transposed] [--prefill-logits all|last|none] "
                        "[--step-logits] [--nocache]\n", argv[0]);
        return 2;
    }
    const char *weights = argv[1], *inventory = argv[2], *config = argv[3], *ids_path = argv[4];
    size_t n_seq = (size_t)atol(argv[5]), n_prompt = (size_t)atol(argv[6]);
    size_t n_new = (size_t)atol(argv[7]);
    const char *out_path = argv[8];
    size_t first = 0;
    int transposed = 0, step_logits = 0, nocache = 0, K = 2, prefill_topk = 0;
    const char *pl = "none";
    const char *time_ctx = NULL;
    int rounds = 1;
    for (int i = 9; i < argc; ++i) {
        if (!strcmp(argv[i], "--first-seq") && i + 1 < argc) first = (size_t)atol(argv[++i]);
        else if (!strcmp(argv[i], "--cproj") && i + 1 < argc) transposed = !strcmp(argv[++i], "transposed");
        else if (!strcmp(argv[i], "--prefill-logits") && i + 1 < argc) pl = argv[++i];
        else if (!strcmp(argv[i], "--step-logits")) step_logits = 1;
        else if (!strcmp(argv[i], "--nocache")) nocache = 1;
        else if (!strcmp(argv[i], "--topk") && i + 1 < argc) K = atoi(argv[++i]);
        else if (!strcmp(argv[i], "--prefill-topk")) prefill_topk = 1;
        else if (!strcmp(argv[i], "--time-contexts") && i + 1 < argc) time_ctx = argv[++i];
        else if (!strcmp(argv[i], "--rounds") && i + 1 < argc) rounds = atoi(argv[++i]);
        else { fprintf(stderr, "unknown flag %s\n", argv[i]); return 2; }
    }
    if (K < 1 || K > 64) { fprintf(stderr, "--topk must be in [1, 64]\n"); return 2; }
    if (n_prompt == 0 || n_new == 0) { fprintf(stderr, "n_prompt and n_new must be > 0\n"); return 2; }

    FILE *fi = fopen(ids_path, "rb");
    if (!fi) { fprintf(stderr, "cannot open %s\n", ids_path); return 1; }
    fseek(fi, 0, SEEK_END);
    long ids_bytes = ftell(fi);
    fseek(fi, 0, SEEK_SET);
    size_t rows_in_file = (size_t)ids_bytes / (n_prompt * sizeof(int32_t));
    if (first + n_seq > rows_in_file) { fprintf(stderr, "ids file too short\n"); fclose(fi); return 1; }
    int32_t *all_ids = (int32_t *)malloc((size_t)ids_bytes);
    if (fread(all_ids, 1, (size_t)ids_bytes, fi) != (size_t)ids_bytes) { fclose(fi); return 1; }
    fclose(fi);

    double t0 = now_ms();
    model *m = NULL;
    model_status rc = model_load(weights, inventory, config,
                                 transposed ? MODEL_CPROJ_TRANSPOSED : MODEL_CPROJ_AS_STORED, &m);
    if (rc != MODEL_OK) { fprintf(stderr, "model_load: %s\n", model_strerror(rc)); return 1; }
    double load_ms = now_ms() - t0;
    const model_config *c = model_config_of(m);
    const size_t V = (size_t)c->vocab_size, total = n_prompt + n_new;
    if (total > (size_t)c->n_ctx + 1) { fprintf(stderr, "prompt + new exceeds n_ctx\n"); return 1; }

    if (!nocache) {
        model_set_decode_path(m, MODEL_PATH_CACHE);
        rc = model_kv_reserve(m, total - 1 < (size_t)c->n_ctx ? total - 1 : (size_t)c->n_ctx);
        if (rc != MODEL_OK) { fprintf(stderr, "kv_reserve: %s\n", model_strerror(rc)); return 1; }
    }
    rc = model_reserve(m, total);
    if (rc != MODEL_OK) { fprintf(stderr, "reserve: %s\n", model_strerror(rc)); return 1; }

    float *plog = (float *)malloc(n_prompt * V * sizeof(float));
    float *one = (float *)malloc(V * sizeof(float));
    int32_t *ids = (int32_t *)malloc(total * sizeof(int32_t));
    int32_t *gen = (int32_t *)malloc(n_new * sizeof(int32_t));
    int32_t *kid = (int32_t *)malloc(n_new * K * sizeof(int32_t));
    float *kval = (float *)malloc(n_new * K * sizeof(float));
    int32_t *pid = (int32_t *)malloc(n_prompt * K * sizeof(int32_t));
    float *pval = (float *)malloc(n_prompt * K * sizeof(float));
    float *steps = step_logits ? (float *)malloc((n_new > 1 ? n_new - 1 : 1) * V * sizeof(float)) : NULL;
    FILE *fo = fopen(out_path, "wb");
    if (!plog || !one || !ids || !gen || !kid || !kval || !pid || !pval || !fo ||
        (step_logits && !steps)) {
        fprintf(stderr, "allocation or output open failed\n");
        return 1;
    }

    if (time_ctx) {
        fclose(fo);
        int ctx[64], n_ctx = 0;
        for (const char *c = time_ctx; strcmp(time_ctx, "none") != 0 && *c && n_ctx < 64;) {
            ctx[n_ctx++] = atoi(c);
            const char *comma = strchr(c, ',');
            if (!comma) break;
            c = comma + 1;
        }
        for (int i = 0; i < n_ctx; ++i)
            if (ctx[i] <= (int)n_prompt || (size_t)ctx[i] > total - 1 || rounds < 1) {
                fprintf(stderr, "--time-contexts: each context must be in (n_prompt, n_prompt + n_new - 1]\n");
                return 2;
            }
        memcpy(ids, all_ids + first * n_prompt, n_prompt * sizeof(int32_t));
        double a = now_ms();
        rc = model_prefill(m, ids, n_prompt, plog, n_prompt * V);
        const double prefill_ms = now_ms() - a;
        if (rc != MODEL_OK) { fprintf(stderr, "prefill: %s\n", model_strerror(rc)); return 1; }
        const int32_t fill = model_argmax(plog + (n_prompt - 1) * V, V);
        for (size_t t = n_prompt; t < total; ++t) ids[t] = fill;
        printf("{\"load_ms\": %.3f, \"mode\": \"sampled\", \"n_prompt\": %zu, \"prefill_ms\": %.3f, "
               "\"contexts\": [", load_ms, n_prompt, prefill_ms);
        for (int i = 0; i < n_ctx; ++i) printf("%s%d", i ? ", " : "", ctx[i]);
        printf("], \"rounds\": [");
        for (int r = 0; r < rounds; ++r) {
            printf("%s[", r ? ", " : "");
            for (int i = 0; i < n_ctx; ++i) {
                if (model_kv_set_length(m, ctx[i] - 1) != MODEL_OK) { fprintf(stderr, "kv_set_length\n"); return 1; }
                a = now_ms();
                rc = model_decode_step_cached(m, ids, (size_t)ctx[i], one, V);
                const double ms = now_ms() - a;
                if (rc != MODEL_OK) { fprintf(stderr, "decode at %d: %s\n", ctx[i], model_strerror(rc)); return 1; }
                printf("%s%.3f", i ? ", " : "", ms);
            }
            printf("]");
            fflush(stdout);
        }
        printf("]}\n");
        model_free(m);
        return 0;
    }

    printf("{\"load_ms\": %.3f, \"n_seq\": %zu, \"n_prompt\": %zu, \"n_new\": %zu, \"seqs\": [",
           load_ms, n_seq, n_prompt, n_new);
    for (size_t s = 0; s < n_seq; ++s) {
        memcpy(ids, all_ids + (first + s) * n_prompt, n_prompt * sizeof(int32_t));
        size_t n = n_prompt;
        double a = now_ms();
        rc = model_prefill(m, ids, n, plog, n * V);
        double prefill_ms = now_ms() - a;
        if (rc != MODEL_OK) { fprintf(stderr, "prefill: %s\n", model_strerror(rc)); return 1; }
        const float *row = plog + (n - 1) * V;
        gen[0] = model_argmax(row, V);
        topk(row, V, K, kid, kval);
        if (prefill_topk)
            for (size_t t = 0; t < n_prompt; ++t)
                topk(plog + t * V, V, K, pid + t * K, pval + t * K);
        double decode_ms = 0.0;
        for (size_t g = 1; g < n_new; ++g) {
            ids[n++] = gen[g - 1];
            a = now_ms();
            rc = nocache ? model_decode_step(m, ids, n, one, V)
                         : model_decode_step_cached(m, ids, n, one, V);
            decode_ms += now_ms() - a;
            if (rc != MODEL_OK) { fprintf(stderr, "decode at %zu: %s\n", n, model_strerror(rc)); return 1; }
            gen[g] = model_argmax(one, V);
            topk(one, V, K, kid + g * K, kval + g * K);
            if (steps) memcpy(steps + (g - 1) * V, one, V * sizeof(float));
        }
        fwrite(gen, sizeof(int32_t), n_new, fo);
        fwrite(kid, sizeof(int32_t), n_new * K, fo);
        fwrite(kval, sizeof(float), n_new * K, fo);
        if (prefill_topk) {
            fwrite(pid, sizeof(int32_t), n_prompt * K, fo);
            fwrite(pval, sizeof(float), n_prompt * K, fo);
        }
        if (!strcmp(pl, "all")) fwrite(plog, sizeof(float), n_prompt * V, fo);
        else if (!strcmp(pl, "last")) fwrite(plog + (n_prompt - 1) * V, sizeof(float), V, fo);
        if (steps && n_new > 1) fwrite(steps, sizeof(float), (n_new - 1) * V, fo);
        printf("%s{\"prefill_ms\": %.3f, \"decode_ms\": %.3f, \"decode_steps\": %zu}",
               s ? ", " : "", prefill_ms, decode_ms, n_new - 1);
        fflush(stdout);
    }
    printf("]}\n");
    fclose(fo);
    model_free(m);
    free(plog); free(one); free(ids); free(gen); free(kid); free(kval); free(pid); free(pval);
    free(steps); free(all_ids);
    return 0;
}
