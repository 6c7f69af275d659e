/* gpt2_oracle.c -- CPU restatement of the reference GPT-2 token loop.
 *
 * TEST INFRASTRUCTURE, NOT PRODUCT. Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg load this library, and only as the checker the
 * CUDA path is compared with. The product library never links it.
 *
 * It restates, operation for operation, the arithmetic of the reference's
 * src/model.c forward pass and src/gemm/gemm_naive.c, so that when both are
 * built with the same flags (oracle/Makefile) their logits agree BIT FOR BIT.
 * That agreement is checked by tests/test_oracle.py against the reference
 * binary (oracle/_ref/ref_gpt2) and against the committed golden vectors.
 *
 * The arithmetic being restated, with the reference line it follows:
 *   matmul          one float accumulator per output, k ascending, C written
 *                   (gemm_naive.c:30-60)
 *   LayerNorm       mean and biased variance in double, inv = (float)(1/sqrt),
 *                   then float gain and shift (model.c:593-610)
 *   gelu_new        0.5x(1 + tanhf(sqrt(2/pi)(x + 0.044715x^3))) in float
 *                   (model.c:615-623)
 *   softmax         float max, expf, double sum, float reciprocal, float scale
 *                   (model.c:629-639)
 *   block           LN1, QKV + bias, per-head scaled causal softmax attention,
 *                   projection + bias + residual, LN2, FC + bias, gelu,
 *                   MLP projection + bias + residual (model.c:671-757)
 *   head            the tied wte as the transposed operand (model.c:778-780)
 *   cached step     one token through the blocks, keys/values appended
 *                   before attention (model.c:794-868)
 *   argmax          strict '>' scan, lowest index wins ties (model.c:920-925)
 *
 * One restatement liberty, equivalent in every finite case: the reference
 * computes the full T x T score square and P.V over all T columns with the
 * upper triangle zeroed (model.c:713-731); this file stops each row at the
 * diagonal. Adding the zeroed products (+-0) to a nonzero float sum never
 * changes it.
 *
 * Weights are passed in as flat float arrays in the canonical tensor order
 * (wte, wpe, ln_f.weight, ln_f.bias, then per layer ln_1.w, ln_1.b, c_attn.w,
 * c_attn.b, c_proj.w, c_proj.b, ln_2.w, ln_2.b, c_fc.w, c_fc.b, mlp.c_proj.w,
 * mlp.c_proj.b), in the file's [input, output] layout. The caller keeps them
 * alive for the life of the oracle.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    int   n_layer, n_head, n_embd, n_ctx, vocab;
    float eps;
} orc_config;

typedef struct {
    const float *ln1_w, *ln1_b, *qkv_w, *qkv_b, *proj_w, *proj_b;
    const float *ln2_w, *ln2_b, *fc_w, *fc_b, *mlp_w, *mlp_b;
} orc_layer;

typedef struct {
    orc_config   c;
    const float *wte, *wpe, *lnf_w, *lnf_b;
    orc_layer   *layers;
    float       *proj_t;          /* transposed copies, for the TRANSPOSED reading */
    /* key/value store: per layer [capacity, n_embd], the activation layout
     * (reference kv_cache.h:10-18) */
    float       *kcache, *vcache;
    int          kv_cap, kv_len;
    /* scratch, sized for n_ctx tokens */
    float *x, *xb, *qkv, *attn, *ff, *scores;
} orc_model;

enum { ORC_OK = 0, ORC_ERR_ARG = 1, ORC_ERR_RANGE = 2, ORC_ERR_CAPACITY = 3, ORC_ERR_NOMEM = 4 };

/* ---------------------------------------------------------------- matmul -- */

/* C[MxN] = A[MxK] . B[KxN], single accumulator, k ascending (gemm_naive.c:30-44) */
void orc_gemm_naive(int M, int N, int K, const float *A, int lda, const float *B, int ldb,
                    float *C, int ldc)
{
    for (int i = 0; i < M; ++i)
        for (int j = 0; j < N; ++j) {
            float acc = 0.0f;
            for (int k = 0; k < K; ++k) acc += A[(size_t)i * lda + k] * B[(size_t)k * ldb + j];
            C[(size_t)i * ldc + j] = acc;
        }
}

/* C[MxN] = A[MxK] . Bt[NxK]^T (gemm_naive.c:46-60) */
void orc_gemm_naive_bt(int M, int N, int K, const float *A, int lda, const float *Bt, int ldbt,
                       float *C, int ldc)
{
    for (int i = 0; i < M; ++i)
        for (int j = 0; j < N; ++j) {
            float acc = 0.0f;
            for (int k = 0; k < K; ++k) acc += A[(size_t)i * lda + k] * Bt[(size_t)j * ldbt + k];
            C[(size_t)i * ldc + j] = acc;
        }
}

/* ---------------------------------------------------------- elementwise -- */

/* model.c:593-603 */
void orc_layernorm_normalize(const float *x, int n, float eps, float *out)
{
    double mean = 0.0, var = 0.0;
    for (int i = 0; i < n; ++i) mean += x[i];
    mean /= (double)n;
    for (int i = 0; i < n; ++i) { double d = x[i] - mean; var += d * d; }
    var /= (double)n;
    float inv = (float)(1.0 / sqrt(var + (double)eps));
    for (int i = 0; i < n; ++i) out[i] = (float)((x[i] - mean) * inv);
}

/* model.c:605-610 */
static void ln_affine(const float *x, const float *g, const float *b, int n, float eps, float *out)
{
    orc_layernorm_normalize(x, n, eps, out);
    for (int i = 0; i < n; ++i) out[i] = out[i] * g[i] + b[i];
}

/* model.c:615-623 */
static void gelu_new(float *v, size_t n)
{
    const float k = 0.7978845608028654f;
    for (size_t i = 0; i < n; ++i) {
        float x = v[i];
        float inner = k * (x + 0.044715f * x * x * x);
        v[i] = 0.5f * x * (1.0f + tanhf(inner));
    }
}

/* model.c:629-639 */
static void softmax_row(float *v, int n)
{
    float mx = v[0];
    for (int i = 1; i < n; ++i) if (v[i] > mx) mx = v[i];
    double sum = 0.0;
    for (int i = 0; i < n; ++i) { float e = expf(v[i] - mx); v[i] = e; sum += e; }
    float inv = (float)(1.0 / sum);
    for (int i = 0; i < n; ++i) v[i] *= inv;
}

/* model.c:920-925 */
int32_t orc_argmax(const float *v, size_t n)
{
    int32_t best = 0;
    for (size_t i = 1; i < n; ++i) if (v[i] > v[best]) best = (int32_t)i;
    return best;
}

/* ------------------------------------------------------------- lifetime -- */

void orc_free(orc_model *m)
{
    if (!m) return;
    free(m->layers); free(m->proj_t); free(m->kcache); free(m->vcache);
    free(m->x); free(m->xb); free(m->qkv); free(m->attn); free(m->ff); free(m->scores);
    free(m);
}

orc_model *orc_create(const orc_config *cfg, const float *const *t, int cproj_transposed,
                      int kv_capacity)
{
    if (!cfg || !t || cfg->n_head <= 0 || cfg->n_embd % cfg->n_head) return NULL;
    orc_model *m = (orc_model *)calloc(1, sizeof *m);
    if (!m) return NULL;
    m->c = *cfg;
    const int L = cfg->n_layer, E = cfg->n_embd;
    const size_t Tm = (size_t)cfg->n_ctx;
    m->wte = t[0]; m->wpe = t[1]; m->lnf_w = t[2]; m->lnf_b = t[3];
    m->layers = (orc_layer *)calloc((size_t)L, sizeof *m->layers);
    if (cproj_transposed) m->proj_t = (float *)malloc((size_t)L * E * E * sizeof(float));
    m->kv_cap = kv_capacity;
    if (kv_capacity > 0) {
        m->kcache = (float *)calloc((size_t)L * kv_capacity * E, sizeof(float));
        m->vcache = (float *)calloc((size_t)L * kv_capacity * E, sizeof(float));
    }
    m->x = (float *)malloc(Tm * E * sizeof(float));
    m->xb = (float *)malloc(Tm * E * sizeof(float));
    m->qkv = (float *)malloc(Tm * 3 * E * sizeof(float));
    m->attn = (float *)malloc(Tm * E * sizeof(float));
    m->ff = (float *)malloc(Tm * 4 * E * sizeof(float));
    m->scores = (float *)malloc(Tm * sizeof(float));
    if (!m->layers || (cproj_transposed && !m->proj_t) ||
        (kv_capacity > 0 && (!m->kcache || !m->vcache)) ||
        !m->x || !m->xb || !m->qkv || !m->attn || !m->ff || !m->scores) {
        orc_free(m);
        return NULL;
    }
    for (int l = 0; l < L; ++l) {
        const float *const *p = t + 4 + 12 * l;
        orc_layer *y = &m->layers[l];
        y->ln1_w = p[0]; y->ln1_b = p[1]; y->qkv_w = p[2]; y->qkv_b = p[3];
        y->proj_w = p[4]; y->proj_b = p[5]; y->ln2_w = p[6]; y->ln2_b = p[7];
        y->fc_w = p[8]; y->fc_b = p[9]; y->mlp_w = p[10]; y->mlp_b = p[11];
        if (cproj_transposed) {           /* model.c:435, transpose_square at load */
            float *d = m->proj_t + (size_t)l * E * E;
            for (int i = 0; i < E; ++i)
                for (int j = 0; j < E; ++j) d[(size_t)i * E + j] = p[4][(size_t)j * E + i];
            y->proj_w = d;
        }
    }
    return m;
}

int  orc_kv_length(const orc_model *m) { return m ? m->kv_len : 0; }
int  orc_kv_set_length(orc_model *m, int n)
{
    if (!m || n < 0) return ORC_ERR_ARG;
    if (n > m->kv_cap) return ORC_ERR_CAPACITY;
    m->kv_len = n;
    return ORC_OK;
}

/* --------------------------------------------------------------- forward -- */

/* One causal attention row: query q (stride-free, D floats) against keys/values
 * rows 0..n-1 at stride ld, output D floats. The same reduction order as
 * mul_bt(1, n, D) + scale + softmax + mul(1, D, n) (model.c:713-731, 836-849). */
static void attend_row(const float *q, const float *k, const float *v, int ld, int n, int D,
                       float scale, float *scores, float *out)
{
    for (int j = 0; j < n; ++j) {
        float acc = 0.0f;
        for (int d = 0; d < D; ++d) acc += q[d] * k[(size_t)j * ld + d];
        scores[j] = acc;
    }
    for (int j = 0; j < n; ++j) scores[j] *= scale;
    softmax_row(scores, n);
    for (int d = 0; d < D; ++d) {
        float acc = 0.0f;
        for (int j = 0; j < n; ++j) acc += scores[j] * v[(size_t)j * ld + d];
        out[d] = acc;
    }
}

/* The blocks over T tokens starting at position p0 of x (rows p0..p0+T-1 hold
 * fresh embeddings). Keys/values of attention come from the activation buffer
 * (prefill, cache==NULL use) or from the cache (cached step). Leaves LN_f(x) in
 * xb. model.c:647-763 and 794-868. */
static int run_blocks(orc_model *m, const int32_t *ids, int T, int write_cache, int cached_step)
{
    const orc_config *c = &m->c;
    const int E = c->n_embd, H = c->n_head, D = E / H, E3 = 3 * E, E4 = 4 * E;
    const float scale = (float)(1.0 / sqrt((double)D));
    const int first_pos = cached_step ? T - 1 : 0;   /* position of row 0 */
    const int rows = cached_step ? 1 : T;

    for (int r = 0; r < rows; ++r) {                 /* model.c:671-676, 805-809 */
        const int pos = first_pos + r;
        const float *we = m->wte + (size_t)ids[pos] * E, *pe = m->wpe + (size_t)pos * E;
        for (int i = 0; i < E; ++i) m->x[(size_t)r * E + i] = we[i] + pe[i];
    }
    for (int l = 0; l < c->n_layer; ++l) {
        const orc_layer *y = &m->layers[l];
        float *kc = m->kcache ? m->kcache + (size_t)l * m->kv_cap * E : NULL;
        float *vc = m->vcache ? m->vcache + (size_t)l * m->kv_cap * E : NULL;
        for (int r = 0; r < rows; ++r)
            ln_affine(m->x + (size_t)r * E, y->ln1_w, y->ln1_b, E, c->eps, m->xb + (size_t)r * E);
        orc_gemm_naive(rows, E3, E, m->xb, E, y->qkv_w, E3, m->qkv, E3);
        for (int r = 0; r < rows; ++r)
            for (int j = 0; j < E3; ++j) m->qkv[(size_t)r * E3 + j] += y->qkv_b[j];
        if (write_cache || cached_step)              /* model.c:697-703, 822-824 */
            for (int r = 0; r < rows; ++r) {
                memcpy(kc + (size_t)(first_pos + r) * E, m->qkv + (size_t)r * E3 + E, E * sizeof(float));
                memcpy(vc + (size_t)(first_pos + r) * E, m->qkv + (size_t)r * E3 + 2 * E, E * sizeof(float));
            }
        for (int h = 0; h < H; ++h)
            for (int r = 0; r < rows; ++r) {
                const float *q = m->qkv + (size_t)r * E3 + (size_t)h * D;
                float *o = m->attn + (size_t)r * E + (size_t)h * D;
                if (cached_step)
                    attend_row(q, kc + (size_t)h * D, vc + (size_t)h * D, E, T, D, scale, m->scores, o);
                else
                    attend_row(q, m->qkv + E + (size_t)h * D, m->qkv + 2 * E + (size_t)h * D, E3,
                               r + 1, D, scale, m->scores, o);
            }
        orc_gemm_naive(rows, E, E, m->attn, E, y->proj_w, E, m->xb, E);   /* model.c:734-737 */
        for (int r = 0; r < rows; ++r)
            for (int i = 0; i < E; ++i)
                m->x[(size_t)r * E + i] += m->xb[(size_t)r * E + i] + y->proj_b[i];
        for (int r = 0; r < rows; ++r)
            ln_affine(m->x + (size_t)r * E, y->ln2_w, y->ln2_b, E, c->eps, m->xb + (size_t)r * E);
        orc_gemm_naive(rows, E4, E, m->xb, E, y->fc_w, E4, m->ff, E4);     /* model.c:744-747 */
        for (int r = 0; r < rows; ++r)
            for (int j = 0; j < E4; ++j) m->ff[(size_t)r * E4 + j] += y->fc_b[j];
        gelu_new(m->ff, (size_t)rows * E4);
        orc_gemm_naive(rows, E, E4, m->ff, E4, y->mlp_w, E, m->xb, E);     /* model.c:749-752 */
        for (int r = 0; r < rows; ++r)
            for (int i = 0; i < E; ++i)
                m->x[(size_t)r * E + i] += m->xb[(size_t)r * E + i] + y->mlp_b[i];
    }
    for (int r = 0; r < rows; ++r)
        ln_affine(m->x + (size_t)r * E, m->lnf_w, m->lnf_b, E, c->eps, m->xb + (size_t)r * E);
    if (write_cache || cached_step) m->kv_len = T;
    return ORC_OK;
}

static int check_ids(const orc_model *m, const int32_t *ids, int T)
{
    if (!m || !ids || T <= 0) return ORC_ERR_ARG;
    if (T > m->c.n_ctx) return ORC_ERR_RANGE;
    for (int t = 0; t < T; ++t) if (ids[t] < 0 || ids[t] >= m->c.vocab) return ORC_ERR_RANGE;
    return ORC_OK;
}

/* Prefill (model.c:765-782): logits at every position into logits_all (T x V)
 * when it is non-NULL, and the last row into logits_last when that is. */
int orc_prefill(orc_model *m, const int32_t *ids, int T, float *logits_all, float *logits_last,
                int write_cache)
{
    int rc = check_ids(m, ids, T);
    if (rc) return rc;
    if (write_cache && T > m->kv_cap) return ORC_ERR_CAPACITY;
    run_blocks(m, ids, T, write_cache, 0);
    const int E = m->c.n_embd, V = m->c.vocab;
    if (logits_all) orc_gemm_naive_bt(T, V, E, m->xb, E, m->wte, E, logits_all, V);
    if (logits_last)
        orc_gemm_naive_bt(1, V, E, m->xb + (size_t)(T - 1) * E, E, m->wte, E, logits_last, V);
    return ORC_OK;
}

/* Cached decode step at context T (model.c:870-896). */
int orc_decode_cached(orc_model *m, const int32_t *ids, int T, float *logits)
{
    int rc = check_ids(m, ids, T);
    if (rc) return rc;
    if (!m->kcache || T > m->kv_cap) return ORC_ERR_CAPACITY;
    if (m->kv_len != T - 1) return ORC_ERR_ARG;
    run_blocks(m, ids, T, 0, 1);
    const int E = m->c.n_embd, V = m->c.vocab;
    orc_gemm_naive_bt(1, V, E, m->xb, E, m->wte, E, logits, V);
    return ORC_OK;
}

/* No-cache decode step (model.c:898-918): the whole context again, head once. */
int orc_decode_nocache(orc_model *m, const int32_t *ids, int T, float *logits)
{
    return orc_prefill(m, ids, T, NULL, logits, 0);
}

/* The greedy loop of main.c:274-287 on the cached path: prefill, then one
 * cached step per further token. Records each chosen token and the top-1 and
 * runner-up logit of the row it came from. */
int orc_greedy(orc_model *m, const int32_t *prompt, int T, int n_new, int32_t *out,
               float *top1, float *top2)
{
    if (!m || !prompt || !out || T <= 0 || n_new <= 0) return ORC_ERR_ARG;
    if (T + n_new - 1 > m->kv_cap) return ORC_ERR_CAPACITY;
    const int V = m->c.vocab;
    int32_t *ids = (int32_t *)malloc((size_t)(T + n_new) * sizeof(int32_t));
    float *row = (float *)malloc((size_t)V * sizeof(float));
    if (!ids || !row) { free(ids); free(row); return ORC_ERR_NOMEM; }
    memcpy(ids, prompt, (size_t)T * sizeof(int32_t));
    int rc = orc_prefill(m, ids, T, NULL, row, 1);
    int n = T;
    for (int g = 0; rc == ORC_OK && g < n_new; ++g) {
        if (g > 0) rc = orc_decode_cached(m, ids, n, row);
        if (rc) break;
        int32_t b = orc_argmax(row, (size_t)V);
        float second = -3.4e38f;
        for (int i = 0; i < V; ++i) if (i != b && row[i] > second) second = row[i];
        out[g] = b;
        if (top1) top1[g] = row[b];
        if (top2) top2[g] = second;
        ids[n++] = b;
    }
    free(ids); free(row);
    return rc;
}
