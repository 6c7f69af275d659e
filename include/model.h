/* model.h -- GPT-2 forward, prefill and decode on one B200 (sm_100a).
 *
 * Drop-in for the reference's src/model.h (lines 53-249). Every declaration the
 * reference exports is here with the same name, signature, enum values and
 * struct layout, so a caller written against the reference (its gpt2_tool, its
 * timing driver, its unit tests) builds against this header unchanged. The one
 * ABI addition is MODEL_ERR_DEVICE, appended to the status enum.
 *
 * What runs underneath: model_load uploads the weights to device memory once;
 * every forward pass after that is hand-written sm_100a kernels (embedding,
 * LayerNorm, streaming GEMV / tiled GEMM with fused epilogues, paged causal
 * attention, tied head with fused argmax). No arithmetic of the token loop runs
 * on the CPU.
 *
 * Contract kept from the reference:
 *   - every architecture value comes from config.json, every tensor's dtype,
 *     shape, offset and length from the inventory cross-checked against the
 *     weight file header (model.h:5-10, model.c:287-317, 354-389);
 *   - caller-owned HOST output buffers with capacities in floats, checked before
 *     any work (model.h:27-30);
 *   - refusals happen before any arithmetic and leave the cache untouched
 *     (model.c:660-668, 878-883);
 *   - the decode-path switch defaults to no-cache, and the cache is allocated
 *     lazily (model.h:79-93, 186-192);
 *   - a model is owned by one host thread at a time (model.c:229-236).
 *
 * Differences a caller can observe, each deliberate:
 *   - model_token_embedding / model_head_weight return the same DEVICE pointer
 *     (the tie is storage identity, as in the reference; do not dereference it
 *     on the host);
 *   - model_set_gemm records the caller's choice but the forward pass always
 *     runs the engine's own kernels (there is no CPU matmul to substitute);
 *     model_gemm_of returns &gemm_impl_sm100a;
 *   - logits are computed in fp32 with a different summation order than the
 *     reference's single-accumulator loops, so they agree with it to a
 *     tolerance (max-abs <= 1e-3 by contract), not bit for bit.
 */
#ifndef TIE_B200_MODEL_H
#define TIE_B200_MODEL_H

#include <stddef.h>
#include <stdint.h>

#include "gemm.h"
#include "kv_cache.h"

#ifdef __cplusplus
extern "C" {
#endif

/* reference src/model.h:53-66, plus MODEL_ERR_DEVICE (additive, last) */
typedef enum {
    MODEL_OK = 0,
    MODEL_ERR_OPEN,           /* an artifact could not be opened                 */
    MODEL_ERR_CONFIG,         /* config.json lacks a field, or names an
                                 unsupported architecture                        */
    MODEL_ERR_INVENTORY,      /* inventory missing a tensor or disagreeing with
                                 the weight file header                          */
    MODEL_ERR_WEIGHTS,        /* the weight file failed to open, parse or read   */
    MODEL_ERR_SHAPE,          /* a tensor's shape contradicts the config         */
    MODEL_ERR_DTYPE,          /* a tensor is not F32                             */
    MODEL_ERR_RANGE,          /* token id or position out of the model's range   */
    MODEL_ERR_CAPACITY,       /* a caller-owned buffer or the cache is too small */
    MODEL_ERR_NOMEM,          /* host or device allocation failed                */
    MODEL_ERR_ARG,            /* null or unusable argument                       */
    MODEL_ERR_DEVICE          /* a CUDA call failed (no device, launch error)    */
} model_status;

/* reference src/model.h:74-77 */
typedef enum {
    MODEL_CPROJ_AS_STORED  = 0,
    MODEL_CPROJ_TRANSPOSED = 1
} model_cproj_reading;

/* reference src/model.h:90-93 */
typedef enum {
    MODEL_PATH_NOCACHE = 0,
    MODEL_PATH_CACHE   = 1
} model_decode_path;

/* reference src/model.h:97-106 (identical layout) */
typedef struct {
    int    n_layer;
    int    n_head;
    int    n_embd;
    int    n_ctx;
    int    vocab_size;
    int    head_dim;
    float  layer_norm_epsilon;
    char   activation_function[32];
} model_config;

typedef struct model model;

/* reference model.h:117-122. Loads onto the current CUDA device. The
 * h.*.attn.bias mask buffers are not read (causality is a loop bound). */
model_status model_load(const char *weights_path,
                        const char *inventory_path,
                        const char *config_path,
                        model_cproj_reading cproj_reading,
                        model **out);
void model_free(model *m);

/* reference model.h:124-125 */
const model_config *model_config_of(const model *m);
model_cproj_reading model_cproj_reading_of(const model *m);

/* reference model.h:133-142 (identical layout) */
typedef struct {
    char name[64];
    char stored_shape[32];
    char inventory_orientation[48];
    int  transposed_at_load;
    char reconciliation[96];
} model_tensor_record;

size_t                     model_tensor_record_count(const model *m);
const model_tensor_record *model_tensor_record_at(const model *m, size_t i);

/* reference model.h:146-147 (see the header note on what set_gemm does here) */
void              model_set_gemm(model *m, const gemm_impl *impl);
const gemm_impl  *model_gemm_of(const model *m);

/* reference model.h:152. Grows device scratch for prefills of up to
 * max_tokens; call it outside timed regions. */
model_status model_reserve(model *m, size_t max_tokens);

/* reference model.h:166-167. Logits for every position into a HOST buffer of
 * logits_cap floats (>= n_ids * vocab_size). Under MODEL_PATH_CACHE also
 * writes every position's keys and values and sets the cache length. */
model_status model_prefill(model *m, const int32_t *ids, size_t n_ids,
                           float *logits_out, size_t logits_cap);

/* reference model.h:176-177. Logits of the last position only. */
model_status model_decode_step(model *m, const int32_t *ids, size_t n_ids,
                               float *logits_out, size_t logits_cap);

/* reference model.h:183-184 */
void              model_set_decode_path(model *m, model_decode_path p);
model_decode_path model_decode_path_of(const model *m);

/* reference model.h:192-201 */
model_status    model_kv_reserve(model *m, size_t capacity);
size_t          model_kv_footprint_bytes(const model *m);
int             model_kv_capacity(const model *m);
int             model_kv_length(const model *m);
model_status    model_kv_set_length(model *m, int length);
const kv_cache *model_kv_cache_of(const model *m);

/* reference model.h:219-220. Positions 0..n_ids-2 must already be cached. */
model_status model_decode_step_cached(model *m, const int32_t *ids, size_t n_ids,
                                      float *logits_out, size_t logits_cap);

/* reference model.h:223. Host scan over a host buffer, lowest index on ties. */
int32_t model_argmax(const float *logits, size_t n);

/* reference model.h:231-232. Same device pointer for both (tied head). */
const float *model_token_embedding(const model *m);
const float *model_head_weight(const model *m);

/* reference model.h:239. Host utility with the engine's LayerNorm
 * normalisation (double statistics); x and out are host arrays. */
void model_layernorm_normalize(const float *x, int n, float eps, float *out);

/* reference model.h:245-247. When enabled, every softmax row the device
 * computes contributes its sum to a min/max pair (read back after each call). */
void model_collect_attn_stats(model *m, int enable);
void model_attn_rowsum_range(const model *m, double *out_min, double *out_max,
                             size_t *out_rows);

/* reference model.h:249 */
const char *model_strerror(model_status s);

#ifdef __cplusplus
}
#endif

#endif /* TIE_B200_MODEL_H */
