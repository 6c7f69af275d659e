/* tie_b200.h -- additive entry points of the B200 GPT-2 engine.
 *
 * Nothing here replaces a reference declaration; these are the additions that
 * the reference's single-sequence, host-logits API cannot express, listed in
 * the reference's own terms:
 *
 *   - a greedy step that keeps the logits on the device and returns only the
 *     argmax (the reference's greedy loop, src/main.c:274-287, copies a full
 *     vocabulary row to the host every step and scans it there);
 *   - batches of independent sequences sharing one model and one paged KV pool
 *     (the reference has exactly one sequence per model, src/model.c:216-245);
 *   - a whole greedy generation (prefill + every decode step) in one call, with
 *     the token ids staying on the device between steps;
 *   - access to the device and stream the model runs on, for callers that time
 *     or order work around it.
 *
 * All functions validate their arguments before launching any work and return
 * a model_status (include/model.h).
 */
#ifndef TIE_B200_TIE_H
#define TIE_B200_TIE_H

#include <stddef.h>
#include <stdint.h>

#include "model.h"

#ifdef __cplusplus
extern "C" {
#endif

/* model_load onto an explicit CUDA device ordinal (model_load uses the
 * calling thread's current device). */
model_status model_load_on_device(const char *weights_path, const char *inventory_path,
                                  const char *config_path, model_cproj_reading cproj_reading,
                                  int device, model **out);

/* The device ordinal and the cudaStream_t (as void*) every kernel of this model
 * is launched on. */
int   model_device(const model *m);
void *model_stream(const model *m);

/* Device bytes held by the weights (all layouts), and the number of kernels
 * this library has launched for the model since load (graph replays count each
 * node). */
size_t   model_weight_device_bytes(const model *m);
uint64_t model_kernel_launches(const model *m);

/* Cached decode step at context n_ids (same preconditions as
 * model_decode_step_cached) that returns only the greedy choice. */
model_status model_decode_step_greedy(model *m, const int32_t *ids, size_t n_ids, int32_t *next_id);

/* ---- batches of independent sequences --------------------------------------
 * model_batch_reserve sizes a paged KV pool and scratch for n_seq sequences of
 * up to `capacity` positions each (pages of KV_CACHE_PAGE_ROWS positions, page
 * tables on the device). It is separate from the single-sequence cache of
 * model_kv_reserve; the batch calls below use only the pool. Extends the
 * reference's kv_cache_create (src/kv_cache.c:150-190) to many sequences. */
model_status model_batch_reserve(model *m, size_t n_seq, size_t capacity);

/* The same pool over a bounded number of physical pages: n_pages pages of
 * KV_CACHE_PAGE_ROWS positions per layer (0: enough for every sequence's whole
 * capacity, which is what model_batch_reserve reserves), plus one scratch page.
 * No page belongs to a sequence until a batch call needs it: prefill assigns
 * the pages its prompt covers, each decode step the page its new position
 * opens, from a free list. A call that finds too few free pages returns
 * MODEL_ERR_CAPACITY before it launches the step (pages assigned by earlier
 * steps stay assigned). n_pages above n_seq * ceil(capacity / 16) is
 * MODEL_ERR_ARG. */
model_status model_batch_reserve_pages(model *m, size_t n_seq, size_t capacity, size_t n_pages);

/* Returns sequence `seq`'s pages to the pool's free list (a finished sequence,
 * so that others can grow into its pages). Its positions are then unmapped;
 * the next prefill that includes it assigns pages again. */
model_status model_batch_release(model *m, size_t seq);

/* Pages of the pool not assigned to any sequence (0 without a pool). */
size_t model_batch_free_pages(const model *m);

/* Prefill of n_seq sequences of n_ids tokens each (ids: host, n_seq * n_ids,
 * row-major). Writes every position's keys and values into the pool and sets
 * each sequence's length to n_ids. logits_out (host, n_seq * n_ids * vocab
 * floats, or NULL for none) receives all positions' logits; next_ids (host,
 * n_seq, or NULL) receives each sequence's greedy choice at its last position. */
model_status model_prefill_batch(model *m, const int32_t *ids, size_t n_seq, size_t n_ids,
                                 float *logits_out, size_t logits_cap, int32_t *next_ids);

/* One cached decode step for every sequence of the batch: token ids[s] is
 * appended at sequence s's current length, which then grows by one. logits_out
 * (host, n_seq * vocab floats, or NULL) and next_ids (host, n_seq, or NULL). */
model_status model_decode_step_batch(model *m, const int32_t *ids, size_t n_seq,
                                     float *logits_out, size_t logits_cap, int32_t *next_ids);

/* Greedy generation: prefill of n_prompt tokens for each of n_seq sequences,
 * then n_new greedy tokens each (n_new - 1 decode steps; the first new token
 * comes from the prefill's last row), all on the device. prompts: host,
 * n_seq * n_prompt; out_ids: host, n_seq * n_new. Requires a prior
 * model_batch_reserve covering n_seq sequences of n_prompt + n_new - 1
 * positions. The decode steps run as CUDA-graph replays. */
model_status model_generate_greedy(model *m, const int32_t *prompts, size_t n_seq,
                                   size_t n_prompt, size_t n_new, int32_t *out_ids);

/* Device-resident variant for timing the kernels alone: prompts and out_ids are
 * DEVICE buffers of the same shapes; no host copies, no synchronisation. */
model_status model_generate_greedy_device(model *m, const int32_t *d_prompts, size_t n_seq,
                                          size_t n_prompt, size_t n_new, int32_t *d_out_ids);

/* ---- diagnostics --------------------------------------------------------
 * Times `iters` back-to-back launches of one kernel of the forward pass, alone,
 * on the model's stream with CUDA events, and stores the average milliseconds
 * per launch (the numbers a roofline is computed from). It runs on the batch
 * pool and scratch of model_batch_reserve, which must cover `rows` sequences of
 * `context` positions, and overwrites their contents and the decode state.
 *   TIE_KERNEL_DECODE_ATTENTION  one layer's decode attention (split + merge),
 *                                `rows` sequences at context `context`
 *   TIE_KERNEL_DECODE_QKV        the QKV matmul of a decode step, `rows` rows
 *   TIE_KERNEL_DECODE_FC         the MLP up-projection (+ GELU) of a decode step
 *   TIE_KERNEL_DECODE_MLP_PROJ   the MLP down-projection (+ residual)
 *   TIE_KERNEL_DECODE_HEAD       the tied head with its fused argmax
 *   TIE_KERNEL_PREFILL_ATTENTION causal attention over `context` tokens x `rows`
 *   TIE_KERNEL_PREFILL_FC        the MLP up-projection over rows * context tokens
 *   TIE_KERNEL_DECODE_STEP       one whole decode step of `rows` (<= 4) sequences
 *                                at context `context` as the persistent kernel */
enum {
    TIE_KERNEL_DECODE_ATTENTION = 0,
    TIE_KERNEL_DECODE_QKV = 1,
    TIE_KERNEL_DECODE_FC = 2,
    TIE_KERNEL_DECODE_MLP_PROJ = 3,
    TIE_KERNEL_DECODE_HEAD = 4,
    TIE_KERNEL_PREFILL_ATTENTION = 5,
    TIE_KERNEL_PREFILL_FC = 6,
    TIE_KERNEL_DECODE_STEP = 7
};
model_status model_time_kernel(model *m, int kernel, size_t rows, size_t context, int iters,
                               float *avg_ms);

/* ---- weight formats --------------------------------------------------------
 * The reference computes in fp32 only. These formats trade weight precision
 * for HBM traffic in the memory-bound decode:
 *   TIE_WEIGHTS_F32   the loaded weights (the default).
 *   TIE_WEIGHTS_BF16  each matrix element rounded to nearest-even bf16.
 *   TIE_WEIGHTS_INT8  per output channel (a row of each [out, in] matrix):
 *                     scale = absmax(row) / 127 in fp32, q = rint(w / scale)
 *                     (ties to even) clamped to +-127; the weight is q * scale.
 * The formats apply to the five matrix kinds -- qkv, attention proj, fc, mlp
 * proj, and the tied wte (head and embedding lookup alike); LayerNorm, biases
 * and wpe stay fp32. Accumulation is fp32 throughout. Decode steps of at most
 * 8 sequences stream the compact copies (2 or 1 byte per element); every other
 * path computes with the fp32 values the copies stand for, so the model is the
 * same model whichever kernels run. A format's copies are built on the device
 * on first selection and kept. */
enum { TIE_WEIGHTS_F32 = 0, TIE_WEIGHTS_BF16 = 1, TIE_WEIGHTS_INT8 = 2 };
model_status model_set_weight_format(model *m, int fmt);
int model_weight_format(const model *m);

/* The last CUDA failure behind a MODEL_ERR_DEVICE on the calling thread: the
 * error's name and text and the failing call, or "" if none yet. With the
 * environment variable TIE_DEBUG set, each such failure is also printed to
 * stderr. */
const char *tie_last_device_error(void);

/* The causal prefill attention of the engine (model.c:705-732, the step
 * between the QKV projection and the output projection) over HOST arrays, for
 * tests of the kernel alone: qkv is n_seq x T rows of 3 * n_head * 64 floats
 * (q, k, v of every head, the layout of the fused projection's output) and out
 * receives n_seq x T rows of n_head * 64. Runs on the current device; returns
 * MODEL_ERR_ARG for a null pointer or a non-positive size, MODEL_ERR_DEVICE on
 * a CUDA failure or an expired wait. */
model_status tie_attention_prefill(const float *qkv, int n_seq, int T, int n_head, float *out);

/* ---- how small decode steps run ------------------------------------------
 * A decode step of at most 8 sequences runs as a chain of per-layer kernels
 * linked by programmatic dependent launch: TIE_STEP_CHAINED, the default
 * (LayerNorm, QKV + the step's K/V rows, attention, projection + residual,
 * LayerNorm, FC + GELU, MLP projection + residual; each matmul's weights are
 * loaded into registers ahead of its dependency wait). TIE_STEP_STREAM runs
 * the same arithmetic as five kernels per layer: the weights are bulk-copied
 * into shared memory ahead of the wait, and LayerNorm, the embedding lookup
 * and the merge of attention chunk partials run in the matmuls' prologues. With
 * TIE_STEP_PERSISTENT a step of at most 4 sequences (fp32 weights, without
 * attention statistics) runs as ONE persistent kernel. All three form every
 * sum in the same order, so they return identical logits and tokens; the
 * switch exists to compare and time them. MODEL_ERR_ARG for any other value. */
enum { TIE_STEP_PERSISTENT = 0, TIE_STEP_CHAINED = 1, TIE_STEP_STREAM = 2 };

/* Failure drill for the bounded waits: the next decode step that runs on the
 * default chained path (at most 8 sequences, no attention statistics) has its
 * first matmul wait on a shared-memory barrier that nothing completes. The
 * wait gives up after limit_ns nanoseconds, the kernel records the expiry in
 * the model's device error flag and returns, and the step's call returns
 * MODEL_ERR_DEVICE with the cache length unchanged; the next step runs
 * normally. Every bounded wait of the engine's kernels reports through the
 * same flag. MODEL_ERR_ARG for a NULL model or a zero limit. No counterpart in
 * the reference (its CPU engine has no device waits). */
model_status model_debug_wait_drill(model *m, uint64_t limit_ns);

/* Trace of one decode step of `rows` (<= 8) sequences at context `context` on
 * the TIE_STEP_STREAM path (the batch pool must cover them; contents are
 * overwritten as for model_time_kernel): for each of its 4 * n_layer + 1
 * streaming matmul kernels in launch order, *per_kernel global-timer stamps
 * (ns) -- 256 CTA slots of 8 events: entry, dependency wait over, input rows
 * built, first weights landed, last stage done, exit, producer done (0 where
 * no CTA ran) -- written to out (host, cap >= *per_kernel * *n_kernels;
 * *per_kernel and *n_kernels are set even when the capacity is short, which
 * returns MODEL_ERR_CAPACITY). MODEL_ERR_ARG when the step would not take that
 * path. No counterpart in the reference. */
model_status model_stream_trace(model *m, size_t rows, size_t context, uint64_t *out, size_t cap,
                                size_t *per_kernel, size_t *n_kernels);

model_status model_set_step_kernel(model *m, int kind);

/* Trace of one persistent decode step of `rows` (<= 4) sequences at context
 * `context` on the batch pool (model_batch_reserve must cover them; contents
 * are overwritten as for model_time_kernel): per CTA, *per_cta global-timer
 * stamps in nanoseconds, *n_cta CTAs, written to out (host, cap >= per_cta *
 * n_cta, else MODEL_ERR_CAPACITY after filling the two counts). Stamp order per
 * CTA: [0] start; [1 + 3 * (5 * layer + stage) + k] for stage 0..4 (LN1+qkv,
 * attention, proj, LN2+fc, mlp) with k = 0 inputs ready, 1 rows staged, 2 done,
 * the head as stage 5 * n_layer; then the CTA's end; then, per weight matrix in
 * stream order (qkv, proj, fc, mlp per layer, then wte), when its last copy was
 * issued. */
model_status model_step_trace(model *m, size_t rows, size_t context, uint64_t *out, size_t cap,
                              size_t *per_cta, size_t *n_cta);

/* ---- the greedy head without allocation --------------------------------
 * No counterpart in the reference (its head is a CPU matmul over host memory).
 * For callers that cannot allocate device memory -- a serving framework whose
 * caching allocator already holds the GPU's memory, a plugin inside a runtime
 * that forbids allocations outside its own allocator, a latency-bound loop that
 * cannot take cudaMalloc's implicit device synchronisation.
 *
 * next[r] = argmax_j (x[r] . w[j]) for r < rows (lowest index on ties), and,
 * when `logits` is non-NULL, logits[r * ldl + j] = x[r] . w[j]. x (rows x k,
 * leading dimension ldx), w (vocab x k, ldw), logits and next are DEVICE
 * pointers; x and w 16-byte aligned, k, ldx and ldw multiples of 4. Work is
 * enqueued on `stream` (a cudaStream_t; NULL for the legacy default stream)
 * and not waited for.
 *
 * Limits: rows <= 16 and vocab <= 65536, else MODEL_ERR_CAPACITY. The per-block
 * partial maxima live in a fixed 512 KiB array inside the library, present on
 * every GPU that loads it until the process exits; nothing is allocated per
 * call. The array's device address is looked up on the first call made on each
 * device (with that device current); make that first call before any stream
 * capture. Every call shares the array, so calls that overlap on the GPU race
 * on it. */
model_status tie_head_argmax_noalloc(const float *x, int ldx, const float *w, int ldw, int rows,
                                     int vocab, int k, float *logits, int ldl, int32_t *next,
                                     void *stream);

#ifdef __cplusplus
}
#endif

#endif /* TIE_B200_TIE_H */
