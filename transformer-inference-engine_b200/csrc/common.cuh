// common.cuh -- shared device helpers and launcher declarations of the engine.
#pragma once

#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace tie {

// ---------------------------------------------------------------- epilogues --
// Matmul epilogues, in the reference's operation order (src/model.c):
//   EPI_STORE       y = acc
//   EPI_BIAS        y = acc + b                       (qkv += b, model.c:687-688)
//   EPI_BIAS_GELU   y = gelu_new(acc + b)             (model.c:745-747, 615-623)
//   EPI_BIAS_RESID  x = x + (acc + b), in place       (model.c:735-737, 750-752)
//   EPI_QKV_KV      y = acc + b, and columns [E, 3E) also stored as this step's
//                   K and V rows in the paged cache   (model.c:686-688, 822-824)
enum Epi : int { EPI_STORE = 0, EPI_BIAS = 1, EPI_BIAS_GELU = 2, EPI_BIAS_RESID = 3, EPI_QKV_KV = 4 };

// Programmatic dependent launch: a kernel launched with launch_pdl may start
// while its predecessor is still running; it must call pdl_wait() before it
// reads anything the predecessor writes, and calls pdl_trigger() once the
// next kernel may be scheduled. Both are no-ops for a kernel launched without
// the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// gelu_new with every product and sum rounded separately, in the reference's
// evaluation order: inner = k * (x + ((0.044715 * x) * x) * x);
// out = (0.5 * x) * (1 + tanhf(inner)).
__device__ __forceinline__ float gelu_new_ref(float x) {
    const float k = 0.7978845608028654f;
    float cube = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
    float inner = __fmul_rn(k, __fadd_rn(x, cube));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner)));
}

template <int EPI>
__device__ __forceinline__ float apply_epi(float acc, const float* __restrict__ bias, int j,
                                           const float* resid_in) {
    if constexpr (EPI == EPI_STORE) {
        return acc;
    } else if constexpr (EPI == EPI_BIAS) {
        return __fadd_rn(acc, bias[j]);
    } else if constexpr (EPI == EPI_BIAS_GELU) {
        return gelu_new_ref(__fadd_rn(acc, bias[j]));
    } else {
        return __fadd_rn(*resid_in, __fadd_rn(acc, bias[j]));
    }
}

// ------------------------------------------------------------- LayerNorm --
// The engine's one LayerNorm arithmetic (model.c:593-610 in double, summed in a
// fixed order of its own): mean and biased variance in double, inv =
// (float)(1 / sqrt(var + eps)), y = fl(fl(fl((x - mean) * inv) * g) + b).
// Both sums run in the canonical order below, whichever kernel computes them,
// so every path normalises a row to the same bits:
//   256 virtual lanes v = 32 w + l (w = 0..7, l = 0..31); lane v adds its terms
//   i = v, v + 256, v + 512, ... in increasing i; each group w of 32 lanes is
//   reduced by an xor butterfly (offsets 16, 8, 4, 2, 1); the group sums are
//   added in group order, G0 + G1 + ... + G7.
constexpr int kLnGroups = 8;

__device__ __forceinline__ double ln_warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Group w's sum (every lane of the calling warp gets it): lane l adds the
// terms of virtual lane 32 w + l, then the butterfly.
template <typename Term>
__device__ __forceinline__ double ln_group_sum(const Term& term, int K, int w, int lane) {
    double s = 0.0;
    for (int i = 32 * w + lane; i < K; i += 32 * kLnGroups) s = __dadd_rn(s, term(i));
    return ln_warp_sum_d(s);
}

// The whole canonical sum by one warp.
template <typename Term>
__device__ __forceinline__ double ln_sum_warp(const Term& term, int K, int lane) {
    double S = ln_group_sum(term, K, 0, lane);
#pragma unroll 1
    for (int w = 1; w < kLnGroups; ++w) S = __dadd_rn(S, ln_group_sum(term, K, w, lane));
    return S;
}

// mean and inv of row xr (K floats, any memory) by one warp
__device__ __forceinline__ void ln_stats_warp(const float* xr, int K, float eps, int lane, double& mean,
                                              float& inv) {
    const double S = ln_sum_warp([&](int i) { return (double)xr[i]; }, K, lane);
    mean = S / (double)K;
    const double m = mean;
    const double V = ln_sum_warp([&](int i) {
        const double d = __dadd_rn((double)xr[i], -m);
        return __dmul_rn(d, d);
    }, K, lane);
    inv = (float)(1.0 / sqrt(__dadd_rn(V / (double)K, (double)eps)));
}

__device__ __forceinline__ float ln_apply(float x, double mean, float inv, float g, float b) {
    const float nrm = (float)__dmul_rn(__dadd_rn((double)x, -mean), (double)inv);
    return __fadd_rn(__fmul_rn(nrm, g), b);
}

// ------------------------------------------------------------ paged KV view --
// One layer's keys and values: rows of n_embd floats grouped into pages of
// kPageRows positions. Position p of sequence s lives at physical row
// page_table[s * pages_per_seq + p / kPageRows] * kPageRows + p % kPageRows.
constexpr int kPageRows = 16;

struct PagedKV {
    float* k;
    float* v;
    const int* page_table;
    int pages_per_seq;
    int n_embd;
    __device__ __forceinline__ size_t row(int seq, int pos) const {
        int page = page_table[seq * pages_per_seq + (pos >> 4)];
        return (size_t)page * kPageRows + (pos & (kPageRows - 1));
    }
};

// Attention softmax row-sum statistics (the reference's model_collect_attn_stats,
// model.c:719-726): min and max as the bit patterns of positive doubles, and
// the number of rows.
struct AttnStats {
    unsigned long long min_bits;
    unsigned long long max_bits;
    unsigned long long rows;
};

// -------------------------------------------------------------- launchers --
// All launchers enqueue on `st` and return cudaGetLastError().

// x[r] = wte[ids[r]] + wpe[r % T] for r in [0, rows)          (model.c:671-676)
cudaError_t launch_embed_prefill(const int32_t* ids, int rows, int T, const float* wte,
                                 const float* wpe, float* x, int E, int V, cudaStream_t st);
// x[b] = wte[tokens[b]] + wpe[lens[b]] for b in [0, B)       (model.c:805-809)
cudaError_t launch_embed_decode(const int32_t* tokens, const int32_t* lens, int B,
                                const float* wte, const float* wpe, float* x, int E, int V,
                                cudaStream_t st);
// y[r] = LN(x[r]) * g + b, statistics in double               (model.c:593-610)
// y (fp32) and/or its tf32 split y_hi/y_lo (the tensor-core matmul's input);
// either may be NULL.
cudaError_t launch_layernorm(const float* x, const float* g, const float* b, float* y, int rows,
                             int E, float eps, cudaStream_t st, float* y_hi = nullptr,
                             float* y_lo = nullptr);

// C[M,N] (epilogue) = A[M,K] . W[N,K]^T, tiled fp32 SIMT GEMM (prefill)
cudaError_t launch_gemm_tn(const float* A, int lda, const float* W, int ldw, const float* bias,
                           float* C, int ldc, int M, int N, int K, int epi, cudaStream_t st);
// Y[M,N] (epilogue) = X[M,K] . W[N,K]^T, streaming GEMV for small M (decode)
cudaError_t launch_gemv(const float* X, int ldx, const float* W, int ldw, const float* bias,
                        float* Y, int ldy, int M, int N, int K, int epi, cudaStream_t st);
// Head GEMV with fused argmax: logits[M,V] (optional) and per-block partial
// maxima; finalize writes next[M] (lowest index on ties, NaN never wins).
// Vocabulary rows one block of the greedy-head GEMV (launch_gemv_argmax) covers;
// its launch has gemv_argmax_blocks(N) blocks, one partial maximum per (block, row).
constexpr int kGemvArgmaxRowsPerBlock = 16;
int gemv_argmax_blocks(int N);
cudaError_t launch_gemv_argmax(const float* X, int ldx, const float* W, int ldw, float* logits,
                               int ldl, int M, int N, int K, float* part_val, int* part_idx,
                               cudaStream_t st);
cudaError_t launch_argmax_finalize(const float* part_val, const int* part_idx, int n_parts, int M,
                                   int32_t* next, cudaStream_t st);
// argmax over rows of a logits matrix (prefill last rows): next[b] = argmax(L[rows[b]])
cudaError_t launch_argmax_rows(const float* L, int ldl, int M, int N, int row_stride,
                               int row_offset, int32_t* next, cudaStream_t st);

// Stores the K and V thirds of qkv rows into the paged cache.
//   prefill: rows r = s * T + t go to (seq s, pos t)             (model.c:697-703)
//   decode:  row b goes to (seq b, pos lens[b])                  (model.c:822-824)
cudaError_t launch_kv_store_prefill(const float* qkv, int n_seq, int T, PagedKV kv, int first_seq,
                                    cudaStream_t st);
cudaError_t launch_kv_store_decode(const float* qkv, const int32_t* lens, int B, PagedKV kv,
                                   cudaStream_t st);

// Causal attention over T tokens per sequence from the fused qkv activations
// (prefill, model.c:705-732): out[r, h*D:(h+1)*D] (fp32 and/or its tf32 split).
// The outputs come from the tensor-core kernel (k_tc_attn.cu); with `stats` a
// second, FFMA pass records the softmax row sums and writes nothing else.
// `err` (may be null) is set when a bounded wait of the tensor-core kernel expires.
cudaError_t launch_attn_prefill(const float* qkv, int n_seq, int T, int H, float* out,
                                AttnStats* stats, cudaStream_t st, float* out_hi = nullptr,
                                float* out_lo = nullptr, int* err = nullptr);
cudaError_t launch_tc_attn_prefill(const float* qkv, int n_seq, int T, int H, float* out, float* out_hi,
                                   float* out_lo, int* err, cudaStream_t st);
// One query per sequence against its cached positions 0..lens[b] (the new
// position included), split over position chunks, then combined
// (model.c:826-850).
int attn_decode_max_splits(int capacity);
int attn_decode_kernels(int B);
// With `counters` (B * H ints, zero on first use; the kernel leaves them zero)
// and no statistics, one fused kernel; else split + merge kernels. `err` is
// set when a bounded wait of the large-batch kernel expires.
cudaError_t launch_attn_decode(const float* qkv, const int32_t* lens, int B, int H, PagedKV kv,
                               int max_splits, float* part, float* out, AttnStats* stats,
                               cudaStream_t st, float* out_hi = nullptr, float* out_lo = nullptr,
                               int* counters = nullptr, int* err = nullptr);

// Chunk partials of decode attention for the stream path: per (sequence b,
// head h, 16-position chunk c) the partial (max, sum, 64 weighted sums) at
// part[((b * H + h) * max_chunks + c) * 66]; merged by launch_stream_gemv's
// STREAM_PRO_MERGE prologue.
cudaError_t launch_attn_chunks(const float* qkv, const int32_t* lens, int B, int H, PagedKV kv, int max_chunks,
                               float* part, cudaStream_t st);

// Small-batch (<= 16 rows) decode matmuls with optional LayerNorm prologue
// (ln_g non-NULL) and PDL chaining (k_decode.cu). Weights fp32 (W), or with wt
// 1 / 2 the bf16 / int8 copy wq (int8 with per-row scales).
enum WeightFormat : int { WF_F32 = 0, WF_BF16 = 1, WF_INT8 = 2 };
cudaError_t launch_dec_gemv(const float* x, int ldx, const float* ln_g, const float* ln_b, float eps,
                            const float* W, const float* bias, float* y, int ldy, int M, int N, int K,
                            int epi, const PagedKV* kv, const int32_t* lens, cudaStream_t st, int wt = WF_F32,
                            const void* wq = nullptr, const float* scale = nullptr);
int dec_head_blocks(int V, int K, int wt, int M);

// The stream path for decode steps of 1-8 rows (k_decode.cu): each matmul's
// weights are staged in shared memory by bulk copies issued before the
// kernel's dependency wait, and the kernel's prologue builds its input rows --
// a copy, LayerNorm, the embedding lookup plus LayerNorm, or the merge of
// decode-attention chunk partials -- so no separate LayerNorm, embedding or
// merge kernel runs. Arithmetic and results are those of the separate kernels.
enum StreamPro : int { STREAM_PRO_PLAIN = 0, STREAM_PRO_LN = 1, STREAM_PRO_EMBED_LN = 2, STREAM_PRO_MERGE = 3 };
struct StreamParams {
    int epi;                      // EPI_BIAS, EPI_BIAS_GELU, EPI_BIAS_RESID, EPI_QKV_KV (ignored for the head)
    int head;                     // the tied head: per-CTA greedy partials instead of an epilogue
    int pro;                      // StreamPro
    int wt;                       // WeightFormat
    const float* x;               // input rows [M][ldx] (PLAIN, LN)
    int ldx;
    const float *ln_g, *ln_b;     // LN, EMBED_LN
    float eps;
    const int32_t* tokens;        // EMBED_LN: x = wte[tokens[m]] + wpe[lens[m]], also stored to x_out
    const float *wte, *wpe;
    float* x_out;
    int V;
    const float* apart;           // MERGE: launch_attn_chunks partials
    int H, max_chunks;
    const int32_t* lens;          // EMBED_LN, MERGE, EPI_QKV_KV
    const float* W;               // [N][K] fp32, or Wq bf16 / int8 with per-row scales
    const void* Wq;
    const float* scale;
    const float* bias;
    float* y;                     // [M][ldy] output (and residual input), logits for the head (optional)
    int ldy;
    int M, N, K;
    PagedKV kv;                   // EPI_QKV_KV
    float* part_val;              // head: [grid][M] partial maxima
    int* part_idx;
    int* err;                     // set when a bounded wait expires
    int stall;                    // failure drill: wait on a barrier nothing completes
    unsigned long long wait_ns;   // the bounded waits' limit (0: one second)
    unsigned long long* trace;    // NULL, or [grid][kStreamTraceEvents] global-timer stamps per CTA
};
// Stream-kernel trace, per CTA (global-timer ns): 0 entry, 1 dependency wait
// over, 2 input rows built, 3 first stage's weights landed, 4 last stage
// finished, 5 exit, 6 the producer issued its last copy.
constexpr int kStreamTraceEvents = 8;
// Whether every matmul of a decode step of M rows of a model of width E (and
// MLP width 4E) runs on the stream path; the choice depends on M and E only.
bool stream_applies(int M, int E, int wt);
// CTAs (greedy partials) of the head's launch.
int stream_head_blocks(int V, int K, int wt, int M);
cudaError_t launch_stream_gemv(const StreamParams& p, cudaStream_t st);
int dec_head_blocks_max(int V, int K);
cudaError_t launch_dec_head(const float* x, int ldx, const float* ln_g, const float* ln_b, float eps,
                            const float* W, float* logits, int ldl, int M, int V, int K, float* part_val,
                            int* part_idx, cudaStream_t st, int wt = WF_F32, const void* wq = nullptr,
                            const float* scale = nullptr);

// The reduced weight formats (k_quant.cu). bf16: q = rn(w); int8: per row,
// scale = absmax / 127, q = clamp(rint(w / scale)). deq receives the weights
// the formats stand for, in fp32.
cudaError_t launch_to_bf16(const float* w, void* q, float* deq, size_t n, cudaStream_t st);
cudaError_t launch_quant_rows(const float* w, void* q, float* scale, float* deq, int N, int K, cudaStream_t st);

// Step bookkeeping for device-resident greedy generation: tokens[b] = next[b];
// out[b * ld + *step] = next[b]; lens[b] += 1; (block 0 thread 0) *step += 1.
cudaError_t launch_step_advance(const int32_t* next, int32_t* tokens, int32_t* lens,
                                int32_t* out, int ld_out, int32_t* step, int B, cudaStream_t st);

// The naive matmul on the device (gemm_naive.c order, separately rounded).
cudaError_t launch_gemm_naive(int M, int N, int K, const float* A, int lda, const float* B,
                              int ldb, float* C, int ldc, bool bt, cudaStream_t st);
// out[c][r] = in[r][c] for an R x Cc matrix (load-time weight transpose)
cudaError_t launch_transpose(const float* in, float* out, int R, int Cc, cudaStream_t st);

// ------------------------------------------------- the persistent decode step --
// One layer's weights as the persistent step kernel reads them (k_step.cu).
struct StepLayer {
    const float *ln1_g, *ln1_b, *qkv_w, *qkv_b, *proj_w, *proj_b;
    const float *ln2_g, *ln2_b, *fc_w, *fc_b, *mlp_w, *mlp_b;
};

struct StepParams {
    const StepLayer* layers;     // [n_layer], device memory
    int n_layer, E, H, V, M;     // M: sequences of the step (1..4)
    float eps, scale;            // LayerNorm epsilon, attention 1/sqrt(head dim)
    const float *wte, *wpe, *lnf_g, *lnf_b;
    // the paged cache: layer l's rows start at k + l * layer_stride
    float *k, *v;
    size_t layer_stride;
    const int* page_table;
    int pages_per_seq;
    int max_splits;              // attention partial slots per (sequence, head)
    int32_t *tokens, *lens;      // this step's input token and position per sequence
    float *x, *qkv, *attn, *ff;  // activations, rows of E, 3E, E, 4E
    float* logits;               // [M][ldl] or NULL
    int ldl;
    float* part;                 // attention partials
    int* head_cnt;               // [M * H] arrival counters, zero between steps
    unsigned* sync;              // [step_sync_words] stage counters, zero between steps
    float* am_val;               // [grid][M] per-CTA argmax partials
    int* am_idx;
    int32_t* next;               // [M] argmax
    int advance;                 // tokens = next, lens += 1, out[m][*step] = next, *step += 1
    int32_t* out;
    int ld_out;
    int32_t* step;
    int* err;                    // set when a bounded wait expires
    int slots;                   // ring slots (from step_supported)
    int head_prefetch;           // bytes of its head rows each CTA prefetches into L2 during the layers
    unsigned long long* trace;   // [grid][step_trace_events] global-timer stamps, or NULL
};

// Whether the persistent step runs M sequences of a model of width E with H
// heads and n_layer layers on the current device; fills the ring slots and the
// grid (one CTA per SM). Each launch also needs a cache of at most
// step_max_pages() pages per sequence.
bool step_supported(int M, int E, int H, int n_layer, int* slots, int* grid);
int step_max_pages();
// The whole decode step in one cooperative launch.
cudaError_t launch_step(const StepParams& p, int grid, cudaStream_t st);
// Counters the step kernel needs zeroed: 5 per layer + 1.
inline size_t step_sync_words(int n_layer) { return 5 * (size_t)n_layer + 1; }

// Trace of one step, per CTA (global-timer nanoseconds):
//   [0]                           the consumers start
//   [1 + 3 * (5 * l + s) + k]     stage s (0..4 = A..E) of layer l; the head is
//                                 stage 5 * n_layer; k = 0 inputs ready (the
//                                 wait is over), 1 activation rows staged,
//                                 2 stage done
//   [step_trace_end(L)]           this CTA done
//   [step_trace_end(L) + 1 + i]   the producer has issued all of matrix i
//                                 (4 per layer: qkv, proj, fc, mlp; then wte)
__host__ __device__ inline int step_trace_end(int n_layer) { return 1 + 3 * (5 * n_layer + 1); }
//   [step_trace_fine(L) + 16 k + 4 j + e]  layer 1, matrix k (qkv, proj, fc,
//       mlp), ring packet j < 4: e = 0 loop top, 1 slot ready, 2 products
//       done, 3 epilogue done (consumer thread 0)
__host__ __device__ inline int step_trace_fine(int n_layer) { return step_trace_end(n_layer) + 1 + 4 * n_layer + 1; }
__host__ __device__ inline int step_trace_events(int n_layer) { return step_trace_fine(n_layer) + 64; }

}  // namespace tie
