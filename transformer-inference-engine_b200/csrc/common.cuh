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
// (prefill, model.c:705-732): out[r, h*D:(h+1)*D].
cudaError_t launch_attn_prefill(const float* qkv, int n_seq, int T, int H, float* out,
                                AttnStats* stats, cudaStream_t st, float* out_hi = nullptr,
                                float* out_lo = nullptr);
// One query per sequence against its cached positions 0..lens[b] (the new
// position included), split over position chunks, then combined
// (model.c:826-850).
int attn_decode_max_splits(int capacity);
// With `counters` (B * H ints, zero on first use; the kernel leaves them zero)
// and no statistics, one fused kernel; else split + merge kernels.
cudaError_t launch_attn_decode(const float* qkv, const int32_t* lens, int B, int H, PagedKV kv,
                               int max_splits, float* part, float* out, AttnStats* stats,
                               cudaStream_t st, float* out_hi = nullptr, float* out_lo = nullptr,
                               int* counters = nullptr);

// Small-batch (<= 16 rows) decode matmuls with optional LayerNorm prologue
// (ln_g non-NULL) and PDL chaining (k_decode.cu).
cudaError_t launch_dec_gemv(const float* x, int ldx, const float* ln_g, const float* ln_b, float eps,
                            const float* W, const float* bias, float* y, int ldy, int M, int N, int K,
                            int epi, const PagedKV* kv, const int32_t* lens, cudaStream_t st);
int dec_head_blocks(int V);
cudaError_t launch_dec_head(const float* x, int ldx, const float* ln_g, const float* ln_b, float eps,
                            const float* W, float* logits, int ldl, int M, int V, int K, float* part_val,
                            int* part_idx, cudaStream_t st);

// Step bookkeeping for device-resident greedy generation: tokens[b] = next[b];
// out[b * ld + *step] = next[b]; lens[b] += 1; (block 0 thread 0) *step += 1.
cudaError_t launch_step_advance(const int32_t* next, int32_t* tokens, int32_t* lens,
                                int32_t* out, int ld_out, int32_t* step, int B, cudaStream_t st);

// The naive matmul on the device (gemm_naive.c order, separately rounded).
cudaError_t launch_gemm_naive(int M, int N, int K, const float* A, int lda, const float* B,
                              int ldb, float* C, int ldc, bool bt, cudaStream_t st);
// out[c][r] = in[r][c] for an R x Cc matrix (load-time weight transpose)
cudaError_t launch_transpose(const float* in, float* out, int R, int Cc, cudaStream_t st);

}  // namespace tie
