/* gemm.h -- the matmul interface of the GPT-2 engine, served on a B200.
 *
 * Drop-in for the reference's src/gemm/gemm.h (lines 55-89): the same two
 * operation types, the same gemm_impl record and the same exported names, so a
 * caller written against the reference compiles and links unchanged.
 *
 * Semantics kept from the reference (gemm.h:14-42):
 *   row-major operands with explicit leading dimensions;
 *   mul:    C[M,N] = A[M,K] . B[K,N]      B(k,j) at B[k*ldb + j]
 *   mul_bt: C[M,N] = A[M,K] . Bt[N,K]^T   Bt(j,k) at Bt[j*ldbt + k]
 *   C is written, never accumulated; K == 0 writes zeros; M == 0 or N == 0
 *   writes nothing.
 *
 * What is different, and why: every product here is computed on the GPU.
 * Operands may be device pointers (the fast case) or host pointers; host
 * operands are staged through device memory for the duration of the call, so
 * the reference's own unit tests can call these functions unmodified. There is
 * no CPU arithmetic path.
 */
#ifndef TIE_B200_GEMM_H
#define TIE_B200_GEMM_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* reference src/gemm/gemm.h:55-58 */
typedef void (*gemm_fn)(int M, int N, int K,
                        const float *A,  int lda,
                        const float *B,  int ldb,
                        float *C, int ldc);

/* reference src/gemm/gemm.h:60-63 */
typedef void (*gemm_bt_fn)(int M, int N, int K,
                           const float *A,  int lda,
                           const float *Bt, int ldbt,
                           float *C, int ldc);

/* reference src/gemm/gemm.h:67-71 */
typedef struct {
    const char *name;
    gemm_fn     mul;
    gemm_bt_fn  mul_bt;
} gemm_impl;

/* reference src/gemm/gemm.h:78-86 (gemm_naive, gemm_naive_bt).
 * The naive algorithm, on the device: one thread per output element, one float
 * accumulator, k ascending, multiply and add rounded separately. That is the
 * reference's arithmetic exactly, so results are bit-identical to its CPU
 * gemm_naive for the same operands. Slow by design (a serial chain per output);
 * it exists for ABI compatibility and as an exact cross-check. */
void gemm_naive(int M, int N, int K,
                const float *A, int lda,
                const float *B, int ldb,
                float *C, int ldc);

void gemm_naive_bt(int M, int N, int K,
                   const float *A,  int lda,
                   const float *Bt, int ldbt,
                   float *C, int ldc);

/* reference src/gemm/gemm.h:89. name "gemm_naive_sm100a". */
extern const gemm_impl gemm_impl_naive;

/* Additive: the engine's own sm_100a kernels behind the same two signatures,
 * name "tie_b200_sm100a" (what model_gemm_of() reports). mul_bt runs the
 * tensor-core matmul (tcgen05, operands split into two tf32 halves, three MMAs
 * per product, fp32 accumulate: relative error near 2^-21 per product) when K
 * is a multiple of 32 and the leading dimensions of 4, else the tiled fp32
 * FFMA kernel; mul runs the tiled fp32 FFMA kernel. Tolerance-equal to the
 * naive order, not bit-equal. */
extern const gemm_impl gemm_impl_sm100a;

#ifdef __cplusplus
}
#endif

#endif /* TIE_B200_GEMM_H */
