// tc_gemm.h -- the tensor-core (tcgen05, 3xTF32) matmul's host interface.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace tie {

// What the epilogue writes.
enum TcOut : int {
    TC_OUT_F32 = 0,       // C = y (fp32)
    TC_OUT_HILO = 1,      // C_hi, C_lo = the tf32 split of y (input of the next matmul)
    TC_OUT_F32_HILO = 2   // both
};

// A = a_hi + a_lo: M x K rows of lda floats; B = b_hi + b_lo: N x K rows of ldb.
struct TcOperands {
    const float* a_hi;
    const float* a_lo;
    int lda;
    const float* b_hi;
    const float* b_lo;
    int ldb;
    const float* b_f32 = nullptr;   // B itself (the tied head reads it and splits in shared memory)
};

struct TcArgs {
    int M, N, K;
    int kb_per_split;        // filled in by the launcher
    int splits;              // filled in by the launcher
    const float* bias;       // [N] (epilogues with bias)
    float* C;                // [M, ldc] fp32 out (and the residual input)
    float* C_hi;             // [M, ldc] tf32-split outputs
    float* C_lo;
    int ldc;
    int* err;                // device error flag (set when a bounded wait expires)
};

// hi = x rounded to tf32 (low 13 mantissa bits zero); x - hi is exact in fp32.
__device__ __forceinline__ float tf32_hi(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// The same rounding with integer operations (round to nearest, ties away
// from zero, at the 13th mantissa bit: half a tf32 ulp is added to the
// magnitude bits and the low 13 bits cleared; a carry out of the mantissa moves
// into the exponent). Equal to tf32_hi for every finite x; it runs on the
// integer pipe instead of the conversion unit.
__device__ __forceinline__ float tf32_hi_int(float x) {
    return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}

bool tc_gemm_supported(int M, int N, int K, int lda, int ldb);
// The tied head of a decode step over 1-256 activation rows (op.a_*: a.M rows)
// against a.N vocabulary rows (op.b_*): the weights are the MMA's 128-row
// operand, each CTA one tile over the whole of K, logits stored to a.C.
cudaError_t launch_tc_head(const TcOperands& op, const TcArgs& a, cudaStream_t st);
int tc_splits_for(int N, int K);
cudaError_t launch_tc_gemm(const TcOperands& op, const TcArgs& a, int epi, int out, int splits,
                           cudaStream_t st);
// hi/lo = the tf32 split of x[0..n)
cudaError_t launch_split_hilo(const float* x, float* hi, float* lo, long long n, cudaStream_t st);

}  // namespace tie
