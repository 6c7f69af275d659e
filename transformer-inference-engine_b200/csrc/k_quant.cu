// k_quant.cu -- the reduced weight formats, built on the device from the fp32
// weights.
//
//   bf16  q = the fp32 weight rounded to nearest-even bf16;
//         the weight the model then computes with is exactly q.
//   int8  per output channel (a row of a [out, in] matrix): scale = absmax(row)
//         / 127 in fp32, q = rint(w / scale) (ties to even) clamped to +-127, and
//         0 for an all-zero row; the weight is q * scale.
//
// Each conversion also writes the dequantised fp32 matrix, which the fp32
// paths (prefill, large-batch decode, embeddings) then use, so that every path
// computes with the same weights.
#include <cuda_bf16.h>

#include <algorithm>

#include "common.cuh"

namespace tie {
namespace {

__global__ void to_bf16_kernel(const float* __restrict__ w, __nv_bfloat16* __restrict__ q, float* __restrict__ deq,
                               size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const __nv_bfloat16 b = __float2bfloat16_rn(w[i]);
        q[i] = b;
        deq[i] = __bfloat162float(b);
    }
}

// one block of 256 threads per row
__global__ void __launch_bounds__(256) quant_rows_kernel(const float* __restrict__ w, int8_t* __restrict__ q,
                                                         float* __restrict__ scale, float* __restrict__ deq, int K) {
    const size_t row = blockIdx.x;
    const float* wr = w + row * K;
    float m = 0.f;
    for (int i = threadIdx.x; i < K; i += 256) m = fmaxf(m, fabsf(wr[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    __shared__ float sm[8];
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = m;
    __syncthreads();
    float absmax = sm[0];
    for (int k = 1; k < 8; ++k) absmax = fmaxf(absmax, sm[k]);
    const float s = absmax / 127.0f;
    for (int i = threadIdx.x; i < K; i += 256) {
        float v = s > 0.f ? rintf(wr[i] / s) : 0.f;
        v = fminf(127.f, fmaxf(-127.f, v));
        q[row * K + i] = (int8_t)v;
        deq[row * K + i] = v * s;
    }
    if (threadIdx.x == 0) scale[row] = s;
}

}  // namespace

cudaError_t launch_to_bf16(const float* w, void* q, float* deq, size_t n, cudaStream_t st) {
    const int grid = (int)std::min<size_t>((n + 255) / 256, 148 * 32);
    to_bf16_kernel<<<grid, 256, 0, st>>>(w, reinterpret_cast<__nv_bfloat16*>(q), deq, n);
    return cudaGetLastError();
}

cudaError_t launch_quant_rows(const float* w, void* q, float* scale, float* deq, int N, int K, cudaStream_t st) {
    if (N <= 0) return cudaSuccess;
    quant_rows_kernel<<<N, 256, 0, st>>>(w, reinterpret_cast<int8_t*>(q), scale, deq, K);
    return cudaGetLastError();
}

}  // namespace tie
