// k_gemv.cu -- decode matmuls for a handful of rows: Y[M,N] = X[M,K] . W[N,K]^T.
//
// Memory-bound weight streaming. Each warp owns RPW output features (rows of
// the K-major weight W); its lanes walk the row in 16-byte chunks (chunk c is
// read by lane c % 32) with loads that bypass L1, accumulate one fp32 FMA chain
// per lane, and combine the 32 lane sums with a fixed xor-butterfly. The
// activations X (a few KB) are read through the read-only L1 path and shared
// by every warp of the block.
//
// The per-output arithmetic depends only on K, never on M, N or the launch
// shape, so a sequence's results are identical whatever batch it is decoded
// in (batch invariance) and whatever GPU its shard lands on.
#include "common.cuh"

namespace tie {
namespace {

constexpr int kWarps = 4;  // warps per block
constexpr int kMT = 8;     // activation rows per pass
constexpr int kU = 4;      // 16-byte chunks in flight per lane per row

__device__ __forceinline__ float4 ld_stream(const float* p) {
    float4 v;
    asm("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
        : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
        : "l"(p));
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ bool beats(float v, int i, float bv, int bi) {
    return bi < 0 || v > bv || (v == bv && i < bi);
}

template <int EPI, int RPW, bool ARGMAX>
__global__ void __launch_bounds__(kWarps * 32)
gemv_kernel(const float* __restrict__ X, int ldx, const float* __restrict__ W, int ldw,
            const float* __restrict__ bias, float* Y, int ldy, int M, int N, int K,
            float* __restrict__ part_val, int* __restrict__ part_idx) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = (blockIdx.x * kWarps + warp) * RPW;
    const int K4 = K >> 2;
    __shared__ float s_val[kWarps][kMT];
    __shared__ int s_idx[kWarps][kMT];

    for (int m0 = 0; m0 < M; m0 += kMT) {
        float acc[RPW][kMT];
#pragma unroll
        for (int r = 0; r < RPW; ++r)
#pragma unroll
            for (int m = 0; m < kMT; ++m) acc[r][m] = 0.f;

        if (row0 < N) {
            for (int cb = 0; cb < K4; cb += 32 * kU) {
                float4 w[kU][RPW];
#pragma unroll
                for (int u = 0; u < kU; ++u) {
                    const int c = cb + u * 32 + lane;
#pragma unroll
                    for (int r = 0; r < RPW; ++r)
                        w[u][r] = (c < K4 && row0 + r < N)
                                      ? ld_stream(W + (size_t)(row0 + r) * ldw + 4 * c)
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int u = 0; u < kU; ++u) {
                    const int c = cb + u * 32 + lane;
                    if (c < K4) {
#pragma unroll
                        for (int m = 0; m < kMT; ++m) {
                            if (m0 + m < M) {
                                const float4 x =
                                    __ldg(reinterpret_cast<const float4*>(X + (size_t)(m0 + m) * ldx) + c);
#pragma unroll
                                for (int r = 0; r < RPW; ++r) {
                                    float a = acc[r][m];
                                    a = fmaf(w[u][r].x, x.x, a);
                                    a = fmaf(w[u][r].y, x.y, a);
                                    a = fmaf(w[u][r].z, x.z, a);
                                    a = fmaf(w[u][r].w, x.w, a);
                                    acc[r][m] = a;
                                }
                            }
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < RPW; ++r)
#pragma unroll
            for (int m = 0; m < kMT; ++m) acc[r][m] = warp_sum(acc[r][m]);

        if constexpr (!ARGMAX) {
            if (lane == 0 && row0 < N) {
#pragma unroll
                for (int r = 0; r < RPW; ++r)
#pragma unroll
                    for (int m = 0; m < kMT; ++m) {
                        const int j = row0 + r;
                        if (j < N && m0 + m < M) {
                            float* y = Y + (size_t)(m0 + m) * ldy + j;
                            *y = apply_epi<EPI>(acc[r][m], bias, j, y);
                        }
                    }
            }
        } else {
            // logits (optional) and the best (value, index) of this warp's rows
            if (lane == 0) {
#pragma unroll
                for (int m = 0; m < kMT; ++m) {
                    float bv = 0.f;
                    int bi = -1;
#pragma unroll
                    for (int r = 0; r < RPW; ++r) {
                        const int j = row0 + r;
                        if (j < N && m0 + m < M) {
                            const float v = acc[r][m];
                            if (Y) Y[(size_t)(m0 + m) * ldy + j] = v;
                            if (j == 0 && !(v == v)) bi = -2;
                            else if (bi != -2 && v == v && beats(v, j, bv, bi)) { bv = v; bi = j; }
                        }
                    }
                    s_val[warp][m] = bv;
                    s_idx[warp][m] = bi;
                }
            }
            __syncthreads();
            if (threadIdx.x < kMT && m0 + (int)threadIdx.x < M) {
                const int m = threadIdx.x;
                float bv = 0.f;
                int bi = -1;
                bool nan0 = false;
                for (int w = 0; w < kWarps; ++w) {
                    const int i = s_idx[w][m];
                    if (i == -2) nan0 = true;
                    else if (i >= 0 && beats(s_val[w][m], i, bv, bi)) { bv = s_val[w][m]; bi = i; }
                }
                part_val[(size_t)blockIdx.x * M + m0 + m] = bv;
                part_idx[(size_t)blockIdx.x * M + m0 + m] = nan0 ? -2 : bi;
            }
            __syncthreads();
        }
    }
}

template <int EPI>
cudaError_t gemv_dispatch(const float* X, int ldx, const float* W, int ldw, const float* bias,
                          float* Y, int ldy, int M, int N, int K, cudaStream_t st) {
    if (N >= 16384) {
        const int grid = (N + kWarps * 4 - 1) / (kWarps * 4);
        gemv_kernel<EPI, 4, false><<<grid, kWarps * 32, 0, st>>>(X, ldx, W, ldw, bias, Y, ldy, M,
                                                                 N, K, nullptr, nullptr);
    } else {
        const int grid = (N + kWarps - 1) / kWarps;
        gemv_kernel<EPI, 1, false><<<grid, kWarps * 32, 0, st>>>(X, ldx, W, ldw, bias, Y, ldy, M,
                                                                 N, K, nullptr, nullptr);
    }
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemv(const float* X, int ldx, const float* W, int ldw, const float* bias,
                        float* Y, int ldy, int M, int N, int K, int epi, cudaStream_t st) {
    if ((K & 3) || (ldx & 3) || (ldw & 3)) return cudaErrorInvalidValue;
    switch (epi) {
        case EPI_STORE: return gemv_dispatch<EPI_STORE>(X, ldx, W, ldw, bias, Y, ldy, M, N, K, st);
        case EPI_BIAS: return gemv_dispatch<EPI_BIAS>(X, ldx, W, ldw, bias, Y, ldy, M, N, K, st);
        case EPI_BIAS_GELU:
            return gemv_dispatch<EPI_BIAS_GELU>(X, ldx, W, ldw, bias, Y, ldy, M, N, K, st);
        case EPI_BIAS_RESID:
            return gemv_dispatch<EPI_BIAS_RESID>(X, ldx, W, ldw, bias, Y, ldy, M, N, K, st);
    }
    return cudaErrorInvalidValue;
}

static_assert(kWarps * 4 == kGemvArgmaxRowsPerBlock, "the head's rows per block, as declared");
int gemv_argmax_blocks(int N) { return (N + kGemvArgmaxRowsPerBlock - 1) / kGemvArgmaxRowsPerBlock; }

cudaError_t launch_gemv_argmax(const float* X, int ldx, const float* W, int ldw, float* logits,
                               int ldl, int M, int N, int K, float* part_val, int* part_idx,
                               cudaStream_t st) {
    if ((K & 3) || (ldx & 3) || (ldw & 3)) return cudaErrorInvalidValue;
    gemv_kernel<EPI_STORE, 4, true><<<gemv_argmax_blocks(N), kWarps * 32, 0, st>>>(
        X, ldx, W, ldw, nullptr, logits, ldl, M, N, K, part_val, part_idx);
    return cudaGetLastError();
}

}  // namespace tie
