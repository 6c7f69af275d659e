// k_gemm.cu -- tiled fp32 SIMT matmul with fused epilogues (prefill path and the
// public gemm_impl_sm100a).
//
//   C[M,N] (epilogue) = A[M,K] . W[N,K]^T      (BT: weights K-major, the engine's layout)
//   C[M,N]            = A[M,K] . B[K,N]        (!BT: the reference's mul layout)
//
// 128x128 output tile per 256-thread block, 16-deep k slices double-buffered
// through shared memory, 8x8 outputs per thread (two 4x4 quadrants per axis so
// shared-memory reads are conflict-free 16-byte loads). Every output is one fp32
// FMA chain over k ascending, independent of M and of the tile it lands in.
#include "common.cuh"

namespace tie {
namespace {

constexpr int BM = 128, BN = 128, BK = 16, PAD = 4, THREADS = 256;

template <bool VEC>
__device__ __forceinline__ float4 load4_rowmajor(const float* base, int ld, int r, int c, int R,
                                                 int Cc) {
    // 4 consecutive elements (r, c..c+3) of an R x Cc row-major matrix, zero outside
    if constexpr (VEC) {
        if (r < R && c + 3 < Cc) return *reinterpret_cast<const float4*>(base + (size_t)r * ld + c);
    }
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < R) {
        const float* p = base + (size_t)r * ld;
        if (c + 0 < Cc) v.x = p[c + 0];
        if (c + 1 < Cc) v.y = p[c + 1];
        if (c + 2 < Cc) v.z = p[c + 2];
        if (c + 3 < Cc) v.w = p[c + 3];
    }
    return v;
}

template <int EPI, bool BT, bool VEC>
__global__ void __launch_bounds__(THREADS)
gemm_tiled_kernel(const float* __restrict__ A, int lda, const float* __restrict__ B, int ldb,
                  const float* __restrict__ bias, float* C, int ldc, int M, int N, int K) {
    __shared__ __align__(16) float As[2][BK][BM + PAD];
    __shared__ __align__(16) float Bs[2][BK][BN + PAD];

    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;

    // loader coordinates: A (and B when BT) as 128 rows x 4 float4 k-chunks
    const int lr = tid >> 2, lk = (tid & 3) * 4;
    // B when !BT: 16 k-rows x 32 float4 n-chunks
    const int bk = tid >> 5, bn = (tid & 31) * 4;

    float4 ra[2], rb[2];
    auto load_tile = [&](int k0) {
#pragma unroll
        for (int p = 0; p < 2; ++p) ra[p] = load4_rowmajor<VEC>(A, lda, m0 + lr + 64 * p, k0 + lk, M, K);
        if constexpr (BT) {
#pragma unroll
            for (int p = 0; p < 2; ++p)
                rb[p] = load4_rowmajor<VEC>(B, ldb, n0 + lr + 64 * p, k0 + lk, N, K);
        } else {
#pragma unroll
            for (int p = 0; p < 2; ++p) rb[p] = load4_rowmajor<VEC>(B, ldb, k0 + bk + 8 * p, n0 + bn, K, N);
        }
    };
    auto store_tile = [&](int buf) {
#pragma unroll
        for (int p = 0; p < 2; ++p) {
            As[buf][lk + 0][lr + 64 * p] = ra[p].x;
            As[buf][lk + 1][lr + 64 * p] = ra[p].y;
            As[buf][lk + 2][lr + 64 * p] = ra[p].z;
            As[buf][lk + 3][lr + 64 * p] = ra[p].w;
        }
        if constexpr (BT) {
#pragma unroll
            for (int p = 0; p < 2; ++p) {
                Bs[buf][lk + 0][lr + 64 * p] = rb[p].x;
                Bs[buf][lk + 1][lr + 64 * p] = rb[p].y;
                Bs[buf][lk + 2][lr + 64 * p] = rb[p].z;
                Bs[buf][lk + 3][lr + 64 * p] = rb[p].w;
            }
        } else {
#pragma unroll
            for (int p = 0; p < 2; ++p) *reinterpret_cast<float4*>(&Bs[buf][bk + 8 * p][bn]) = rb[p];
        }
    };

    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

    const int n_tiles = (K + BK - 1) / BK;
    if (n_tiles > 0) {
        load_tile(0);
        store_tile(0);
        __syncthreads();
    }
    for (int t = 0; t < n_tiles; ++t) {
        const int buf = t & 1;
        if (t + 1 < n_tiles) load_tile((t + 1) * BK);
#pragma unroll
        for (int k = 0; k < BK; ++k) {
            const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][k][ty * 4]);
            const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][k][64 + ty * 4]);
            const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][k][tx * 4]);
            const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][k][64 + tx * 4]);
            const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        if (t + 1 < n_tiles) {
            store_tile(buf ^ 1);
            __syncthreads();
        }
    }

#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int r = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
        if (r >= M) continue;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int c = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
            if (c < N) {
                float* out = C + (size_t)r * ldc + c;
                *out = apply_epi<EPI>(acc[i][j], bias, c, out);
            }
        }
    }
}

template <int EPI, bool BT>
cudaError_t gemm_dispatch(const float* A, int lda, const float* B, int ldb, const float* bias,
                          float* C, int ldc, int M, int N, int K, cudaStream_t st) {
    if (M <= 0 || N <= 0) return cudaSuccess;
    if ((M + BM - 1) / BM > 65535) return cudaErrorInvalidValue;
    dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
    const bool vec = ((lda | ldb) & 3) == 0 && (reinterpret_cast<uintptr_t>(A) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(B) & 15) == 0;
    if (vec)
        gemm_tiled_kernel<EPI, BT, true><<<grid, THREADS, 0, st>>>(A, lda, B, ldb, bias, C, ldc, M, N, K);
    else
        gemm_tiled_kernel<EPI, BT, false><<<grid, THREADS, 0, st>>>(A, lda, B, ldb, bias, C, ldc, M, N, K);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemm_tn(const float* A, int lda, const float* W, int ldw, const float* bias,
                           float* C, int ldc, int M, int N, int K, int epi, cudaStream_t st) {
    switch (epi) {
        case EPI_STORE: return gemm_dispatch<EPI_STORE, true>(A, lda, W, ldw, bias, C, ldc, M, N, K, st);
        case EPI_BIAS: return gemm_dispatch<EPI_BIAS, true>(A, lda, W, ldw, bias, C, ldc, M, N, K, st);
        case EPI_BIAS_GELU:
            return gemm_dispatch<EPI_BIAS_GELU, true>(A, lda, W, ldw, bias, C, ldc, M, N, K, st);
        case EPI_BIAS_RESID:
            return gemm_dispatch<EPI_BIAS_RESID, true>(A, lda, W, ldw, bias, C, ldc, M, N, K, st);
    }
    return cudaErrorInvalidValue;
}

// C = A . B (B row-major K x N), epilogue-free: the public mul of gemm_impl_sm100a.
cudaError_t launch_gemm_nn(const float* A, int lda, const float* B, int ldb, float* C, int ldc,
                           int M, int N, int K, cudaStream_t st) {
    return gemm_dispatch<EPI_STORE, false>(A, lda, B, ldb, nullptr, C, ldc, M, N, K, st);
}

}  // namespace tie
