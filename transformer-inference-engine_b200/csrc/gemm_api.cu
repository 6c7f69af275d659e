// gemm_api.cu -- the gemm.h entry points (reference src/gemm/gemm.h:55-89).
//
// Operands may live in device memory (used as they are) or in host memory
// (copied to the device for the call and C copied back); the arithmetic is
// always a kernel. Calls are synchronous, like the reference's.
#include "../../include/gemm.h"
#include "internal.h"
#include "tc_gemm.h"

#include <cstdio>

using namespace tie;

namespace {

bool on_device(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) { cudaGetLastError(); return false; }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

// Span in floats of an R x Cc block with leading dimension ld.
size_t span(int R, int Cc, int ld) { return R <= 0 || Cc <= 0 ? 0 : (size_t)(R - 1) * ld + Cc; }

// Makes `p` (n floats) usable by a kernel: returns p itself when it is device
// memory, else a device copy (made only if `copy_in`) that the caller frees.
float* devicify(const float* p, size_t n, bool copy_in, bool* owned) {
    *owned = false;
    if (!p || n == 0 || on_device(p)) return const_cast<float*>(p);
    float* d = nullptr;
    if (cudaMalloc(&d, n * sizeof(float)) != cudaSuccess) { cudaGetLastError(); return nullptr; }
    if (copy_in && cudaMemcpy(d, p, n * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(d);
        return nullptr;
    }
    *owned = true;
    return d;
}

enum Kind { NAIVE_NN, NAIVE_BT, TILED_NN, TILED_BT };

void run(Kind kind, int M, int N, int K, const float* A, int lda, const float* B, int ldb, float* C,
         int ldc) {
    if (M <= 0 || N <= 0 || !C) return;  // nothing to write
    const bool bt = kind == NAIVE_BT || kind == TILED_BT;
    const size_t nA = K > 0 ? span(M, K, lda) : 0;
    const size_t nB = K > 0 ? (bt ? span(N, K, ldb) : span(K, N, ldb)) : 0;
    const size_t nC = span(M, N, ldc);
    bool oa = false, ob = false, oc = false;
    float* dA = devicify(A, nA, true, &oa);
    float* dB = devicify(B, nB, true, &ob);
    float* dC = devicify(C, nC, true, &oc);  // copied in: columns past N must survive
    cudaError_t e = cudaSuccess;
    if ((nA && !dA) || (nB && !dB) || !dC) {
        e = cudaErrorMemoryAllocation;
    } else if (kind == NAIVE_NN || kind == NAIVE_BT) {
        e = launch_gemm_naive(M, N, K, dA, lda, dB, ldb, dC, ldc, bt, nullptr);
    } else if (kind == TILED_BT && K > 0 && tc_gemm_supported(M, N, K, lda, ldb)) {
        // the tensor-core path: split both operands into tf32 halves, then 3xTF32
        float* sp = nullptr;
        const size_t na = span(M, K, lda), nb = span(N, K, ldb);  // what the kernel reads
        e = cudaMalloc(&sp, 2 * (na + nb) * sizeof(float));
        if (e == cudaSuccess) {
            float *ah = sp, *al = sp + na, *bh = sp + 2 * na, *bl = bh + nb;
            e = launch_split_hilo(dA, ah, al, (long long)na, nullptr);
            if (e == cudaSuccess) e = launch_split_hilo(dB, bh, bl, (long long)nb, nullptr);
            TcOperands op{ah, al, lda, bh, bl, ldb};
            TcArgs a{};
            a.M = M; a.N = N; a.K = K; a.C = dC; a.ldc = ldc;
            int* err = nullptr;
            if (e == cudaSuccess) e = cudaMalloc(&err, sizeof(int));
            if (e == cudaSuccess) e = cudaMemset(err, 0, sizeof(int));
            a.err = err;
            if (e == cudaSuccess) e = launch_tc_gemm(op, a, EPI_STORE, TC_OUT_F32, 1, nullptr);
            if (e == cudaSuccess) e = cudaDeviceSynchronize();
            int flag = 0;
            if (e == cudaSuccess) e = cudaMemcpy(&flag, err, sizeof flag, cudaMemcpyDeviceToHost);
            if (e == cudaSuccess && flag) e = cudaErrorLaunchTimeout;
            cudaFree(err);
            cudaFree(sp);
        }
    } else if (kind == TILED_BT) {
        e = launch_gemm_tn(dA, lda, dB, ldb, nullptr, dC, ldc, M, N, K, EPI_STORE, nullptr);
    } else {
        e = launch_gemm_nn(dA, lda, dB, ldb, dC, ldc, M, N, K, nullptr);
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess && oc) e = cudaMemcpy(C, dC, nC * sizeof(float), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) {
        std::fprintf(stderr, "tie_b200 gemm: %s\n", cudaGetErrorString(e));
        cudaGetLastError();
    }
    if (oa) cudaFree(dA);
    if (ob) cudaFree(dB);
    if (oc) cudaFree(dC);
}

void tiled_mul(int M, int N, int K, const float* A, int lda, const float* B, int ldb, float* C, int ldc) {
    run(TILED_NN, M, N, K, A, lda, B, ldb, C, ldc);
}
void tiled_mul_bt(int M, int N, int K, const float* A, int lda, const float* B, int ldb, float* C, int ldc) {
    run(TILED_BT, M, N, K, A, lda, B, ldb, C, ldc);
}

}  // namespace

extern "C" {

void gemm_naive(int M, int N, int K, const float* A, int lda, const float* B, int ldb, float* C, int ldc) {
    run(NAIVE_NN, M, N, K, A, lda, B, ldb, C, ldc);
}

void gemm_naive_bt(int M, int N, int K, const float* A, int lda, const float* Bt, int ldbt, float* C,
                   int ldc) {
    run(NAIVE_BT, M, N, K, A, lda, Bt, ldbt, C, ldc);
}

const gemm_impl gemm_impl_naive = {"gemm_naive_sm100a", gemm_naive, gemm_naive_bt};
const gemm_impl gemm_impl_sm100a = {"tie_b200_sm100a", tiled_mul, tiled_mul_bt};

}  // extern "C"
