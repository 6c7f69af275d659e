// k_misc.cu -- embedding, LayerNorm, KV stores, argmax reductions, greedy-step
// bookkeeping, the load-time transpose and the naive (reference-order) matmul.
#include "common.cuh"
#include "tc_gemm.h"

#include <cfloat>
#include <climits>

namespace tie {

namespace {

// ------------------------------------------------------------- embedding --
// model.c:671-676 / 805-809: x = wte[id] + wpe[pos], one float add per element.
// An id outside [0, V) (only possible through the device-buffer entry point,
// whose ids the host cannot check) yields a NaN row instead of a wild read.
__global__ void embed_prefill_kernel(const int32_t* __restrict__ ids, int rows, int T,
                                     const float* __restrict__ wte,
                                     const float* __restrict__ wpe, float* __restrict__ x,
                                     int E, int V) {
    const int E4 = E >> 2;
    const long long n = (long long)rows * E4;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(i / E4), c = (int)(i % E4);
        const int t = r % T;
        const int id = ids[r];
        if ((unsigned)id >= (unsigned)V) {
            reinterpret_cast<float4*>(x + (size_t)r * E)[c] = make_float4(NAN, NAN, NAN, NAN);
            continue;
        }
        const float4 a = reinterpret_cast<const float4*>(wte + (size_t)id * E)[c];
        const float4 b = reinterpret_cast<const float4*>(wpe + (size_t)t * E)[c];
        reinterpret_cast<float4*>(x + (size_t)r * E)[c] =
            make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z),
                        __fadd_rn(a.w, b.w));
    }
}

__global__ void embed_decode_kernel(const int32_t* __restrict__ tokens,
                                    const int32_t* __restrict__ lens, int B,
                                    const float* __restrict__ wte,
                                    const float* __restrict__ wpe, float* __restrict__ x, int E, int V) {
    pdl_trigger();
    pdl_wait();
    const int E4 = E >> 2;
    const int n = B * E4;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int b = i / E4, c = i % E4;
        const int id = tokens[b];
        if ((unsigned)id >= (unsigned)V) {
            reinterpret_cast<float4*>(x + (size_t)b * E)[c] = make_float4(NAN, NAN, NAN, NAN);
            continue;
        }
        const float4 a = reinterpret_cast<const float4*>(wte + (size_t)id * E)[c];
        const float4 p = reinterpret_cast<const float4*>(wpe + (size_t)lens[b] * E)[c];
        reinterpret_cast<float4*>(x + (size_t)b * E)[c] =
            make_float4(__fadd_rn(a.x, p.x), __fadd_rn(a.y, p.y), __fadd_rn(a.z, p.z),
                        __fadd_rn(a.w, p.w));
    }
}

// ------------------------------------------------------------- LayerNorm --
// model.c:593-610 with the engine's canonical summation order (ln_stats_warp,
// common.cuh). One warp per row; the row is first staged in shared memory
// with all its 16-byte loads in flight, so the statistics do not wait on one
// load at a time.
// One block of kLnGroups warps per row: warp w is canonical group w, so the
// eight group butterflies run at once; the group sums are then added in group
// order by every thread (common.cuh's order exactly).
constexpr int kLnThreads = 32 * kLnGroups;   // 256 virtual lanes
constexpr int kLnMaxPer = 8;                 // terms per thread: E <= 2048

__global__ void __launch_bounds__(kLnThreads)
layernorm_kernel(const float* __restrict__ x, const float* __restrict__ g,
                 const float* __restrict__ bvec, float* __restrict__ y,
                 float* __restrict__ y_hi, float* __restrict__ y_lo,
                 int rows, int E, float eps) {
    __shared__ double s_grp[2][kLnGroups];
    const int v = threadIdx.x, w = v >> 5;
    const int row = blockIdx.x;
    // in a programmatic-dependent chain: let the next kernel start loading its
    // weights, then wait for x
    pdl_trigger();
    pdl_wait();
    if (row >= rows) return;
    const float* xr = x + (size_t)row * E;
    float xv[kLnMaxPer];
#pragma unroll
    for (int j = 0; j < kLnMaxPer; ++j) xv[j] = v + kLnThreads * j < E ? xr[v + kLnThreads * j] : 0.f;
    // mean: virtual lane v adds its terms v, v + 256, ... in order
    double s = 0.0;
#pragma unroll
    for (int j = 0; j < kLnMaxPer; ++j)
        if (v + kLnThreads * j < E) s = __dadd_rn(s, (double)xv[j]);
    s = ln_warp_sum_d(s);
    if ((v & 31) == 0) s_grp[0][w] = s;
    __syncthreads();
    double S = s_grp[0][0];
#pragma unroll
    for (int k = 1; k < kLnGroups; ++k) S = __dadd_rn(S, s_grp[0][k]);
    const double mean = S / (double)E;
    // biased variance, same order
    double q = 0.0;
#pragma unroll
    for (int j = 0; j < kLnMaxPer; ++j)
        if (v + kLnThreads * j < E) {
            const double d = __dadd_rn((double)xv[j], -mean);
            q = __dadd_rn(q, __dmul_rn(d, d));
        }
    q = ln_warp_sum_d(q);
    if ((v & 31) == 0) s_grp[1][w] = q;
    __syncthreads();
    double V = s_grp[1][0];
#pragma unroll
    for (int k = 1; k < kLnGroups; ++k) V = __dadd_rn(V, s_grp[1][k]);
    const float inv = (float)(1.0 / sqrt(__dadd_rn(V / (double)E, (double)eps)));
    const size_t off = (size_t)row * E;
#pragma unroll
    for (int j = 0; j < kLnMaxPer; ++j) {
        const int i = v + kLnThreads * j;
        if (i >= E) break;
        const float val = ln_apply(xv[j], mean, inv, g[i], bvec[i]);
        if (y) y[off + i] = val;
        if (y_hi) {
            const float h = tf32_hi(val);
            y_hi[off + i] = h;
            y_lo[off + i] = __fsub_rn(val, h);
        }
    }
}

// ------------------------------------------------------------- KV stores --
__global__ void kv_store_prefill_kernel(const float* __restrict__ qkv, int n_seq, int T,
                                        PagedKV kv, int first_seq) {
    const int E = kv.n_embd, E4 = E >> 2;
    const long long n = (long long)n_seq * T * E4;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const int c = (int)(i % E4);
        const long long r = i / E4;
        const int t = (int)(r % T), s = (int)(r / T);
        const float4* src = reinterpret_cast<const float4*>(qkv + (size_t)r * 3 * E);
        const size_t row = kv.row(first_seq + s, t);
        reinterpret_cast<float4*>(kv.k + row * E)[c] = src[E4 + c];
        reinterpret_cast<float4*>(kv.v + row * E)[c] = src[2 * E4 + c];
    }
}

__global__ void kv_store_decode_kernel(const float* __restrict__ qkv,
                                       const int32_t* __restrict__ lens, int B, PagedKV kv) {
    const int E = kv.n_embd, E4 = E >> 2;
    const int n = B * E4;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int b = i / E4, c = i % E4;
        const float4* src = reinterpret_cast<const float4*>(qkv + (size_t)b * 3 * E);
        const size_t row = kv.row(b, lens[b]);
        reinterpret_cast<float4*>(kv.k + row * E)[c] = src[E4 + c];
        reinterpret_cast<float4*>(kv.v + row * E)[c] = src[2 * E4 + c];
    }
}

// -------------------------------------------------------------- argmax --
// Candidates (value, index); index -1 means "none yet". A candidate beats the
// current best when it is larger, or equal with a lower index: the result of
// the reference's strict '>' scan from index 0 (model.c:920-925). NaN values
// never become candidates; a partial whose range starts with a NaN at index 0
// reports index -2, which makes the final answer 0 (the scan never moves off
// index 0 when v[0] is NaN).
__device__ __forceinline__ bool beats(float v, int i, float bv, int bi) {
    return bi < 0 || v > bv || (v == bv && i < bi);
}

__global__ void argmax_finalize_kernel(const float* __restrict__ pv, const int* __restrict__ pi,
                                       int n_parts, int M, int32_t* __restrict__ next) {
    pdl_trigger();
    pdl_wait();
    const int m = blockIdx.x;
    if (m >= M) return;
    float bv = 0.f;
    int bi = -1;
    bool nan0 = false;
    // 8 partials per thread per round, all loaded before any is compared
    for (int p0 = threadIdx.x; p0 < n_parts; p0 += 8 * blockDim.x) {
        int ii[8];
        float vv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int p = p0 + u * blockDim.x;
            ii[u] = p < n_parts ? pi[(size_t)p * M + m] : -1;
            vv[u] = p < n_parts ? pv[(size_t)p * M + m] : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            if (ii[u] == -2) nan0 = true;
            else if (ii[u] >= 0 && beats(vv[u], ii[u], bv, bi)) { bv = vv[u]; bi = ii[u]; }
        }
    }
    __shared__ float sv[32];
    __shared__ int si[32];
    __shared__ int snan;
    if (threadIdx.x == 0) snan = 0;
    __syncthreads();
    if (nan0) atomicOr(&snan, 1);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oi >= 0 && beats(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) { sv[w] = bv; si[w] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int k = 1; k < (int)(blockDim.x >> 5); ++k)
            if (si[k] >= 0 && beats(sv[k], si[k], bv, bi)) { bv = sv[k]; bi = si[k]; }
        next[m] = snan ? 0 : (bi < 0 ? 0 : bi);
    }
}

// argmax of full rows of a logits matrix: row b = row_offset + b * row_stride
__global__ void argmax_rows_kernel(const float* __restrict__ L, int ldl, int N, int row_stride,
                                   int row_offset, int32_t* __restrict__ next) {
    const int b = blockIdx.x;
    const float* r = L + (size_t)(row_offset + (size_t)b * row_stride) * ldl;
    float bv = 0.f;
    int bi = -1;
    auto take = [&](float v, int i) {
        if (v == v && beats(v, i, bv, bi)) { bv = v; bi = i; }
    };
    // The winner is the maximum of a total order (value, then lower index),
    // so the scan may visit the row in any order. Rows start anywhere (the
    // row length is the vocabulary), so up to three scalars lead to a 16-byte
    // boundary; the body goes in float4s, kArgU of them in flight per thread.
    constexpr int kArgU = 4;
    const int head = min(N, (int)((16u - ((uint32_t)(uintptr_t)r & 15u)) & 15u) / 4);
    if ((int)threadIdx.x < head) take(r[threadIdx.x], threadIdx.x);
    const float4* r4 = reinterpret_cast<const float4*>(r + head);
    const int n4 = (N - head) >> 2, T = blockDim.x;
    int c = threadIdx.x;
    for (; c + (kArgU - 1) * T < n4; c += kArgU * T) {
        float4 v[kArgU];
#pragma unroll
        for (int u = 0; u < kArgU; ++u) v[u] = __ldg(r4 + c + u * T);
#pragma unroll
        for (int u = 0; u < kArgU; ++u) {
            const int i = head + 4 * (c + u * T);
            take(v[u].x, i);
            take(v[u].y, i + 1);
            take(v[u].z, i + 2);
            take(v[u].w, i + 3);
        }
    }
    for (; c < n4; c += T) {
        const float4 v = __ldg(r4 + c);
        const int i = head + 4 * c;
        take(v.x, i);
        take(v.y, i + 1);
        take(v.z, i + 2);
        take(v.w, i + 3);
    }
    for (int i = head + 4 * n4 + threadIdx.x; i < N; i += T) take(r[i], i);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oi >= 0 && beats(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    __shared__ float sv[32];
    __shared__ int si[32];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) { sv[w] = bv; si[w] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int k = 1; k < (int)(blockDim.x >> 5); ++k)
            if (si[k] >= 0 && beats(sv[k], si[k], bv, bi)) { bv = sv[k]; bi = si[k]; }
        const bool nan0 = !(r[0] == r[0]);
        next[b] = nan0 ? 0 : (bi < 0 ? 0 : bi);
    }
}

// ----------------------------------------------------- greedy bookkeeping --
__global__ void step_advance_kernel(const int32_t* __restrict__ next, int32_t* __restrict__ tokens,
                                    int32_t* __restrict__ lens, int32_t* __restrict__ out,
                                    int ld_out, int32_t* __restrict__ step, int B) {
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    const int s = *step;
    __syncthreads();
    if (b < B) {
        const int32_t t = next[b];
        tokens[b] = t;
        out[(size_t)b * ld_out + s] = t;
        lens[b] += 1;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) *step = s + 1;
}

// ------------------------------------------------------------ transpose --
__global__ void transpose_kernel(const float* __restrict__ in, float* __restrict__ out, int R,
                                 int Cc) {
    __shared__ float tile[32][33];
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int r = r0 + i, c = c0 + threadIdx.x;
        if (r < R && c < Cc) tile[i][threadIdx.x] = in[(size_t)r * Cc + c];
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int c = c0 + i, r = r0 + threadIdx.x;
        if (r < R && c < Cc) out[(size_t)c * R + r] = tile[threadIdx.x][i];
    }
}

// ---------------------------------------------------------- naive matmul --
// gemm_naive.c:30-60 on the device: one thread per output, one accumulator,
// k ascending, product and sum rounded separately (no fused multiply-add).
__global__ void gemm_naive_kernel(int M, int N, int K, const float* __restrict__ A, int lda,
                                  const float* __restrict__ B, int ldb, float* __restrict__ C,
                                  int ldc, int bt) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    const int i = blockIdx.y;
    if (i >= M || j >= N) return;
    float acc = 0.0f;
    const float* a = A + (size_t)i * lda;
    if (bt) {
        const float* b = B + (size_t)j * ldb;
        for (int k = 0; k < K; ++k) acc = __fadd_rn(acc, __fmul_rn(a[k], b[k]));
    } else {
        for (int k = 0; k < K; ++k) acc = __fadd_rn(acc, __fmul_rn(a[k], B[(size_t)k * ldb + j]));
    }
    C[(size_t)i * ldc + j] = acc;
}

inline int grid_for(long long n, int block) {
    long long g = (n + block - 1) / block;
    if (g > 148 * 32) g = 148 * 32;
    return (int)(g < 1 ? 1 : g);
}

}  // namespace

cudaError_t launch_embed_prefill(const int32_t* ids, int rows, int T, const float* wte,
                                 const float* wpe, float* x, int E, int V, cudaStream_t st) {
    embed_prefill_kernel<<<grid_for((long long)rows * (E / 4), 256), 256, 0, st>>>(ids, rows, T,
                                                                                    wte, wpe, x, E, V);
    return cudaGetLastError();
}

cudaError_t launch_embed_decode(const int32_t* tokens, const int32_t* lens, int B,
                                const float* wte, const float* wpe, float* x, int E, int V,
                                cudaStream_t st) {
    embed_decode_kernel<<<grid_for((long long)B * (E / 4), 256), 256, 0, st>>>(tokens, lens, B,
                                                                                wte, wpe, x, E, V);
    return cudaGetLastError();
}

cudaError_t launch_layernorm(const float* x, const float* g, const float* b, float* y, int rows,
                             int E, float eps, cudaStream_t st, float* y_hi, float* y_lo) {
    if (E > kLnThreads * kLnMaxPer) return cudaErrorInvalidValue;
    if (rows <= 0) return cudaSuccess;
    cudaError_t e = launch_pdl(layernorm_kernel, dim3(rows), dim3(kLnThreads), 0, st, x, g, b, y, y_hi, y_lo,
                               rows, E, eps);
    return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_kv_store_prefill(const float* qkv, int n_seq, int T, PagedKV kv, int first_seq,
                                    cudaStream_t st) {
    kv_store_prefill_kernel<<<grid_for((long long)n_seq * T * (kv.n_embd / 4), 256), 256, 0, st>>>(
        qkv, n_seq, T, kv, first_seq);
    return cudaGetLastError();
}

cudaError_t launch_kv_store_decode(const float* qkv, const int32_t* lens, int B, PagedKV kv,
                                   cudaStream_t st) {
    kv_store_decode_kernel<<<grid_for((long long)B * (kv.n_embd / 4), 256), 256, 0, st>>>(
        qkv, lens, B, kv);
    return cudaGetLastError();
}

cudaError_t launch_argmax_finalize(const float* part_val, const int* part_idx, int n_parts, int M,
                                   int32_t* next, cudaStream_t st) {
    cudaError_t e = launch_pdl(argmax_finalize_kernel, dim3(M), dim3(256), 0, st, part_val, part_idx, n_parts, M, next);
    return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_argmax_rows(const float* L, int ldl, int M, int N, int row_stride,
                               int row_offset, int32_t* next, cudaStream_t st) {
    argmax_rows_kernel<<<M, 512, 0, st>>>(L, ldl, N, row_stride, row_offset, next);
    return cudaGetLastError();
}

cudaError_t launch_step_advance(const int32_t* next, int32_t* tokens, int32_t* lens,
                                int32_t* out, int ld_out, int32_t* step, int B, cudaStream_t st) {
    // One block: every thread reads *step before thread 0 advances it.
    if (B > 1024) return cudaErrorInvalidValue;
    cudaError_t e = launch_pdl(step_advance_kernel, dim3(1), dim3(1024), 0, st, next, tokens, lens, out, ld_out, step, B);
    return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_transpose(const float* in, float* out, int R, int Cc, cudaStream_t st) {
    dim3 grid((Cc + 31) / 32, (R + 31) / 32);
    transpose_kernel<<<grid, dim3(32, 8), 0, st>>>(in, out, R, Cc);
    return cudaGetLastError();
}

cudaError_t launch_gemm_naive(int M, int N, int K, const float* A, int lda, const float* B,
                              int ldb, float* C, int ldc, bool bt, cudaStream_t st) {
    if (M <= 0 || N <= 0) return cudaSuccess;
    if (M > 65535) return cudaErrorInvalidValue;
    dim3 grid((N + 127) / 128, M);
    gemm_naive_kernel<<<grid, 128, 0, st>>>(M, N, K, A, lda, B, ldb, C, ldc, bt ? 1 : 0);
    return cudaGetLastError();
}

}  // namespace tie
