// k_decode.cu -- the small-batch decode step (at most 16 sequences), fused and
// chained with programmatic dependent launch.
//
// A decode step at batch 1 moves ~0.5 GB of fp32 weights through a few dozen
// matmuls whose individual transfers take ~1 us at HBM speed, so the step is
// bound by the gaps between kernels as much as by bandwidth. Two measures:
//
//   * fusion: LayerNorm runs inside the matmul that consumes it (every block
//     normalises the <= 16 input rows itself, in shared memory, with the same
//     double-precision statistics as the standalone kernel), the K/V rows of a
//     step are stored by the QKV matmul's epilogue, and LN_f runs inside the
//     tied head;
//   * programmatic dependent launch: every kernel first issues the loads of its
//     own weight rows (which no earlier kernel writes), then lets the next
//     kernel launch (griddepcontrol.launch_dependents), and only then waits for
//     its predecessor's results (griddepcontrol.wait). Weight streaming thus
//     overlaps the previous kernel's tail and the launch latency.
//
// Each warp holds all of its weight chunks in registers (loaded before the
// dependency wait), so a matrix is in flight in one round trip.
#include "common.cuh"

namespace tie {
namespace {

constexpr int kWarps = 4;
constexpr int kMaxRows = 16;
constexpr int kStageFloats = 0;               // activation rows copied to shared memory up to this many floats (0: read through L1)

__device__ __forceinline__ float4 ld_stream(const float* p) {
    float4 v;
    asm("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
        : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
        : "l"(p));
    return v;
}

// LayerNorm of rows [0, M) of x (row stride ldx) into xs (row stride K), the
// arithmetic of layernorm_kernel (k_misc.cu). Each row is first copied into
// xs with all of the block's 16-byte loads in flight; the statistics (one warp
// per row, the canonical order of ln_stats_warp) and the normalisation then
// run out of shared memory, in place.
__device__ void ln_rows_to_smem(const float* __restrict__ x, int ldx, const float* __restrict__ g,
                                const float* __restrict__ b, float eps, int M, int K, float* xs) {
    const int K4 = K >> 2;
    for (int i = threadIdx.x; i < M * K4; i += kWarps * 32) {
        const int m = i / K4, c = i % K4;
        reinterpret_cast<float4*>(xs + (size_t)m * K)[c] =
            __ldg(reinterpret_cast<const float4*>(x + (size_t)m * ldx) + c);
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int m = warp; m < M; m += kWarps) {
        float* xr = xs + (size_t)m * K;
        double mean;
        float inv;
        ln_stats_warp(xr, K, eps, lane, mean, inv);
        for (int i = lane; i < K; i += 32) xr[i] = ln_apply(xr[i], mean, inv, g[i], b[i]);
    }
}

struct DecArgs {
    const float* x;   // input rows [M][ldx] (pre-normalisation when LN)
    int ldx;
    const float* ln_g;
    const float* ln_b;
    float eps;
    const float* W;   // [N][K], K-major (fp32)
    const void* Wq;   // [N][K] bf16 or int8 (reduced weight formats)
    const float* scale;   // [N] int8 per-row scales
    const float* bias;
    float* y;         // [M][ldy]
    int ldy;
    int M, N, K;
    // QKV epilogue: columns [E, 3E) are also this step's K and V rows
    PagedKV kv;
    const int32_t* lens;
    // head: partial maxima per block
    float* part_val;
    int* part_idx;
};

enum : int { DEC_BIAS = 0, DEC_BIAS_GELU = 1, DEC_BIAS_RESID = 2, DEC_QKV_KV = 3, DEC_HEAD = 4 };

__device__ __forceinline__ bool beats(float v, int i, float bv, int bi) {
    return bi < 0 || v > bv || (v == bv && i < bi);
}

// A block of 4 warps covers RPB = (4 / WS) * RPW weight rows; each row's K is
// cut into WS slices of K / WS and each warp owns RPW rows of one slice. A warp
// loads ALL of its weight chunks (at most CPL 16-byte chunks per lane per row)
// into registers before the dependency wait, so the whole matrix is in flight
// at once; after the wait it only reads the <= 16 activation rows (shared
// memory when normalised here, else global through L1) and reduces.
// Per (row, activation row) the sum is: within a slice, lane c accumulates
// chunks c, c + 32, ... (four FMAs per chunk, in order), then an xor-butterfly
// across lanes; the WS slice sums are added in slice order. The order depends
// only on K, so results do not depend on the batch a sequence decodes in.
// Weight formats: WT 0 fp32 (4 elements per 16-byte chunk), 1 bf16 (8), 2 int8
// (16, times the row's scale after the sum). For the reduced formats the
// elements of a chunk are added in element order against the matching
// activations; everything else is as for fp32.
template <int WT> constexpr int elems_per_chunk() { return WT == 0 ? 4 : (WT == 1 ? 8 : 16); }

// element e of a 16-byte chunk of a reduced format
template <int WT>
__device__ __forceinline__ float chunk_elem(const float4& c, int e) {
    if constexpr (WT == 0) return e == 0 ? c.x : e == 1 ? c.y : e == 2 ? c.z : c.w;
    else {
    const uint32_t w = __float_as_uint(e >> (WT == 1 ? 1 : 2) == 0 ? c.x
                                        : e >> (WT == 1 ? 1 : 2) == 1 ? c.y
                                        : e >> (WT == 1 ? 1 : 2) == 2 ? c.z : c.w);
    if constexpr (WT == 1) return __uint_as_float((e & 1) ? (w & 0xffff0000u) : (w << 16));
    else return (float)(int8_t)(w >> (8 * (e & 3)));
    }
}

// The kernel is persistent: a block normalises (or stages) the activation
// rows once and then walks row groups blockIdx.x, + gridDim.x, ... The first
// group's weights are loaded before the dependency wait; each later group's
// are loaded while the previous group's sums are finished.
template <int EPI, bool LN, int RPW, int WS, int CPL, int WT = 0>
__global__ void __launch_bounds__(kWarps * 32)
dec_gemv_kernel(DecArgs a) {
    extern __shared__ __align__(16) float xs[];  // [M][K] when LN
    constexpr int GROUPS = kWarps / WS;          // row groups per block
    constexpr int RPB = GROUPS * RPW;            // rows per block iteration
    __shared__ float s_part[GROUPS][WS][RPW][kMaxRows];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int grp = warp / WS, ks = warp % WS;
    constexpr int EPC = elems_per_chunk<WT>();
    const int K4 = a.K / EPC;                       // 16-byte chunks per row
    const int slice = (K4 + WS - 1) / WS;          // 16-byte chunks per slice
    const int c0 = ks * slice, c1 = min(K4, c0 + slice);
    const int n_iter_rows = a.N;

    // this warp's weight chunks of one row group (registers)
    float4 w[RPW][CPL];
    auto load = [&](int row0) {
#pragma unroll
        for (int r = 0; r < RPW; ++r)
#pragma unroll
            for (int u = 0; u < CPL; ++u) {
                const int c = c0 + u * 32 + lane;
                const bool in = row0 + r < a.N && c < c1;
                if constexpr (WT == 0)
                    w[r][u] = in ? ld_stream(a.W + (size_t)(row0 + r) * a.K + 4 * c) : make_float4(0.f, 0.f, 0.f, 0.f);
                else
                    w[r][u] = in ? ld_stream(reinterpret_cast<const float*>(
                                       reinterpret_cast<const char*>(a.Wq) + ((size_t)(row0 + r) * K4 + c) * 16))
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
            }
    };

    // 1. the first group's weights, before the dependency wait
    load((blockIdx.x * GROUPS + grp) * RPW);
    pdl_trigger();
    pdl_wait();

    // 2. the activation rows, once per block: normalised into shared memory,
    //    or copied there when they fit (kStageFloats), else read through L1
    const float* X = a.x;
    int ldx = a.ldx;
    const bool staged = LN || a.M * a.K <= kStageFloats;
    if constexpr (LN) {
        ln_rows_to_smem(a.x, a.ldx, a.ln_g, a.ln_b, a.eps, a.M, a.K, xs);
        __syncthreads();
        X = xs;
        ldx = a.K;
    } else if (staged) {
        const int K4x = a.K >> 2;
        for (int i = threadIdx.x; i < a.M * K4x; i += kWarps * 32) {
            const int m = i / K4x, c = i - m * K4x;
            reinterpret_cast<float4*>(xs + (size_t)m * a.K)[c] =
                __ldg(reinterpret_cast<const float4*>(a.x + (size_t)m * a.ldx) + c);
        }
        __syncthreads();
        X = xs;
        ldx = a.K;
    }

    // head: this block's best (value, index) per activation row, over all its rows
    float bv = 0.f;
    int bi = -1;
    bool nan0 = false;

    for (int blk = blockIdx.x; blk * RPB < n_iter_rows; blk += gridDim.x) {
        const int row0 = (blk * GROUPS + grp) * RPW;
        // 3. slice sums
        float acc[RPW][kMaxRows];
#pragma unroll
        for (int r = 0; r < RPW; ++r)
#pragma unroll
            for (int m = 0; m < kMaxRows; ++m) acc[r][m] = 0.f;
#pragma unroll
        for (int u = 0; u < CPL; ++u) {
            const int c = c0 + u * 32 + lane;
            if (c < c1) {
                if constexpr (WT == 0 && RPW == 1 && WS == 1 && CPL <= 8) {
                    // every row's activation chunk first, then the sums
                    float4 xv[kMaxRows];
#pragma unroll
                    for (int m = 0; m < kMaxRows; ++m)
                        if (m < a.M)
                            xv[m] = staged ? *reinterpret_cast<const float4*>(X + (size_t)m * ldx + 4 * c)
                                           : __ldg(reinterpret_cast<const float4*>(X + (size_t)m * ldx) + c);
#pragma unroll
                    for (int m = 0; m < kMaxRows; ++m) {
                        if (m < a.M) {
#pragma unroll
                            for (int r = 0; r < RPW; ++r) {
                                float t = acc[r][m];
                                t = fmaf(w[r][u].x, xv[m].x, t);
                                t = fmaf(w[r][u].y, xv[m].y, t);
                                t = fmaf(w[r][u].z, xv[m].z, t);
                                t = fmaf(w[r][u].w, xv[m].w, t);
                                acc[r][m] = t;
                            }
                        }
                    }
                } else {
#pragma unroll
                for (int m = 0; m < kMaxRows; ++m) {
                    if (m < a.M) {
                        {
#pragma unroll
                            for (int q4 = 0; q4 < EPC / 4; ++q4) {
                                // (fp32: EPC / 4 == 1 and chunk_elem is the float4's lanes)
                                const float* xp = X + (size_t)m * ldx + (size_t)c * EPC + 4 * q4;
                                const float4 xv = staged ? *reinterpret_cast<const float4*>(xp)
                                                         : __ldg(reinterpret_cast<const float4*>(xp));
#pragma unroll
                                for (int r = 0; r < RPW; ++r) {
                                    float t = acc[r][m];
                                    t = fmaf(chunk_elem<WT>(w[r][u], 4 * q4 + 0), xv.x, t);
                                    t = fmaf(chunk_elem<WT>(w[r][u], 4 * q4 + 1), xv.y, t);
                                    t = fmaf(chunk_elem<WT>(w[r][u], 4 * q4 + 2), xv.z, t);
                                    t = fmaf(chunk_elem<WT>(w[r][u], 4 * q4 + 3), xv.w, t);
                                    acc[r][m] = t;
                                }
                            }
                        }
                    }
                }
                }
            }
        }
        // the next group's weights go out while this group is finished
        if ((blk + gridDim.x) * RPB < n_iter_rows) load(((blk + gridDim.x) * GROUPS + grp) * RPW);
#pragma unroll
        for (int r = 0; r < RPW; ++r)
#pragma unroll
            for (int m = 0; m < kMaxRows; ++m) {
                if (m >= a.M) break;  // uniform across the block
                float v = acc[r][m];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                acc[r][m] = v;
            }
        if (lane == 0) {
#pragma unroll
            for (int r = 0; r < RPW; ++r)
#pragma unroll
                for (int m = 0; m < kMaxRows; ++m) s_part[grp][ks][r][m] = acc[r][m];
        }
        __syncthreads();

        // 4. epilogue: slice sums in slice order; thread t of a row group
        //    handles (row r, activation row m) pairs
        if constexpr (EPI != DEC_HEAD) {
            const int t = threadIdx.x % (WS * 32);
            if (warp % WS == 0 || WS == 1) {
                for (int q = (WS == 1 ? lane : t); q < RPW * a.M; q += (WS == 1 ? 32 : WS * 32)) {
                    const int r = q / a.M, m = q % a.M;
                    const int j = row0 + r;
                    if (j >= a.N) continue;
                    float sum = s_part[grp][0][r][m];
#pragma unroll
                    for (int k = 1; k < WS; ++k) sum += s_part[grp][k][r][m];
                    if constexpr (WT == 2) sum = sum * __ldg(a.scale + j);
                    float* yp = a.y + (size_t)m * a.ldy + j;
                    float v;
                    if constexpr (EPI == DEC_BIAS || EPI == DEC_QKV_KV) v = apply_epi<EPI_BIAS>(sum, a.bias, j, yp);
                    else if constexpr (EPI == DEC_BIAS_GELU) v = apply_epi<EPI_BIAS_GELU>(sum, a.bias, j, yp);
                    else v = apply_epi<EPI_BIAS_RESID>(sum, a.bias, j, yp);
                    *yp = v;
                    if constexpr (EPI == DEC_QKV_KV) {
                        const int E = a.kv.n_embd;
                        if (j >= E) {
                            const size_t row = a.kv.row(m, a.lens[m]);
                            if (j < 2 * E) a.kv.k[row * E + (j - E)] = v;
                            else a.kv.v[row * E + (j - 2 * E)] = v;
                        }
                    }
                }
            }
        } else {
            // logits (optional) and the running best per activation row; NaN
            // at index 0 is reported as index -2 (the reference's scan never
            // leaves index 0 then)
            if ((int)threadIdx.x < a.M) {
                const int m = threadIdx.x;
                for (int g = 0; g < GROUPS; ++g)
                    for (int r = 0; r < RPW; ++r) {
                        const int j = (blk * GROUPS + g) * RPW + r;
                        if (j >= a.N) continue;
                        float v = s_part[g][0][r][m];
                        for (int k = 1; k < WS; ++k) v += s_part[g][k][r][m];
                        if constexpr (WT == 2) v = v * __ldg(a.scale + j);
                        if (a.y) a.y[(size_t)m * a.ldy + j] = v;
                        if (j == 0 && !(v == v)) nan0 = true;
                        else if (v == v && beats(v, j, bv, bi)) { bv = v; bi = j; }
                    }
            }
        }
        __syncthreads();   // s_part is rewritten by the next group
    }
    if constexpr (EPI == DEC_HEAD) {
        if ((int)threadIdx.x < a.M) {
            a.part_val[(size_t)blockIdx.x * a.M + threadIdx.x] = bv;
            a.part_idx[(size_t)blockIdx.x * a.M + threadIdx.x] = nan0 ? -2 : bi;
        }
    }
}

// Blocks of a launch: one per row group up to four per SM; the kernel walks
// the remaining groups itself.
int gemv_grid(int N, int rows_per_block) {
    static int cap = 0;
    if (!cap) {
        int dev = 0, sms = 148;
        if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) !=
                                                      cudaSuccess) {
            cudaGetLastError();
            sms = 148;
        }
        cap = 4 * sms;
    }
    const int need = (N + rows_per_block - 1) / rows_per_block;
    return need < cap ? need : cap;
}

template <int EPI, bool LN, int RPW, int WS, int CPL, int WT = 0>
cudaError_t dec_launch(const DecArgs& a, cudaStream_t st) {
    // the kernel stages the activation rows whenever it normalises them or
    // they fit kStageFloats; that is exactly when it needs this much
    const bool staged = LN || a.M * a.K <= kStageFloats;
    const size_t smem = staged ? (size_t)a.M * a.K * sizeof(float) : 0;
    auto k = dec_gemv_kernel<EPI, LN, RPW, WS, CPL, WT>;
    if (smem > 32 * 1024) {   // with the static shared memory, beyond the default 48 KB
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    constexpr int rows_per_block = (kWarps / WS) * RPW;
    const int grid = gemv_grid(a.N, rows_per_block);
    cudaError_t e = launch_pdl(k, dim3(grid), dim3(kWarps * 32), smem, st, a);
    return e != cudaSuccess ? e : cudaGetLastError();
}

// The slicing of K for a matrix: each lane holds at most 8 chunks per row.
//   at most 256 chunks per row: whole rows, WS = 1
//   at most 1024: WS = 4; at most 2048 (fp32 only): WS = 4 with 16 chunks per lane
template <int EPI, bool LN, int WT>
cudaError_t dec_dispatch(const DecArgs& a, cudaStream_t st) {
    const int KC = a.K / elems_per_chunk<WT>();
    if (KC <= 256) return dec_launch<EPI, LN, 1, 1, 8, WT>(a, st);
    if (KC <= 1024) return dec_launch<EPI, LN, 1, 4, 8, WT>(a, st);
    if constexpr (WT == 0)
        if (KC <= 2048) return dec_launch<EPI, LN, 1, 4, 16, WT>(a, st);
    return cudaErrorInvalidValue;
}

template <int EPI, int WT>
cudaError_t dec_dispatch_ln(const DecArgs& a, bool ln, cudaStream_t st) {
    return ln ? dec_dispatch<EPI, true, WT>(a, st) : dec_dispatch<EPI, false, WT>(a, st);
}

template <int WT>
cudaError_t dec_dispatch_epi(const DecArgs& a, int epi, bool ln, cudaStream_t st) {
    switch (epi) {
        case EPI_BIAS: return dec_dispatch_ln<DEC_BIAS, WT>(a, ln, st);
        case EPI_BIAS_GELU: return dec_dispatch_ln<DEC_BIAS_GELU, WT>(a, ln, st);
        case EPI_BIAS_RESID: return dec_dispatch_ln<DEC_BIAS_RESID, WT>(a, ln, st);
        case EPI_QKV_KV: return dec_dispatch_ln<DEC_QKV_KV, WT>(a, ln, st);
    }
    return cudaErrorInvalidValue;
}

template <int WT>
cudaError_t head_dispatch(const DecArgs& a, bool ln, cudaStream_t st) {
    const int KC = a.K / elems_per_chunk<WT>();
    if (KC <= 256)
        return ln ? dec_launch<DEC_HEAD, true, 4, 1, 8, WT>(a, st) : dec_launch<DEC_HEAD, false, 4, 1, 8, WT>(a, st);
    if (KC <= 1024)
        return ln ? dec_launch<DEC_HEAD, true, 1, 4, 8, WT>(a, st) : dec_launch<DEC_HEAD, false, 1, 4, 8, WT>(a, st);
    return cudaErrorInvalidValue;
}

int chunk_elems(int wt) { return wt == 0 ? 4 : (wt == 1 ? 8 : 16); }

}  // namespace

// Rows per head block: 4 rows in each of 4 warps while a row is at most 256
// chunks (RPW 4, WS 1), else one row cut into 4 slices (RPW 1, WS 4).
int dec_head_blocks(int V, int K, int wt) {
    const int rows = K / chunk_elems(wt) <= 256 ? kWarps * 4 : 1;
    return gemv_grid(V, rows);
}

// y = [LN](x) . W^T (+ epilogue) for M <= 16 rows, chained with PDL. Weights
// fp32 (W), or with wt 1 / 2 bf16 / int8 (wq, int8 with per-row scales).
cudaError_t launch_dec_gemv(const float* x, int ldx, const float* ln_g, const float* ln_b, float eps,
                            const float* W, const float* bias, float* y, int ldy, int M, int N, int K,
                            int epi, const PagedKV* kv, const int32_t* lens, cudaStream_t st, int wt,
                            const void* wq, const float* scale) {
    if (M <= 0 || M > kMaxRows || (ldx & 3) || wt < 0 || wt > 2 || K % chunk_elems(wt)) return cudaErrorInvalidValue;
    if ((wt != 0 && !wq) || (wt == 2 && !scale)) return cudaErrorInvalidValue;
    if (epi == EPI_QKV_KV && (!kv || !lens)) return cudaErrorInvalidValue;
    DecArgs a{};
    a.x = x; a.ldx = ldx; a.ln_g = ln_g; a.ln_b = ln_b; a.eps = eps; a.W = W; a.bias = bias;
    a.Wq = wq; a.scale = scale;
    a.y = y; a.ldy = ldy; a.M = M; a.N = N; a.K = K;
    if (kv) a.kv = *kv;
    a.lens = lens;
    const bool ln = ln_g != nullptr;
    if (wt == 1) return dec_dispatch_epi<1>(a, epi, ln, st);
    if (wt == 2) return dec_dispatch_epi<2>(a, epi, ln, st);
    return dec_dispatch_epi<0>(a, epi, ln, st);
}

// The tied head with LN_f in its prologue: logits (optional) and per-block
// partial maxima for launch_argmax_finalize.
cudaError_t launch_dec_head(const float* x, int ldx, const float* ln_g, const float* ln_b, float eps,
                            const float* W, float* logits, int ldl, int M, int V, int K, float* part_val,
                            int* part_idx, cudaStream_t st, int wt, const void* wq, const float* scale) {
    if (M <= 0 || M > kMaxRows || (ldx & 3) || wt < 0 || wt > 2 || K % chunk_elems(wt)) return cudaErrorInvalidValue;
    if ((wt != 0 && !wq) || (wt == 2 && !scale)) return cudaErrorInvalidValue;
    DecArgs a{};
    a.x = x; a.ldx = ldx; a.ln_g = ln_g; a.ln_b = ln_b; a.eps = eps; a.W = W; a.Wq = wq; a.scale = scale;
    a.y = logits; a.ldy = ldl; a.M = M; a.N = V; a.K = K; a.part_val = part_val; a.part_idx = part_idx;
    const bool ln = ln_g != nullptr;
    if (wt == 1) return head_dispatch<1>(a, ln, st);
    if (wt == 2) return head_dispatch<2>(a, ln, st);
    return head_dispatch<0>(a, ln, st);
}

}  // namespace tie
