// k_decode.cu -- the small-batch decode matmuls (up to 16 rows; the decode step
// sends batches of at most 8 sequences here, larger ones to the tensor cores),
// chained with programmatic dependent launch.
//
// A decode step at batch 1 moves ~0.5 GB of fp32 weights through a few dozen
// matmuls whose individual transfers take ~1 us at HBM speed, so the step is
// bound by the gaps between kernels as much as by bandwidth. Two measures:
//
//   * fusion: the K/V rows of a step are stored by the QKV matmul's epilogue,
//     bias, GELU and the residual add run in the epilogues, and the tied head
//     keeps a running greedy argmax (LayerNorm runs once per row before the
//     matmul that consumes it, in layernorm_kernel);
//   * programmatic dependent launch: every kernel first issues the loads of its
//     own weight rows (which no earlier kernel writes), then lets the next
//     kernel launch (griddepcontrol.launch_dependents), and only then waits for
//     its predecessor's results (griddepcontrol.wait). Weight streaming thus
//     overlaps the previous kernel's tail and the launch latency.
//
// Each warp holds all of its weight chunks of a row group in registers (loaded
// before the dependency wait), so a matrix is in flight in one round trip. The
// kernel is compiled per row bucket (1, 2, 4, 8 or 16 activation rows), so its
// accumulators, registers and code are those of the batch it runs.
#include <algorithm>

#include "common.cuh"

namespace tie {
namespace {

constexpr int kWarps = 4;
constexpr int kMaxRows = 16;
constexpr int kFreeSms = 16;   // SMs a GEMV's grid leaves to the next kernel

__device__ __forceinline__ float4 ld_stream(const float* p) {
    float4 v;
    // volatile: the compiler keeps the load where it is written, ahead of
    // griddepcontrol.wait; a plain asm without memory operands may be moved
    // past the wait, putting the whole weight round trip after it
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
        : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
        : "l"(p));
    return v;
}

struct DecArgs {
    const float* x;   // input rows [M][ldx]
    int ldx;
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
// at once; after the wait it only reads the activation rows (through L1) and
// reduces.
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

// The kernel is persistent (one wave: the grid is what fits on the GPU at
// once) and walks row groups blockIdx.x, + gridDim.x, ... The first group's
// weights are loaded before the dependency wait; each later group's are
// loaded while the previous group's sums are finished. MB is the row bucket:
// a.M <= MB activation rows.
// At one activation row the matrices need up to 768 blocks (GPT-2 small's FC
// and MLP): seven resident blocks per SM (at most 72 registers) keep them in
// one wave; the fp32 and bf16 variants of up to 8 chunks fit without spills.
// Every other variant gives 0, which leaves the minimum unspecified: an
// explicit 1 is not neutral, ptxas then spends registers freely (the 8-row
// MLP variant went from 166 to 214 registers, 3 to 2 blocks per SM, and
// GPT-2 medium at batch 8 lost a fifth of its throughput).
template <int EPI, int MB, int CPL, int WT>
constexpr int dec_min_blocks() { return EPI != DEC_HEAD && MB == 1 && CPL <= 8 && WT != 2 ? 7 : 0; }

template <int EPI, int MB, int RPW, int WS, int CPL, int WT = 0>
__global__ void __launch_bounds__(kWarps * 32, dec_min_blocks<EPI, MB, CPL, WT>())
dec_gemv_kernel(DecArgs a) {
    constexpr int GROUPS = kWarps / WS;          // row groups per block
    constexpr int RPB = GROUPS * RPW;            // rows per block iteration
    __shared__ float s_part[GROUPS][WS][RPW][MB];
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

    // The epilogue's operands. A thread finishes at most one (row, activation
    // row) pair of a group: pair q = lane of the slice-0 warp, row q / M and
    // activation row q % M. Its bias and int8 scale are weights, loaded with
    // the group's weights before the dependency wait; its residual and
    // sequence length are read right after the wait (or after the previous
    // group's epilogue), so no load is left between the sums and the store.
    static_assert(EPI == DEC_HEAD || RPW * MB <= 32, "one epilogue pair per thread");
    const bool ep_on = EPI != DEC_HEAD && warp % WS == 0 && lane < RPW * a.M;
    const int ep_r = ep_on ? lane / a.M : 0, ep_m = ep_on ? lane % a.M : 0;
    float ep_bias = 0.f, ep_scale = 1.f, ep_res = 0.f;
    int ep_len = 0;
    auto ep_weights = [&](int row0, float& b, float& sc) {
        if (ep_on && row0 + ep_r < a.N) {
            b = __ldg(a.bias + row0 + ep_r);
            if constexpr (WT == 2) sc = __ldg(a.scale + row0 + ep_r);
        }
    };
    auto ep_inputs = [&](int row0) {
        if (ep_on && row0 + ep_r < a.N) {
            if constexpr (EPI == DEC_BIAS_RESID) ep_res = a.y[(size_t)ep_m * a.ldy + row0 + ep_r];
            if constexpr (EPI == DEC_QKV_KV) ep_len = a.lens[ep_m];
        }
    };

    // 1. the first group's weights, before the dependency wait
    load((blockIdx.x * GROUPS + grp) * RPW);
    ep_weights((blockIdx.x * GROUPS + grp) * RPW, ep_bias, ep_scale);
    pdl_trigger();
    pdl_wait();
    ep_inputs((blockIdx.x * GROUPS + grp) * RPW);

    const float* X = a.x;
    const int ldx = a.ldx;

    // head: this block's best (value, index) per activation row, over all its rows
    float bv = 0.f;
    int bi = -1;
    bool nan0 = false;

    for (int blk = blockIdx.x; blk * RPB < n_iter_rows; blk += gridDim.x) {
        const int row0 = (blk * GROUPS + grp) * RPW;
        // 3. slice sums
        float acc[RPW][MB];
#pragma unroll
        for (int r = 0; r < RPW; ++r)
#pragma unroll
            for (int m = 0; m < MB; ++m) acc[r][m] = 0.f;
#pragma unroll
        for (int u = 0; u < CPL; ++u) {
            const int c = c0 + u * 32 + lane;
            if (c < c1) {
                if constexpr (WT == 0 && RPW == 1 && WS == 1 && CPL <= 8) {
                    // every row's activation chunk first, then the sums
                    float4 xv[MB];
#pragma unroll
                    for (int m = 0; m < MB; ++m)
                        if (m < a.M) xv[m] = __ldg(reinterpret_cast<const float4*>(X + (size_t)m * ldx) + c);
#pragma unroll
                    for (int m = 0; m < MB; ++m) {
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
                for (int m = 0; m < MB; ++m) {
                    if (m < a.M) {
                        {
#pragma unroll
                            for (int q4 = 0; q4 < EPC / 4; ++q4) {
                                // (fp32: EPC / 4 == 1 and chunk_elem is the float4's lanes)
                                const float* xp = X + (size_t)m * ldx + (size_t)c * EPC + 4 * q4;
                                const float4 xv = __ldg(reinterpret_cast<const float4*>(xp));
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
        const bool more = (blk + gridDim.x) * RPB < n_iter_rows;
        const int next0 = ((blk + gridDim.x) * GROUPS + grp) * RPW;
        float nbias = 0.f, nscale = 1.f;
        if (more) {
            load(next0);
            ep_weights(next0, nbias, nscale);
        }
#pragma unroll
        for (int r = 0; r < RPW; ++r)
#pragma unroll
            for (int m = 0; m < MB; ++m) {
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
                for (int m = 0; m < MB; ++m) s_part[grp][ks][r][m] = acc[r][m];
        }
        __syncthreads();

        // 4. epilogue: slice sums in slice order; thread t of a row group
        //    handles (row r, activation row m) pairs
        if constexpr (EPI != DEC_HEAD) {
            const int j = row0 + ep_r;
            if (ep_on && j < a.N) {
                const int r = ep_r, m = ep_m;
                float sum = s_part[grp][0][r][m];
#pragma unroll
                for (int k = 1; k < WS; ++k) sum += s_part[grp][k][r][m];
                if constexpr (WT == 2) sum = sum * ep_scale;
                // bias, GELU or residual as apply_epi (common.cuh) computes them
                float v = __fadd_rn(sum, ep_bias);
                if constexpr (EPI == DEC_BIAS_GELU) v = gelu_new_ref(v);
                if constexpr (EPI == DEC_BIAS_RESID) v = __fadd_rn(ep_res, v);
                a.y[(size_t)m * a.ldy + j] = v;
                if constexpr (EPI == DEC_QKV_KV) {
                    const int E = a.kv.n_embd;
                    if (j >= E) {
                        const size_t row = a.kv.row(m, ep_len);
                        if (j < 2 * E) a.kv.k[row * E + (j - E)] = v;
                        else a.kv.v[row * E + (j - 2 * E)] = v;
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
        if (more) {
            ep_bias = nbias;
            ep_scale = nscale;
            ep_inputs(next0);
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

// Blocks of a launch: one per row group, up to what fits on the GPU at once
// (the kernel's occupancy, so the persistent grid is one wave); the kernel
// walks the remaining groups itself.
int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) !=
                                                      cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = 148;
        }
    }
    return n;
}

template <int EPI, int MB, int RPW, int WS, int CPL, int WT = 0>
int resident_blocks() {
    static int per_sm = 0;
    if (!per_sm) {
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, dec_gemv_kernel<EPI, MB, RPW, WS, CPL, WT>,
                                                          kWarps * 32, 0) != cudaSuccess || per_sm <= 0) {
            cudaGetLastError();
            per_sm = 1;
        }
    }
    // all but kFreeSms SMs: the blocks of the next kernel in the chain (a
    // LayerNorm row, the attention heads) become resident under programmatic
    // dependent launch while this one runs (measured on B200: GPT-2 medium,
    // batch 8, 4086 -> 4213 tok/s; batch 1 unchanged within 1%)
    return per_sm * (sm_count() - kFreeSms);
}

template <int EPI, int MB, int RPW, int WS, int CPL, int WT = 0>
cudaError_t dec_launch(const DecArgs& a, cudaStream_t st) {
    constexpr int rows_per_block = (kWarps / WS) * RPW;
    const int need = (a.N + rows_per_block - 1) / rows_per_block;
    const int grid = std::min(need, resident_blocks<EPI, MB, RPW, WS, CPL, WT>());
    cudaError_t e = launch_pdl(dec_gemv_kernel<EPI, MB, RPW, WS, CPL, WT>, dim3(grid), dim3(kWarps * 32), 0, st, a);
    return e != cudaSuccess ? e : cudaGetLastError();
}

// The row bucket of M activation rows
template <int EPI, int RPW, int WS, int CPL, int WT>
cudaError_t dec_launch_m(const DecArgs& a, cudaStream_t st) {
    if (a.M <= 1) return dec_launch<EPI, 1, RPW, WS, CPL, WT>(a, st);
    if (a.M <= 2) return dec_launch<EPI, 2, RPW, WS, CPL, WT>(a, st);
    if (a.M <= 4) return dec_launch<EPI, 4, RPW, WS, CPL, WT>(a, st);
    if (a.M <= 8) return dec_launch<EPI, 8, RPW, WS, CPL, WT>(a, st);
    return dec_launch<EPI, 16, RPW, WS, CPL, WT>(a, st);
}

// The slicing of K for a matrix: each lane holds at most 8 chunks per row.
//   at most 256 chunks per row: whole rows, WS = 1
//   at most 1024: WS = 4; at most 2048 (fp32 only): WS = 4 with 16 chunks per lane
template <int EPI, int WT>
cudaError_t dec_dispatch(const DecArgs& a, cudaStream_t st) {
    const int KC = a.K / elems_per_chunk<WT>();
    if (KC <= 256) return dec_launch_m<EPI, 1, 1, 8, WT>(a, st);
    if (KC <= 1024) return dec_launch_m<EPI, 1, 4, 8, WT>(a, st);
    if constexpr (WT == 0)
        if (KC <= 2048) return dec_launch_m<EPI, 1, 4, 16, WT>(a, st);
    return cudaErrorInvalidValue;
}

template <int WT>
cudaError_t dec_dispatch_epi(const DecArgs& a, int epi, cudaStream_t st) {
    switch (epi) {
        case EPI_BIAS: return dec_dispatch<DEC_BIAS, WT>(a, st);
        case EPI_BIAS_GELU: return dec_dispatch<DEC_BIAS_GELU, WT>(a, st);
        case EPI_BIAS_RESID: return dec_dispatch<DEC_BIAS_RESID, WT>(a, st);
        case EPI_QKV_KV: return dec_dispatch<DEC_QKV_KV, WT>(a, st);
    }
    return cudaErrorInvalidValue;
}

template <int WT>
cudaError_t head_dispatch(const DecArgs& a, cudaStream_t st) {
    const int KC = a.K / elems_per_chunk<WT>();
    if (KC <= 256) return dec_launch_m<DEC_HEAD, 4, 1, 8, WT>(a, st);
    if (KC <= 1024) return dec_launch_m<DEC_HEAD, 1, 4, 8, WT>(a, st);
    return cudaErrorInvalidValue;
}

int chunk_elems(int wt) { return wt == 0 ? 4 : (wt == 1 ? 8 : 16); }

// Blocks of the tied head's launch for M rows (one partial best per block
// and row): 4 rows in each of 4 warps while a row is at most 256 chunks
// (RPW 4, WS 1), else one row cut into 4 slices (RPW 1, WS 4).
template <int WT>
int head_blocks_wt(int V, int K, int M) {
    const bool whole = K / elems_per_chunk<WT>() <= 256;
    const int rows = whole ? kWarps * 4 : 1;
    const int need = (V + rows - 1) / rows;
    int cap;
    if (whole) {
        cap = M <= 1 ? resident_blocks<DEC_HEAD, 1, 4, 1, 8, WT>() : M <= 2 ? resident_blocks<DEC_HEAD, 2, 4, 1, 8, WT>()
            : M <= 4 ? resident_blocks<DEC_HEAD, 4, 4, 1, 8, WT>() : M <= 8 ? resident_blocks<DEC_HEAD, 8, 4, 1, 8, WT>()
            : resident_blocks<DEC_HEAD, 16, 4, 1, 8, WT>();
    } else {
        cap = M <= 1 ? resident_blocks<DEC_HEAD, 1, 1, 4, 8, WT>() : M <= 2 ? resident_blocks<DEC_HEAD, 2, 1, 4, 8, WT>()
            : M <= 4 ? resident_blocks<DEC_HEAD, 4, 1, 4, 8, WT>() : M <= 8 ? resident_blocks<DEC_HEAD, 8, 1, 4, 8, WT>()
            : resident_blocks<DEC_HEAD, 16, 1, 4, 8, WT>();
    }
    return std::min(need, cap);
}

}  // namespace

// Blocks (one partial best per block and row) of the tied head's launch for
// M rows; and the most any row count or weight format uses (buffer sizing).
int dec_head_blocks(int V, int K, int wt, int M) {
    return wt == 1 ? head_blocks_wt<1>(V, K, M) : wt == 2 ? head_blocks_wt<2>(V, K, M) : head_blocks_wt<0>(V, K, M);
}

int dec_head_blocks_max(int V, int K) {
    int n = 0;
    for (int wt : {0, 1, 2})
        for (int M : {1, 2, 4, 8, 16}) n = std::max(n, dec_head_blocks(V, K, wt, M));
    return n;
}

// y = x . W^T (+ epilogue) for M <= 16 rows, chained with PDL. Weights fp32
// (W), or with wt 1 / 2 bf16 / int8 (wq, int8 with per-row scales).
cudaError_t launch_dec_gemv(const float* x, int ldx, const float* ln_g, const float* ln_b, float eps,
                            const float* W, const float* bias, float* y, int ldy, int M, int N, int K,
                            int epi, const PagedKV* kv, const int32_t* lens, cudaStream_t st, int wt,
                            const void* wq, const float* scale) {
    (void)eps;
    if (M <= 0 || M > kMaxRows || (ldx & 3) || wt < 0 || wt > 2 || K % chunk_elems(wt)) return cudaErrorInvalidValue;
    if (ln_g || ln_b) return cudaErrorInvalidValue;   // LayerNorm runs in layernorm_kernel
    if ((wt != 0 && !wq) || (wt == 2 && !scale)) return cudaErrorInvalidValue;
    if (epi == EPI_QKV_KV && (!kv || !lens)) return cudaErrorInvalidValue;
    DecArgs a{};
    a.x = x; a.ldx = ldx; a.W = W; a.bias = bias;
    a.Wq = wq; a.scale = scale;
    a.y = y; a.ldy = ldy; a.M = M; a.N = N; a.K = K;
    if (kv) a.kv = *kv;
    a.lens = lens;
    if (wt == 1) return dec_dispatch_epi<1>(a, epi, st);
    if (wt == 2) return dec_dispatch_epi<2>(a, epi, st);
    return dec_dispatch_epi<0>(a, epi, st);
}

cudaError_t launch_dec_head(const float* x, int ldx, const float* ln_g, const float* ln_b, float eps,
                            const float* W, float* logits, int ldl, int M, int V, int K, float* part_val,
                            int* part_idx, cudaStream_t st, int wt, const void* wq, const float* scale) {
    (void)eps;
    if (M <= 0 || M > kMaxRows || (ldx & 3) || wt < 0 || wt > 2 || K % chunk_elems(wt)) return cudaErrorInvalidValue;
    if (ln_g || ln_b) return cudaErrorInvalidValue;   // LN_f runs in layernorm_kernel
    if ((wt != 0 && !wq) || (wt == 2 && !scale)) return cudaErrorInvalidValue;
    DecArgs a{};
    a.x = x; a.ldx = ldx; a.W = W; a.Wq = wq; a.scale = scale;
    a.y = logits; a.ldy = ldl; a.M = M; a.N = V; a.K = K; a.part_val = part_val; a.part_idx = part_idx;
    if (wt == 1) return head_dispatch<1>(a, st);
    if (wt == 2) return head_dispatch<2>(a, st);
    return head_dispatch<0>(a, st);
}

}  // namespace tie
