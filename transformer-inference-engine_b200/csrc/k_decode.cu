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
#include "mbar.cuh"

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

// ---------------------------------------------------------------------------
// The stream path (launch_stream_gemv): decode matmuls of 1-8 rows with the
// weights staged in shared memory by the bulk-copy engine.
//
// A CTA owns a contiguous range of weight-row groups of g rows; a group is
// g * K contiguous weight bytes, one bulk copy into one stage of a ring. The
// producer warp issues the first stages as soon as the CTA starts (no kernel
// writes weights, so nothing waits for the predecessor) and refills stages as
// the compute warps release them. A CTA takes at most ~110 KB of shared memory
// and 288 threads, so the next kernel's CTAs are resident beside it under
// programmatic dependent launch and have their own weights in flight while
// this one computes: the weight stream runs ahead of the dependency chain.
//
// After the dependency wait the eight compute warps build the input rows in
// shared memory (the prologue) and reduce each stage: warp w takes row w / WS
// of the stage and K-slice w % WS, with dec_gemv_kernel's arithmetic -- lane c
// of a slice accumulates 16-byte chunks c, c + 32, ... (elements in order),
// an xor butterfly, then the WS slice sums in slice order. The prologue's
// LayerNorm is the canonical order of common.cuh, and the merge of attention
// chunk partials is merge_warp's (k_attn.cu), so a step on this path is
// bit-identical to the chain of separate kernels.
constexpr int kSgCompute = 8;                       // compute warps
constexpr int kSgThreads = (kSgCompute + 1) * 32;   // + the producer warp
constexpr int kSgMaxRows = 8;                       // activation rows
constexpr int kSgMaxStages = 8;
constexpr int kSgStageTarget = 24 * 1024;           // bytes of weights per stage, about
constexpr int kSgSmemBudget = 100 * 1024;           // two consecutive kernels' CTAs share an SM
constexpr int kSgHeadBudget = 200 * 1024;           // the head, last in the chain, takes the SM
constexpr int kSgXsMax = 48 * 1024;                 // input rows staged in shared memory up to this size
constexpr int kAttnD = 64, kAttnPart = kAttnD + 2, kAttnPg = 16;

struct SgArgs {
    int epi, head, pro;   // DEC_* epilogue, the tied head, StreamPro
    const float* x;
    int ldx;
    const float *ln_g, *ln_b;
    float eps;
    const int32_t* tokens;
    const float *wte, *wpe;
    float* x_out;
    int V;
    const float* apart;
    int H, max_chunks;
    const int32_t* lens;
    const char* W;        // fp32 / bf16 / int8 rows, K elements each
    const float* scale;
    const float* bias;
    float* y;
    int ldy;
    int M, N, K;
    PagedKV kv;
    float* part_val;
    int* part_idx;
    int g, ws, stages, gpc;   // rows per stage, slices per row, ring stages, groups per CTA
    int xs;                   // input rows in shared memory (else read from global memory)
    uint32_t stage_bytes;     // ring stride
    uint32_t off_x, off_ring; // shared-memory offsets (bytes)
    int* err;
    int stall;
    unsigned long long wait_ns;
    unsigned long long* trace;
};

// fixed part of the shared-memory layout: barriers, reductions, partial sums,
// per-row epilogue operands; then x rows, then the ring
struct SgFixed {
    static constexpr uint32_t bars = 0;                                   // full[8], empty[8], never, flag
    static constexpr uint32_t red = 256;                                  // double [2][8 rows][8 groups]
    static constexpr uint32_t part = red + 2 * kSgMaxRows * 8 * 8;        // float [2][8 warps][8 rows]
    static constexpr uint32_t best = part + 2 * kSgCompute * kSgMaxRows * 4;  // (float, int) [16 warps][8]
    static constexpr uint32_t lens = best + kSgCompute * kSgMaxRows * 8;  // int [8]
    static constexpr uint32_t epi = lens + kSgMaxRows * 4;                // bias [R], scale [R], resid [M][R]
};

__host__ __device__ inline uint32_t sg_align(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

// bounded wait; also gives up once `stop` is set (another warp gave up)
__device__ __forceinline__ bool sg_wait(uint64_t* bar, uint32_t parity, unsigned long long limit,
                                        volatile int* stop) {
    if (mbar_test(bar, parity)) return true;
    const unsigned long long t0 = gtime();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try(bar, parity)) return true;
        if ((i & 63u) == 0) {
            if (*stop) return false;
            if (gtime() - t0 > limit) return false;
        }
    }
}

template <int WT, int MB>
__global__ void __launch_bounds__(kSgThreads, 2)
stream_gemv_kernel(const __grid_constant__ SgArgs a) {
    extern __shared__ __align__(128) uint8_t sg_smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(sg_smem + SgFixed::bars);
    uint64_t* empty = full + kSgMaxStages;
    uint64_t* never = empty + kSgMaxStages;
    // set once any warp gives up a bounded wait; the others then stop waiting
    volatile int* stop = reinterpret_cast<volatile int*>(never + 1);
    double* s_red = reinterpret_cast<double*>(sg_smem + SgFixed::red);
    float* s_part = reinterpret_cast<float*>(sg_smem + SgFixed::part);
    float* s_bv = reinterpret_cast<float*>(sg_smem + SgFixed::best);
    int* s_bi = reinterpret_cast<int*>(sg_smem + SgFixed::best + kSgCompute * kSgMaxRows * 4);
    int* s_lens = reinterpret_cast<int*>(sg_smem + SgFixed::lens);
    const int R = a.gpc * a.g;   // weight rows of this CTA's range
    float* s_bias = reinterpret_cast<float*>(sg_smem + SgFixed::epi);
    float* s_scale = s_bias + R;
    float* s_res = s_scale + R;
    float* x_s = reinterpret_cast<float*>(sg_smem + a.off_x);
    uint8_t* ring = sg_smem + a.off_ring;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int EPI = a.head ? (int)DEC_HEAD : a.epi, PRO = a.pro;
    constexpr int EPC = elems_per_chunk<WT>();
    constexpr int BPE = WT == 0 ? 4 : (WT == 1 ? 2 : 1);
    const int M = a.M, K = a.K, S = a.stages;
    const int g0 = blockIdx.x * a.gpc;                                   // first group
    const int ng = max(0, min(a.gpc, (a.N + a.g - 1) / a.g - g0));      // groups of this CTA
    const int row_base = g0 * a.g;
    const unsigned long long limit = a.wait_ns ? a.wait_ns : kWaitNs;
    unsigned long long* tr = a.trace ? a.trace + (size_t)blockIdx.x * kStreamTraceEvents : nullptr;
    if (tr && tid == 0) tr[0] = gtime();

    if (tid == 0) {
        for (int s = 0; s < kSgMaxStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kSgCompute);
        }
        mbar_init(never, 1);
        *stop = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    pdl_trigger();

    if (warp == kSgCompute) {
        // ------------------------------------------------------- producer
        if (lane == 0) {
            const uint64_t pol = evict_first_policy();
            const size_t row_bytes = (size_t)K * BPE;
            int issued = 0;
            for (int i = 0; i < ng; ++i) {
                const int slot = i % S;
                if (i >= S && !sg_wait(&empty[slot], (uint32_t)((i / S) - 1) & 1u, limit, stop)) {
                    *stop = 1;
                    atomicExch(a.err, 1);
                    break;
                }
                const int row0 = (g0 + i) * a.g;
                const uint32_t bytes = (uint32_t)(min(a.g, a.N - row0) * row_bytes);
                mbar_expect_tx(&full[slot], bytes);
                bulk_load(ring + (size_t)slot * a.stage_bytes, a.W + (size_t)row0 * row_bytes, bytes, &full[slot], pol);
                ++issued;
            }
            if (tr) tr[6] = gtime();
            // every copy this thread started has landed before the CTA may exit
            for (int j = issued > S ? issued - S : 0; j < issued; ++j)
                if (!sg_wait(&full[j % S], (uint32_t)(j / S) & 1u, limit, stop)) {
                    const unsigned long long t0 = gtime();
                    while (!mbar_try(&full[j % S], (uint32_t)(j / S) & 1u) && gtime() - t0 < limit) {
                    }
                }
        }
        return;
    }

    // ------------------------------------------------------------ compute
    // operands that no earlier kernel writes: before the dependency wait
    if (EPI != DEC_HEAD) {
        for (int t = tid; t < R; t += kSgCompute * 32)
            s_bias[t] = row_base + t < a.N ? __ldg(a.bias + row_base + t) : 0.f;
    }
    if constexpr (WT == 2) {
        for (int t = tid; t < R; t += kSgCompute * 32)
            s_scale[t] = row_base + t < a.N ? __ldg(a.scale + row_base + t) : 1.f;
    }
    float gam[8], bet[8];   // LayerNorm gain and shift of elements tid + 256 j (threads < 256)
    if ((PRO == STREAM_PRO_LN || PRO == STREAM_PRO_EMBED_LN) && tid < 256) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int i = tid + 256 * j;
            gam[j] = i < K ? __ldg(a.ln_g + i) : 0.f;
            bet[j] = i < K ? __ldg(a.ln_b + i) : 0.f;
        }
    }
    pdl_wait();
    if (tr && tid == 0) tr[1] = gtime();

    // ----------------------------------------------------------- prologue
    if (tid < M && (PRO == STREAM_PRO_EMBED_LN || PRO == STREAM_PRO_MERGE || EPI == DEC_QKV_KV))
        s_lens[tid] = __ldcg(a.lens + tid);
    if (EPI == DEC_BIAS_RESID) {
        for (int t = tid; t < M * R; t += kSgCompute * 32) {
            const int m = t / R, r = t % R;
            s_res[t] = row_base + r < a.N ? __ldcg(a.y + (size_t)m * a.ldy + row_base + r) : 0.f;
        }
    }
    const int K4 = K >> 2;
    if (PRO == STREAM_PRO_PLAIN || PRO == STREAM_PRO_LN) {
        if (a.xs)
            for (int t = tid; t < M * K4; t += kSgCompute * 32) {
                const int m = t / K4, c = t % K4;
                reinterpret_cast<float4*>(x_s)[t] = __ldcg(reinterpret_cast<const float4*>(a.x + (size_t)m * a.ldx) + c);
            }
    }
    if (PRO == STREAM_PRO_EMBED_LN) {
        bar_sync(1, kSgCompute * 32);   // s_lens
        for (int t = tid; t < M * K4; t += kSgCompute * 32) {
            const int m = t / K4, c = t % K4;
            const int id = __ldcg(a.tokens + m);
            float4 v;
            if ((unsigned)id >= (unsigned)a.V) {
                v = make_float4(NAN, NAN, NAN, NAN);
            } else {
                const float4 e = __ldg(reinterpret_cast<const float4*>(a.wte + (size_t)id * K) + c);
                const float4 p = __ldg(reinterpret_cast<const float4*>(a.wpe + (size_t)s_lens[m] * K) + c);
                v = make_float4(__fadd_rn(e.x, p.x), __fadd_rn(e.y, p.y), __fadd_rn(e.z, p.z), __fadd_rn(e.w, p.w));
            }
            reinterpret_cast<float4*>(x_s)[t] = v;
            if (blockIdx.x == 0) reinterpret_cast<float4*>(a.x_out + (size_t)m * K)[c] = v;
        }
    }
    if (PRO == STREAM_PRO_LN || PRO == STREAM_PRO_EMBED_LN) {
        // LayerNorm of every row in place, the canonical order: thread tid is
        // virtual lane tid, warp w group w
        bar_sync(1, kSgCompute * 32);
        // the canonical sums are formed by threads 0..255 (virtual lanes), warps 0..7 (groups)
        const bool vl = tid < 256;
        double acc[MB];
#pragma unroll
        for (int m = 0; m < MB; ++m) {
            acc[m] = 0.0;
            if (m < M && vl)
                for (int i = tid; i < K; i += 256) acc[m] = __dadd_rn(acc[m], (double)x_s[m * K + i]);
            acc[m] = ln_warp_sum_d(acc[m]);
        }
        if (lane == 0 && vl)
#pragma unroll
            for (int m = 0; m < MB; ++m) s_red[m * 8 + warp] = acc[m];
        bar_sync(1, kSgCompute * 32);
        double mean[MB];
#pragma unroll
        for (int m = 0; m < MB; ++m) {
            double S_ = s_red[m * 8];
#pragma unroll
            for (int w = 1; w < kLnGroups; ++w) S_ = __dadd_rn(S_, s_red[m * 8 + w]);
            mean[m] = S_ / (double)K;
            acc[m] = 0.0;
            if (m < M && vl)
                for (int i = tid; i < K; i += 256) {
                    const double d = __dadd_rn((double)x_s[m * K + i], -mean[m]);
                    acc[m] = __dadd_rn(acc[m], __dmul_rn(d, d));
                }
            acc[m] = ln_warp_sum_d(acc[m]);
        }
        if (lane == 0 && vl)
#pragma unroll
            for (int m = 0; m < MB; ++m) s_red[kSgMaxRows * 8 + m * 8 + warp] = acc[m];
        bar_sync(1, kSgCompute * 32);
#pragma unroll
        for (int m = 0; m < MB; ++m) {
            if (m >= M) break;
            double V_ = s_red[kSgMaxRows * 8 + m * 8];
#pragma unroll
            for (int w = 1; w < kLnGroups; ++w) V_ = __dadd_rn(V_, s_red[kSgMaxRows * 8 + m * 8 + w]);
            const float inv = (float)(1.0 / sqrt(__dadd_rn(V_ / (double)K, (double)a.eps)));
            if (vl)
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int i = tid + 256 * j;
                    if (i < K) x_s[m * K + i] = ln_apply(x_s[m * K + i], mean[m], inv, gam[j], bet[j]);
                }
        }
    }
    if (PRO == STREAM_PRO_MERGE) {
        // attention rows from the chunk partials: warp per (row, head), the
        // arithmetic of merge_warp
        bar_sync(1, kSgCompute * 32);   // s_lens
        for (int p = warp; p < M * a.H; p += kSgCompute) {
            const int m = p / a.H, h = p % a.H;
            const int ns = (s_lens[m] + 1 + kAttnPg - 1) / kAttnPg;
            const float* P = a.apart + (size_t)(m * a.H + h) * a.max_chunks * kAttnPart;
            float mx = -INFINITY;
            for (int k = lane; k < ns; k += 32) mx = fmaxf(mx, __ldcg(P + (size_t)k * kAttnPart));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            float lt = 0.f, o0 = 0.f, o1 = 0.f;
            for (int k0 = 0; k0 < ns; k0 += 16) {
                float2 ml[16], ov[16];
#pragma unroll
                for (int k = 0; k < 16; ++k)
                    if (k0 + k < ns) {
                        ml[k] = __ldcg(reinterpret_cast<const float2*>(P + (size_t)(k0 + k) * kAttnPart));
                        ov[k] = __ldcg(reinterpret_cast<const float2*>(P + (size_t)(k0 + k) * kAttnPart + 2 + 2 * lane));
                    }
#pragma unroll
                for (int k = 0; k < 16; ++k)
                    if (k0 + k < ns) {
                        const float cf = expf(ml[k].x - mx);
                        lt = fmaf(ml[k].y, cf, lt);
                        o0 = fmaf(ov[k].x, cf, o0);
                        o1 = fmaf(ov[k].y, cf, o1);
                    }
            }
            *reinterpret_cast<float2*>(x_s + (size_t)m * K + h * kAttnD + 2 * lane) = make_float2(o0 / lt, o1 / lt);
        }
    }
    bar_sync(1, kSgCompute * 32);
    if (tr && tid == 0) tr[2] = gtime();

    // failure drill: a barrier that nothing completes; the bounded wait expires
    if (a.stall && !sg_wait(never, 0, limit, stop)) {
        if (tid == 0) atomicExch(a.err, 1);
        *stop = 1;
    }

    // -------------------------------------------------------------- stages
    // Warps run through the stages independently (a warp that gives up keeps
    // going without computing, so every barrier below is met by all of its
    // warps). With WS = 1 a warp owns a whole row and finishes it itself;
    // with WS = 4 the four warps of a row meet on a 128-thread barrier and the
    // slice-0 warp adds the slice sums in order.
    const int K4c = K / EPC;                              // 16-byte chunks per row
    const int slice = (K4c + a.ws - 1) / a.ws;
    const int my_r = warp / a.ws, my_s = warp % a.ws;
    const int c0 = my_s * slice, c1 = min(K4c, c0 + slice);
    float bv = 0.f;   // head: this lane's best (value, index) for activation row `lane`, and NaN at 0
    int bi = -1;
    bool nan0 = false;
    for (int i = 0; i < ng; ++i) {
        const int slot = i % S, buf = i & 1;
        const int row0 = (g0 + i) * a.g, rows = min(a.g, a.N - row0);
        const bool ok = sg_wait(&full[slot], (uint32_t)(i / S) & 1u, limit, stop);
        if (tr && tid == 0 && i == 0) tr[3] = gtime();
        if (!ok) {
            *stop = 1;
            if (lane == 0) atomicExch(a.err, 1);
        }
        float acc[MB];
#pragma unroll
        for (int m = 0; m < MB; ++m) acc[m] = 0.f;
        if (ok && my_r < rows) {
            const uint8_t* wrow = ring + (size_t)slot * a.stage_bytes + (size_t)my_r * K * BPE;
            for (int c = c0 + lane; c < c1; c += 32) {
                const float4 wv = *reinterpret_cast<const float4*>(wrow + (size_t)c * 16);
#pragma unroll
                for (int m = 0; m < MB; ++m) {
                    if (m < M) {
                        float t = acc[m];
#pragma unroll
                        for (int q4 = 0; q4 < EPC / 4; ++q4) {
                            const size_t xi = (size_t)m * (a.xs ? K : a.ldx) + (size_t)c * EPC + 4 * q4;
                            const float4 xv = a.xs ? *reinterpret_cast<const float4*>(x_s + xi)
                                                   : __ldcg(reinterpret_cast<const float4*>(a.x + xi));
                            t = fmaf(chunk_elem<WT>(wv, 4 * q4 + 0), xv.x, t);
                            t = fmaf(chunk_elem<WT>(wv, 4 * q4 + 1), xv.y, t);
                            t = fmaf(chunk_elem<WT>(wv, 4 * q4 + 2), xv.z, t);
                            t = fmaf(chunk_elem<WT>(wv, 4 * q4 + 3), xv.w, t);
                        }
                        acc[m] = t;
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);   // the ring slot is read
#pragma unroll
        for (int m = 0; m < MB; ++m) {
            float v = acc[m];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            acc[m] = v;
        }
        // lane m's value for activation row m
        float mine = acc[0];
#pragma unroll
        for (int m = 1; m < MB; ++m)
            if (lane == m) mine = acc[m];
        bool fin = my_r < rows && lane < M;   // this lane finishes (row my_r, activation row lane)
        if (a.ws > 1) {
            if (lane < M) s_part[(buf * kSgCompute + warp) * kSgMaxRows + lane] = mine;
            bar_sync(2 + my_r, 32 * a.ws);
            if (my_s != 0) fin = false;
            else if (fin) {
                mine = s_part[(buf * kSgCompute + warp) * kSgMaxRows + lane];
                for (int k = 1; k < a.ws; ++k) mine += s_part[(buf * kSgCompute + warp + k) * kSgMaxRows + lane];
            }
        }
        if (fin && ok) {
            const int m = lane, j = row0 + my_r, lr = i * a.g + my_r;
            float sum = mine;
            if constexpr (WT == 2) sum = sum * s_scale[lr];
            if (EPI == DEC_HEAD) {
                if (a.y) a.y[(size_t)m * a.ldy + j] = sum;
                if (j == 0 && !(sum == sum)) nan0 = true;
                else if (sum == sum && beats(sum, j, bv, bi)) { bv = sum; bi = j; }
            } else {
                float v = __fadd_rn(sum, s_bias[lr]);
                if (EPI == DEC_BIAS_GELU) v = gelu_new_ref(v);
                if (EPI == DEC_BIAS_RESID) v = __fadd_rn(s_res[m * R + lr], v);
                a.y[(size_t)m * a.ldy + j] = v;
                if (EPI == DEC_QKV_KV) {
                    const int E = a.kv.n_embd;
                    if (j >= E) {
                        const size_t row = a.kv.row(m, s_lens[m]);
                        if (j < 2 * E) a.kv.k[row * E + (j - E)] = v;
                        else a.kv.v[row * E + (j - 2 * E)] = v;
                    }
                }
            }
        }
    }
    if (tr && tid == 0) tr[4] = gtime();
    if (EPI == DEC_HEAD) {
        // this CTA's best per activation row over the warps' bests
        if (lane < kSgMaxRows) {
            s_bv[warp * kSgMaxRows + lane] = bv;
            s_bi[warp * kSgMaxRows + lane] = nan0 ? -2 : bi;
        }
        bar_sync(1, kSgCompute * 32);
        if (tid < M) {
            float b2 = 0.f;
            int i2 = -1;
            bool n2 = false;
            for (int w = 0; w < kSgCompute; ++w) {
                const int t = w * kSgMaxRows + tid;
                if (s_bi[t] == -2) n2 = true;
                else if (s_bi[t] >= 0 && beats(s_bv[t], s_bi[t], b2, i2)) { b2 = s_bv[t]; i2 = s_bi[t]; }
            }
            a.part_val[(size_t)blockIdx.x * M + tid] = b2;
            a.part_idx[(size_t)blockIdx.x * M + tid] = n2 ? -2 : i2;
        }
    }
    if (tr && tid == 0) tr[5] = gtime();
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

// ------------------------------------------------------- the stream path --
namespace {

struct SgGeom {
    int g, ws, gpc, grid, stages, xs;
    uint32_t stage_bytes, off_x, off_ring, smem;
};

// The launch geometry of one stream-path matmul, from its shape, weight format
// and kinds only (never from which rows are in the batch beyond their count):
// false when the path cannot run it.
bool sg_geometry(int M, int N, int K, int wt, int pro, int epi, bool head, SgGeom* o) {
    const int bpe = wt == 0 ? 4 : (wt == 1 ? 2 : 1);
    const int epc = 16 / bpe;
    if (M < 1 || M > kSgMaxRows || N < 1 || K < 4 || K % epc || K % 4) return false;
    const int k4c = K / epc;
    if (k4c > (wt == 0 ? 2048 : 1024)) return false;
    if ((pro == STREAM_PRO_LN || pro == STREAM_PRO_EMBED_LN) && K > 8 * 256) return false;
    const int ws = k4c <= 256 ? 1 : 4;      // dec_dispatch's slicing
    const int row_bytes = K * bpe;
    const int g = std::max(1, std::min(kSgStageTarget / row_bytes, kSgCompute / ws));
    const int ng = (N + g - 1) / g;
    const int sms = sm_count();
    const int gpc = (ng + sms - 1) / sms;
    const int R = gpc * g;
    const uint32_t xbytes = (uint32_t)M * K * 4;
    const int xs = xbytes <= (uint32_t)kSgXsMax;
    if (pro != STREAM_PRO_PLAIN && !xs) return false;
    // per-row epilogue operands: R bias slots, R scale slots, then M x R residuals
    const uint32_t epi_span = 4u * (2 * R + (!head && epi == EPI_BIAS_RESID ? M * R : 0));
    o->g = g;
    o->ws = ws;
    o->gpc = gpc;
    o->grid = (ng + gpc - 1) / gpc;
    o->xs = xs;
    o->off_x = sg_align(SgFixed::epi + epi_span, 128);
    o->off_ring = sg_align(o->off_x + (xs ? xbytes : 0), 128);
    o->stage_bytes = sg_align((uint32_t)(g * row_bytes), 128);
    const int budget = (head ? kSgHeadBudget : kSgSmemBudget) - (int)o->off_ring;
    o->stages = std::min({kSgMaxStages, gpc, budget / (int)o->stage_bytes});
    if (o->stages < 1) return false;
    o->smem = o->off_ring + (uint32_t)o->stages * o->stage_bytes;
    return true;
}

template <int WT, int MB>
cudaError_t sg_launch(const SgArgs& a, const SgGeom& g, cudaStream_t st) {
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(stream_gemv_kernel<WT, MB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kSgHeadBudget);
        if (e != cudaSuccess) return e;
        // the whole unified array as shared memory: two CTAs of consecutive kernels fit
        e = cudaFuncSetAttribute(stream_gemv_kernel<WT, MB>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    cudaError_t e = launch_pdl(stream_gemv_kernel<WT, MB>, dim3(g.grid), dim3(kSgThreads), g.smem, st, a);
    return e != cudaSuccess ? e : cudaGetLastError();
}

template <int WT>
cudaError_t sg_launch_m(const SgArgs& a, const SgGeom& g, cudaStream_t st) {
    if (a.M <= 1) return sg_launch<WT, 1>(a, g, st);
    if (a.M <= 2) return sg_launch<WT, 2>(a, g, st);
    if (a.M <= 4) return sg_launch<WT, 4>(a, g, st);
    return sg_launch<WT, 8>(a, g, st);
}

}  // namespace

bool stream_applies(int M, int E, int wt) {
    SgGeom g;
    return sg_geometry(M, 3 * E, E, wt, STREAM_PRO_EMBED_LN, EPI_QKV_KV, false, &g) &&
           sg_geometry(M, E, E, wt, STREAM_PRO_MERGE, EPI_BIAS_RESID, false, &g) &&
           sg_geometry(M, 4 * E, E, wt, STREAM_PRO_LN, EPI_BIAS_GELU, false, &g) &&
           sg_geometry(M, E, 4 * E, wt, STREAM_PRO_PLAIN, EPI_BIAS_RESID, false, &g) &&
           sg_geometry(M, 50257, E, wt, STREAM_PRO_LN, EPI_STORE, true, &g);
}

int stream_head_blocks(int V, int K, int wt, int M) {
    SgGeom g;
    return sg_geometry(M, V, K, wt, STREAM_PRO_LN, EPI_STORE, true, &g) ? g.grid : 0;
}

cudaError_t launch_stream_gemv(const StreamParams& p, cudaStream_t st) {
    if (p.wt < 0 || p.wt > 2 || (p.wt == 0 && !p.W) || (p.wt != 0 && !p.Wq) || (p.wt == 2 && !p.scale) || !p.err)
        return cudaErrorInvalidValue;
    if (!p.head && p.epi != EPI_BIAS && p.epi != EPI_BIAS_GELU && p.epi != EPI_BIAS_RESID && p.epi != EPI_QKV_KV)
        return cudaErrorInvalidValue;
    if (p.head && (!p.part_val || !p.part_idx)) return cudaErrorInvalidValue;
    if (!p.head && (!p.bias || !p.y)) return cudaErrorInvalidValue;
    if ((p.pro == STREAM_PRO_LN || p.pro == STREAM_PRO_EMBED_LN) && (!p.ln_g || !p.ln_b)) return cudaErrorInvalidValue;
    if (p.pro == STREAM_PRO_EMBED_LN && (!p.tokens || !p.wte || !p.wpe || !p.x_out || !p.lens)) return cudaErrorInvalidValue;
    if (p.pro == STREAM_PRO_MERGE && (!p.apart || !p.lens || p.H * kAttnD != p.K)) return cudaErrorInvalidValue;
    if ((p.pro == STREAM_PRO_PLAIN || p.pro == STREAM_PRO_LN) && (!p.x || (p.ldx & 3))) return cudaErrorInvalidValue;
    if (p.epi == EPI_QKV_KV && !p.head && !p.lens) return cudaErrorInvalidValue;
    SgGeom g;
    if (!sg_geometry(p.M, p.N, p.K, p.wt, p.pro, p.epi, p.head != 0, &g)) return cudaErrorInvalidValue;
    SgArgs a{};
    a.epi = p.epi == EPI_BIAS ? DEC_BIAS : p.epi == EPI_BIAS_GELU ? DEC_BIAS_GELU
          : p.epi == EPI_BIAS_RESID ? DEC_BIAS_RESID : DEC_QKV_KV;
    a.head = p.head;
    a.pro = p.pro;
    a.x = p.x; a.ldx = p.ldx; a.ln_g = p.ln_g; a.ln_b = p.ln_b; a.eps = p.eps;
    a.tokens = p.tokens; a.wte = p.wte; a.wpe = p.wpe; a.x_out = p.x_out; a.V = p.V;
    a.apart = p.apart; a.H = p.H; a.max_chunks = p.max_chunks; a.lens = p.lens;
    a.W = p.wt == 0 ? reinterpret_cast<const char*>(p.W) : reinterpret_cast<const char*>(p.Wq);
    a.scale = p.scale; a.bias = p.bias; a.y = p.y; a.ldy = p.ldy;
    a.M = p.M; a.N = p.N; a.K = p.K; a.kv = p.kv;
    a.part_val = p.part_val; a.part_idx = p.part_idx;
    a.g = g.g; a.ws = g.ws; a.stages = g.stages; a.gpc = g.gpc; a.xs = g.xs;
    a.stage_bytes = g.stage_bytes; a.off_x = g.off_x; a.off_ring = g.off_ring;
    a.err = p.err; a.stall = p.stall; a.wait_ns = p.wait_ns; a.trace = p.trace;
    if (p.wt == 1) return sg_launch_m<1>(a, g, st);
    if (p.wt == 2) return sg_launch_m<2>(a, g, st);
    return sg_launch_m<0>(a, g, st);
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
