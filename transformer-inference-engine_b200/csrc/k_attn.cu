// k_attn.cu -- causal attention for GPT-2 (head_dim 64), fp32.
//
// Prefill (reference model.c:705-732) runs on the tensor cores (k_tc_attn.cu).
// The FFMA kernel here is the statistics pass of model_collect_attn_stats: per
// (sequence, head, 64-query tile) one block streams 64-key tiles up to the
// diagonal through shared memory with an online softmax (running max and sum);
// the T x T score square is never materialised. Scores are q.k scaled by
// 1/sqrt(64), the reference's order (dot product, then scale).
//
// Decode (reference model.c:826-850): one query per sequence against its cached
// positions, read through the page table. Positions are split into 64-position
// chunks, one block each (flash-decoding), and the chunk partials (max, sum,
// unnormalised output) are merged in chunk order -- by the last block of each
// (sequence, head) in the fused kernel, or by a second kernel.
//
// With statistics enabled (reference model_collect_attn_stats) a second pass
// recomputes each row's normalised probabilities from the same scores and
// records the min and max of their double-precision sums.
#include <algorithm>

#include "common.cuh"
#include "tc_gemm.h"

#include <cfloat>

namespace tie {
namespace {

constexpr int D = 64;
constexpr int BQ = 64, BKEY = 64, LDS = D + 4;
constexpr int CH = 64;  // decode positions per split

__device__ __forceinline__ void stats_update(AttnStats* st, double rowsum) {
    const unsigned long long bits = (unsigned long long)__double_as_longlong(rowsum);
    atomicMin(&st->min_bits, bits);
    atomicMax(&st->max_bits, bits);
    atomicAdd(&st->rows, 1ull);
}

// ------------------------------------------------------------------ prefill --
template <bool STATS>
__global__ void __launch_bounds__(128)
attn_prefill_kernel(const float* __restrict__ qkv, int T, int H, float scale,
                    float* __restrict__ out, float* __restrict__ out_hi, float* __restrict__ out_lo,
                    AttnStats* stats) {
    extern __shared__ __align__(16) float smem[];
    float* Qs = smem;                  // [BQ][LDS]
    float* Ks = Qs + BQ * LDS;         // [BKEY][LDS]
    float* Vs = Ks + BKEY * LDS;       // [BKEY][LDS]
    float* Pt = Vs + BKEY * LDS;       // [BKEY][BQ + 4], probabilities transposed

    const int E = H * D, E3 = 3 * E;
    // heavy (late) query tiles first
    const int qt = gridDim.x - 1 - blockIdx.x;
    const int h = blockIdx.y, seq = blockIdx.z;
    const int q0 = qt * BQ;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ty = lane >> 3, tx = lane & 7;
    const float* base = qkv + (size_t)seq * T * E3;

    for (int i = tid; i < BQ * (D / 4); i += blockDim.x) {
        const int r = i / (D / 4), c = (i % (D / 4)) * 4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (q0 + r < T) v = *reinterpret_cast<const float4*>(base + (size_t)(q0 + r) * E3 + h * D + c);
        *reinterpret_cast<float4*>(Qs + r * LDS + c) = v;
    }

    int rows[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) rows[i] = warp * 16 + ty * 4 + i;
    float m_i[4], l_i[4], o[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m_i[i] = -INFINITY;
        l_i[i] = 0.f;
#pragma unroll
        for (int d = 0; d < 8; ++d) o[i][d] = 0.f;
    }

    const int last_row = min(q0 + BQ, T) - 1;
    const int n_kt = last_row / BKEY + 1;

    auto load_kv = [&](int kt) {
        for (int i = tid; i < BKEY * (D / 4); i += blockDim.x) {
            const int r = i / (D / 4), c = (i % (D / 4)) * 4;
            const int key = kt * BKEY + r;
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (key < T) {
                const float* p = base + (size_t)key * E3 + h * D + c;
                kv = *reinterpret_cast<const float4*>(p + E);
                vv = *reinterpret_cast<const float4*>(p + 2 * E);
            }
            *reinterpret_cast<float4*>(Ks + r * LDS + c) = kv;
            *reinterpret_cast<float4*>(Vs + r * LDS + c) = vv;
        }
    };
    // s[i][j]: row rows[i], key kt*BKEY + tx + 8*j
    auto scores = [&](int kt, float (&s)[4][8]) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 8; ++j) s[i][j] = 0.f;
#pragma unroll 4
        for (int d = 0; d < D; d += 4) {
            float4 q[4], k[8];
#pragma unroll
            for (int i = 0; i < 4; ++i) q[i] = *reinterpret_cast<const float4*>(Qs + rows[i] * LDS + d);
#pragma unroll
            for (int j = 0; j < 8; ++j) k[j] = *reinterpret_cast<const float4*>(Ks + (tx + 8 * j) * LDS + d);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    float a = s[i][j];
                    a = fmaf(q[i].x, k[j].x, a);
                    a = fmaf(q[i].y, k[j].y, a);
                    a = fmaf(q[i].z, k[j].z, a);
                    a = fmaf(q[i].w, k[j].w, a);
                    s[i][j] = a;
                }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int t = q0 + rows[i];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int key = kt * BKEY + tx + 8 * j;
                s[i][j] = key <= t ? s[i][j] * scale : -INFINITY;
            }
        }
    };

    for (int kt = 0; kt < n_kt; ++kt) {
        __syncthreads();
        load_kv(kt);
        __syncthreads();
        float s[4][8];
        scores(kt, s);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float mt = s[i][0];
#pragma unroll
            for (int j = 1; j < 8; ++j) mt = fmaxf(mt, s[i][j]);
            mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
            mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
            mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 4));
            const float m_new = fmaxf(m_i[i], mt);
            const float alpha = (m_i[i] == -INFINITY) ? 0.f : expf(m_i[i] - m_new);
            float ps = 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float p = (s[i][j] == -INFINITY) ? 0.f : expf(s[i][j] - m_new);
                Pt[(tx + 8 * j) * (BQ + 4) + rows[i]] = p;
                ps += p;
            }
            ps += __shfl_xor_sync(0xffffffffu, ps, 1);
            ps += __shfl_xor_sync(0xffffffffu, ps, 2);
            ps += __shfl_xor_sync(0xffffffffu, ps, 4);
            l_i[i] = l_i[i] * alpha + ps;
            m_i[i] = m_new;
#pragma unroll
            for (int d = 0; d < 8; ++d) o[i][d] *= alpha;
        }
        __syncwarp();
        const int kmax = min(BKEY, T - kt * BKEY);
        for (int j = 0; j < kmax; ++j) {
            const float4 p4 = *reinterpret_cast<const float4*>(Pt + j * (BQ + 4) + warp * 16 + ty * 4);
            const float4 v0 = *reinterpret_cast<const float4*>(Vs + j * LDS + tx * 4);
            const float4 v1 = *reinterpret_cast<const float4*>(Vs + j * LDS + 32 + tx * 4);
            const float p[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                o[i][0] = fmaf(p[i], v0.x, o[i][0]);
                o[i][1] = fmaf(p[i], v0.y, o[i][1]);
                o[i][2] = fmaf(p[i], v0.z, o[i][2]);
                o[i][3] = fmaf(p[i], v0.w, o[i][3]);
                o[i][4] = fmaf(p[i], v1.x, o[i][4]);
                o[i][5] = fmaf(p[i], v1.y, o[i][5]);
                o[i][6] = fmaf(p[i], v1.z, o[i][6]);
                o[i][7] = fmaf(p[i], v1.w, o[i][7]);
            }
        }
        __syncwarp();
    }

#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int t = q0 + rows[i];
        if (t < T) {
            const float inv = 1.0f / l_i[i];
            const size_t ob = ((size_t)seq * T + t) * E + h * D;
            float v[8];
#pragma unroll
            for (int d = 0; d < 8; ++d) v[d] = o[i][d] * inv;
            if (out) {
                *reinterpret_cast<float4*>(out + ob + tx * 4) = make_float4(v[0], v[1], v[2], v[3]);
                *reinterpret_cast<float4*>(out + ob + 32 + tx * 4) = make_float4(v[4], v[5], v[6], v[7]);
            }
            if (out_hi) {
                float hv[8], lv[8];
#pragma unroll
                for (int d = 0; d < 8; ++d) {
                    hv[d] = tf32_hi(v[d]);
                    lv[d] = __fsub_rn(v[d], hv[d]);
                }
                *reinterpret_cast<float4*>(out_hi + ob + tx * 4) = make_float4(hv[0], hv[1], hv[2], hv[3]);
                *reinterpret_cast<float4*>(out_hi + ob + 32 + tx * 4) = make_float4(hv[4], hv[5], hv[6], hv[7]);
                *reinterpret_cast<float4*>(out_lo + ob + tx * 4) = make_float4(lv[0], lv[1], lv[2], lv[3]);
                *reinterpret_cast<float4*>(out_lo + ob + 32 + tx * 4) = make_float4(lv[4], lv[5], lv[6], lv[7]);
            }
        }
    }

    if constexpr (STATS) {
        // second pass: the normalised probabilities of each row, summed in double
        // (reference softmax check, model.c:635-638)
        double rs[4] = {0.0, 0.0, 0.0, 0.0};
        float inv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) inv[i] = (float)(1.0 / (double)l_i[i]);
        for (int kt = 0; kt < n_kt; ++kt) {
            __syncthreads();
            load_kv(kt);
            __syncthreads();
            float s[4][8];
            scores(kt, s);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    if (s[i][j] != -INFINITY) rs[i] += (double)__fmul_rn(expf(s[i][j] - m_i[i]), inv[i]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            rs[i] += __shfl_xor_sync(0xffffffffu, rs[i], 1);
            rs[i] += __shfl_xor_sync(0xffffffffu, rs[i], 2);
            rs[i] += __shfl_xor_sync(0xffffffffu, rs[i], 4);
            if (tx == 0 && q0 + rows[i] < T) stats_update(stats, rs[i]);
        }
    }
}

// ------------------------------------------------------------------- decode --
// part layout per (b, h, split): [0] max, [1] sum, [2..2+D) unnormalised output
constexpr int PART = D + 2;

template <bool STATS>
__global__ void __launch_bounds__(128)
attn_decode_split_kernel(const float* __restrict__ qkv, const int32_t* __restrict__ lens, int H,
                         PagedKV kv, int max_splits, float scale, float* __restrict__ part,
                         float* __restrict__ e_out, int e_ld) {
    const int s = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int ctx = lens[b] + 1;
    const int p0 = s * CH;
    if (p0 >= ctx) return;
    const int n = min(CH, ctx - p0);
    const int E = kv.n_embd;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    __shared__ float s_e[CH];
    __shared__ float s_o[2][D];

    const float2 q = *reinterpret_cast<const float2*>(qkv + (size_t)b * 3 * E + h * D + 2 * lane);
    for (int i = warp; i < n; i += 4) {
        const size_t row = kv.row(b, p0 + i);
        const float2 k = *reinterpret_cast<const float2*>(kv.k + row * E + h * D + 2 * lane);
        float a = fmaf(q.x, k.x, q.y * k.y);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        if (lane == 0) s_e[i] = a * scale;
    }
    __syncthreads();
    float mx = s_e[0];
    for (int i = 1; i < n; ++i) mx = fmaxf(mx, s_e[i]);
    __syncthreads();
    if (tid < n) s_e[tid] = expf(s_e[tid] - mx);
    __syncthreads();
    float l = 0.f;
    for (int i = 0; i < n; ++i) l += s_e[i];

    const int d = tid & (D - 1), half = tid >> 6;
    float acc = 0.f;
    for (int i = half; i < n; i += 2) {
        const size_t row = kv.row(b, p0 + i);
        acc = fmaf(s_e[i], kv.v[row * E + h * D + d], acc);
    }
    s_o[half][d] = acc;
    __syncthreads();
    float* pp = part + ((size_t)(b * H + h) * max_splits + s) * PART;
    if (tid < D) pp[2 + tid] = s_o[0][tid] + s_o[1][tid];
    if (tid == 0) { pp[0] = mx; pp[1] = l; }
    if constexpr (STATS) {
        if (tid < n) e_out[(size_t)(b * H + h) * e_ld + p0 + tid] = s_e[tid];
    }
}

template <bool STATS>
__global__ void __launch_bounds__(D)
attn_decode_combine_kernel(const int32_t* __restrict__ lens, int H, int max_splits,
                           const float* __restrict__ part, float* __restrict__ out,
                           float* __restrict__ out_hi, float* __restrict__ out_lo,
                           const float* __restrict__ e_in, int e_ld, AttnStats* stats) {
    const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
    const int ctx = lens[b] + 1;
    const int ns = (ctx + CH - 1) / CH;
    const float* pp = part + (size_t)(b * H + h) * max_splits * PART;
    float m = pp[0];
    for (int s = 1; s < ns; ++s) m = fmaxf(m, pp[s * PART]);
    float l = 0.f, o = 0.f;
    for (int s = 0; s < ns; ++s) {
        const float c = expf(pp[s * PART] - m);
        l = fmaf(pp[s * PART + 1], c, l);
        o = fmaf(pp[s * PART + 2 + d], c, o);
    }
    const float y = o / l;
    const size_t oi = (size_t)b * H * D + h * D + d;
    if (out) out[oi] = y;
    if (out_hi) {
        const float hv = tf32_hi(y);
        out_hi[oi] = hv;
        out_lo[oi] = __fsub_rn(y, hv);
    }
    if constexpr (STATS) {
        if (d == 0) {
            const float inv = (float)(1.0 / (double)l);
            double rs = 0.0;
            for (int s = 0; s < ns; ++s) {
                const float c = expf(pp[s * PART] - m);
                const int n = min(CH, ctx - s * CH);
                for (int i = 0; i < n; ++i)
                    rs += (double)__fmul_rn(__fmul_rn(e_in[(size_t)(b * H + h) * e_ld + s * CH + i], c), inv);
            }
            stats_update(stats, rs);
        }
    }
}


// Decode attention, one kernel: each block stages its 64-position chunk of K
// and V with cp.async (all 16-byte copies in flight at once), computes the
// chunk's scores, max, exponentials, sum and unnormalised output, and writes
// them as a partial. The last block of a (sequence, head) to finish -- counted
// with an atomic -- merges all partials in chunk order (so the result does not
// depend on which block was last) and resets the counter for the next launch.
constexpr int KLD = D + 8;  // padded row: conflict-free 16-byte reads
// chunk partials the merging block stages in shared memory: a 1024-position
// context at chunk size CHT (longer contexts read the rest from global)
template <int CHT>
constexpr int merge_splits() { return 1024 / CHT; }

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
                 "l"(gmem)
                 : "memory");
}

template <int CHT>
__global__ void __launch_bounds__(128)
attn_decode_fused_kernel(const float* __restrict__ qkv, const int32_t* __restrict__ lens, int H, PagedKV kv,
                         int max_splits, float scale, float* __restrict__ part, int* __restrict__ counters,
                         float* __restrict__ out, float* __restrict__ out_hi, float* __restrict__ out_lo) {
    const int s = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    pdl_trigger();
    pdl_wait();
    const int ctx = lens[b] + 1;
    const int ns = (ctx + CHT - 1) / CHT;
    if (s >= ns) return;
    const int p0 = s * CHT, n = min(CHT, ctx - p0);
    const int E = kv.n_embd;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    __shared__ __align__(16) float Ks[CHT * KLD];
    __shared__ __align__(16) float Vs[CHT * KLD];
    constexpr int kMergeSplits = merge_splits<CHT>();
    __shared__ float s_merge[kMergeSplits * PART];
    __shared__ float s_e[CHT];
    __shared__ float s_red[8][D];
    __shared__ float s_w[4];
    __shared__ int s_last;

    // stage K and V: n rows x 16 chunks of 16 bytes each
    for (int i = tid; i < n * 16; i += 128) {
        const int r = i >> 4, c = (i & 15) * 4;
        const size_t row = kv.row(b, p0 + r);
        cp_async16(&Ks[r * KLD + c], kv.k + row * E + h * D + c);
        cp_async16(&Vs[r * KLD + c], kv.v + row * E + h * D + c);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    // this thread's half of the query: dims 4*(2j + half) .. +3, j = 0..7
    const int pi = tid >> 1, half = tid & 1;
    const float* q = qkv + (size_t)b * 3 * E + h * D;
    float4 qv[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) qv[j] = *reinterpret_cast<const float4*>(q + 4 * (2 * j + half));
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();

    // scores: two threads per position
    float a = 0.f;
    if (pi < n) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float4 k4 = *reinterpret_cast<const float4*>(&Ks[pi * KLD + 4 * (2 * j + half)]);
            a = fmaf(qv[j].x, k4.x, a);
            a = fmaf(qv[j].y, k4.y, a);
            a = fmaf(qv[j].z, k4.z, a);
            a = fmaf(qv[j].w, k4.w, a);
        }
    }
    a += __shfl_xor_sync(0xffffffffu, a, 1);
    const float sc = pi < n ? a * scale : -INFINITY;
    // chunk max
    float mx = sc;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) s_w[warp] = mx;
    __syncthreads();
    mx = fmaxf(fmaxf(s_w[0], s_w[1]), fmaxf(s_w[2], s_w[3]));
    if (pi < n && half == 0) s_e[pi] = expf(sc - mx);
    __syncthreads();
    // chunk sum, in position order (every thread the same value)
    float l = 0.f;
    for (int i = 0; i < n; ++i) l += s_e[i];
    // unnormalised output: 16 threads per position group, 8 groups
    const int d4 = tid & 15, g = tid >> 4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i = g; i < n; i += 8) {
        const float e = s_e[i];
        const float4 v = *reinterpret_cast<const float4*>(&Vs[i * KLD + 4 * d4]);
        acc.x = fmaf(e, v.x, acc.x);
        acc.y = fmaf(e, v.y, acc.y);
        acc.z = fmaf(e, v.z, acc.z);
        acc.w = fmaf(e, v.w, acc.w);
    }
    *reinterpret_cast<float4*>(&s_red[g][4 * d4]) = acc;
    __syncthreads();
    float* pp = part + ((size_t)(b * H + h) * max_splits + s) * PART;
    if (tid < D) {
        float o = s_red[0][tid];
#pragma unroll
        for (int k = 1; k < 8; ++k) o += s_red[k][tid];
        pp[2 + tid] = o;
    }
    if (tid == 0) { pp[0] = mx; pp[1] = l; }

    // the last block of this (sequence, head) merges the partials
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(&counters[b * H + h], 1) == ns - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // the partials of this (sequence, head) into shared memory, all loads in
    // flight together (beyond kMergeSplits of them, read from global)
    const float* base = part + (size_t)(b * H + h) * max_splits * PART;
    const int staged = min(ns, kMergeSplits);
    for (int i = tid; i < staged * PART; i += 128) s_merge[i] = __ldcg(base + i);
    __syncthreads();
    auto P = [&](int i) { return i < staged * PART ? s_merge[i] : __ldcg(base + i); };
    if (tid < D) {
        float m = P(0);
        for (int k = 1; k < ns; ++k) m = fmaxf(m, P(k * PART));
        float lt = 0.f, o = 0.f;
        for (int k = 0; k < ns; ++k) {
            const float c = expf(P(k * PART) - m);
            lt = fmaf(P(k * PART + 1), c, lt);
            o = fmaf(P(k * PART + 2 + tid), c, o);
        }
        const float y = o / lt;
        const size_t oi = (size_t)b * H * D + h * D + tid;
        if (out) out[oi] = y;
        if (out_hi) {
            const float hv = tf32_hi(y);
            out_hi[oi] = hv;
            out_lo[oi] = __fsub_rn(y, hv);
        }
    }
    if (tid == 0) counters[b * H + h] = 0;
}

constexpr int PG = 16;   // positions per page and per chunk
static_assert(PG == kPageRows, "a chunk is one page");

// Small batches: a block of 8 warps per (sequence, head, 256 positions). Warp
// w reduces chunks c0 + w and c0 + w + 8 of its range, both chunks' keys and
// values loaded into registers before either is reduced, with the arithmetic
// of attn_decode_fused_kernel<16>; the chunk partials go to shared memory.
// When one block covers the whole context (<= 256 positions) it merges them
// in chunk order itself (no global partials, no counters); otherwise the
// partials go to global memory and the block completing a (sequence, head)'s
// count merges all of them. Results are bit-identical to the fused kernel.
constexpr int kSeqWarps = 8;
constexpr int kSeqChunks = 2 * kSeqWarps;   // chunks per block

struct ChunkRegs {
    float4 k[8];
    float2 v[PG];
};

__device__ __forceinline__ void chunk_load(ChunkRegs& r, const PagedKV& kv, int b, int h, int c, int n, int lane) {
    const int pi = lane >> 1, half = lane & 1, E = kv.n_embd;
    const size_t row0 = kv.row(b, c * PG);
    if (pi < n) {
        const float* kp = kv.k + (row0 + pi) * E + h * D;
#pragma unroll
        for (int j = 0; j < 8; ++j) r.k[j] = __ldcs(reinterpret_cast<const float4*>(kp + 4 * (2 * j + half)));
    }
    const float* vp = kv.v + row0 * E + h * D + 2 * lane;
#pragma unroll
    for (int i = 0; i < PG; ++i)
        r.v[i] = i < n ? __ldcs(reinterpret_cast<const float2*>(vp + (size_t)i * E)) : make_float2(0.f, 0.f);
}

// chunk partial (max, sum, 64 weighted sums) of registers r into out
__device__ __forceinline__ void chunk_reduce(const ChunkRegs& r, const float4 (&qv)[8], int n, float scale, int lane,
                                             float* out) {
    const int pi = lane >> 1;
    float a = 0.f;
    if (pi < n) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            a = fmaf(qv[j].x, r.k[j].x, a);
            a = fmaf(qv[j].y, r.k[j].y, a);
            a = fmaf(qv[j].z, r.k[j].z, a);
            a = fmaf(qv[j].w, r.k[j].w, a);
        }
    }
    a += __shfl_xor_sync(0xffffffffu, a, 1);
    const float sc = pi < n ? a * scale : -INFINITY;
    float mx = sc;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float e = pi < n ? expf(sc - mx) : 0.f;
    float l = 0.f;
#pragma unroll
    for (int i = 0; i < PG; ++i) {
        const float ei = __shfl_sync(0xffffffffu, e, 2 * i);
        if (i < n) l += ei;
    }
    float ox = 0.f, oy = 0.f;
#pragma unroll
    for (int g = 0; g < 8; ++g) {
        const float e0 = __shfl_sync(0xffffffffu, e, 2 * g);
        const float e1 = __shfl_sync(0xffffffffu, e, 2 * (g + 8));
        float ax = 0.f, ay = 0.f;
        if (g < n) {
            ax = fmaf(e0, r.v[g].x, ax);
            ay = fmaf(e0, r.v[g].y, ay);
        }
        if (g + 8 < n) {
            ax = fmaf(e1, r.v[g + 8].x, ax);
            ay = fmaf(e1, r.v[g + 8].y, ay);
        }
        if (g == 0) { ox = ax; oy = ay; }
        else { ox += ax; oy += ay; }
    }
    *reinterpret_cast<float2*>(out + 2 + 2 * lane) = make_float2(ox, oy);
    if (lane == 0) *reinterpret_cast<float2*>(out) = make_float2(mx, l);
}

// merge of ns chunk partials P(k) (chunk order) by one warp: lane l writes
// dims 2l, 2l + 1 of the head's output
template <typename PF>
__device__ __forceinline__ void merge_warp(const PF& P, int ns, int lane, float* out, float* out_hi, float* out_lo,
                                           size_t oi) {
    float m = -INFINITY;
    for (int k = lane; k < ns; k += 32) m = fmaxf(m, P(k, 0));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float lt = 0.f, o0 = 0.f, o1 = 0.f;
    for (int k = 0; k < ns; ++k) {
        const float cf = expf(P(k, 0) - m);
        lt = fmaf(P(k, 1), cf, lt);
        o0 = fmaf(P(k, 2 + 2 * lane), cf, o0);
        o1 = fmaf(P(k, 3 + 2 * lane), cf, o1);
    }
    const float y0 = o0 / lt, y1 = o1 / lt;
    if (out) *reinterpret_cast<float2*>(out + oi) = make_float2(y0, y1);
    if (out_hi) {
        const float h0 = tf32_hi(y0), h1 = tf32_hi(y1);
        *reinterpret_cast<float2*>(out_hi + oi) = make_float2(h0, h1);
        *reinterpret_cast<float2*>(out_lo + oi) = make_float2(__fsub_rn(y0, h0), __fsub_rn(y1, h1));
    }
}

__global__ void __launch_bounds__(kSeqWarps * 32, 1)
attn_decode_seq_kernel(const float* __restrict__ qkv, const int32_t* __restrict__ lens, int H, PagedKV kv,
                       int max_splits, float scale, float* __restrict__ part, int* __restrict__ counters,
                       float* __restrict__ out, float* __restrict__ out_hi, float* __restrict__ out_lo) {
    const int h = blockIdx.x, b = blockIdx.y, sp = blockIdx.z;
    __shared__ __align__(16) float s_part[kSeqChunks][PART + 2];
    __shared__ int s_last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_trigger();
    pdl_wait();
    const int ctx = lens[b] + 1, ns = (ctx + PG - 1) / PG;
    const int nsp = (ns + kSeqChunks - 1) / kSeqChunks;
    if (sp >= nsp) return;
    const int c0 = sp * kSeqChunks, c1 = min(ns, c0 + kSeqChunks);
    const int E = kv.n_embd;
    float4 qv[8];
    {
        const float* q = qkv + (size_t)b * 3 * E + h * D;
#pragma unroll
        for (int j = 0; j < 8; ++j) qv[j] = *reinterpret_cast<const float4*>(q + 4 * (2 * j + (lane & 1)));
    }
    const int ca = c0 + warp, cb = c0 + warp + kSeqWarps;
    ChunkRegs ra, rb;
    if (ca < c1) chunk_load(ra, kv, b, h, ca, min(PG, ctx - ca * PG), lane);
    if (cb < c1) chunk_load(rb, kv, b, h, cb, min(PG, ctx - cb * PG), lane);
    if (ca < c1) chunk_reduce(ra, qv, min(PG, ctx - ca * PG), scale, lane, s_part[warp]);
    if (cb < c1) chunk_reduce(rb, qv, min(PG, ctx - cb * PG), scale, lane, s_part[warp + kSeqWarps]);
    __syncthreads();
    const size_t oi = (size_t)b * H * D + h * D + 2 * lane;
    if (nsp == 1) {
        if (warp == 0)
            merge_warp([&](int k, int f) { return s_part[k][f]; }, ns, lane, out, out_hi, out_lo, oi);
        return;
    }
    // several blocks per (sequence, head): partials to global, the last merges
    float* pbase = part + (size_t)(b * H + h) * max_splits * PART;
    for (int i = threadIdx.x; i < (c1 - c0) * PART; i += kSeqWarps * 32)
        pbase[(size_t)c0 * PART + i] = s_part[i / PART][i % PART];
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(&counters[b * H + h], 1) == nsp - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (warp == 0) {
        merge_warp([&](int k, int f) { return __ldcg(pbase + (size_t)k * PART + f); }, ns, lane, out, out_hi, out_lo,
                   oi);
        if (lane == 0) counters[b * H + h] = 0;
    }
}

// Large batches, persistent, one warp per unit: a unit is up to kUnitChunks
// consecutive 16-position chunks of one (sequence, head). Units are numbered
// (sequence, split, head), head fastest; each CTA takes a contiguous range of
// them and its warps take the range's units in turn, so a CTA reads a few
// neighbouring pages at a time.
//
// A warp keeps its chunk's keys and values in registers -- lane 2 pi + half
// the half of key pi it scores (8 x 16 bytes), lane l value dims 2l, 2l + 1
// of all 16 positions -- and software-pipelines across chunks in those same
// registers: as soon as a chunk's scores are formed its key registers receive
// the next chunk's keys, and once its weighted values are summed the value
// registers receive the next chunk's values. Page-table entries are looked up
// one chunk ahead and the next unit's query is fetched while the current unit
// runs, so loads stay in flight through the whole loop. Decode attention reads
// every K and V element exactly once; nothing is staged in shared memory.
//
// Each chunk is reduced with the arithmetic of attn_decode_fused_kernel<16>
// -- lane 2 pi + half scores position pi over its half of the dims, then the
// chunk max, the probabilities summed in position order, and the weighted
// values as eight position groups added in group order -- and its partial
// (max, sum, 64 weighted sums) is written to `part`. The loop carries no
// counters or merges: attn_decode_merge_kernel, chained after it with
// programmatic dependent launch, merges every (sequence, head) with the fused
// kernel's formula, so results are bit-identical to the small-batch path.
// Units of two chunks balance the warps best (measured on B200, 256
// sequences at context 64-512: 83 us per launch against 86 us with four and
// 87 us with eight); the unit only changes which warp reduces which chunks.
constexpr int kUnitChunks = 2;
constexpr int kWarpThreads = 256;
constexpr int kWarpsPerCta = kWarpThreads / 32;
constexpr int kWarpMaxSeqs = 8192;

__device__ __forceinline__ float4 ld_stream4(const float* p) { return __ldcs(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ float2 ld_stream2(const float* p) { return __ldcs(reinterpret_cast<const float2*>(p)); }

// the sequence holding unit u, searching s_start[0..B] (s_start[B] = total)
__device__ __forceinline__ int unit_seq(const int* s_start, int B, int u) {
    int lo = 0, hi = B;   // s_start[lo] <= u < s_start[hi]
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (s_start[mid] <= u) lo = mid;
        else hi = mid;
    }
    return lo;
}

__device__ __forceinline__ int units_of(int ctx, int H) {
    return H * ((ctx + PG * kUnitChunks - 1) / (PG * kUnitChunks));
}

// a warp's position in its chunk sequence: unit u (valid while u < end),
// sequence b, head h, chunk c of the unit's chunks [.., c1), context ctx
struct ChunkCursor {
    int u, b, h, c, c1, ctx;
    __device__ __forceinline__ void unit(int uu, const int* s_start, const int* s_ctx, int B, int H, int end) {
        u = uu;
        if (u >= end) return;
        b = unit_seq(s_start, B, u);
        const int r = u - s_start[b], split = r / H;
        h = r - split * H;
        ctx = s_ctx[b];
        c = split * kUnitChunks;
        c1 = min((ctx + PG - 1) / PG, c + kUnitChunks);
    }
    // the next chunk; returns true when it starts a new unit
    __device__ __forceinline__ bool next(const int* s_start, const int* s_ctx, int B, int H, int end) {
        if (++c < c1) return false;
        unit(u + kWarpsPerCta, s_start, s_ctx, B, H, end);
        return true;
    }
    __device__ __forceinline__ int rows() const { return min(PG, ctx - c * PG); }
};

__global__ void __launch_bounds__(kWarpThreads, 2)
attn_decode_warp_kernel(const float* __restrict__ qkv, const int32_t* __restrict__ lens, int B, int H, PagedKV kv,
                        int max_splits, float scale, float* __restrict__ part) {
    extern __shared__ int s_seq[];
    int* s_start = s_seq;           // [B + 1] unit offsets
    int* s_ctx = s_seq + B + 1;     // [B] contexts
    __shared__ float4 s_q[kWarpsPerCta][D / 4];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    pdl_trigger();
    pdl_wait();
    {
        // contexts and unit offsets of every sequence: a block-wide exclusive scan
        const int seg = (B + kWarpThreads - 1) / kWarpThreads, j0 = min(B, tid * seg), j1 = min(B, j0 + seg);
        int local = 0;
        for (int j = j0; j < j1; ++j) {
            s_ctx[j] = lens[j] + 1;
            local += units_of(s_ctx[j], H);
        }
        int v = local;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) v += y;
        }
        __shared__ int s_wsum[kWarpsPerCta];
        if (lane == 31) s_wsum[warp] = v;
        __syncthreads();
        int run = v - local;
        for (int w = 0; w < warp; ++w) run += s_wsum[w];
        for (int j = j0; j < j1; ++j) {
            s_start[j] = run;
            run += units_of(s_ctx[j], H);
        }
        if (j0 < j1 && j1 == B) s_start[B] = run;
        __syncthreads();
    }
    const int total = s_start[B];
    const int u_lo = (int)((long long)blockIdx.x * total / gridDim.x);
    const int end = (int)((long long)(blockIdx.x + 1) * total / gridDim.x);
    if (u_lo + warp >= end) return;
    const int E = kv.n_embd;
    const int pi = lane >> 1, half = lane & 1;
    const float4* qs = s_q[warp];
    auto q_ptr = [&](const ChunkCursor& q) { return qkv + (size_t)q.b * 3 * E + q.h * D; };

    ChunkCursor cc, nx;
    cc.unit(u_lo + warp, s_start, s_ctx, B, H, end);
    if (lane < D / 4) s_q[warp][lane] = *reinterpret_cast<const float4*>(q_ptr(cc) + 4 * lane);
    float4 k4[8];
    float2 v2[PG];
    {
        const size_t row0 = kv.row(cc.b, cc.c * PG);
        const int n = cc.rows();
        const float* kp = kv.k + (row0 + pi) * E + cc.h * D;
        if (pi < n) {
#pragma unroll
            for (int j = 0; j < 8; ++j) k4[j] = ld_stream4(kp + 4 * (2 * j + half));
        }
#pragma unroll
        for (int i = 0; i < PG; ++i)
            if (i < n) v2[i] = ld_stream2(kv.v + (row0 + i) * E + cc.h * D + 2 * lane);
    }
    nx = cc;
    bool nx_new = nx.next(s_start, s_ctx, B, H, end);
    float4 qn = make_float4(0.f, 0.f, 0.f, 0.f);   // lanes < 16: the next unit's query
    size_t nx_row = 0;
    if (nx.u < end) {
        nx_row = kv.row(nx.b, nx.c * PG);
        if (nx_new && lane < D / 4) qn = *reinterpret_cast<const float4*>(q_ptr(nx) + 4 * lane);
    }
    __syncwarp();
    while (true) {
        const int n = cc.rows();
        const bool more = nx.u < end;
        const int nn = more ? nx.rows() : 0;
        // scores of this chunk; then the key registers take the next chunk's keys
        float a = 0.f;
        if (pi < n) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float4 q4 = qs[2 * j + half];
                a = fmaf(q4.x, k4[j].x, a);
                a = fmaf(q4.y, k4[j].y, a);
                a = fmaf(q4.z, k4[j].z, a);
                a = fmaf(q4.w, k4[j].w, a);
            }
        }
        if (pi < nn) {
            const float* kp = kv.k + (nx_row + pi) * E + nx.h * D;
#pragma unroll
            for (int j = 0; j < 8; ++j) k4[j] = ld_stream4(kp + 4 * (2 * j + half));
        }
        a += __shfl_xor_sync(0xffffffffu, a, 1);
        const float sc = pi < n ? a * scale : -INFINITY;
        float mx = sc;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const float e = pi < n ? expf(sc - mx) : 0.f;
        float l = 0.f;
#pragma unroll
        for (int i = 0; i < PG; ++i) {
            const float ei = __shfl_sync(0xffffffffu, e, 2 * i);
            if (i < n) l += ei;
        }
        // weighted values; then the value registers take the next chunk's values
        float ox = 0.f, oy = 0.f;
#pragma unroll
        for (int g = 0; g < 8; ++g) {
            const float e0 = __shfl_sync(0xffffffffu, e, 2 * g);
            const float e1 = __shfl_sync(0xffffffffu, e, 2 * (g + 8));
            float ax = 0.f, ay = 0.f;
            if (g < n) {
                ax = fmaf(e0, v2[g].x, ax);
                ay = fmaf(e0, v2[g].y, ay);
            }
            if (g + 8 < n) {
                ax = fmaf(e1, v2[g + 8].x, ax);
                ay = fmaf(e1, v2[g + 8].y, ay);
            }
            if (g == 0) { ox = ax; oy = ay; }
            else { ox += ax; oy += ay; }
        }
#pragma unroll
        for (int i = 0; i < PG; ++i)
            if (i < nn) v2[i] = ld_stream2(kv.v + (nx_row + i) * E + nx.h * D + 2 * lane);
        float* pbase = part + (size_t)(cc.b * H + cc.h) * max_splits * PART;
        float* pp = pbase + (size_t)cc.c * PART;
        *reinterpret_cast<float2*>(pp + 2 + 2 * lane) = make_float2(ox, oy);
        if (lane == 0) *reinterpret_cast<float2*>(pp) = make_float2(mx, l);

        if (!more) break;
        // advance: the next chunk becomes current
        if (nx_new) {
            __syncwarp();
            if (lane < D / 4) s_q[warp][lane] = qn;
            __syncwarp();
        }
        cc = nx;
        nx_new = nx.next(s_start, s_ctx, B, H, end);
        if (nx.u < end) {
            nx_row = kv.row(nx.b, nx.c * PG);
            if (nx_new && lane < D / 4) qn = *reinterpret_cast<const float4*>(q_ptr(nx) + 4 * lane);
        }
    }
}

// One warp per (sequence, head): its chunk partials from `part` merged in
// chunk order with the formula of attn_decode_fused_kernel<16> (lane l: dims
// 2l and 2l + 1); the chunk maxima and sums are read by lane k for chunk k and
// shuffled, each lane's weighted sums eight chunks at a time.
constexpr int kMergeWarps = 8;

__global__ void __launch_bounds__(kMergeWarps * 32)
attn_decode_merge_kernel(const int32_t* __restrict__ lens, int B, int H, int max_splits,
                         const float* __restrict__ part, float* __restrict__ out, float* __restrict__ out_hi,
                         float* __restrict__ out_lo) {
    pdl_trigger();
    pdl_wait();
    const int gw = blockIdx.x * kMergeWarps + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (gw >= B * H) return;
    const int b = gw / H, h = gw - b * H;
    const int ns = (lens[b] + PG) / PG;   // chunks of context lens[b] + 1
    const float* pbase = part + (size_t)gw * max_splits * PART;
    float m = -INFINITY;
    for (int k = lane; k < ns; k += 32) m = fmaxf(m, __ldcg(pbase + (size_t)k * PART));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float lt = 0.f, o0 = 0.f, o1 = 0.f;
    for (int k0 = 0; k0 < ns; k0 += 32) {
        float2 ml = make_float2(0.f, 0.f);
        if (k0 + lane < ns) ml = __ldcg(reinterpret_cast<const float2*>(pbase + (size_t)(k0 + lane) * PART));
        const int kn = min(32, ns - k0);
        for (int k1 = 0; k1 < kn; k1 += 8) {
            float2 ov[8];
#pragma unroll
            for (int k = 0; k < 8; ++k)
                if (k1 + k < kn)
                    ov[k] = __ldcg(reinterpret_cast<const float2*>(pbase + (size_t)(k0 + k1 + k) * PART + 2 + 2 * lane));
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float mk = __shfl_sync(0xffffffffu, ml.x, (k1 + k) & 31);
                const float lk = __shfl_sync(0xffffffffu, ml.y, (k1 + k) & 31);
                if (k1 + k < kn) {
                    const float cf = expf(mk - m);
                    lt = fmaf(lk, cf, lt);
                    o0 = fmaf(ov[k].x, cf, o0);
                    o1 = fmaf(ov[k].y, cf, o1);
                }
            }
        }
    }
    const float y0 = o0 / lt, y1 = o1 / lt;
    const size_t oi = (size_t)b * H * D + h * D + 2 * lane;
    if (out) *reinterpret_cast<float2*>(out + oi) = make_float2(y0, y1);
    if (out_hi) {
        const float h0 = tf32_hi(y0), h1 = tf32_hi(y1);
        *reinterpret_cast<float2*>(out_hi + oi) = make_float2(h0, h1);
        *reinterpret_cast<float2*>(out_lo + oi) = make_float2(__fsub_rn(y0, h0), __fsub_rn(y1, h1));
    }
}

// Small batches ahead of the fused projection (k_decode.cu's stream path): a
// warp per 16-position chunk of one (sequence, head), four chunks per block,
// writing the chunk partial (max, sum, 64 weighted sums) to `part` with the
// arithmetic of chunk_reduce; the projection kernel that follows merges them
// in chunk order with merge_warp's formula, so the step's numbers are the
// small-batch kernel's bit for bit. Sequence lengths are fixed for a step, so
// every cached row (positions below the current one, written by earlier
// steps) is loaded before the dependency wait; only the current position's
// row and the query, which the QKV matmul just wrote, are read after it. All
// loads go through L2 only (another kernel wrote every one of them).
constexpr int kChunkWarps = 4;

__device__ __forceinline__ void chunk_load_rows(ChunkRegs& r, const PagedKV& kv, int b, int h, int c, int lo, int hi,
                                                int lane) {
    const int pi = lane >> 1, half = lane & 1, E = kv.n_embd;
    const size_t row0 = kv.row(b, c * PG);
    if (pi >= lo && pi < hi) {
        const float* kp = kv.k + (row0 + pi) * E + h * D;
#pragma unroll
        for (int j = 0; j < 8; ++j) r.k[j] = __ldcg(reinterpret_cast<const float4*>(kp + 4 * (2 * j + half)));
    }
    const float* vp = kv.v + row0 * E + h * D + 2 * lane;
#pragma unroll
    for (int i = 0; i < PG; ++i)
        if (i >= lo && i < hi) r.v[i] = __ldcg(reinterpret_cast<const float2*>(vp + (size_t)i * E));
}

__global__ void __launch_bounds__(kChunkWarps * 32)
attn_chunk_kernel(const float* __restrict__ qkv, const int32_t* __restrict__ lens, int H, PagedKV kv,
                  int max_chunks, float scale, float* __restrict__ part) {
    const int h = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = blockIdx.x * kChunkWarps + warp;
    pdl_trigger();
    const int ctx = __ldcg(lens + b) + 1, ns = (ctx + PG - 1) / PG;
    const bool act = c < ns && c < max_chunks;
    const int n = act ? min(PG, ctx - c * PG) : 0;
    const bool last = c == ns - 1;   // holds the current position
    ChunkRegs r;
#pragma unroll
    for (int j = 0; j < 8; ++j) r.k[j] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = 0; i < PG; ++i) r.v[i] = make_float2(0.f, 0.f);
    if (act) chunk_load_rows(r, kv, b, h, c, 0, last ? n - 1 : n, lane);
    pdl_wait();
    if (!act) return;
    if (last) chunk_load_rows(r, kv, b, h, c, n - 1, n, lane);
    const int E = kv.n_embd;
    float4 qv[8];
    const float* q = qkv + (size_t)b * 3 * E + h * D;
#pragma unroll
    for (int j = 0; j < 8; ++j) qv[j] = __ldcg(reinterpret_cast<const float4*>(q + 4 * (2 * j + (lane & 1))));
    chunk_reduce(r, qv, n, scale, lane, part + ((size_t)(b * H + h) * max_chunks + c) * PART);
}

}  // namespace

// Kernels one launch_attn_decode issues with counters and without statistics:
// the streaming kernel and its merge for batches above 16 (up to the
// sequences it indexes), else one.
int attn_decode_kernels(int B) { return B > 16 && B <= kWarpMaxSeqs ? 2 : 1; }

// Partial-buffer sizing: the finest chunking any launch uses (16 positions).
int attn_decode_max_splits(int capacity) { return (capacity + 15) / 16; }

cudaError_t launch_attn_prefill(const float* qkv, int n_seq, int T, int H, float* out,
                                AttnStats* stats, cudaStream_t st, float* out_hi, float* out_lo, int* err) {
    if (T <= 0 || n_seq <= 0) return cudaSuccess;
    cudaError_t e = launch_tc_attn_prefill(qkv, n_seq, T, H, out, out_hi, out_lo, err, st);
    if (e != cudaSuccess || !stats) return e;
    // the statistics pass: same scores and softmax, no outputs
    const size_t smem = (size_t)(BQ * LDS * 3 + BKEY * (BQ + 4)) * sizeof(float);
    const float scale = (float)(1.0 / sqrt((double)D));
    dim3 grid((T + BQ - 1) / BQ, H, n_seq);
    cudaFuncSetAttribute(attn_prefill_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attn_prefill_kernel<true><<<grid, 128, smem, st>>>(qkv, T, H, scale, nullptr, nullptr, nullptr, stats);
    return cudaGetLastError();
}

cudaError_t launch_attn_chunks(const float* qkv, const int32_t* lens, int B, int H, PagedKV kv, int max_chunks,
                               float* part, cudaStream_t st) {
    if (B <= 0) return cudaSuccess;
    const float scale = (float)(1.0 / sqrt((double)D));
    cudaError_t e = launch_pdl(attn_chunk_kernel, dim3((max_chunks + kChunkWarps - 1) / kChunkWarps, H, B),
                               dim3(kChunkWarps * 32), 0, st, qkv, lens, H, kv, max_chunks, scale, part);
    return e != cudaSuccess ? e : cudaGetLastError();
}

// part: B * H * max_splits * (D + 2) floats. With stats, `part` must also hold
// B * H * max_splits * CH floats after the partials for the probabilities.
cudaError_t launch_attn_decode(const float* qkv, const int32_t* lens, int B, int H, PagedKV kv,
                               int max_splits, float* part, float* out, AttnStats* stats,
                               cudaStream_t st, float* out_hi, float* out_lo, int* counters, int* err) {
    if (B <= 0) return cudaSuccess;
    const float scale = (float)(1.0 / sqrt((double)D));
    if (stats || !counters) max_splits = (max_splits * 16 + CH - 1) / CH;  // 64-position chunks
    dim3 g1(max_splits, H, B), g2(H, B);
    if (stats) {
        float* e = part + (size_t)B * H * max_splits * PART;
        const int e_ld = max_splits * CH;
        attn_decode_split_kernel<true><<<g1, 128, 0, st>>>(qkv, lens, H, kv, max_splits, scale, part, e, e_ld);
        attn_decode_combine_kernel<true><<<g2, D, 0, st>>>(lens, H, max_splits, part, out, out_hi, out_lo, e, e_ld, stats);
    } else if (counters) {
        // 16-position chunks, a block each, while the batch is small; the
        // persistent warp-per-unit kernel for larger batches; 64-position
        // chunks beyond the sequences it indexes; `max_splits` is the sizing bound
        const int capacity = max_splits * 16;
        const bool fine = B <= 16;
        const int splits = fine ? max_splits : (capacity + CH - 1) / CH;
        if (!fine && B <= kWarpMaxSeqs && kv.n_embd == H * D) {
            // persistent, a warp per unit, loads pipelined in registers
            int dev = 0, sms = 0;
            cudaGetDevice(&dev);
            cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
            if (e != cudaSuccess) return e;
            const size_t smem = (size_t)(2 * B + 1) * sizeof(int);
            if (smem > 48 * 1024) {
                e = cudaFuncSetAttribute(attn_decode_warp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
                if (e != cudaSuccess) return e;
            }
            const long long units = (long long)B * H * ((max_splits + kUnitChunks - 1) / kUnitChunks);
            const int grid = (int)std::min<long long>((units + kWarpsPerCta - 1) / kWarpsPerCta, 2LL * sms);
            e = launch_pdl(attn_decode_warp_kernel, dim3(grid), dim3(kWarpThreads), smem, st, qkv, lens, B, H, kv,
                           max_splits, scale, part);
            if (e != cudaSuccess) return e;
            e = launch_pdl(attn_decode_merge_kernel, dim3((B * H + kMergeWarps - 1) / kMergeWarps),
                           dim3(kMergeWarps * 32), 0, st, lens, B, H, max_splits, part, out, out_hi, out_lo);
            return e != cudaSuccess ? e : cudaGetLastError();
        }
        if (fine) {
            // a block per (sequence, head, 256 positions)
            const int nsp = (max_splits + kSeqChunks - 1) / kSeqChunks;
            cudaError_t e = launch_pdl(attn_decode_seq_kernel, dim3(H, B, nsp), dim3(kSeqWarps * 32), 0, st, qkv,
                                       lens, H, kv, max_splits, scale, part, counters, out, out_hi, out_lo);
            return e != cudaSuccess ? e : cudaGetLastError();
        }
        cudaError_t e = fine ? launch_pdl(attn_decode_fused_kernel<16>, dim3(splits, H, B), dim3(128), 0, st, qkv,
                                          lens, H, kv, splits, scale, part, counters, out, out_hi, out_lo)
                             : launch_pdl(attn_decode_fused_kernel<CH>, dim3(splits, H, B), dim3(128), 0, st, qkv,
                                          lens, H, kv, splits, scale, part, counters, out, out_hi, out_lo);
        if (e != cudaSuccess) return e;
    } else {
        attn_decode_split_kernel<false><<<g1, 128, 0, st>>>(qkv, lens, H, kv, max_splits, scale, part, nullptr, 0);
        attn_decode_combine_kernel<false><<<g2, D, 0, st>>>(lens, H, max_splits, part, out, out_hi, out_lo, nullptr, 0, nullptr);
    }
    return cudaGetLastError();
}

}  // namespace tie
