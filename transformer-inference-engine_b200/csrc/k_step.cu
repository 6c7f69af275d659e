// k_step.cu -- one whole decode step of a small batch (1..4 sequences) as a
// single persistent kernel: embedding, every layer, LN_f, the tied head, the
// greedy argmax and the step bookkeeping.
//
// Why: at batch 1 a step moves ~0.5 GB of fp32 weights (GPT-2 small), 77 us at
// HBM speed, through ~60 dependent matmuls and attentions. As separate kernels
// each costs its launch, its ramp and its drain; here each dependency is one
// release/acquire counter in global memory instead.
//
// Layout of a CTA (one per SM, all co-resident: cooperative launch):
//   warp 0           the producer, two lanes. Lane 0 walks the step's
//                    matrices in order (per layer qkv, proj, fc, mlp; then wte
//                    for the head) and streams this CTA's rows of each into a
//                    ring of 32 KB shared-memory slots; lane 1 copies each
//                    stage's small parameters (LayerNorm gain and shift, this
//                    CTA's slice of the bias) into one of two parameter
//                    buffers. All copies are bulk asynchronous copies
//                    (cp.async.bulk) completing on mbarriers. Nothing they copy
//                    is computed in the step, so the weights run ahead of the
//                    consumers by the whole ring, across stage boundaries.
//   warps 1..7       the consumers. Per stage they wait for the stage's inputs
//                    (a counter reaching its target), stage the activation rows
//                    in shared memory (LayerNorm applied there where the stage
//                    starts with one), and reduce each weight row of the slots
//                    against them.
//
// Stages of layer l and what they wait for:
//   A  LN1 + qkv (+ this step's K/V rows into the cache)    E of layer l-1
//   B  attention: one unit per (sequence, head, 16-position chunk),
//      dealt to every consumer warp of the grid; merged by the
//      warp completing a (sequence, head)                     A
//   C  proj + residual                                       all merges of B
//   D  LN2 + fc + gelu                                       C
//   E  mlp + residual                                        D
// then the head (LN_f + wte rows + per-CTA argmax) and, in the last CTA to
// finish it, the final argmax and the step bookkeeping.
//
// Every sum is formed in the order of the small-batch kernels (k_decode.cu:
// rows of K/4 <= 256 chunks whole, longer rows in four slices whose sums are
// added in slice order; LayerNorm in the canonical order of common.cuh;
// attention as attn_decode_fused_kernel<16>), so the two paths give
// bit-identical results.
//
// Waits are bounded (1 s on the global timer); on expiry the kernel sets *err,
// lets its copies in flight land and returns.
#include "common.cuh"
#include "mbar.cuh"

#include <cstddef>

namespace tie {
namespace {

constexpr int kCons = 7;                        // consumer warps (8 warps in all: 255 registers each)
constexpr int kThreads = (kCons + 1) * 32;      // + the producer warp
constexpr int kSlot = 32 * 1024;                // bytes per ring slot
constexpr int kMaxSlots = 8;
constexpr int kRowsMax = 4;                     // sequences per step
constexpr int D = 64;                           // head dim
constexpr int PART = D + 2;                     // attention partial: max, sum, D sums
constexpr int CHT = 16;                         // positions per attention chunk
constexpr int kMaxPages = 64;
constexpr int kMaxResid = 32;                   // residual columns a CTA keeps
constexpr int kRegChunks = 6;                   // activation chunks per lane kept in registers (batch 1)

__device__ __forceinline__ void cons_sync() { bar_sync(1, kCons * 32); }
// activations written earlier in this kernel by other CTAs: read at L2, never
// from a possibly stale L1 line
__device__ __forceinline__ float4 ld_cg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ float2 ld_cg2(const float* p) { return __ldcg(reinterpret_cast<const float2*>(p)); }

// one stamp of the optional trace (consumer thread 0 / the producer thread)
__device__ __forceinline__ void stamp(const StepParams& p, int ev) {
    if (p.trace) p.trace[(size_t)blockIdx.x * step_trace_events(p.n_layer) + ev] = gtime();
}
__device__ __forceinline__ int ev_stage(int layer, int stage, int k) { return 1 + 3 * (5 * layer + stage) + k; }

__device__ __forceinline__ bool beats(float v, int i, float bv, int bi) {
    return bi < 0 || v > bv || (v == bv && i < bi);
}

// Floats of one parameter buffer: gain and shift (E each) and a bias slice of
// at most ceil(4E / grid) rows widened to 4-row boundaries.
__host__ __device__ __forceinline__ int param_floats(int E, int grid) {
    return 2 * E + (((4 * E + grid - 1) / grid + 8 + 3) & ~3);
}

// The matrices in stream order: 4 per layer, then the head.
struct MatDesc {
    const float* W;
    const float* bias;      // NULL for the head
    const float* ln_g;      // NULL for stages without a LayerNorm
    const float* ln_b;
    int N, K;               // rows, row length
    int lws;                // log2 of the slices per row (0 or 2)
    int sc;                 // chunks (16 bytes) per slice
    int P;                  // segments (row slices) per ring slot, a multiple of the slices per row
    int kind;               // 0..3 per layer (qkv, proj, fc, mlp), 4 the head
};

__device__ __forceinline__ MatDesc mat_desc(const StepParams& p, const StepLayer* tab, int i) {
    MatDesc d;
    const int E = p.E;
    if (i == 4 * p.n_layer) {
        d.W = p.wte; d.bias = nullptr; d.ln_g = p.lnf_g; d.ln_b = p.lnf_b; d.N = p.V; d.K = E; d.kind = 4;
    } else {
        const StepLayer& l = tab[i >> 2];
        d.kind = i & 3;
        switch (i & 3) {
            case 0: d.W = l.qkv_w; d.bias = l.qkv_b; d.ln_g = l.ln1_g; d.ln_b = l.ln1_b; d.N = 3 * E; d.K = E; break;
            case 1: d.W = l.proj_w; d.bias = l.proj_b; d.ln_g = nullptr; d.ln_b = nullptr; d.N = E; d.K = E; break;
            case 2: d.W = l.fc_w; d.bias = l.fc_b; d.ln_g = l.ln2_g; d.ln_b = l.ln2_b; d.N = 4 * E; d.K = E; break;
            default: d.W = l.mlp_w; d.bias = l.mlp_b; d.ln_g = nullptr; d.ln_b = nullptr; d.N = E; d.K = 4 * E; break;
        }
    }
    const int K4 = d.K >> 2;
    d.lws = K4 <= 256 ? 0 : 2;
    const int WS = 1 << d.lws;
    d.sc = (K4 + WS - 1) / WS;
    int P = kSlot / (d.sc * 16);
    if (P > kCons) P = kCons;
    d.P = P - P % WS;
    return d;
}
// float offset of segment g (row g / WS, slice g % WS) from the matrix start
__device__ __forceinline__ size_t seg_off(const MatDesc& d, int g) {
    const int r = g >> d.lws, s = g & ((1 << d.lws) - 1);
    return (size_t)r * d.K + 4 * (size_t)min(d.K >> 2, s * d.sc);
}

struct Smem {
    uint64_t full[kMaxSlots];
    uint64_t empty[kMaxSlots];
    uint64_t pfull[2];
    uint64_t pempty[2];
    double ln_s[kRowsMax][kLnGroups];   // LayerNorm group sums: mean pass
    double ln_v[kRowsMax][kLnGroups];   // variance pass
    double ln_mean[kRowsMax];
    float ln_inv[kRowsMax];
    float pk_sum[kCons][kRowsMax];      // segment sums of one slot (sliced rows)
    float best_v[kCons][kRowsMax];
    int best_i[kCons][kRowsMax];
    long long kvrow[kRowsMax];          // this step's physical K/V row per sequence
    int r0[5], r1[5];                   // this CTA's rows of each matrix kind
    float resid[kRowsMax][kMaxResid];   // this CTA's columns of the residual stream
    int pt[kRowsMax][kMaxPages];        // page tables of the step's sequences
    int nan0[kRowsMax];
    int lens[kRowsMax];
    int abort;
    int last;
};

// ------------------------------------------------------------ the producer --
// Two lanes of warp 0, each its own sequence of bounded waits: lane 0 streams
// the weight rows of every matrix in order through the ring, running ahead of
// the consumers by the ring's whole depth; lane 1 copies each stage's small
// parameters into the two parameter buffers as they free up. Neither waits on
// the other.
__device__ void producer_weights(const StepParams& p, Smem& sm, char* ring, const StepLayer* tab) {
    const uint64_t policy = evict_first_policy(), keep = evict_last_policy();
    const int n_mats = 4 * p.n_layer + 1, E = p.E;
    // this CTA's rows of the tied head go into L2 a layer's share at a time:
    // the layers' stages wait on one another and leave HBM mostly idle
    const char* head0 = reinterpret_cast<const char*>(p.wte + (size_t)sm.r0[4] * E);
    const size_t head_bytes = (size_t)(sm.r1[4] - sm.r0[4]) * E * 4;
    const size_t pf_total = min(head_bytes, (size_t)p.head_prefetch) & ~(size_t)15;
    const size_t pf_step = ((pf_total / p.n_layer) + 15) & ~(size_t)15;
    size_t pf_done = 0;
    uint32_t pk = 0;
    bool ok = true;
    for (int i = 0; i < n_mats && ok; ++i) {
        const MatDesc d = mat_desc(p, tab, i);
        const int r0 = sm.r0[d.kind], r1 = sm.r1[d.kind];
        if ((i & 3) == 0 && d.kind != 4 && pf_done < pf_total) {
            const size_t n = min(pf_step, pf_total - pf_done);
            for (size_t o = 0; o < n; o += 32768)
                bulk_prefetch_l2(head0 + pf_done + o, (uint32_t)min((size_t)32768, n - o), keep);
            pf_done += n;
        }
        const int g1 = r1 << d.lws;
        for (int g = r0 << d.lws; g < g1; g += d.P, ++pk) {
            const int slot = pk % p.slots;
            const uint32_t par = (pk / p.slots) & 1;
            if (sm.abort || !mbar_wait(&sm.empty[slot], par ^ 1)) { ok = false; break; }
            const int ge = min(g + d.P, g1);
            const size_t o0 = seg_off(d, g), o1 = seg_off(d, ge);
            const uint32_t bytes = (uint32_t)((o1 - o0) * sizeof(float));
            mbar_expect_tx(&sm.full[slot], bytes);
            bulk_load(ring + (size_t)slot * kSlot, d.W + o0, bytes, &sm.full[slot], policy);
        }
        stamp(p, step_trace_end(p.n_layer) + 1 + i);
    }
    if (!ok) {
        atomicExch(p.err, 1);
        // let every copy still in flight land before the CTA's shared memory goes
        const uint32_t n = pk < (uint32_t)p.slots ? pk : (uint32_t)p.slots;
        for (uint32_t k = pk - n; k < pk; ++k) mbar_wait(&sm.full[k % p.slots], (k / p.slots) & 1);
    }
}

__device__ void producer_params(const StepParams& p, Smem& sm, float* params, const StepLayer* tab) {
    const int n_mats = 4 * p.n_layer + 1, E = p.E;
    const int pfl = param_floats(E, gridDim.x);
    int np = 0;   // parameter blocks issued
    bool ok = true;
    for (int i = 0; i < n_mats; ++i) {
        const MatDesc d = mat_desc(p, tab, i);
        const int r0 = sm.r0[d.kind], r1 = sm.r1[d.kind];
        const int ps = i & 1;
        if (sm.abort || !mbar_wait(&sm.pempty[ps], ((i >> 1) & 1) ^ 1)) { ok = false; break; }
        float* dst = params + (size_t)ps * pfl;
        const uint32_t ln_bytes = d.ln_g ? 2u * E * 4u : 0u;
        const int r0a = r0 & ~3, r1a = (r1 + 3) & ~3;
        const uint32_t b_bytes = (d.bias && r1 > r0) ? (uint32_t)(r1a - r0a) * 4u : 0u;
        if (ln_bytes + b_bytes == 0) mbar_arrive(&sm.pfull[ps]);
        else {
            mbar_expect_tx(&sm.pfull[ps], ln_bytes + b_bytes);
            if (ln_bytes) {
                bulk_load(dst, d.ln_g, E * 4u, &sm.pfull[ps]);
                bulk_load(dst + E, d.ln_b, E * 4u, &sm.pfull[ps]);
            }
            if (b_bytes) bulk_load(dst + 2 * E, d.bias + r0a, b_bytes, &sm.pfull[ps]);
        }
        ++np;
    }
    if (!ok) {
        atomicExch(p.err, 1);
        for (int j = max(0, np - 2); j < np; ++j) mbar_wait(&sm.pfull[j & 1], (j >> 1) & 1);
    }
}

// ------------------------------------------------------------ consumers --
// Consumer thread 0 waits for *ctr >= target (when ctr is given) and for the
// parameters of matrix `mi` (when mi >= 0); the others learn the outcome at the
// barrier. Returns false (everyone) when the kernel is giving up.
__device__ bool stage_begin(const StepParams& p, Smem& sm, const unsigned* ctr, unsigned target, int mi) {
    const int t = threadIdx.x - 32;
    if (t == 0 && !sm.abort) {
        if (ctr) {
            const unsigned long long t0 = gtime();
            while (ld_acquire(ctr) < target) {
                if (gtime() - t0 > kWaitNs) {
                    atomicExch(p.err, 1);
                    sm.abort = 1;
                    break;
                }
            }
        }
        if (mi >= 0 && !sm.abort && !mbar_wait(&sm.pfull[mi & 1], (mi >> 1) & 1)) {
            atomicExch(p.err, 1);
            sm.abort = 1;
        }
    }
    cons_sync();
    return !sm.abort;
}
// the stage's parameter buffer may be refilled (after a barrier that ends the stage)
__device__ __forceinline__ void stage_params_done(Smem& sm, int mi) {
    if (threadIdx.x == 32) mbar_arrive(&sm.pempty[mi & 1]);
}

// LayerNorm of rows [0, M) of xs (row stride K) in place, all consumer warps:
// the canonical order of common.cuh, each row's 8 groups spread over the
// row's kCons / M warps.
__device__ void ln_rows(Smem& sm, float* xs, int M, int K, const float* g, const float* b, float eps) {
    const int t = threadIdx.x - 32, warp = t >> 5, lane = t & 31;
    const int wpr = kCons / M;                        // warps per row
    const int m = warp / wpr, wr = warp % wpr;
    const float* xr = xs + (size_t)m * K;
    if (m < M)
        for (int w = wr; w < kLnGroups; w += wpr) {
            const double s = ln_group_sum([&](int i) { return (double)xr[i]; }, K, w, lane);
            if (lane == 0) sm.ln_s[m][w] = s;
        }
    cons_sync();
    if (m < M) {
        double S = sm.ln_s[m][0];
        for (int w = 1; w < kLnGroups; ++w) S = __dadd_rn(S, sm.ln_s[m][w]);
        const double mean = S / (double)K;
        for (int w = wr; w < kLnGroups; w += wpr) {
            const double v = ln_group_sum([&](int i) {
                const double d = __dadd_rn((double)xr[i], -mean);
                return __dmul_rn(d, d);
            }, K, w, lane);
            if (lane == 0) sm.ln_v[m][w] = v;
        }
        if (wr == 0 && lane == 0) sm.ln_mean[m] = mean;
    }
    cons_sync();
    if (t < M) {
        double V = sm.ln_v[t][0];
        for (int w = 1; w < kLnGroups; ++w) V = __dadd_rn(V, sm.ln_v[t][w]);
        sm.ln_inv[t] = (float)(1.0 / sqrt(__dadd_rn(V / (double)K, (double)eps)));
    }
    cons_sync();
    for (int i = t; i < M * K; i += kCons * 32) {
        const int r = i / K, k = i - r * K;
        xs[i] = ln_apply(xs[i], sm.ln_mean[r], sm.ln_inv[r], g[k], b[k]);
    }
    cons_sync();
}

// Rows [0, M) of the global activations `src` (row stride lds) into xs (row
// stride K), then LayerNorm in place when g != NULL.
__device__ void stage_rows(Smem& sm, const float* src, int lds, int M, int K, const float* g, const float* b,
                           float eps, float* xs) {
    const int t = threadIdx.x - 32, K4 = K >> 2;
#pragma unroll 4
    for (int i = t; i < M * K4; i += kCons * 32) {
        const int m = i / K4, c = i - m * K4;
        reinterpret_cast<float4*>(xs + (size_t)m * K)[c] = ld_cg4(src + (size_t)m * lds + 4 * c);
    }
    cons_sync();
    if (g) ln_rows(sm, xs, M, K, g, b, eps);
}

// The embedding of this step's tokens (embed_decode_kernel's arithmetic) into
// xs, and this CTA's columns of it into its share of the residual stream.
__device__ void stage_embed(const StepParams& p, Smem& sm, float* xs) {
    const int t = threadIdx.x - 32, E4 = p.E >> 2;
    for (int i = t; i < p.M * E4; i += kCons * 32) {
        const int m = i / E4, c = i % E4;
        const int id = p.tokens[m];
        float4 r;
        if ((unsigned)id >= (unsigned)p.V) r = make_float4(NAN, NAN, NAN, NAN);
        else {
            const float4 a = __ldg(reinterpret_cast<const float4*>(p.wte + (size_t)id * p.E) + c);
            const float4 q = __ldg(reinterpret_cast<const float4*>(p.wpe + (size_t)sm.lens[m] * p.E) + c);
            r = make_float4(__fadd_rn(a.x, q.x), __fadd_rn(a.y, q.y), __fadd_rn(a.z, q.z), __fadd_rn(a.w, q.w));
        }
        reinterpret_cast<float4*>(xs + (size_t)m * p.E)[c] = r;
    }
    cons_sync();
    // this CTA's columns of the residual stream (proj and mlp rows)
    for (int i = t; i < p.M * (sm.r1[1] - sm.r0[1]); i += kCons * 32) {
        const int w = sm.r1[1] - sm.r0[1], m = i / w, j = i % w;
        sm.resid[m][j] = xs[(size_t)m * p.E + sm.r0[1] + j];
    }
}

enum : int { ST_QKV = 0, ST_PROJ = 1, ST_FC = 2, ST_MLP = 3, ST_HEAD = 4 };

// A thread's running best logit of the head for its sequence.
struct Best {
    float v;
    int i;
    int m;   // the sequence this thread's logits belong to (-1: none yet)
};

// The epilogue of output column j of sequence m; `bias` is the stage's bias
// slice, starting at row r0a.
template <int KIND>
__device__ __forceinline__ void epilogue(const StepParams& p, Smem& sm, int layer, float sum, int j, int m,
                                         const float* bias, int r0a, Best& best) {
    const int E = p.E;
    if constexpr (KIND == ST_HEAD) {
        if (p.logits) p.logits[(size_t)m * p.ldl + j] = sum;
        best.m = m;
        if (j == 0 && !(sum == sum)) sm.nan0[m] = 1;
        else if (sum == sum && beats(sum, j, best.v, best.i)) { best.v = sum; best.i = j; }
    } else {
        const float bj = bias[j - r0a];
        if constexpr (KIND == ST_QKV) {
            const float v = __fadd_rn(sum, bj);
            p.qkv[(size_t)m * 3 * E + j] = v;
            if (j >= E) {
                float* base = (j < 2 * E ? p.k : p.v) + (size_t)layer * p.layer_stride;
                base[(size_t)sm.kvrow[m] * E + (j < 2 * E ? j - E : j - 2 * E)] = v;
            }
        } else if constexpr (KIND == ST_FC) {
            p.ff[(size_t)m * 4 * E + j] = gelu_new_ref(__fadd_rn(sum, bj));
        } else {
            // proj or mlp: the residual stream, x = x + (acc + b); this CTA
            // owns the column and keeps its running value in shared memory
            float& xr = sm.resid[m][j - sm.r0[1]];
            xr = __fadd_rn(xr, __fadd_rn(sum, bj));
            p.x[(size_t)m * E + j] = xr;
        }
    }
}

__device__ __forceinline__ float pick(const float (&a)[kRowsMax], int i) {
    float v = a[0];
#pragma unroll
    for (int k = 1; k < kRowsMax; ++k) v = i == k ? a[k] : v;
    return v;
}

// This CTA's rows of matrix `mi` against the staged rows xs. `pk` is the ring
// position, advanced exactly as the producer advances it. Warp w reduces
// segment w of each slot; rows cut into slices are finished once all their
// slices are in (every slot holds whole rows).
template <int KIND>
__device__ bool stage_matmul(const StepParams& p, Smem& sm, const StepLayer* tab, const char* ring,
                             const float* xs, const float* params, int mi, uint32_t& pk, Best& best) {
    const MatDesc d = mat_desc(p, tab, mi);
    const int layer = mi >> 2;
    const int t = threadIdx.x - 32, warp = t >> 5, lane = t & 31;
    const int M = p.M, K4 = d.K >> 2, WS = 1 << d.lws;
    const int r0 = sm.r0[d.kind], r1 = sm.r1[d.kind];
    const float* bias = params + 2 * p.E;
    const int r0a = r0 & ~3;
    const int g1 = r1 << d.lws;
    // Batch 1 with at most kRegChunks chunks per lane: this warp's activation
    // chunks in registers for the whole stage (its slice of every row it
    // reduces is slice warp mod WS), so the shared-memory traffic is the
    // weights alone.
    const bool xreg = M == 1 && (d.sc + 31) / 32 <= kRegChunks;
    float4 xr[kRegChunks];
    if (xreg) {
        const int c0 = (warp & (WS - 1)) * d.sc, nc = min(K4, c0 + d.sc) - c0;
#pragma unroll
        for (int u = 0; u < kRegChunks; ++u)
            xr[u] = 32 * u + lane < nc ? reinterpret_cast<const float4*>(xs)[c0 + 32 * u + lane]
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const bool fine = p.trace && t == 0 && layer == 1;
    const int fine0 = step_trace_fine(p.n_layer) + 16 * (mi & 3);
    int pkt = 0;
    for (int g = r0 << d.lws; g < g1; g += d.P, ++pk, ++pkt) {
        const int slot = pk % p.slots;
        const uint32_t par = (pk / p.slots) & 1;
        const int ge = min(g + d.P, g1);
        const int gs = g + warp;   // this warp's segment
        const bool fs = fine && pkt < 4;
        if (fs) stamp(p, fine0 + 4 * pkt);
        float acc[kRowsMax] = {0.f, 0.f, 0.f, 0.f};
        bool have = false;
        if (gs < ge && !sm.abort) {
            if (!mbar_wait(&sm.full[slot], par)) {
                atomicExch(p.err, 1);
                sm.abort = 1;
            } else {
                have = true;
                if (fs) stamp(p, fine0 + 4 * pkt + 1);
                const float* w = reinterpret_cast<const float*>(ring + (size_t)slot * kSlot) +
                                 (seg_off(d, gs) - seg_off(d, g));
                const int s = gs & (WS - 1);
                const int c0 = s * d.sc, nc = min(K4, c0 + d.sc) - c0;
                if (xreg) {
                    // batch 1: the activation chunks are in registers
#pragma unroll
                    for (int u = 0; u < kRegChunks; ++u) {
                        if (32 * u + lane < nc) {
                            const float4 wv = reinterpret_cast<const float4*>(w)[32 * u + lane];
                            float a = acc[0];
                            a = fmaf(wv.x, xr[u].x, a);
                            a = fmaf(wv.y, xr[u].y, a);
                            a = fmaf(wv.z, xr[u].z, a);
                            a = fmaf(wv.w, xr[u].w, a);
                            acc[0] = a;
                        }
                    }
                } else
                for (int c = lane; c < nc; c += 32) {
                    const float4 wv = reinterpret_cast<const float4*>(w)[c];
#pragma unroll
                    for (int m = 0; m < kRowsMax; ++m) {
                        if (m < M) {
                            const float4 xv = reinterpret_cast<const float4*>(xs + (size_t)m * d.K)[c0 + c];
                            float a = acc[m];
                            a = fmaf(wv.x, xv.x, a);
                            a = fmaf(wv.y, xv.y, a);
                            a = fmaf(wv.z, xv.z, a);
                            a = fmaf(wv.w, xv.w, a);
                            acc[m] = a;
                        }
                    }
                }
#pragma unroll
                for (int m = 0; m < kRowsMax; ++m) {
                    if (m < M) {
                        float v = acc[m];
#pragma unroll
                        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                        acc[m] = v;
                    }
                }
            }
        }
        __syncwarp();
        if (fs) stamp(p, fine0 + 4 * pkt + 2);
        if (lane == 0) mbar_arrive(&sm.empty[slot]);
        if (WS == 1) {
            if (have && lane < M) epilogue<KIND>(p, sm, layer, pick(acc, lane), gs, lane, bias, r0a, best);
        } else {
            // slice sums in slice order, then the epilogue
            if (lane == 0)
#pragma unroll
                for (int m = 0; m < kRowsMax; ++m) sm.pk_sum[warp][m] = acc[m];
            cons_sync();
            const int rows = (ge - g) >> d.lws;
            if (t < rows * M && !sm.abort) {
                const int r = t / M, m = t % M;
                float sum = sm.pk_sum[r * WS][m];
                for (int k = 1; k < WS; ++k) sum += sm.pk_sum[r * WS + k][m];
                epilogue<KIND>(p, sm, layer, sum, (g >> d.lws) + r, m, bias, r0a, best);
            }
            cons_sync();
        }
        if (fs) stamp(p, fine0 + 4 * pkt + 3);
    }
    cons_sync();
    return !sm.abort;
}

// One 16-position chunk of one (sequence, head) by one warp, with the
// arithmetic of attn_decode_fused_kernel<16> (k_attn.cu): lane 2 pi + half
// takes position pi's score over its half of the dims; probabilities from the
// chunk max; the sum of probabilities in position order; the weighted values
// as eight position groups g (positions g, g + 8) added in group order. Lane l
// finishes dims 2l and 2l + 1. Writes max, sum and the 64 sums to out.
__device__ void attn_chunk(const StepParams& p, const Smem& sm, const float* kl, const float* vl, int b, int h,
                           int p0, int n, const float4 (&qv)[8], int lane, float* out) {
    const int E = p.E;
    const int pi = lane >> 1, half = lane & 1;
    auto row = [&](int pos) { return (size_t)sm.pt[b][pos >> 4] * kPageRows + (pos & 15); };
    float a = 0.f;
    if (pi < n) {
        const float* kp = kl + row(p0 + pi) * E + h * D;
        float4 kv[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) kv[j] = ld_cg4(kp + 4 * (2 * j + half));
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            a = fmaf(qv[j].x, kv[j].x, a);
            a = fmaf(qv[j].y, kv[j].y, a);
            a = fmaf(qv[j].z, kv[j].z, a);
            a = fmaf(qv[j].w, kv[j].w, a);
        }
    }
    // the values of this chunk (dims 2 lane, 2 lane + 1), loaded while the scores finish
    float2 vv[CHT];
#pragma unroll
    for (int i = 0; i < CHT; ++i)
        vv[i] = i < n ? ld_cg2(vl + row(p0 + i) * E + h * D + 2 * lane) : make_float2(0.f, 0.f);
    a += __shfl_xor_sync(0xffffffffu, a, 1);
    const float sc = pi < n ? a * p.scale : -INFINITY;
    float mx = sc;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float e = pi < n ? expf(sc - mx) : 0.f;
    float l = 0.f;
#pragma unroll
    for (int i = 0; i < CHT; ++i) {
        const float ei = __shfl_sync(0xffffffffu, e, 2 * i);
        if (i < n) l += ei;
    }
    float ox = 0.f, oy = 0.f;
#pragma unroll
    for (int g = 0; g < 8; ++g) {
        const float e0 = __shfl_sync(0xffffffffu, e, 2 * g);
        const float e1 = __shfl_sync(0xffffffffu, e, 2 * (g + 8));
        float ax = 0.f, ay = 0.f;
        if (g < n) { ax = fmaf(e0, vv[g].x, ax); ay = fmaf(e0, vv[g].y, ay); }
        if (g + 8 < n) { ax = fmaf(e1, vv[g + 8].x, ax); ay = fmaf(e1, vv[g + 8].y, ay); }
        if (g == 0) { ox = ax; oy = ay; }
        else { ox += ax; oy += ay; }
    }
    out[2 + 2 * lane] = ox;
    out[3 + 2 * lane] = oy;
    if (lane == 0) { out[0] = mx; out[1] = l; }
}

// Attention of layer `layer`: one unit per (sequence, head, 16-position
// chunk), dealt round-robin to every consumer warp of the grid (unit u: CTA
// u % G, warp (u / G) % kCons), so a batch-1 step spreads its chunks over the
// whole GPU. Each warp writes its chunk partial; the warp that completes a
// (sequence, head)'s count merges the partials in chunk order (the merge of
// attn_decode_fused_kernel<16>), writes the head's 64 outputs and counts the
// head on `ctr`.
__device__ void stage_attention(const StepParams& p, Smem& sm, int layer, unsigned* ctr) {
    const int t = threadIdx.x - 32, warp = t >> 5, lane = t & 31;
    const int H = p.H, E = p.E, G = gridDim.x;
    // units per sequence: H x its chunks; offsets by a scan over the (<= 4) sequences
    int off[kRowsMax + 1];
    off[0] = 0;
    for (int m = 0; m < p.M; ++m) off[m + 1] = off[m] + H * ((sm.lens[m] + CHT) / CHT);
    const int units = off[p.M];
    const float* kl = p.k + (size_t)layer * p.layer_stride;
    const float* vl = p.v + (size_t)layer * p.layer_stride;
    for (int u = warp * G + blockIdx.x; u < units; u += G * kCons) {
        int b = 0;
        while (u >= off[b + 1]) ++b;
        const int ctx = sm.lens[b] + 1, ns = (ctx + CHT - 1) / CHT;
        const int r = u - off[b], h = r / ns, c = r - h * ns;
        float4 qv[8];
        const float* qp = p.qkv + (size_t)b * 3 * E + h * D;
#pragma unroll
        for (int j = 0; j < 8; ++j) qv[j] = ld_cg4(qp + 4 * (2 * j + (lane & 1)));
        float* part_g = p.part + (size_t)(b * H + h) * p.max_splits * PART;
        const int p0 = c * CHT;
        attn_chunk(p, sm, kl, vl, b, h, p0, min(CHT, ctx - p0), qv, lane, part_g + (size_t)c * PART);
        __syncwarp();
        int last = 0;
        if (lane == 0) {
            int old;
            asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(&p.head_cnt[b * H + h]) : "memory");
            last = old == ns - 1;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (!last) continue;
        __syncwarp();   // lane 0 acquired the other warps' partials for the whole warp
        float mm = -INFINITY;
        for (int k = lane; k < ns; k += 32) mm = fmaxf(mm, __ldcg(part_g + (size_t)k * PART));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, o));
        float lt = 0.f, o0 = 0.f, o1 = 0.f;
        for (int k0 = 0; k0 < ns; k0 += 32) {
            float2 ml = make_float2(0.f, 0.f);
            if (k0 + lane < ns) ml = ld_cg2(part_g + (size_t)(k0 + lane) * PART);
            const int kn = min(32, ns - k0);
            for (int k1 = 0; k1 < kn; k1 += 8) {
                float2 ov[8];
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    if (k1 + k < kn) ov[k] = ld_cg2(part_g + (size_t)(k0 + k1 + k) * PART + 2 + 2 * lane);
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const float mk = __shfl_sync(0xffffffffu, ml.x, (k1 + k) & 31);
                    const float lk = __shfl_sync(0xffffffffu, ml.y, (k1 + k) & 31);
                    if (k1 + k < kn) {
                        const float cf = expf(mk - mm);
                        lt = fmaf(lk, cf, lt);
                        o0 = fmaf(ov[k].x, cf, o0);
                        o1 = fmaf(ov[k].y, cf, o1);
                    }
                }
            }
        }
        *reinterpret_cast<float2*>(p.attn + (size_t)b * E + h * D + 2 * lane) = make_float2(o0 / lt, o1 / lt);
        __syncwarp();
        if (lane == 0) {
            p.head_cnt[b * H + h] = 0;
            signal(ctr);
        }
    }
}

__device__ void consumers(const StepParams& p, Smem& sm, const StepLayer* tab, const char* ring, float* xs,
                          float* params) {
    const int t = threadIdx.x - 32;
    const int E = p.E, M = p.M, G = gridDim.x;
    const int pfl = param_floats(E, G);
    uint32_t pk = 0;
    Best best{0.f, -1, -1};
    const bool tr = p.trace && t == 0;
    if (tr) stamp(p, 0);
    for (int l = 0; l < p.n_layer; ++l) {
        unsigned* ctr = p.sync + 5 * l;
        const int mq = 4 * l, mp = 4 * l + 1, mf = 4 * l + 2, mm = 4 * l + 3;
        float* pq = params + (size_t)(mq & 1) * pfl;
        float* pp = params + (size_t)(mp & 1) * pfl;
        // A: LN1 + qkv
        if (!stage_begin(p, sm, l == 0 ? nullptr : ctr - 1, G, mq)) return;
        if (tr) stamp(p, ev_stage(l, 0, 0));
        if (l == 0) {
            stage_embed(p, sm, xs);
            ln_rows(sm, xs, M, E, pq, pq + E, p.eps);
        } else {
            stage_rows(sm, p.x, E, M, E, pq, pq + E, p.eps, xs);
        }
        if (tr) stamp(p, ev_stage(l, 0, 1));
        if (!stage_matmul<ST_QKV>(p, sm, tab, ring, xs, pq, mq, pk, best)) return;
        stage_params_done(sm, mq);
        if (t == 0) signal(ctr + 0);
        if (tr) stamp(p, ev_stage(l, 0, 2));
        // B: attention
        if (!stage_begin(p, sm, ctr + 0, G, -1)) return;
        if (tr) { stamp(p, ev_stage(l, 1, 0)); stamp(p, ev_stage(l, 1, 1)); }
        stage_attention(p, sm, l, ctr + 1);
        if (tr) stamp(p, ev_stage(l, 1, 2));
        // C: proj + residual
        if (!stage_begin(p, sm, ctr + 1, (unsigned)(M * p.H), mp)) return;
        if (tr) stamp(p, ev_stage(l, 2, 0));
        stage_rows(sm, p.attn, E, M, E, nullptr, nullptr, 0.f, xs);
        if (tr) stamp(p, ev_stage(l, 2, 1));
        if (!stage_matmul<ST_PROJ>(p, sm, tab, ring, xs, pp, mp, pk, best)) return;
        stage_params_done(sm, mp);
        if (t == 0) signal(ctr + 2);
        if (tr) stamp(p, ev_stage(l, 2, 2));
        // D: LN2 + fc + gelu
        float* pf = params + (size_t)(mf & 1) * pfl;
        if (!stage_begin(p, sm, ctr + 2, G, mf)) return;
        if (tr) stamp(p, ev_stage(l, 3, 0));
        stage_rows(sm, p.x, E, M, E, pf, pf + E, p.eps, xs);
        if (tr) stamp(p, ev_stage(l, 3, 1));
        if (!stage_matmul<ST_FC>(p, sm, tab, ring, xs, pf, mf, pk, best)) return;
        stage_params_done(sm, mf);
        if (t == 0) signal(ctr + 3);
        if (tr) stamp(p, ev_stage(l, 3, 2));
        // E: mlp + residual
        float* pm = params + (size_t)(mm & 1) * pfl;
        if (!stage_begin(p, sm, ctr + 3, G, mm)) return;
        if (tr) stamp(p, ev_stage(l, 4, 0));
        stage_rows(sm, p.ff, 4 * E, M, 4 * E, nullptr, nullptr, 0.f, xs);
        if (tr) stamp(p, ev_stage(l, 4, 1));
        if (!stage_matmul<ST_MLP>(p, sm, tab, ring, xs, pm, mm, pk, best)) return;
        stage_params_done(sm, mm);
        if (t == 0) signal(ctr + 4);
        if (tr) stamp(p, ev_stage(l, 4, 2));
    }
    // the head: LN_f, wte rows, this CTA's best per sequence
    const int mh = 4 * p.n_layer, eh = 1 + 3 * 5 * p.n_layer;
    float* ph = params + (size_t)(mh & 1) * pfl;
    if (!stage_begin(p, sm, p.sync + 5 * p.n_layer - 1, G, mh)) return;
    if (tr) stamp(p, eh + 0);
    stage_rows(sm, p.x, E, M, E, ph, ph + E, p.eps, xs);
    if (tr) stamp(p, eh + 1);
    if (!stage_matmul<ST_HEAD>(p, sm, tab, ring, xs, ph, mh, pk, best)) return;
    stage_params_done(sm, mh);
    if (tr) stamp(p, eh + 2);
    const int warp = t >> 5, lane = t & 31;
    for (int m = 0; m < M; ++m) {
        float bv = best.m == m ? best.v : 0.f;
        int bi = best.m == m ? best.i : -1;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi >= 0 && beats(ov, oi, bv, bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) { sm.best_v[warp][m] = bv; sm.best_i[warp][m] = bi; }
    }
    cons_sync();
    if (t < M) {
        float bv = sm.best_v[0][t];
        int bi = sm.best_i[0][t];
        for (int k = 1; k < kCons; ++k)
            if (sm.best_i[k][t] >= 0 && beats(sm.best_v[k][t], sm.best_i[k][t], bv, bi)) {
                bv = sm.best_v[k][t];
                bi = sm.best_i[k][t];
            }
        p.am_val[(size_t)blockIdx.x * M + t] = bv;
        p.am_idx[(size_t)blockIdx.x * M + t] = sm.nan0[t] ? -2 : bi;
    }
    cons_sync();
    unsigned* ticket = p.sync + 5 * p.n_layer;
    if (t == 0) {
        __threadfence();
        sm.last = atomicAdd(ticket, 1u) == (unsigned)(G - 1);
    }
    cons_sync();
    if (tr) stamp(p, step_trace_end(p.n_layer));
    if (!sm.last) return;
    // the last CTA: final argmax, bookkeeping, counters back to zero
    __threadfence();
    if (t < M) {
        float bv = 0.f;
        int bi = -1;
        bool nan0 = false;
        for (int c = 0; c < G; ++c) {
            const int i = __ldcg(p.am_idx + (size_t)c * M + t);
            const float v = __ldcg(p.am_val + (size_t)c * M + t);
            if (i == -2) nan0 = true;
            else if (i >= 0 && beats(v, i, bv, bi)) { bv = v; bi = i; }
        }
        const int32_t nx = nan0 ? 0 : (bi < 0 ? 0 : bi);
        p.next[t] = nx;
        if (p.advance) {
            const int s = *p.step;
            p.tokens[t] = nx;
            p.out[(size_t)t * p.ld_out + s] = nx;
            p.lens[t] = sm.lens[t] + 1;
        }
    }
    cons_sync();
    if (t == 0 && p.advance) *p.step += 1;
    for (int i = t; i <= 5 * p.n_layer; i += kCons * 32) p.sync[i] = 0;
}

__global__ void __launch_bounds__(kThreads, 1) step_kernel(const StepParams p) {
    extern __shared__ __align__(128) char dyn[];
    __shared__ Smem sm;
    char* ring = dyn;
    float* xs = reinterpret_cast<float*>(dyn + (size_t)p.slots * kSlot);
    float* params = xs + (size_t)p.M * 4 * p.E;
    StepLayer* tab = reinterpret_cast<StepLayer*>(params + 2 * (size_t)param_floats(p.E, gridDim.x));
    // bulk copies land 16-byte aligned; refuse to run otherwise
    if (smem_u32(dyn) & 15) {
        if (threadIdx.x == 0) atomicExch(p.err, 2);
        return;
    }
    // the layer table, the step's page tables and positions into shared memory
    {
        const unsigned long long* src = reinterpret_cast<const unsigned long long*>(p.layers);
        unsigned long long* dst = reinterpret_cast<unsigned long long*>(tab);
        const int words = p.n_layer * (int)(sizeof(StepLayer) / 8);
        for (int i = threadIdx.x; i < words; i += kThreads) dst[i] = src[i];
        for (int i = threadIdx.x; i < p.M * p.pages_per_seq; i += kThreads)
            sm.pt[i / p.pages_per_seq][i % p.pages_per_seq] = p.page_table[i];
        if (threadIdx.x < kRowsMax) {
            sm.lens[threadIdx.x] = (int)threadIdx.x < p.M ? p.lens[threadIdx.x] : 0;
            sm.nan0[threadIdx.x] = 0;
        }
        if (threadIdx.x < 5) {
            const int E = p.E;
            const int N = threadIdx.x == 0 ? 3 * E : threadIdx.x == 2 ? 4 * E : threadIdx.x == 4 ? p.V : E;
            sm.r0[threadIdx.x] = (int)((long long)N * blockIdx.x / gridDim.x);
            sm.r1[threadIdx.x] = (int)((long long)N * (blockIdx.x + 1) / gridDim.x);
        }
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < p.slots; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], kCons);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&sm.pfull[s], 1);
            mbar_init(&sm.pempty[s], 1);
        }
        sm.abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if ((int)threadIdx.x < p.M) {
        const int m = threadIdx.x, pos = sm.lens[m];
        sm.kvrow[m] = (long long)sm.pt[m][pos >> 4] * kPageRows + (pos & (kPageRows - 1));
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        if (threadIdx.x == 0) producer_weights(p, sm, ring, tab);
        else if (threadIdx.x == 1) producer_params(p, sm, params, tab);
        return;
    }
    consumers(p, sm, tab, ring, xs, params);
}

// Shared memory of a launch: the ring, the activation rows, two parameter
// buffers and the layer table.
size_t step_smem(int slots, int M, int E, int n_layer, int grid) {
    return (size_t)slots * kSlot + (size_t)M * 4 * E * sizeof(float) +
           2 * (size_t)param_floats(E, grid) * sizeof(float) + (size_t)n_layer * sizeof(StepLayer);
}

}  // namespace

int step_max_pages() { return kMaxPages; }

// Whether the persistent step applies: M <= 4 sequences, head dim 64, one row
// of every matrix fits a ring slot, and at least two slots fit next to the
// other buffers. Fills *slots and *grid. (Caches of at most step_max_pages()
// pages per sequence are a further condition of each launch.)
bool step_supported(int M, int E, int H, int n_layer, int* slots, int* grid) {
    if (M < 1 || M > kRowsMax || E % 4 || E % H || E / H != D) return false;
    const int K4s[2] = {E / 4, E};
    for (int K4 : K4s) {
        const int WS = K4 <= 256 ? 1 : 4;
        if (K4 > 2048) return false;
        const int sc = (K4 + WS - 1) / WS;
        int P = kSlot / (sc * 16);
        if (P > kCons) P = kCons;
        if (P - P % WS < WS) return false;
    }
    int dev = 0, optin = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) return false;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return false;
    if ((E + sms - 1) / sms > kMaxResid) return false;
    const size_t budget = (size_t)optin - sizeof(Smem) - 1024;
    int s = kMaxSlots;
    while (s >= 2 && step_smem(s, M, E, n_layer, sms) > budget) --s;
    if (s < 2) return false;
    const size_t smem = step_smem(s, M, E, n_layer, sms);
    // the attribute is an upper bound shared by every batch size: the whole budget
    if (cudaFuncSetAttribute(step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(budget & ~(size_t)15)) !=
        cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, step_kernel, kThreads, smem) != cudaSuccess ||
        per_sm < 1) {
        cudaGetLastError();
        return false;
    }
    *slots = s;
    *grid = sms;
    return true;
}

cudaError_t launch_step(const StepParams& p, int grid, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = step_smem(p.slots, p.M, p.E, p.n_layer, grid);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, step_kernel, p);
    return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace tie
