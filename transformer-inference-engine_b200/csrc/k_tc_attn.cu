// k_tc_attn.cu -- causal prefill attention on the tensor cores (head_dim 64).
//
// Reference: model.c:705-732 (per head: scores q.k scaled by 1/sqrt(64), the
// causal mask, a max-subtracted softmax, the probability-weighted sum of V).
//
// One CTA per (sequence, head, 128-query block), heavy (late) blocks first. It
// walks 64-key blocks up to the diagonal with an online softmax, both products
// on tcgen05 in the fp32-accurate 3xTF32 form of k_tc_gemm.cu (every operand
// split x = hi + lo, three kind::tf32 MMAs per k-step into fp32 TMEM):
//
//   S  = Q . K^T      M = 128 queries, N = 64 keys, K = 64 dims   (TMEM cols 0..127, two blocks)
//   O += P . V        M = 128 queries, N = 64 dims, K = 64 keys   (TMEM cols 128..191)
//
// Warp roles (416 threads):
//   warps 0-7  softmax: warp (q, hf) = (warp % 4, warp / 4) owns TMEM lane
//              quarter q (query rows 32 q .. 32 q + 31, one per thread) and half
//              hf of the 64 columns. Per block it loads its half of the S row,
//              masks and scales it, exchanges the partial row maximum with its
//              partner warp (TMEM exchange column + named barrier), updates the
//              running max and its half of the sum, writes its probabilities
//              (hi/lo) to shared memory as the A operand of P . V, and rescales
//              its half of the running output row O in TMEM by
//              alpha = 2^((m_old - m_new) log2 e) before the block's P . V
//              accumulates onto it. At the end it divides by the row sum and
//              stores its 32 dims.
//   warps 8-11 loaders: plain 16-byte loads of Q (once) and of each key block's
//              K and V rows from the qkv activations, split into hi/lo and
//              stored in the 128-byte-swizzled K-major layout the MMA reads
//              (V transposed: dims are its rows, keys its k). The next block's
//              rows are loaded into registers while the current one computes.
//   warp 12    allocates TMEM and issues the MMAs (one thread): S of blocks 0
//              and 1, then per block j: O += P_j . V_j, S of block j + 2.
//
// Shared memory (224 KB, one CTA per SM): Q hi/lo, two key-block buffers
// (K hi/lo), V^T hi/lo, P hi/lo. TMEM (256 columns): S of two blocks, O, and
// the exchange columns. The steps are ordered by mbarriers: k_full[2] and
// v_full (loaders -> MMA), s_full[2] (S ready), p_full (probabilities written,
// O rescaled), o_full (P . V done: V and P free again). Every wait is bounded;
// on expiry the CTA records the error flag, the loader and MMA loops end, the
// softmax warps finish their blocks without storing, the MMAs issued are
// drained and TMEM is freed before the CTA returns.
//
// A row's result does not depend on T or on the other rows: the MMA computes
// each row independently, key blocks past a row's diagonal contribute exact
// zeros (p = 0, alpha = 1), and padded rows and keys are zero.
#include <cuda.h>

#include <cstdint>

#include "common.cuh"
#include "tc_gemm.h"

namespace tie {
namespace {

#include "tc_ptx.cuh"

constexpr int D = 64;
constexpr int BQ = 128, BKY = 64;
constexpr int kThreads = 416;
constexpr unsigned long long kAttnWaitNs = 2000000000ull;  // 2 s

// shared-memory regions (bytes from the 1024-aligned base); each region is a
// K-major operand with 128-byte rows in 8-row, 1024-byte swizzle atoms. Only
// the B operands live here (two key blocks, two value blocks); Q and P, the A
// operands, are in TMEM.
constexpr uint32_t kKRegion = BKY * 128;           // 64 keys x 32 dims
constexpr uint32_t kVRegion = D * 128;             // 64 dims x 32 keys
constexpr uint32_t kKBuf = 4 * kKRegion;           // one key block: hi (2 regions), lo (2 regions)
constexpr uint32_t kVBuf = 4 * kVRegion;           // one value block, transposed: hi, lo
constexpr uint32_t kOffK = 0;                      // two key-block buffers
constexpr uint32_t kOffV = kOffK + 2 * kKBuf;      // two value-block buffers
constexpr uint32_t kOffBars = kOffV + 2 * kVBuf;
constexpr size_t kSmemBytes = 1024 + kOffBars + 128;
static_assert(kOffBars == 128u * 1024u, "operand layout");
// TMEM columns (all 512): S of two blocks, the running output O, the exchange
// columns of the softmax warp pairs, Q and P (hi and lo)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 128;                    // 128..191
constexpr uint32_t kXchMax = 192;                  // 192..195: partial row maxima (block parity x half)
constexpr uint32_t kXchSum = 196;                  // 196..197: partial row sums (half)
constexpr uint32_t kColQhi = 256, kColQlo = 320;   // Q: 64 dims each
constexpr uint32_t kColPhi = 384, kColPlo = 448;   // P: 64 keys each

// byte offset of element (row, c), c < 32, in a 128-byte-swizzled region
__device__ __forceinline__ uint32_t sw128_off(int row, int c) {
    return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((((c >> 2) ^ (row & 7))) << 4) + (c & 3) * 4);
}

// 16 bytes (4 consecutive elements c..c+3, c % 4 == 0) at (row, c)
__device__ __forceinline__ uint32_t sw128_off4(int row, int c) {
    return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((((c >> 2) ^ (row & 7))) << 4));
}

// kind::tf32, fp32 accumulate, both operands K-major, M = 128, N = 64
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(64 >> 3) << 17) |
                            ((uint32_t)(128 >> 4) << 24);

// 2^x on the special-function unit (ex2.approx.ftz: relative error about
// 2^-22, results below 2^-126 flush to zero). The softmax computes
// exp(s - m) = 2^((s - m) log2 e) with it: one SFU operation per score, where
// the accurate expf takes several.
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// A 16-byte read-only global load that stays where it is written: volatile,
// so the compiler neither sinks it to the first use of its registers nor moves
// it across the barrier waits (the loaders fetch the next key block's rows
// before they wait, and the loads' latency overlaps the wait).
__device__ __forceinline__ float4 ldg_early(const float* p) {
    float4 v;
    asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void st_split4(uint8_t* hi_base, uint8_t* lo_base, uint32_t off, float4 v) {
    const float4 h = make_float4(tf32_hi_int(v.x), tf32_hi_int(v.y), tf32_hi_int(v.z), tf32_hi_int(v.w));
    const float4 l = make_float4(__fsub_rn(v.x, h.x), __fsub_rn(v.y, h.y), __fsub_rn(v.z, h.z), __fsub_rn(v.w, h.w));
    *reinterpret_cast<float4*>(hi_base + off) = h;
    *reinterpret_cast<float4*>(lo_base + off) = l;
}

__global__ void __launch_bounds__(kThreads, 1)
tc_attn_prefill_kernel(const float* __restrict__ qkv, int T, int H, float scale, float* __restrict__ out,
                       float* __restrict__ out_hi, float* __restrict__ out_lo, int* __restrict__ err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBars);
    uint64_t* k_full = bars + 0;    // [2] key block in buffer b written (128 loader arrivals; the first also Q)
    uint64_t* v_full = bars + 2;    // [2] value block in buffer b written (128 loader arrivals)
    uint64_t* s_full = bars + 4;    // [2] S of buffer b computed: K buffer b free (MMA commit)
    uint64_t* v_free = bars + 6;    // [2] P . V of value buffer b done (MMA commit)
    uint64_t* p_full = bars + 8;    // P written, O rescaled (256 softmax arrivals)
    uint64_t* o_full = bars + 9;    // P . V of the block done: P free (MMA commit)
    uint64_t* drained = bars + 10;  // every MMA done (MMA commit)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 11);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int E = H * D, E3 = 3 * E;
    const int qb = gridDim.x - 1 - blockIdx.x;
    const int h = blockIdx.y, seq = blockIdx.z;
    const int q0 = qb * BQ;
    const int n_kb = (min(q0 + BQ, T) - 1) / BKY + 1;
    const float* base = qkv + (size_t)seq * T * E3 + h * D;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(&k_full[b]), 128);
            mbar_init(smem_u32(&v_full[b]), 128);
            mbar_init(smem_u32(&s_full[b]), 1);
            mbar_init(smem_u32(&v_free[b]), 1);
        }
        mbar_init(smem_u32(p_full), 256);
        mbar_init(smem_u32(o_full), 1);
        mbar_init(smem_u32(drained), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 12) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(tmem_slot)), "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = *tmem_slot;
    // this warp's TMEM lane quarter (warp % 4), column 0
    const uint32_t lane_addr = tmem + ((uint32_t)((warp & 3) * 32) << 16);

    auto wait = [&](const uint64_t* bar, uint32_t parity) -> bool {
        const uint32_t b = smem_u32(bar);
        if (mbar_try_wait(b, parity)) return true;
        const unsigned long long t0 = globaltimer_ns();
        for (uint32_t i = 1;; ++i) {
            if (mbar_try_wait(b, parity)) return true;
            if ((i & 255u) == 0) {
                if (*abort_flag) return false;
                if (globaltimer_ns() - t0 > kAttnWaitNs) break;
            }
        }
        *abort_flag = 1;
        if (err) atomicExch(err, 1);
        return false;
    };

    if (warp >= 8 && warp < 12) {
        // ------------------------------------------------------------ loaders
        const int t = threadIdx.x - 256;   // = TMEM lane of this thread's Q row
        // Q: row t, all 64 dims, split into hi/lo and stored to TMEM (warp-collective)
        {
            const int row = q0 + t;
#pragma unroll 1
            for (int g = 0; g < 2; ++g) {   // dims 32 g .. 32 g + 31
                float x[32];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float4 v = row < T ? __ldg(reinterpret_cast<const float4*>(base + (size_t)row * E3 + 32 * g) + i)
                                             : make_float4(0.f, 0.f, 0.f, 0.f);
                    x[4 * i] = v.x;
                    x[4 * i + 1] = v.y;
                    x[4 * i + 2] = v.z;
                    x[4 * i + 3] = v.w;
                }
                uint32_t w[32];
#pragma unroll
                for (int c = 0; c < 32; ++c) w[c] = __float_as_uint(tf32_hi_int(x[c]));
                tmem_st32(lane_addr + kColQhi + (uint32_t)(32 * g), w);
#pragma unroll
                for (int c = 0; c < 32; ++c) w[c] = __float_as_uint(__fsub_rn(x[c], __uint_as_float(w[c])));
                tmem_st32(lane_addr + kColQlo + (uint32_t)(32 * g), w);
            }
            asm volatile("tcgen05.fence::before_thread_sync;");
        }
        // K and V: key row kr = t / 2, dims [32 half, 32 half + 32)
        const int kr = t >> 1, half = t & 1;
        float4 kv[8], vv[8];
        auto load4 = [&](float4 (&dst)[8], int j, int which) {
            const int key = j * BKY + kr;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                dst[i] = key < T ? ldg_early(base + (size_t)key * E3 + which * E + half * 32 + 4 * i)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
        };
        load4(kv, 0, 1);
        load4(vv, 0, 2);
        const uint32_t vreg = (uint32_t)(kr >> 5) * kVRegion;
        const int kc = kr & 31;
        for (int j = 0; j < n_kb; ++j) {
            const int b = j & 1;
            const uint32_t use = (uint32_t)(j >> 1);
            // key buffer b is free once S of block j - 2 is computed
            if (j >= 2 && !wait(&s_full[b], (use - 1) & 1u)) break;
            uint8_t* kb = smem + kOffK + (uint32_t)b * kKBuf;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                st_split4(kb, kb + 2 * kKRegion, (uint32_t)half * kKRegion + sw128_off4(kr, 4 * i), kv[i]);
            fence_async_smem();
            mbar_arrive(smem_u32(&k_full[b]));
            if (j + 1 < n_kb) load4(kv, j + 1, 1);
            // value buffer b is free once P . V of block j - 2 is done
            if (j >= 2 && !wait(&v_free[b], (use - 1) & 1u)) break;
            uint8_t* vb = smem + kOffV + (uint32_t)b * kVBuf;
            auto st_v = [&](int d, float x) {
                // V transposed: element (key kr, dim d) at row d, column kr % 32 of key region kr / 32
                const uint32_t off = vreg + sw128_off(d, kc);
                const float hv = tf32_hi_int(x);
                *reinterpret_cast<float*>(vb + off) = hv;
                *reinterpret_cast<float*>(vb + 2 * kVRegion + off) = __fsub_rn(x, hv);
            };
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int d = half * 32 + 4 * i;
                st_v(d, vv[i].x);
                st_v(d + 1, vv[i].y);
                st_v(d + 2, vv[i].z);
                st_v(d + 3, vv[i].w);
            }
            fence_async_smem();
            mbar_arrive(smem_u32(&v_full[b]));
            if (j + 1 < n_kb) load4(vv, j + 1, 2);
        }
    } else if (warp == 12) {
        // ---------------------------------------------------------------- MMA
        if (lane == 0) {
            const uint32_t sb = smem_u32(smem);
            // S_j = Q . K_j^T into S[j % 2] over the 64 dims (eight 8-wide k-steps):
            // A = Q from TMEM, B = the key block from shared memory
            auto issue_s = [&](int j) -> bool {
                const int b = j & 1;
                if (!wait(&k_full[b], (uint32_t)(j >> 1) & 1u)) return false;
                asm volatile("tcgen05.fence::after_thread_sync;");
                const uint32_t kb = sb + kOffK + (uint32_t)b * kKBuf;
                const uint32_t d = tmem + 64u * (uint32_t)b;
#pragma unroll
                for (int rg = 0; rg < 2; ++rg)
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) {
                        const uint32_t k0 = (uint32_t)(32 * rg + 8 * ks);
                        const uint64_t b_hi = sw128_desc(kb + rg * kKRegion + ks * 32);
                        const uint64_t b_lo = sw128_desc(kb + 2 * kKRegion + rg * kKRegion + ks * 32);
                        mma_tf32_ta(d, tmem + kColQlo + k0, b_hi, kIdesc, (rg | ks) ? 1u : 0u);
                        mma_tf32_ta(d, tmem + kColQhi + k0, b_lo, kIdesc, 1u);
                        mma_tf32_ta(d, tmem + kColQhi + k0, b_hi, kIdesc, 1u);
                    }
                mma_commit(smem_u32(&s_full[b]));
                return true;
            };
            bool go = issue_s(0) && (n_kb < 2 || issue_s(1));
            for (int j = 0; go && j < n_kb; ++j) {
                const int b = j & 1;
                if (!wait(p_full, (uint32_t)j & 1u) || !wait(&v_full[b], (uint32_t)(j >> 1) & 1u)) break;
                asm volatile("tcgen05.fence::after_thread_sync;");
                // O += P_j . V_j over the 64 keys of the block: A = P from TMEM
                const uint32_t vb = sb + kOffV + (uint32_t)b * kVBuf;
#pragma unroll
                for (int rg = 0; rg < 2; ++rg)
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) {
                        const uint32_t k0 = (uint32_t)(32 * rg + 8 * ks);
                        const uint64_t b_hi = sw128_desc(vb + rg * kVRegion + ks * 32);
                        const uint64_t b_lo = sw128_desc(vb + 2 * kVRegion + rg * kVRegion + ks * 32);
                        mma_tf32_ta(tmem + kColO, tmem + kColPlo + k0, b_hi, kIdesc, (j | rg | ks) ? 1u : 0u);
                        mma_tf32_ta(tmem + kColO, tmem + kColPhi + k0, b_lo, kIdesc, 1u);
                        mma_tf32_ta(tmem + kColO, tmem + kColPhi + k0, b_hi, kIdesc, 1u);
                    }
                mma_commit(smem_u32(o_full));
                mma_commit(smem_u32(&v_free[b]));
                // S of block j + 2 into the buffer block j's softmax has finished reading
                if (j + 2 < n_kb && !issue_s(j + 2)) break;
            }
            // arrives once every MMA issued above has completed (also when cut
            // short); this thread waits for it so that TMEM is freed only
            // after the last MMA (the warp's other lanes wait at the block
            // barrier below, not in a spin beside the issuing lane)
            mma_commit(smem_u32(drained));
            const unsigned long long t0 = globaltimer_ns();
            while (!mbar_try_wait(smem_u32(drained), 0))
                if (globaltimer_ns() - t0 > kAttnWaitNs) {
                    if (err) atomicExch(err, 1);
                    break;
                }
        }
    } else {
        // ------------------------------------------------------------ softmax
        // Warp (q, hf) = (warp % 4, warp / 4): TMEM lane quarter q (query rows
        // 32 q .. 32 q + 31, one per thread) and half hf of the 64 columns (keys
        // of S, dims of O). The two warps of a quarter combine their partial
        // row maxima through two TMEM exchange columns and a named barrier, so
        // both hold the same maximum and alpha; each keeps its half of the row
        // sum, added once at the end.
        const int q = warp & 3, hf = warp >> 2;
        const int r = q * 32 + lane;   // TMEM lane = query row within the block
        const int row = q0 + r;
        const int last_key = min(row, T - 1);   // padded rows (row >= T) see every real key
        // tcgen05.ld / tcgen05.st are warp-collective (.sync.aligned) and the
        // named barrier pairs two warps: every lane of both warps executes each
        // of them on every block. A failed wait therefore does not leave the
        // loop: it clears `ok` (the abort flag makes every later wait return
        // at once), the remaining blocks run on whatever TMEM holds, and
        // nothing is stored.
        auto pair_sync = [&]() {
            asm volatile("tcgen05.fence::before_thread_sync;");
            asm volatile("bar.sync %0, 64;" ::"r"(1 + q) : "memory");
            asm volatile("tcgen05.fence::after_thread_sync;");
        };
        constexpr unsigned kAll = 0xffffffffu;
        constexpr float kLog2e = 1.4426950408889634f;
        const float scale2 = scale * kLog2e;   // q.k to the exp2 domain in one multiply
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < n_kb; ++j) {
            const int b = j & 1;
            ok = __all_sync(kAll, wait(&s_full[b], (uint32_t)(j >> 1) & 1u)) && ok;
            asm volatile("tcgen05.fence::after_thread_sync;");
            const int key0 = j * BKY + 32 * hf;
            float sv[32];
            {
                uint32_t v[32];
                tmem_ld32(lane_addr + 64u * (uint32_t)b + (uint32_t)(32 * hf), v);
#pragma unroll
                for (int c = 0; c < 32; ++c) sv[c] = __uint_as_float(v[c]);
            }
            float mt = -INFINITY;
#pragma unroll
            for (int c = 0; c < 32; ++c)
                if (key0 + c <= last_key) mt = fmaxf(mt, sv[c] * scale);
            tmem_st1(lane_addr + kXchMax + 2u * (uint32_t)b + (uint32_t)hf, __float_as_uint(mt));
            pair_sync();
            mt = fmaxf(mt, __uint_as_float(tmem_ld1(lane_addr + kXchMax + 2u * (uint32_t)b + (uint32_t)(hf ^ 1))));
            const float m_new = fmaxf(m, mt);
            const float alpha = (m == -INFINITY) ? 0.f : ex2_approx((m - m_new) * kLog2e);
            const float mb = m_new * kLog2e;   // the maximum in the exp2 domain
            float ps = 0.f;
#pragma unroll
            for (int c = 0; c < 32; ++c) {
                sv[c] = key0 + c <= last_key ? ex2_approx(fmaf(sv[c], scale2, -mb)) : 0.f;
                ps += sv[c];
            }
            l = l * alpha + ps;
            m = m_new;
            if (j > 0) {
                // P . V of block j - 1 is done: its P may be overwritten, and this
                // warp's half of the running output in TMEM is rescaled to the
                // new maximum before this block's P . V accumulates onto it
                ok = __all_sync(kAll, wait(o_full, (uint32_t)(j - 1) & 1u)) && ok;
                asm volatile("tcgen05.fence::after_thread_sync;");
                if (__any_sync(kAll, alpha != 1.f)) {
                    uint32_t v[32];
                    tmem_ld32(lane_addr + kColO + (uint32_t)(32 * hf), v);
#pragma unroll
                    for (int d = 0; d < 32; ++d) v[d] = __float_as_uint(__uint_as_float(v[d]) * alpha);
                    tmem_st32(lane_addr + kColO + (uint32_t)(32 * hf), v);
                }
            }
            // probabilities of this half's 32 keys, split hi/lo, into the P columns of TMEM
            {
                uint32_t ph[32], pl[32];
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    const float hv = tf32_hi_int(sv[c]);
                    ph[c] = __float_as_uint(hv);
                    pl[c] = __float_as_uint(__fsub_rn(sv[c], hv));
                }
                tmem_st32(lane_addr + kColPhi + (uint32_t)(32 * hf), ph);
                tmem_st32(lane_addr + kColPlo + (uint32_t)(32 * hf), pl);
            }
            asm volatile("tcgen05.fence::before_thread_sync;");
            mbar_arrive(smem_u32(p_full));
        }
        ok = __all_sync(kAll, wait(o_full, (uint32_t)(n_kb - 1) & 1u)) && ok;
        asm volatile("tcgen05.fence::after_thread_sync;");
        // the row sum: half 0's part plus half 1's, the same order in both warps
        tmem_st1(lane_addr + kXchSum + (uint32_t)hf, __float_as_uint(l));
        pair_sync();
        const float l_other = __uint_as_float(tmem_ld1(lane_addr + kXchSum + (uint32_t)(hf ^ 1)));
        const float inv = 1.0f / (hf == 0 ? l + l_other : l_other + l);
        uint32_t o[32];
        tmem_ld32(lane_addr + kColO + (uint32_t)(32 * hf), o);
        if (ok && row < T) {
            const size_t ob = ((size_t)seq * T + row) * E + h * D + 32 * hf;
#pragma unroll
            for (int q4 = 0; q4 < 8; ++q4) {
                const float4 v = make_float4(__uint_as_float(o[4 * q4]) * inv, __uint_as_float(o[4 * q4 + 1]) * inv,
                                             __uint_as_float(o[4 * q4 + 2]) * inv,
                                             __uint_as_float(o[4 * q4 + 3]) * inv);
                if (out) reinterpret_cast<float4*>(out + ob)[q4] = v;
                if (out_hi) {
                    const float4 hv = make_float4(tf32_hi(v.x), tf32_hi(v.y), tf32_hi(v.z), tf32_hi(v.w));
                    reinterpret_cast<float4*>(out_hi + ob)[q4] = hv;
                    reinterpret_cast<float4*>(out_lo + ob)[q4] =
                        make_float4(__fsub_rn(v.x, hv.x), __fsub_rn(v.y, hv.y), __fsub_rn(v.z, hv.z),
                                    __fsub_rn(v.w, hv.w));
                }
            }
        }
    }

    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == 12) {
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

}  // namespace

bool tc_attn_prefill_supported(int T, int H) { return T > 0 && H > 0; }

cudaError_t launch_tc_attn_prefill(const float* qkv, int n_seq, int T, int H, float* out, float* out_hi,
                                   float* out_lo, int* err, cudaStream_t st) {
    if (T <= 0 || n_seq <= 0) return cudaSuccess;
    if ((out_hi == nullptr) != (out_lo == nullptr)) return cudaErrorInvalidValue;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(tc_attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)kSmemBytes);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    const float scale = (float)(1.0 / sqrt((double)D));
    dim3 grid((T + BQ - 1) / BQ, H, n_seq);
    tc_attn_prefill_kernel<<<grid, kThreads, kSmemBytes, st>>>(qkv, T, H, scale, out, out_hi, out_lo, err);
    return cudaGetLastError();
}

}  // namespace tie
