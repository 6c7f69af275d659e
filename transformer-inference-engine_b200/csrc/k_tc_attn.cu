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
//   S  = Q . K^T      M = 128 queries, N = 64 keys, K = 64 dims   (TMEM cols 0..63)
//   O += P . V        M = 128 queries, N = 64 dims, K = 64 keys   (TMEM cols 64..127)
//
// Warp roles (288 threads):
//   warps 0-3  softmax: thread = one query row = one TMEM lane. Loads its S row,
//              masks and scales it, updates the running max and sum, writes its
//              probabilities (hi/lo) to shared memory as the A operand of P . V,
//              and rescales its row of the running output O in TMEM by
//              alpha = exp(m_old - m_new) before the block's P . V accumulates
//              onto it. At the end it divides its row by the sum and stores it.
//   warps 4-7  loaders: plain 16-byte loads of Q (once) and of each key block's
//              K and V rows from the qkv activations, split into hi/lo and
//              stored in the 128-byte-swizzled K-major layout the MMA reads
//              (V transposed: dims are its rows, keys its k). The next block's
//              rows are loaded into registers while the current one computes.
//   warp 8     allocates TMEM and issues the MMAs (one thread).
//
// Shared memory (192 KB, one CTA per SM): Q hi/lo, K hi/lo, V^T hi/lo, P hi/lo.
// Each block's steps are ordered by mbarriers: kv_full (loaders -> MMA),
// s_full (S ready), p_full (probabilities written, O rescaled), o_full (P . V
// done: K, V, P and S free again). Every wait is bounded; on expiry the CTA records the
// error flag, every role leaves its loop, the MMAs it issued are drained and
// TMEM is freed before it returns.
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
constexpr int kThreads = 288;
constexpr unsigned long long kAttnWaitNs = 2000000000ull;  // 2 s

// shared-memory regions (bytes from the 1024-aligned base); each region is a
// K-major operand with 128-byte rows in 8-row, 1024-byte swizzle atoms
constexpr uint32_t kQRegion = BQ * 128;            // 128 rows x 32 dims
constexpr uint32_t kKRegion = BKY * 128;           // 64 keys x 32 dims
constexpr uint32_t kVRegion = D * 128;             // 64 dims x 32 keys
constexpr uint32_t kPRegion = BQ * 128;            // 128 queries x 32 keys
constexpr uint32_t kOffQhi = 0, kOffQlo = kOffQhi + 2 * kQRegion;
constexpr uint32_t kKBuf = 4 * kKRegion;           // one key block: hi (2 regions), lo (2 regions)
constexpr uint32_t kOffK = kOffQlo + 2 * kQRegion;  // two key-block buffers
constexpr uint32_t kOffVhi = kOffK + 2 * kKBuf, kOffVlo = kOffVhi + 2 * kVRegion;
constexpr uint32_t kOffPhi = kOffVlo + 2 * kVRegion, kOffPlo = kOffPhi + 2 * kPRegion;
constexpr uint32_t kOffBars = kOffPlo + 2 * kPRegion;
constexpr size_t kSmemBytes = 1024 + kOffBars + 128;
static_assert(kOffBars == 224u * 1024u && kSmemBytes <= 227u * 1024u, "operand layout");
constexpr uint32_t kTmemCols = 256;                // S[0] 0..63, S[1] 64..127, O 128..191

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

// hi = x rounded to tf32 (nearest, ties away from zero) with integer
// operations: half a tf32 ulp (bit 12) is added to the magnitude bits and the
// low 13 bits are cleared; a carry out of the mantissa moves into the exponent,
// which is the correct rounding up to the next binade. Finite inputs only (the
// scores, probabilities and activations here are finite).
__device__ __forceinline__ float tf32_hi_int(float x) {
    return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
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
    uint64_t* k_full = bars + 0;    // [2] key block in buffer b written (128 loader arrivals)
    uint64_t* v_full = bars + 2;    // V of the block written (128 loader arrivals)
    uint64_t* s_full = bars + 3;    // [2] S of buffer b computed (MMA commit)
    uint64_t* p_full = bars + 5;    // P written, O rescaled (128 softmax arrivals)
    uint64_t* o_full = bars + 6;    // P . V of the block done (MMA commit)
    uint64_t* drained = bars + 7;   // every MMA done (MMA commit)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int E = H * D, E3 = 3 * E;
    const int qb = gridDim.x - 1 - blockIdx.x;
    const int h = blockIdx.y, seq = blockIdx.z;
    const int q0 = qb * BQ;
    const int n_kb = (min(q0 + BQ, T) - 1) / BKY + 1;
    const float* base = qkv + (size_t)seq * T * E3 + h * D;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&k_full[0]), 128);
        mbar_init(smem_u32(&k_full[1]), 128);
        mbar_init(smem_u32(v_full), 128);
        mbar_init(smem_u32(&s_full[0]), 1);
        mbar_init(smem_u32(&s_full[1]), 1);
        mbar_init(smem_u32(p_full), 128);
        mbar_init(smem_u32(o_full), 1);
        mbar_init(smem_u32(drained), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 8) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(tmem_slot)), "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = *tmem_slot;

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

    if (warp >= 4 && warp < 8) {
        // ------------------------------------------------------------ loaders
        const int t = threadIdx.x - 128;
        // Q: row t, all 64 dims (two 32-dim regions)
        {
            const int row = q0 + t;
            float4 qv[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
                qv[i] = row < T ? __ldg(reinterpret_cast<const float4*>(base + (size_t)row * E3) + i)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const uint32_t off = (uint32_t)(i >> 3) * kQRegion + sw128_off4(t, (i & 7) * 4);
                st_split4(smem + kOffQhi, smem + kOffQlo, off, qv[i]);
            }
        }
        // K and V: key row kr = t / 2, dims [32 half, 32 half + 32)
        const int kr = t >> 1, half = t & 1;
        float4 kv[8], vv[8];
        auto load4 = [&](float4 (&dst)[8], int j, int which) {
            const int key = j * BKY + kr;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                dst[i] = key < T ? __ldg(reinterpret_cast<const float4*>(base + (size_t)key * E3 + which * E +
                                                                          half * 32 + 4 * i))
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
        };
        load4(kv, 0, 1);
        load4(vv, 0, 2);
        const uint32_t vreg = (uint32_t)(kr >> 5) * kVRegion;
        const int kc = kr & 31;
        auto st_v = [&](int d, float x) {
            // V transposed: element (key kr, dim d) at row d, column kr % 32 of key region kr / 32
            const uint32_t off = vreg + sw128_off(d, kc);
            const float hv = tf32_hi_int(x);
            *reinterpret_cast<float*>(smem + kOffVhi + off) = hv;
            *reinterpret_cast<float*>(smem + kOffVlo + off) = __fsub_rn(x, hv);
        };
        for (int j = 0; j < n_kb; ++j) {
            const int b = j & 1;
            // key buffer b is free once S of block j - 2 is computed
            if (j >= 2 && !wait(&s_full[b], (uint32_t)((j - 2) >> 1) & 1u)) break;
            uint8_t* kb = smem + kOffK + (uint32_t)b * kKBuf;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                st_split4(kb, kb + 2 * kKRegion, (uint32_t)half * kKRegion + sw128_off4(kr, 4 * i), kv[i]);
            fence_async_smem();
            mbar_arrive(smem_u32(&k_full[b]));
            if (j + 1 < n_kb) load4(kv, j + 1, 1);
            // V is free once P . V of block j - 1 is done
            if (j >= 1 && !wait(o_full, (uint32_t)(j - 1) & 1u)) break;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int d = half * 32 + 4 * i;
                st_v(d, vv[i].x);
                st_v(d + 1, vv[i].y);
                st_v(d + 2, vv[i].z);
                st_v(d + 3, vv[i].w);
            }
            fence_async_smem();
            mbar_arrive(smem_u32(v_full));
            if (j + 1 < n_kb) load4(vv, j + 1, 2);
        }
    } else if (warp == 8) {
        // ---------------------------------------------------------------- MMA
        if (lane == 0) {
            const uint32_t sb = smem_u32(smem);
            // S_j = Q . K_j^T into S[j % 2] over the 64 dims: two 32-dim regions x four 8-wide k-steps
            auto issue_s = [&](int j) -> bool {
                const int b = j & 1;
                if (!wait(&k_full[b], (uint32_t)(j >> 1) & 1u)) return false;
                asm volatile("tcgen05.fence::after_thread_sync;");
                const uint32_t kb = sb + kOffK + (uint32_t)b * kKBuf;
#pragma unroll
                for (int rg = 0; rg < 2; ++rg)
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) {
                        const uint64_t a_hi = sw128_desc(sb + kOffQhi + rg * kQRegion + ks * 32);
                        const uint64_t a_lo = sw128_desc(sb + kOffQlo + rg * kQRegion + ks * 32);
                        const uint64_t b_hi = sw128_desc(kb + rg * kKRegion + ks * 32);
                        const uint64_t b_lo = sw128_desc(kb + 2 * kKRegion + rg * kKRegion + ks * 32);
                        const uint32_t d = tmem + 64u * (uint32_t)b;
                        mma_tf32(d, a_lo, b_hi, kIdesc, (rg | ks) ? 1u : 0u);
                        mma_tf32(d, a_hi, b_lo, kIdesc, 1u);
                        mma_tf32(d, a_hi, b_hi, kIdesc, 1u);
                    }
                mma_commit(smem_u32(&s_full[b]));
                return true;
            };
            bool go = issue_s(0) && (n_kb < 2 || issue_s(1));
            for (int j = 0; go && j < n_kb; ++j) {
                if (!wait(p_full, (uint32_t)j & 1u) || !wait(v_full, (uint32_t)j & 1u)) break;
                asm volatile("tcgen05.fence::after_thread_sync;");
                // O += P_j . V_j over the 64 keys of the block
#pragma unroll
                for (int rg = 0; rg < 2; ++rg)
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) {
                        const uint64_t a_hi = sw128_desc(sb + kOffPhi + rg * kPRegion + ks * 32);
                        const uint64_t a_lo = sw128_desc(sb + kOffPlo + rg * kPRegion + ks * 32);
                        const uint64_t b_hi = sw128_desc(sb + kOffVhi + rg * kVRegion + ks * 32);
                        const uint64_t b_lo = sw128_desc(sb + kOffVlo + rg * kVRegion + ks * 32);
                        mma_tf32(tmem + 128, a_lo, b_hi, kIdesc, (j | rg | ks) ? 1u : 0u);
                        mma_tf32(tmem + 128, a_hi, b_lo, kIdesc, 1u);
                        mma_tf32(tmem + 128, a_hi, b_hi, kIdesc, 1u);
                    }
                mma_commit(smem_u32(o_full));
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
        const int r = warp * 32 + lane;   // TMEM lane = query row within the block
        const int row = q0 + r;
        const int last_key = min(row, T - 1);   // padded rows (row >= T) see every real key
        const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
        // tcgen05.ld / tcgen05.st are warp-collective (.sync.aligned): every
        // lane of the warp executes each of them, so every condition around
        // them is warp-uniform (waits are combined with __all_sync, the
        // rescale is skipped only when no lane needs it, and padded rows load
        // their TMEM row like the others and only skip the store)
        constexpr unsigned kAll = 0xffffffffu;
        constexpr float kLog2e = 1.4426950408889634f;
        const float scale2 = scale * kLog2e;   // q.k to the exp2 domain in one multiply
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < n_kb; ++j) {
            const int b = j & 1;
            ok = __all_sync(kAll, wait(&s_full[b], (uint32_t)(j >> 1) & 1u));
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;");
            const int key0 = j * BKY;
            float sv[BKY];
#pragma unroll
            for (int hc = 0; hc < 2; ++hc) {
                uint32_t v[32];
                tmem_ld32(lane_addr + 64u * (uint32_t)b + (uint32_t)(32 * hc), v);
#pragma unroll
                for (int c = 0; c < 32; ++c) sv[32 * hc + c] = __uint_as_float(v[c]);
            }
            float mt = -INFINITY;
#pragma unroll
            for (int c = 0; c < BKY; ++c)
                if (key0 + c <= last_key) mt = fmaxf(mt, sv[c] * scale);
            const float m_new = fmaxf(m, mt);
            const float alpha = (m == -INFINITY) ? 0.f : ex2_approx((m - m_new) * kLog2e);
            const float mb = m_new * kLog2e;   // the maximum in the exp2 domain
            float ps = 0.f;
#pragma unroll
            for (int c = 0; c < BKY; ++c) {
                sv[c] = key0 + c <= last_key ? ex2_approx(fmaf(sv[c], scale2, -mb)) : 0.f;
                ps += sv[c];
            }
            l = l * alpha + ps;
            m = m_new;
            if (j > 0) {
                // P . V of block j - 1 is done: its P may be overwritten, and the
                // running output in TMEM is rescaled to the new maximum before
                // this block's P . V accumulates onto it
                ok = __all_sync(kAll, wait(o_full, (uint32_t)(j - 1) & 1u));
                if (!ok) break;
                asm volatile("tcgen05.fence::after_thread_sync;");
                if (__any_sync(kAll, alpha != 1.f)) {
#pragma unroll
                    for (int hc = 0; hc < 2; ++hc) {
                        uint32_t v[32];
                        tmem_ld32(lane_addr + 128 + (uint32_t)(32 * hc), v);
#pragma unroll
                        for (int d = 0; d < 32; ++d) v[d] = __float_as_uint(__uint_as_float(v[d]) * alpha);
                        tmem_st32(lane_addr + 128 + (uint32_t)(32 * hc), v);
                    }
                }
            }
            // probabilities, four keys (one 16-byte chunk) at a time
#pragma unroll
            for (int c4 = 0; c4 < BKY / 4; ++c4) {
                const uint32_t off = (uint32_t)(c4 >> 3) * kPRegion + sw128_off4(r, (c4 & 7) * 4);
                st_split4(smem + kOffPhi, smem + kOffPlo, off,
                          make_float4(sv[4 * c4], sv[4 * c4 + 1], sv[4 * c4 + 2], sv[4 * c4 + 3]));
            }
            fence_async_smem();
            asm volatile("tcgen05.fence::before_thread_sync;");
            mbar_arrive(smem_u32(p_full));
        }
        if (ok) ok = __all_sync(kAll, wait(o_full, (uint32_t)(n_kb - 1) & 1u));
        asm volatile("tcgen05.fence::after_thread_sync;");
        if (ok) {
            const float inv = 1.0f / l;
            const size_t ob = ((size_t)seq * T + min(row, T - 1)) * E + h * D;
#pragma unroll
            for (int hc = 0; hc < 2; ++hc) {
                uint32_t o[32];
                tmem_ld32(lane_addr + 128 + (uint32_t)(32 * hc), o);
                if (row >= T) continue;   // padded row: loaded with the warp, not stored
#pragma unroll
                for (int q4 = 0; q4 < 8; ++q4) {
                    const int d4 = 8 * hc + q4;
                    const float4 v = make_float4(__uint_as_float(o[4 * q4]) * inv, __uint_as_float(o[4 * q4 + 1]) * inv,
                                                 __uint_as_float(o[4 * q4 + 2]) * inv,
                                                 __uint_as_float(o[4 * q4 + 3]) * inv);
                    if (out) reinterpret_cast<float4*>(out + ob)[d4] = v;
                    if (out_hi) {
                        const float4 hv = make_float4(tf32_hi(v.x), tf32_hi(v.y), tf32_hi(v.z), tf32_hi(v.w));
                        reinterpret_cast<float4*>(out_hi + ob)[d4] = hv;
                        reinterpret_cast<float4*>(out_lo + ob)[d4] =
                            make_float4(__fsub_rn(v.x, hv.x), __fsub_rn(v.y, hv.y), __fsub_rn(v.z, hv.z),
                                        __fsub_rn(v.w, hv.w));
                    }
                }
            }
        }
    }

    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == 8) {
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
