// k_tc_gemm.cu -- fp32-accurate matmul on the 5th-generation tensor cores.
//
//   C[M,N] (epilogue) = A[M,K] . B[N,K]^T,  A and B K-major fp32
//
// Each operand arrives split in two tf32 halves, x = hi + lo with
// hi = round_to_tf32(x) and lo = x - hi (exact in fp32), and every k-step issues
// three tcgen05.mma (kind::tf32) into the same fp32 TMEM accumulator:
// lo(A).hi(B) + hi(A).lo(B) + hi(A).hi(B). The dropped lo.lo term and the tf32
// rounding of the lo halves leave a relative error near 2^-21 per product --
// fp32-level, where a plain tf32 product would be near 2^-11. (The split is the
// published "3xTF32" scheme.)
//
// Structure (one 128 x BN output tile at a time per CTA, 192 threads):
//   warp 0      TMA producer: 4 tiles per 16-wide k-block (A hi/lo, B hi/lo:
//               64-byte rows, 64-byte swizzled) into a shared-memory ring
//   warp 1      allocates the TMEM accumulator and issues the MMAs (one thread),
//               committing each stage back to the producer
//   warps 2..5  epilogue: tcgen05.ld the accumulator (each warp its 32 TMEM
//               lanes), apply bias / GELU / residual, store fp32 and/or the
//               hi/lo split the next matmul consumes
// tc_gemm_kernel (prefill) is persistent over the output tiles with a double-
// buffered accumulator. tc_gemm_split_kernel (decode shapes) splits K across
// the CTAs of a thread-block cluster and sums the splits through distributed
// shared memory in split order. The split count depends only on N and K,
// never on M, so a row's result does not depend on how many rows are in the
// batch.
//
// Every wait on an mbarrier is bounded; on expiry the kernel records an error
// flag, still drains its own TMA copies and MMAs, frees its TMEM and returns.
#include <cuda.h>

#include <algorithm>

#include "common.cuh"
#include "tc_gemm.h"

namespace tie {
namespace {

constexpr int BM = 128, BK = 16;
// k-block width of the persistent and head kernels: 128-byte rows, 128-byte
// swizzle (the split kernel keeps BK, 64-byte rows, to fit two CTAs an SM)
constexpr int BKD = 32;
constexpr int THREADS = 192;
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

#include "tc_ptx.cuh"

// kind::tf32 instruction descriptor: fp32 accumulate, tf32 A and B, both
// K-major, M = 128, N = BN.
template <int BN>
__device__ __forceinline__ uint32_t idesc_tf32() {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}


// One pipeline stage: A hi/lo (BM x BK) and B hi/lo (BN x BK), 64-byte rows.
template <int BN>
constexpr uint32_t stage_bytes() { return 2u * BM * 64 + 2u * BN * 64; }

template <int BN>
constexpr int stages() { return (int)((192u * 1024) / stage_bytes<BN>()); }

template <int BN>
constexpr size_t smem_bytes() {
    return 1024 /* alignment slack */ + (size_t)stages<BN>() * stage_bytes<BN>() + 256 /* barriers */;
}

// The persistent kernel's tile is MT x 128 rows by BN columns: A (hi and lo)
// MT x 128 rows, B BN rows per 32-wide k-block (128-byte rows).
template <int BN, int MT>
constexpr uint32_t stage_bytes_mt() { return 2u * MT * BM * 128 + 2u * BN * 128; }

template <int BN, int MT>
constexpr int stages_mt() { return (int)((192u * 1024) / stage_bytes_mt<BN, MT>()); }

template <int BN, int MT>
constexpr size_t smem_bytes_mt() {
    return 1024 /* alignment slack */ + (size_t)stages_mt<BN, MT>() * stage_bytes_mt<BN, MT>() + 256 /* barriers */;
}

// Persistent, warp-specialised: each block loops over output tiles
// (blockIdx.x, + gridDim.x, ...) of MT x 128 rows by BN columns; with MT = 2
// each B tile feeds two accumulators (the two 128-row halves), so B crosses
// from memory once per 256 rows. The TMEM accumulators are double-buffered,
// so the epilogue warps drain tile i while the MMA warp accumulates tile i + 1.
template <int BN, int MT, int EPI, int OUT>
__global__ void __launch_bounds__(THREADS, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap ta_hi, const __grid_constant__ CUtensorMap ta_lo,
               const __grid_constant__ CUtensorMap tb_hi, const __grid_constant__ CUtensorMap tb_lo,
               TcArgs p) {
    constexpr int S = stages_mt<BN, MT>();
    constexpr uint32_t kStage = stage_bytes_mt<BN, MT>();
    constexpr uint32_t kTileA = MT * BM * 128, kTileB = BN * 128;
    constexpr uint32_t kAcc = MT * BN;   // TMEM columns of one accumulator buffer
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * kStage);
    uint64_t* full = bars;              // [S]   TMA -> MMA
    uint64_t* empty = bars + S;         // [S]   MMA -> TMA
    uint64_t* tfull = bars + 2 * S;     // [2]   MMA -> epilogue
    uint64_t* tempty = bars + 2 * S + 2;  // [2] epilogue -> MMA
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 4);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_n = (p.N + BN - 1) / BN, tiles_m = (p.M + MT * BM - 1) / (MT * BM);
    const int tiles_mn = tiles_n * tiles_m;
    const int n_tiles = tiles_mn * p.splits;
    const int kb_total = p.K / BKD;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(&tfull[b]), 1);
            mbar_init(smem_u32(&tempty[b]), 4);  // one arrival per epilogue warp
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(tmem_slot)), "r"((uint32_t)(2 * kAcc)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = *tmem_slot;

    auto tile_k_range = [&](int z, int& kb0, int& nkb) {
        kb0 = z * p.kb_per_split;
        nkb = min(p.kb_per_split, kb_total - kb0);
    };
    auto wait = [&](uint32_t bar, uint32_t parity) -> bool {
        if (mbar_try_wait(bar, parity)) return true;
        const unsigned long long t0 = globaltimer_ns();
        for (uint32_t i = 1;; ++i) {
            if (mbar_try_wait(bar, parity)) return true;
            if ((i & 255u) == 0) {
                if (*abort_flag) return false;
                if (globaltimer_ns() - t0 > kWaitLimitNs) break;
            }
        }
        *abort_flag = 1;
        atomicExch(p.err, 1);
        return false;
    };

    if (warp == 0) {
        // ------------------------------------------------------- producer
        if (lane == 0) {
            uint32_t it = 0;  // k-blocks issued so far (ring position)
            bool ok = true;
            for (int t = blockIdx.x; ok && t < n_tiles; t += gridDim.x) {
                const int z = t / tiles_mn, r = t % tiles_mn;
                const int m0 = (r / tiles_n) * MT * BM, n0 = (r % tiles_n) * BN;
                int kb0, nkb;
                tile_k_range(z, kb0, nkb);
                for (int kb = 0; kb < nkb; ++kb, ++it) {
                    const int s = it % S;
                    if (!wait(smem_u32(&empty[s]), ((it / S) & 1u) ^ 1u)) { ok = false; break; }
                    const uint32_t base = smem_u32(smem + s * kStage);
                    const uint32_t fb = smem_u32(&full[s]);
                    mbar_expect_tx(fb, kStage);
                    const int kx = (kb0 + kb) * BKD;
                    tma_load_2d(base, &ta_hi, fb, kx, m0);
                    tma_load_2d(base + kTileA, &ta_lo, fb, kx, m0);
                    tma_load_2d(base + 2 * kTileA, &tb_hi, fb, kx, n0);
                    tma_load_2d(base + 2 * kTileA + kTileB, &tb_lo, fb, kx, n0);
                }
            }
            // drain: every copy this thread started has landed before exit
            for (uint32_t j = it > (uint32_t)S ? it - S : 0; j < it; ++j) {
                const unsigned long long t0 = globaltimer_ns();
                while (!mbar_try_wait(smem_u32(&full[j % S]), (j / S) & 1u))
                    if (globaltimer_ns() - t0 > kWaitLimitNs) { atomicExch(p.err, 1); break; }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA
        if (lane == 0) {
            const uint32_t idesc = idesc_tf32<BN>();
            uint32_t it = 0;
            int i = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < n_tiles; t += gridDim.x, ++i) {
                const int buf = i & 1;
                const uint32_t use = (uint32_t)(i >> 1);
                if (!wait(smem_u32(&tempty[buf]), (use & 1u) ^ 1u)) break;
                asm volatile("tcgen05.fence::after_thread_sync;");
                const uint32_t acc = tmem + (uint32_t)(buf * kAcc);
                int kb0, nkb;
                tile_k_range(t / tiles_mn, kb0, nkb);
                for (int kb = 0; kb < nkb; ++kb, ++it) {
                    const int s = it % S;
                    if (!wait(smem_u32(&full[s]), (it / S) & 1u)) { ok = false; break; }
                    asm volatile("tcgen05.fence::after_thread_sync;");
                    const uint32_t base = smem_u32(smem + s * kStage);
#pragma unroll
                    for (int j = 0; j < BKD / 8; ++j) {  // k-steps of 8 tf32 (32 bytes) within the 128-byte rows
                        const uint64_t b_hi = sw128_desc(base + 2 * kTileA + j * 32);
                        const uint64_t b_lo = sw128_desc(base + 2 * kTileA + kTileB + j * 32);
#pragma unroll
                        for (int mh = 0; mh < MT; ++mh) {   // 128-row halves: rows 128 mh.. of the A tiles
                            const uint64_t a_hi = sw128_desc(base + mh * BM * 128 + j * 32);
                            const uint64_t a_lo = sw128_desc(base + kTileA + mh * BM * 128 + j * 32);
                            const uint32_t d = acc + (uint32_t)(mh * BN);
                            mma_tf32(d, a_lo, b_hi, idesc, (kb > 0 || j > 0) ? 1u : 0u);
                            mma_tf32(d, a_hi, b_lo, idesc, 1u);
                            mma_tf32(d, a_hi, b_hi, idesc, 1u);
                        }
                    }
                    mma_commit(smem_u32(&empty[s]));
                }
                // arrives once this tile's MMAs have completed (also when cut short)
                mma_commit(smem_u32(&tfull[buf]));
            }
        }
    } else {
        // ------------------------------------------------------- epilogue
        const int q = warp & 3;  // this warp's TMEM lane quarter
        int i = 0;
        for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++i) {
            const int buf = i & 1;
            const uint32_t use = (uint32_t)(i >> 1);
            const int r = t % tiles_mn;
            const int n0 = (r % tiles_n) * BN;
            const bool ok = wait(smem_u32(&tfull[buf]), use & 1u);
            asm volatile("tcgen05.fence::after_thread_sync;");
#pragma unroll 1
            for (int cc = 0; cc < MT * (BN / 32); ++cc) {
                const int mh = cc / (BN / 32), c = cc % (BN / 32);
                const int row = (r / tiles_n) * MT * BM + mh * BM + q * 32 + lane;
                uint32_t v[32];
                tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * kAcc + mh * BN + c * 32), v);
                if (!ok || row >= p.M) continue;
                const int col0 = n0 + c * 32;
                const bool full_chunk = col0 + 32 <= p.N;
                {
                    const size_t o = (size_t)row * p.ldc + col0;
                    float y[32];
#pragma unroll
                    for (int k = 0; k < 32; ++k)
                        y[k] = (col0 + k < p.N) ? apply_epi<EPI>(__uint_as_float(v[k]), p.bias, col0 + k, p.C + o + k)
                                                : 0.f;
                    if (full_chunk && (p.ldc & 3) == 0) {
#pragma unroll
                        for (int i4 = 0; i4 < 8; ++i4) {
                            if constexpr (OUT == TC_OUT_F32 || OUT == TC_OUT_F32_HILO)
                                reinterpret_cast<float4*>(p.C + o)[i4] =
                                    make_float4(y[4 * i4], y[4 * i4 + 1], y[4 * i4 + 2], y[4 * i4 + 3]);
                            if constexpr (OUT == TC_OUT_HILO || OUT == TC_OUT_F32_HILO) {
                                float h[4], l[4];
#pragma unroll
                                for (int e = 0; e < 4; ++e) {
                                    h[e] = tf32_hi(y[4 * i4 + e]);
                                    l[e] = __fsub_rn(y[4 * i4 + e], h[e]);
                                }
                                reinterpret_cast<float4*>(p.C_hi + o)[i4] = make_float4(h[0], h[1], h[2], h[3]);
                                reinterpret_cast<float4*>(p.C_lo + o)[i4] = make_float4(l[0], l[1], l[2], l[3]);
                            }
                        }
                    } else {
                        for (int k = 0; k < 32; ++k) {
                            if (col0 + k >= p.N) break;
                            if constexpr (OUT == TC_OUT_F32 || OUT == TC_OUT_F32_HILO) p.C[o + k] = y[k];
                            if constexpr (OUT == TC_OUT_HILO || OUT == TC_OUT_F32_HILO) {
                                const float h = tf32_hi(y[k]);
                                p.C_hi[o + k] = h;
                                p.C_lo[o + k] = __fsub_rn(y[k], h);
                            }
                        }
                    }
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;");
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&tempty[buf]));
            if (!ok) break;
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)(2 * kAcc)));
    }
}

// ---------------------------------------------------------------------------
// Decode-sized matmuls: split-K across a thread-block cluster.
//
// Grid (splits, N tiles, M tiles), cluster (splits, 1, 1): the CTAs of a
// cluster compute the K splits of one 128 x 128 output tile. Each accumulates
// its split in TMEM (the same TMA ring and three MMAs per k-step as
// tc_gemm_kernel, three stages so that two CTAs fit on an SM), then stages the
// raw partial in its own shared memory over the drained ring. After a cluster
// barrier, CTA z sums rows [z R, (z + 1) R) of the tile, R = 128 / splits,
// reading every CTA's partial through distributed shared memory in split
// order (the order of tc_splitk_reduce, so the result does not depend on
// which kernel reduced it), applies the epilogue and stores. No partial goes
// through global memory and there is no second kernel.
//
// Launched with programmatic dependent launch: the weight (B) tiles of the
// first stages are requested before griddepcontrol.wait, the activation (A)
// tiles and every read of a previous kernel's output after it.
constexpr int kSplitStages = 3;
constexpr int kMaxSplits = 16;   // CTAs of a cluster (16 is a non-portable size)
constexpr int kRedLd = 128 + 4;   // staging row stride in floats: conflict-free float4 stores down a column
static_assert((size_t)kSplitStages * (2u * BM * 64 + 2u * 128 * 64) >= (size_t)BM * kRedLd * sizeof(float),
              "the partial overlays the drained ring");

constexpr size_t split_smem_bytes() {
    return 1024 + (size_t)kSplitStages * (2u * BM * 64 + 2u * 128 * 64) + 256;
}

__device__ __forceinline__ uint32_t mapa_cluster(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ float4 ld_cluster4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }

template <int EPI, int OUT>
__global__ void __launch_bounds__(THREADS, 2)
tc_gemm_split_kernel(const __grid_constant__ CUtensorMap ta_hi, const __grid_constant__ CUtensorMap ta_lo,
                     const __grid_constant__ CUtensorMap tb_hi, const __grid_constant__ CUtensorMap tb_lo,
                     TcArgs p) {
    constexpr int BN = 128, S = kSplitStages;
    constexpr uint32_t kStage = stage_bytes<BN>();
    constexpr uint32_t kTileA = BM * 64, kTileB = BN * 64;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * kStage);
    uint64_t* full = bars;          // [S]  TMA -> MMA
    uint64_t* empty = bars + S;     // [S]  MMA -> TMA
    uint64_t* tfull = bars + 2 * S; // [1]  MMA -> epilogue
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* red = reinterpret_cast<float*>(smem);   // [BM][kRedLd] once the ring has drained

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int z = blockIdx.x, splits = gridDim.x;
    const int n0 = blockIdx.y * BN, m0 = blockIdx.z * BM;
    const int kb0 = z * p.kb_per_split;
    const int nkb = min(p.kb_per_split, p.K / BK - kb0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        mbar_init(smem_u32(&tfull[0]), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(tmem_slot)), "r"((uint32_t)BN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = *tmem_slot;
    grid_dep_trigger();

    auto wait = [&](uint32_t bar, uint32_t parity) -> bool {
        if (mbar_try_wait(bar, parity)) return true;
        const unsigned long long t0 = globaltimer_ns();
        for (uint32_t i = 1;; ++i) {
            if (mbar_try_wait(bar, parity)) return true;
            if ((i & 255u) == 0) {
                if (*abort_flag) return false;
                if (globaltimer_ns() - t0 > kWaitLimitNs) break;
            }
        }
        *abort_flag = 1;
        atomicExch(p.err, 1);
        return false;
    };

    if (warp == 0) {
        // ------------------------------------------------------- producer
        if (lane == 0) {
            const int pre = min(S, nkb);
            // weights first: they do not depend on the previous kernel
            for (int kb = 0; kb < pre; ++kb) {
                const uint32_t base = smem_u32(smem + kb * kStage);
                const uint32_t fb = smem_u32(&full[kb]);
                mbar_expect_tx(fb, kStage);
                const int kx = (kb0 + kb) * BK;
                tma_load_2d(base + 2 * kTileA, &tb_hi, fb, kx, n0);
                tma_load_2d(base + 2 * kTileA + kTileB, &tb_lo, fb, kx, n0);
            }
            // the rest of this split's weight boxes go to L2 now: the ring's
            // later refills then wait on L2, not on a DRAM round trip each.
            // One row tile only (measured on B200: 32 rows QKV 12.8 -> 11.7 us,
            // MLP 13.7 -> 12.8; with two row tiles both CTAs of a weight tile
            // request it and the MLP slowed 17.3 -> 18.3 us)
            for (int kb = pre; gridDim.z == 1 && kb < nkb; ++kb) {
                tma_prefetch_2d(&tb_hi, (kb0 + kb) * BK, n0);
                tma_prefetch_2d(&tb_lo, (kb0 + kb) * BK, n0);
            }
            grid_dep_wait();
            for (int kb = 0; kb < pre; ++kb) {
                const uint32_t base = smem_u32(smem + kb * kStage);
                const uint32_t fb = smem_u32(&full[kb]);
                const int kx = (kb0 + kb) * BK;
                tma_load_2d(base, &ta_hi, fb, kx, m0);
                tma_load_2d(base + kTileA, &ta_lo, fb, kx, m0);
            }
            int kb = pre;
            for (; kb < nkb; ++kb) {
                const int s = kb % S;
                if (!wait(smem_u32(&empty[s]), ((kb / S) & 1u) ^ 1u)) break;
                const uint32_t base = smem_u32(smem + s * kStage);
                const uint32_t fb = smem_u32(&full[s]);
                mbar_expect_tx(fb, kStage);
                const int kx = (kb0 + kb) * BK;
                tma_load_2d(base, &ta_hi, fb, kx, m0);
                tma_load_2d(base + kTileA, &ta_lo, fb, kx, m0);
                tma_load_2d(base + 2 * kTileA, &tb_hi, fb, kx, n0);
                tma_load_2d(base + 2 * kTileA + kTileB, &tb_lo, fb, kx, n0);
            }
            // every copy this thread started has landed before the ring is reused
            for (int j = kb > S ? kb - S : 0; j < kb; ++j) {
                const unsigned long long t0 = globaltimer_ns();
                while (!mbar_try_wait(smem_u32(&full[j % S]), (j / S) & 1u))
                    if (globaltimer_ns() - t0 > kWaitLimitNs) { atomicExch(p.err, 1); break; }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA
        if (lane == 0) {
            const uint32_t idesc = idesc_tf32<BN>();
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb % S;
                if (!wait(smem_u32(&full[s]), (kb / S) & 1u)) break;
                asm volatile("tcgen05.fence::after_thread_sync;");
                const uint32_t base = smem_u32(smem + s * kStage);
#pragma unroll
                for (int j = 0; j < BK / 8; ++j) {
                    const uint64_t a_hi = sw64_desc(base + j * 32);
                    const uint64_t a_lo = sw64_desc(base + kTileA + j * 32);
                    const uint64_t b_hi = sw64_desc(base + 2 * kTileA + j * 32);
                    const uint64_t b_lo = sw64_desc(base + 2 * kTileA + kTileB + j * 32);
                    mma_tf32(tmem, a_lo, b_hi, idesc, (kb > 0 || j > 0) ? 1u : 0u);
                    mma_tf32(tmem, a_hi, b_lo, idesc, 1u);
                    mma_tf32(tmem, a_hi, b_hi, idesc, 1u);
                }
                mma_commit(smem_u32(&empty[s]));
            }
            // arrives once every MMA of the tile has completed (also when cut short)
            mma_commit(smem_u32(&tfull[0]));
        }
    } else {
        // ------------------------------------ epilogue: partial -> shared memory
        const int q = warp & 3;   // this warp's TMEM lane quarter
        wait(smem_u32(&tfull[0]), 0);
        asm volatile("tcgen05.fence::after_thread_sync;");
        float* dst = red + (size_t)(q * 32 + lane) * kRedLd;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
            uint32_t v[32];
            tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(c * 32), v);
#pragma unroll
            for (int i4 = 0; i4 < 8; ++i4)
                reinterpret_cast<float4*>(dst + c * 32)[i4] =
                    make_float4(__uint_as_float(v[4 * i4]), __uint_as_float(v[4 * i4 + 1]),
                                __uint_as_float(v[4 * i4 + 2]), __uint_as_float(v[4 * i4 + 3]));
        }
    }
    __syncwarp();
    // every partial of the cluster staged
    cluster_sync_all();
    grid_dep_wait();   // the residual input and the outputs belong to earlier kernels

    // ---------------------------- rows [z R, (z + 1) R): sum in split order
    const int R = BM / splits;
    for (int idx = threadIdx.x; idx < R * (BN / 4); idx += THREADS) {
        const int r = z * R + idx / (BN / 4), c4 = idx % (BN / 4);
        const int row = m0 + r, col = n0 + 4 * c4;
        if (row >= p.M || col >= p.N) continue;
        const uint32_t local = smem_u32(red + (size_t)r * kRedLd + 4 * c4);
        const size_t o = (size_t)row * p.ldc + col;
        // the epilogue's operands (bias, residual) and every split's value in
        // flight at once -- one round trip per item, not one per operand --
        // then the splits summed in split order
        float bv[4] = {0.f, 0.f, 0.f, 0.f}, rv[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int e = 0; e < 4; ++e)
            if (col + e < p.N) {
                if constexpr (EPI != EPI_STORE) bv[e] = __ldg(p.bias + col + e);
                if constexpr (EPI == EPI_BIAS_RESID) rv[e] = p.C[o + e];
            }
        float4 v[kMaxSplits];
#pragma unroll
        for (int s = 0; s < kMaxSplits; ++s)
            if (s < splits) v[s] = ld_cluster4(mapa_cluster(local, (uint32_t)s));
        float4 acc = v[0];
#pragma unroll
        for (int s = 1; s < kMaxSplits; ++s)
            if (s < splits) {
                acc.x = __fadd_rn(acc.x, v[s].x);
                acc.y = __fadd_rn(acc.y, v[s].y);
                acc.z = __fadd_rn(acc.z, v[s].z);
                acc.w = __fadd_rn(acc.w, v[s].w);
            }
        const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            if (col + e >= p.N) break;
            // apply_epi's arithmetic on the operands loaded above
            float y = a4[e];
            if constexpr (EPI == EPI_BIAS) y = __fadd_rn(y, bv[e]);
            else if constexpr (EPI == EPI_BIAS_GELU) y = gelu_new_ref(__fadd_rn(y, bv[e]));
            else if constexpr (EPI == EPI_BIAS_RESID) y = __fadd_rn(rv[e], __fadd_rn(y, bv[e]));
            if constexpr (OUT == TC_OUT_F32 || OUT == TC_OUT_F32_HILO) p.C[o + e] = y;
            if constexpr (OUT == TC_OUT_HILO || OUT == TC_OUT_F32_HILO) {
                const float h = tf32_hi(y);
                p.C_hi[o + e] = h;
                p.C_lo[o + e] = __fsub_rn(y, h);
            }
        }
    }
    // no CTA leaves while another may still read its shared memory
    cluster_sync_all();
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)BN));
    }
}

// ---------------------------------------------------------------------------
// The tied head of a decode step of 9-256 rows, with the WEIGHTS (the token
// embedding, [V, E]) as the 128-row MMA operand:
//
//   tile: D[128 vocabulary rows n0.., nb activation rows] = W[n0.., :] . X[.., :]^T
//
// One MMA per k-step covers every activation row of the step (N = nb, the rows
// rounded up to 16, at most 256; rows past the batch read zeros from TMA), so
// each weight element crosses from memory once per step whatever the batch.
// A CTA owns one tile over the whole of K (no split, so a row's logits do not
// depend on the batch it decodes in): the 3xTF32 MMAs of tc_gemm_kernel into
// TMEM, fed by TMA through a deep ring of 128-byte-swizzled k-blocks (32
// columns), the weight tiles of the first stages requested before
// griddepcontrol.wait. The weights arrive as fp32 (one k-block of 128 rows is
// 16 KB); the epilogue warps, idle until the accumulator is complete, split
// each landed weight tile in shared memory into its tf32 hi half (in place) and
// lo half (the tile's second slot) -- the split the MMAs need, bit for bit the
// one stored for the other matmuls -- so the weights cross from memory once,
// at half the bytes of streaming a stored split. Then the epilogue warps read
// the accumulator back and store it transposed: for each activation row, a
// warp writes 32 consecutive logits.
constexpr int kDecStagesMax = 8;
constexpr int kHeadPrefetch = 8;   // k-blocks of weights requested into L2 ahead of the ring
constexpr uint32_t kDecTileW = BM * 128;   // one k-block of 128 weight rows

__host__ __device__ constexpr uint32_t dec_stage_bytes(int nb) { return 2u * kDecTileW + 2u * (uint32_t)nb * 128u; }

__global__ void __launch_bounds__(THREADS, 1)
tc_head_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx_hi,
               const __grid_constant__ CUtensorMap tx_lo, TcArgs p, int nb, int S, int tcols) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t SB = dec_stage_bytes(nb);
    const uint32_t tileX = (uint32_t)nb * 128u;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (uint32_t)S * SB);
    uint64_t* full = bars;                       // [S]  TMA -> splitters
    uint64_t* empty = bars + kDecStagesMax;      // [S]  MMA -> TMA
    uint64_t* split = bars + 2 * kDecStagesMax;  // [S]  splitters -> MMA (128 arrivals)
    uint64_t* tfull = bars + 3 * kDecStagesMax;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * kDecStagesMax + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BM;
    const int nkb = p.K / BKD;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), 1);
            mbar_init(smem_u32(&split[s]), 128);
        }
        mbar_init(smem_u32(&tfull[0]), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(tmem_slot)), "r"((uint32_t)tcols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = *tmem_slot;
    grid_dep_trigger();

    auto wait = [&](uint32_t bar, uint32_t parity) -> bool {
        if (mbar_try_wait(bar, parity)) return true;
        const unsigned long long t0 = globaltimer_ns();
        for (uint32_t i = 1;; ++i) {
            if (mbar_try_wait(bar, parity)) return true;
            if ((i & 255u) == 0) {
                if (*abort_flag) return false;
                if (globaltimer_ns() - t0 > kWaitLimitNs) break;
            }
        }
        *abort_flag = 1;
        atomicExch(p.err, 1);
        return false;
    };

    if (warp == 0) {
        // ------------------------------------------------------- producer
        if (lane == 0) {
            const int pre = min(S, nkb);
            // weights first: no earlier kernel writes them
            const uint32_t tx_bytes = kDecTileW + 2u * tileX;   // fp32 weights, x hi and lo
            for (int kb = 0; kb < pre; ++kb) {
                const uint32_t base = smem_u32(smem + kb * SB);
                const uint32_t fb = smem_u32(&full[kb]);
                mbar_expect_tx(fb, tx_bytes);
                tma_load_2d(base, &tw, fb, kb * BKD, n0);
            }
            // weight boxes kHeadPrefetch k-blocks ahead of the ring go to L2
            // when the ring is two stages deep (129-256 rows; measured on
            // B200: 256 rows 162 -> 138 us; with the four-stage ring of 32 rows
            // the prefetches slowed it 74 -> 82 us, and a prefetch of the CTA's
            // whole contiguous weight slab slowed every size, 32 rows 74 -> 86)
            const int pf = S <= 2 ? kHeadPrefetch : 0;
            for (int kb = pre; kb < min(nkb, pre + pf); ++kb) tma_prefetch_2d(&tw, kb * BKD, n0);
            grid_dep_wait();
            for (int kb = 0; kb < pre; ++kb) {
                const uint32_t base = smem_u32(smem + kb * SB);
                const uint32_t fb = smem_u32(&full[kb]);
                tma_load_2d(base + 2 * kDecTileW, &tx_hi, fb, kb * BKD, 0);
                tma_load_2d(base + 2 * kDecTileW + tileX, &tx_lo, fb, kb * BKD, 0);
            }
            int kb = pre;
            for (; kb < nkb; ++kb) {
                const int s = kb % S;
                if (!wait(smem_u32(&empty[s]), ((kb / S) & 1u) ^ 1u)) break;
                const uint32_t base = smem_u32(smem + s * SB);
                const uint32_t fb = smem_u32(&full[s]);
                mbar_expect_tx(fb, tx_bytes);
                tma_load_2d(base, &tw, fb, kb * BKD, n0);
                tma_load_2d(base + 2 * kDecTileW, &tx_hi, fb, kb * BKD, 0);
                tma_load_2d(base + 2 * kDecTileW + tileX, &tx_lo, fb, kb * BKD, 0);
                if (pf && kb + pf < nkb) tma_prefetch_2d(&tw, (kb + pf) * BKD, n0);
            }
            // every copy this thread started has landed before the CTA may exit
            for (int j = kb > S ? kb - S : 0; j < kb; ++j) {
                const unsigned long long t0 = globaltimer_ns();
                while (!mbar_try_wait(smem_u32(&full[j % S]), (j / S) & 1u))
                    if (globaltimer_ns() - t0 > kWaitLimitNs) { atomicExch(p.err, 1); break; }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA
        if (lane == 0) {
            const uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(nb >> 3) << 17) |
                                   ((uint32_t)(BM >> 4) << 24);
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb % S;
                if (!wait(smem_u32(&split[s]), (kb / S) & 1u)) break;
                asm volatile("tcgen05.fence::after_thread_sync;");
                const uint32_t base = smem_u32(smem + s * SB);
#pragma unroll
                for (int j = 0; j < BKD / 8; ++j) {   // k-steps of 8 tf32 (32 bytes) within the 128-byte rows
                    const uint64_t w_hi = sw128_desc(base + j * 32);
                    const uint64_t w_lo = sw128_desc(base + kDecTileW + j * 32);
                    const uint64_t x_hi = sw128_desc(base + 2 * kDecTileW + j * 32);
                    const uint64_t x_lo = sw128_desc(base + 2 * kDecTileW + tileX + j * 32);
                    mma_tf32(tmem, w_lo, x_hi, idesc, (kb > 0 || j > 0) ? 1u : 0u);
                    mma_tf32(tmem, w_hi, x_lo, idesc, 1u);
                    mma_tf32(tmem, w_hi, x_hi, idesc, 1u);
                }
                mma_commit(smem_u32(&empty[s]));
            }
            // arrives once every MMA of the tile has completed (also when cut short)
            mma_commit(smem_u32(&tfull[0]));
        }
    } else {
        // ---------------------------- weight splitters, then the epilogue
        // Each landed weight tile (16 KB, 128-byte-swizzled) becomes its hi half
        // in place and its lo half in the tile's second slot; the swizzle is a
        // function of the position only, so the halves keep the tile's layout.
        const int t = threadIdx.x - 64;
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb) {
            const int s = kb % S;
            if (!wait(smem_u32(&full[s]), (kb / S) & 1u)) { ok = false; break; }
            float4* w = reinterpret_cast<float4*>(smem + s * SB);
#pragma unroll
            for (int i = 0; i < (int)(kDecTileW / 16) / 128; ++i) {
                const int e = t + 128 * i;
                const float4 v = w[e];
                const float4 h = make_float4(tf32_hi_int(v.x), tf32_hi_int(v.y), tf32_hi_int(v.z), tf32_hi_int(v.w));
                w[e] = h;
                w[e + kDecTileW / 16] = make_float4(__fsub_rn(v.x, h.x), __fsub_rn(v.y, h.y), __fsub_rn(v.z, h.z),
                                                    __fsub_rn(v.w, h.w));
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive(smem_u32(&split[s]));
        }
        const int q = warp & 3;                // TMEM lane quarter: vocabulary rows n0 + q * 32 + lane
        ok = wait(smem_u32(&tfull[0]), 0) && ok;
        asm volatile("tcgen05.fence::after_thread_sync;");
        const int col = n0 + q * 32 + lane;
        for (int c = 0; c < nb / 32 + (nb % 32 ? 1 : 0); ++c) {
            uint32_t v[32];
            tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(c * 32), v);
            if (!ok || col >= p.N) continue;
#pragma unroll
            for (int k = 0; k < 32; ++k) {
                const int row = c * 32 + k;
                if (row < p.M) p.C[(size_t)row * p.ldc + col] = __uint_as_float(v[k]);
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)tcols));
    }
}

__global__ void split_hilo_kernel(const float* __restrict__ x, float* __restrict__ hi,
                                  float* __restrict__ lo, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const float v = x[i];
        const float h = tf32_hi(v);
        hi[i] = h;
        lo[i] = __fsub_rn(v, h);
    }
}

using EncodeTiledFn = decltype(&cuTensorMapEncodeTiled);

// cuTensorMapEncodeTiled, reached through the runtime's driver entry point.
EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
    return fn;
}

// 2-D map over a rows x cols fp32 matrix (row stride ld floats), box box_cols x
// box_rows: 16 columns with the 64-byte swizzle (the layout sw64_desc
// describes) or 32 columns with the 128-byte swizzle (sw128_desc).
bool make_map(CUtensorMap* map, const float* base, int rows, int cols, int ld, int box_rows, int box_cols = BK) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * sizeof(float)};
    const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, box_cols == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int num_sms() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    }
    return n;
}

template <int BN, int MT, int EPI, int OUT>
cudaError_t launch_bn(const TcOperands& op, const TcArgs& a, int splits, cudaStream_t st) {
    CUtensorMap m[4];
    if (!make_map(&m[0], op.a_hi, a.M, a.K, op.lda, MT * BM, BKD) ||
        !make_map(&m[1], op.a_lo, a.M, a.K, op.lda, MT * BM, BKD) ||
        !make_map(&m[2], op.b_hi, a.N, a.K, op.ldb, BN, BKD) || !make_map(&m[3], op.b_lo, a.N, a.K, op.ldb, BN, BKD))
        return cudaErrorInvalidValue;
    constexpr size_t smem = smem_bytes_mt<BN, MT>();
    cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<BN, MT, EPI, OUT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const int tiles = ((a.N + BN - 1) / BN) * ((a.M + MT * BM - 1) / (MT * BM)) * splits;
    TcArgs b = a;
    b.splits = splits;
    tc_gemm_kernel<BN, MT, EPI, OUT><<<std::min(tiles, num_sms()), THREADS, smem, st>>>(m[0], m[1], m[2], m[3], b);
    return cudaGetLastError();
}

// Decode shapes: one cluster of `splits` CTAs per 128 x 128 tile (splits <= 16),
// programmatic dependent launch.
template <int EPI, int OUT>
cudaError_t launch_split(const TcOperands& op, TcArgs a, int splits, cudaStream_t st) {
    CUtensorMap m[4];
    if (!make_map(&m[0], op.a_hi, a.M, a.K, op.lda, BM) || !make_map(&m[1], op.a_lo, a.M, a.K, op.lda, BM) ||
        !make_map(&m[2], op.b_hi, a.N, a.K, op.ldb, 128) || !make_map(&m[3], op.b_lo, a.N, a.K, op.ldb, 128))
        return cudaErrorInvalidValue;
    constexpr size_t smem = split_smem_bytes();
    cudaError_t e = cudaFuncSetAttribute(tc_gemm_split_kernel<EPI, OUT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    if (splits > 8) {
        e = cudaFuncSetAttribute(tc_gemm_split_kernel<EPI, OUT>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
    }
    a.kb_per_split = (a.K / BK + splits - 1) / splits;
    const int used = (a.K / BK + a.kb_per_split - 1) / a.kb_per_split;
    a.splits = used;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(used, (a.N + 127) / 128, (a.M + BM - 1) / BM);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = used;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 2;
    e = cudaLaunchKernelEx(&cfg, tc_gemm_split_kernel<EPI, OUT>, m[0], m[1], m[2], m[3], a);
    return e != cudaSuccess ? e : cudaGetLastError();
}

template <int EPI, int OUT>
cudaError_t launch_epi(const TcOperands& op, TcArgs a, int splits, cudaStream_t st) {
    if (splits <= 1) {
        a.kb_per_split = a.K / BKD;
        // 129-256 rows (decode batches, the tied head): 256-row tiles, so each
        // B tile crosses from memory once (measured on B200: head over 256
        // rows 250 -> 216-235 us; a prefill FC of 8192 rows slows 300 -> 315
        // us with them, so larger matmuls keep 128-row tiles)
        if (a.M > BM && a.M <= 2 * BM) return launch_bn<128, 2, EPI, OUT>(op, a, 1, st);
        return launch_bn<128, 1, EPI, OUT>(op, a, 1, st);
    }
    return launch_split<EPI, OUT>(op, a, splits, st);
}

// The tied head of a decode step (tc_head_kernel): op.a_* are the activations
// (a.M rows), op.b_* the weights (a.N rows).
cudaError_t launch_head(const TcOperands& op, TcArgs a, cudaStream_t st) {
    const int nb = (a.M + 15) / 16 * 16;
    if (nb < 16 || nb > 256) return cudaErrorInvalidValue;
    CUtensorMap m[3];
    if (!op.b_f32 || !make_map(&m[0], op.b_f32, a.N, a.K, op.ldb, BM, BKD) ||
        !make_map(&m[1], op.a_hi, a.M, a.K, op.lda, nb, BKD) || !make_map(&m[2], op.a_lo, a.M, a.K, op.lda, nb, BKD))
        return cudaErrorInvalidValue;
    // one CTA per SM: a deep ring keeps several stages' copies in flight
    const uint32_t sb = dec_stage_bytes(nb);
    const int S = std::max(2, std::min(kDecStagesMax, (int)((196u * 1024) / sb)));
    const size_t smem = 1024 + (size_t)S * sb + 256;
    int tcols = 32;
    while (tcols < nb) tcols <<= 1;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(tc_head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    cudaError_t e = launch_pdl(tc_head_kernel, dim3((a.N + BM - 1) / BM), dim3(THREADS), smem, st, m[0], m[1], m[2],
                               a, nb, S, tcols);
    return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace

cudaError_t launch_tc_head(const TcOperands& op, const TcArgs& a, cudaStream_t st) {
    if (!tc_gemm_supported(a.M, a.N, a.K, op.lda, op.ldb) || a.M > 256 || a.K % BKD) return cudaErrorInvalidValue;
    return launch_head(op, a, st);
}

bool tc_gemm_supported(int M, int N, int K, int lda, int ldb) {
    return M > 0 && N > 0 && K > 0 && K % BKD == 0 && lda % 4 == 0 && ldb % 4 == 0 && encode_fn() != nullptr;
}

// Split count for a decode-sized matmul, chosen from N and K only, so that a
// row's result never depends on how many rows are in the batch: the largest
// power of two up to a portable cluster (8; 16 below) with N tiles x splits <= 96 --
// two 128-row tiles (the largest decode batch) then make at most 192 CTAs,
// which one wave holds at two CTAs per SM (71 clusters of 4 or 33 of 8 are
// resident at this kernel's shared memory) -- and at least four 16-wide
// k-blocks per split.
int tc_splits_for(int N, int K) {
    const int n_tiles = (N + 127) / 128;
    const int kb = K / BK;
    int s = 1;
    while (s < 8 && n_tiles * s * 2 <= 96 && s * 2 <= kb / 4) s *= 2;
    // narrow matrices with long rows (N <= 768, K >= 3072: the MLP
    // down-projection) take a 16-CTA cluster (non-portable; 14 are resident,
    // two 128-row tiles of N <= 768 need at most 12)
    if (s == 8 && n_tiles * 2 <= 12 && 16 <= kb / 8) s = 16;
    return s;
}

cudaError_t launch_tc_gemm(const TcOperands& op, const TcArgs& a, int epi, int out, int splits,
                           cudaStream_t st) {
    if (!tc_gemm_supported(a.M, a.N, a.K, op.lda, op.ldb)) return cudaErrorInvalidValue;
#define TC_CASE(E, O) \
    if (epi == E && out == O) return launch_epi<E, O>(op, a, splits, st);
    TC_CASE(EPI_STORE, TC_OUT_F32)
    TC_CASE(EPI_BIAS, TC_OUT_F32)
    TC_CASE(EPI_BIAS_RESID, TC_OUT_F32)
    TC_CASE(EPI_BIAS_GELU, TC_OUT_HILO)
    TC_CASE(EPI_BIAS_GELU, TC_OUT_F32_HILO)
    TC_CASE(EPI_BIAS_GELU, TC_OUT_F32)
#undef TC_CASE
    return cudaErrorInvalidValue;
}

cudaError_t launch_split_hilo(const float* x, float* hi, float* lo, long long n, cudaStream_t st) {
    const int grid = (int)std::min<long long>((n + 255) / 256, 148 * 32);
    split_hilo_kernel<<<grid > 0 ? grid : 1, 256, 0, st>>>(x, hi, lo, n);
    return cudaGetLastError();
}

}  // namespace tie
