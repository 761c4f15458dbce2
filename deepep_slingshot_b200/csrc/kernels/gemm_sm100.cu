// Grouped block-scaled FP8 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
//   D[m, n] = sum_kb  sa[m, kb] * sb[e, n/128, kb] * sum_{k in block kb} A[m, k] * B_e[n, k]
//
// A: [rows, K] e4m3, rows grouped by expert e at [offsets[e], offsets[e+1]) (128-aligned blocks, the
//    layout `permute(..., alignment=128)` produces); sa: [rows, K/128] fp32 (1x128 activation scales).
// B: [E, N, K] e4m3 (K-major expert weights); sb: [E, N/128, K/128] fp32 (128x128 weight scales).
// D: [rows, N] bf16.
//
// The reference has no GEMM (its expert compute comes from DeepGEMM via SGLang,
// backend/tests/sglang_dispatcher_smoke.py:107-124); this kernel is new. Structure:
//  * one persistent CTA per SM walks tiles (expert, m-tile, n-tile) with n innermost, so a 128-row A
//    tile and an expert's weights stay in L2 while neighbouring CTAs use them;
//  * warp 0, one thread: TMA 2D loads (128B swizzle, no multicast) of the A and B tiles of every
//    128-wide K block into an S-stage shared-memory ring;
//  * warp 1, one thread: four `tcgen05.mma.cta_group::1.kind::f8f6f4` (M=128, N=128, K=32) per K
//    block into one of the TMEM accumulators (K blocks rotate over 512 / N of them: four at N = 128),
//    then `tcgen05.commit` frees the shared-memory stage and publishes the TMEM buffer;
//  * warps 2..17: read the K-block partial with `tcgen05.ld` (four warps per TMEM lane quarter, one
//    column quarter each), release the TMEM buffer, and accumulate sa*sb*partial in fp32 registers
//    (the per-block scale promotion that fp32 scales need); after the last K block they write bf16 rows.
// Tile width: 256 columns when N allows (default), else 128 (`DEEPEP_B200_GEMM_BN=128` forces it):
// a 256-wide tile stages 48 KiB of A and B per 8.4 MFLOP instead of 32 KiB per 4.2 MFLOP and halves
// the promotion round trips per FLOP (the promotion paces the MMA issuer); the two accumulators then
// fill all 512 TMEM columns and each epilogue thread promotes 64 columns, 8 per TMEM load with the
// next load in flight.
// Every mbarrier wait is bounded (a status is reported, the kernel returns).
#include <algorithm>
#include <cstdlib>
#include <string>

#include <cuda.h>
#include <cuda_bf16.h>

#include "../include/ep/device.cuh"
#include "../include/ep/gemm_combine.cuh"
#include "gemm.h"
#include "tcgen05_common.cuh"

namespace ep {

namespace {

using tc::mma_commit;
using tc::smem_desc_sw128;
using tc::tma_load_2d;
using tc::tmem_ld_16;
using tc::tmem_ld_32;
using tc::tmem_wait_ld;
__device__ __forceinline__ void tc_fence_before() { tc::fence_before(); }
__device__ __forceinline__ void tc_fence_after() { tc::fence_after(); }

constexpr int kBM = 128, kBK = 128;  // BK = 128 fp8 = one 128-byte swizzle row
// Sixteen epilogue warps: four per TMEM lane quarter, each promoting a quarter of the tile's columns,
// so one K block's promotion (TMEM load + scaled FMAs) takes half the time of eight warps and keeps
// up with the MMA issuer (measured: with eight, the tensor pipe idled on the promotion).
constexpr int kEpiWarps = 16;
constexpr int kThreads = (2 + kEpiWarps) * 32;
// Tile width kBN (128 or 256): a stage holds A (kBM x kBK) and B (kBN x kBK); TMEM holds two fp32
// accumulators of kBN columns. 256-wide tiles stage 48 KiB per 8.4 MFLOP instead of 32 KiB per 4.2.
template <int kBN>
constexpr int kStageBytesT = (kBM + kBN) * kBK;
// TMEM accumulators: as many kBN-column buffers as the 512 columns hold (4 at 128 wide, 2 at 256),
// so the MMA issuer runs up to kAcc - 1 K blocks ahead of the epilogue's scale promotion.
template <int kBN>
constexpr int kAccT = 512 / kBN;
template <int kBN>
constexpr uint32_t kTmemColsT = 512;

// Instruction descriptor, kind::f8f6f4: E4M3 x E4M3 -> F32, both K-major, M = 128, N = kBN.
__host__ __device__ constexpr uint32_t idesc_e4m3_f32(int m, int n) {
    return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_f8(uint32_t tmem_d, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Bounded wait; on expiry reports and returns false (the caller abandons the tile loop).
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, const KernelStatus& st) {
    return mbar_wait(bar, parity, st, kErrTimeoutTma);
}

struct TileInfo {
    int e, m0, n0;
};

// Map a linear tile index to (expert, m0, n0) using the per-expert m-tile prefix in shared memory.
template <int kBN>
__device__ __forceinline__ bool tile_of(int t, const int* s_mt_prefix, int E, int n_tiles, const int* offsets, TileInfo& ti) {
    const int total = s_mt_prefix[E] * n_tiles;
    if (t >= total) return false;
    const int mt = t / n_tiles, nt = t % n_tiles;
    int lo = 0, hi = E - 1;  // expert with s_mt_prefix[e] <= mt < s_mt_prefix[e+1]
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (s_mt_prefix[mid] <= mt) lo = mid;
        else hi = mid - 1;
    }
    ti.e = lo;
    ti.m0 = offsets[lo] + (mt - s_mt_prefix[lo]) * kBM;
    ti.n0 = nt * kBN;
    return true;
}

}  // namespace

// kSend: the combine send is the epilogue (GemmArgs::row_dest); the plain instance is unchanged.
template <int kBN, bool kSend>
__global__ void __launch_bounds__(kThreads, 1) grouped_gemm_fp8_kernel(const __grid_constant__ CUtensorMap map_a,
                                                                     const __grid_constant__ CUtensorMap map_b, GemmArgs a) {
    constexpr int kStageBytes = kStageBytesT<kBN>;
    constexpr uint32_t kTmemCols = kTmemColsT<kBN>;
    constexpr int kCols = kBN / 4;  // accumulator columns per epilogue thread (one row, one quarter)
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t s_full[kMaxGemmStages], s_empty[kMaxGemmStages];
    constexpr int kAcc = kAccT<kBN>;
    __shared__ __align__(8) uint64_t s_tfull[kAcc], s_tempty[kAcc];
    __shared__ uint32_t s_tmem_base;
    __shared__ int s_mt_prefix[kMaxGemmExperts + 1];
    __shared__ int s_send_ok;

    const int warp = warp_id(), lane = lane_id();
    const int S = a.stages;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const int KB = a.k / kBK;
    const int n_tiles = a.n / kBN;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&s_full[s], 1);
            mbar_init(&s_empty[s], 1);
        }
        for (int b = 0; b < kAcc; ++b) {
            mbar_init(&s_tfull[b], 1);
            mbar_init(&s_tempty[b], kEpiWarps);
        }
        fence_mbar_init();
        int acc = 0;
        s_mt_prefix[0] = 0;
        for (int e = 0; e < a.num_experts; ++e) {
            const int rows = a.expert_counts != nullptr ? a.expert_counts[e] : a.offsets[e + 1] - a.offsets[e];
            acc += (rows + kBM - 1) / kBM;
            s_mt_prefix[e + 1] = acc;
        }
        if constexpr (kSend) {
            // Every destination's slots must be free: it finished reducing the previous epoch (the
            // wait is normally satisfied at once; the GEMM's own work does not depend on it).
            s_send_ok = 1;
            const SymCtrl* mine = static_cast<const SymCtrl*>(a.gc_regions.base[a.gc_rank]);
            for (int r = 0; r < a.gc_num_ranks; ++r)
                if (!wait_ge(&mine->gc_free[r], a.gc_epoch - 1, a.st, kErrTimeoutCombineReady, r)) {
                    s_send_ok = 0;
                    break;
                }
        }
    }
    if (warp == 1) {  // TMEM allocation: one warp, power-of-two columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem_base)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = s_tmem_base;

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer
        if (lane == 0) {
            uint32_t g = 0;
            bool ok = true;
            TileInfo ti;
            for (int t = blockIdx.x; ok && tile_of<kBN>(t, s_mt_prefix, a.num_experts, n_tiles, a.offsets, ti); t += gridDim.x) {
                for (int kb = 0; kb < KB && ok; ++kb, ++g) {
                    const int s = g % S;
                    ok = wait_bar(&s_empty[s], ((g / S) & 1) ^ 1, a.st);
                    if (!ok) break;
                    uint8_t* sa_tile = smem + (size_t)s * kStageBytes;
                    uint8_t* sb_tile = sa_tile + kBM * kBK;
                    mbar_arrive_expect_tx(&s_full[s], kStageBytes);
                    tma_load_2d(sa_tile, &map_a, kb * kBK, ti.m0, &s_full[s]);
                    tma_load_2d(sb_tile, &map_b, kb * kBK, ti.e * a.n + ti.n0, &s_full[s]);
                }
            }
            // After an expired wait: the loads already issued land before the CTA exits.
            if (!ok) ring_drain(s_full, S, (int)g, a.st, kErrTimeoutTma);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_e4m3_f32(kBM, kBN);
            uint32_t g = 0;
            bool ok = true;
            TileInfo ti;
            for (int t = blockIdx.x; ok && tile_of<kBN>(t, s_mt_prefix, a.num_experts, n_tiles, a.offsets, ti); t += gridDim.x) {
                for (int kb = 0; kb < KB && ok; ++kb, ++g) {
                    const int s = g % S, b = g % kAcc;
                    ok = wait_bar(&s_tempty[b], ((g / kAcc) & 1) ^ 1, a.st) && wait_bar(&s_full[s], (g / S) & 1, a.st);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t sa_addr = smem_u32(smem + (size_t)s * kStageBytes);
                    const uint32_t sb_addr = sa_addr + kBM * kBK;
                    const uint64_t da = smem_desc_sw128(sa_addr), db = smem_desc_sw128(sb_addr);
                    const uint32_t d_tmem = tmem_base + (uint32_t)(b * kBN);
#pragma unroll
                    for (int k = 0; k < kBK / 32; ++k)  // K = 32 per instruction = 32 bytes: +2 in 16-byte units
                        mma_f8(d_tmem, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc, k > 0 ? 1u : 0u);
                    mma_commit(&s_empty[s]);
                    mma_commit(&s_tfull[b]);
                }
            }
            // After an expired wait: the MMAs already issued complete before the TMEM is freed (the
            // last commit tracks every earlier MMA of this thread).
            if (!ok && g > 0) wait_bar(&s_empty[(g - 1) % S], ((g - 1) / S) & 1, a.st);
        }
    } else {
        // ---------------------------------------------------------------- epilogue / scale promotion
        const int ew = warp - 2;
        const int q = warp & 3;      // TMEM lane quarter this warp may access
        const int h = ew >> 2;       // column quarter: [kCols * h, kCols * (h + 1))
        const int row = 32 * q + lane;
        uint32_t g = 0;
        bool ok = true;
        TileInfo ti;
        for (int t = blockIdx.x; ok && tile_of<kBN>(t, s_mt_prefix, a.num_experts, n_tiles, a.offsets, ti); t += gridDim.x) {
            float acc[kCols];
#pragma unroll
            for (int i = 0; i < kCols; ++i) acc[i] = 0.f;
            const int m = ti.m0 + row;
            const float* sa_row = a.sa + (int64_t)m * KB;
            const float* sb_blk = a.sb + ((int64_t)ti.e * (a.n / 128) + (ti.n0 + kCols * h) / 128) * KB;
            // Per K block: wait for its partial, promote it with the block's scale, release the buffer.
            // The scales of block kb + 1 are loaded before block kb's partial is waited for and read
            // (their latency would otherwise stall every K block of the promotion, which paces the MMA
            // issuer).
            float pa = sa_row[0], pb = sb_blk[0];
            for (int kb = 0; kb < KB; ++kb) {
                const int b = g % kAcc;
                const float scale = pa * pb;
                if (kb + 1 < KB) {
                    pa = sa_row[kb + 1];
                    pb = sb_blk[kb + 1];
                }
                int good = 1;
                if (lane == 0) good = wait_bar(&s_tfull[b], (g / kAcc) & 1, a.st) ? 1 : 0;
                if (!__shfl_sync(0xffffffffu, good, 0)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t taddr = tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(b * kBN + kCols * h);
                // TMEM -> registers 8 columns per load with the next load in flight (register budget at
                // 576 threads: the kCols accumulators + 16 staged values), then release the buffer.
                tc::tmem_promote<kCols>(taddr, scale, acc);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&s_tempty[b]);
                ++g;
            }
            if (!ok) break;
            __nv_bfloat16* d = nullptr;
            if (!kSend || a.d != nullptr) d = static_cast<__nv_bfloat16*>(a.d) + (int64_t)m * a.n + ti.n0 + kCols * h;
            __nv_bfloat16* peer = nullptr;  // the row's combine slot on its source rank (kSend)
            if constexpr (kSend) {
                const int dest = (s_send_ok && m < a.rows) ? a.row_dest[m] : -1;
                if (dest >= 0) {
                    const int r = gc_rank_of(dest), slot = gc_slot_of(dest);
                    if (r < a.gc_num_ranks && slot < a.gc_slots)
                        peer = reinterpret_cast<__nv_bfloat16*>(static_cast<uint8_t*>(a.gc_regions.base[r]) + kSymCtrlBytes) +
                               (int64_t)slot * a.n + ti.n0 + kCols * h;
                    else
                        report_error(a.st, kErrBounds, r, slot);
                }
            }
#pragma unroll
            for (int c = 0; c < kCols; c += 8) {
                int4 o;
                __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
                for (int i = 0; i < 4; ++i) o2[i] = __floats2bfloat162_rn(acc[c + 2 * i], acc[c + 2 * i + 1]);
                if constexpr (!kSend) {
                    *reinterpret_cast<int4*>(d + c) = o;
                } else {
                    if (d != nullptr) *reinterpret_cast<int4*>(d + c) = o;
                    if (peer != nullptr) *reinterpret_cast<int4*>(peer + c) = o;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols) : "memory");
    }
    if constexpr (kSend) {
        if (threadIdx.x == 0) {
            // Every thread's slot stores precede the barrier above; the system fence orders them
            // before the counter, and the last CTA publishes the epoch in every rank's gc_done. After
            // an error nothing is published: the reducers' bounded waits then report it too.
            SymCtrl* mine = static_cast<SymCtrl*>(a.gc_regions.base[a.gc_rank]);
            fence_sys();
            const int old = atom_add_acq_rel_gpu(&mine->gc_send_blocks, 1);
            if (old == (int)gridDim.x - 1) {
                mine->gc_send_blocks = 0;
                fence_sys();
                if (!aborted(a.st))
                    for (int r = 0; r < a.gc_num_ranks; ++r)
                        st_release_sys(&static_cast<SymCtrl*>(a.gc_regions.base[r])->gc_done[a.gc_rank], a.gc_epoch);
            }
        }
    }
}

// ------------------------------------------------------------------------------------------------
// CTA-pair variant (`cta_group::2`): a cluster of two CTAs computes a 256 x 256 tile with one MMA
// of M = 256, N = 256 per 32-deep K step. Each CTA stages its own 128 rows of A and its own 128 of
// the tile's 256 rows of B (32 KiB per K block instead of 48 KiB for a 128 x 256 tile on one CTA),
// and the tensor cores read both CTAs' halves of B: per FLOP, half the L2 -> shared-memory traffic
// of the 128 x 128 tile. Roles:
//  * warp 0 of each CTA, one thread: waits for its own stage to be free, TMA-loads its halves with
//    `cta_group::2` loads whose bytes complete on the leader CTA's full barrier (the leader expects
//    the bytes of both CTAs);
//  * warp 1 of the leader (cluster rank 0), one thread: four MMAs per K block into TMEM buffer
//    g % 2 of both CTAs (each CTA's TMEM holds its 128 rows x 256 columns), then one commit to each
//    CTA's empty barrier of the stage and one to each CTA's full barrier of the TMEM buffer;
//  * warps 2..17 of each CTA: the per-K-block scale promotion of its own rows (as in the one-CTA
//    kernel), then an arrive on the leader's TMEM-empty barrier (both CTAs' epilogues must drain a
//    buffer before the next MMA writes it).
// An expert's 128-row m-tiles are paired; the second CTA of an expert's last, odd pair computes
// rows it does not store. Every wait is bounded; both CTAs meet in a cluster barrier before the
// TMEM is freed and before either exits.
// ------------------------------------------------------------------------------------------------
namespace {

constexpr int kPBN = 256;                    // tile columns per pair
constexpr int kPStageBytes = (kBM + 128) * kBK;  // own A rows + own half of B (32 KiB)
// Epilogue warps per CTA: 16 (a quarter of the columns each; the 18 warps put five on two SM
// sub-partitions, a 96-register cap, so the promotion loads TMEM eight columns at a time and waits on
// each) or 8 (half of the columns each; ten warps, at most three per sub-partition, a 168-register
// cap that holds the pipelined promotion with the next load in flight).
template <int kEpi>
constexpr int kPColsT = kPBN / (kEpi / 4);  // accumulator columns per epilogue thread

struct PairTile {
    int e, m0, n0, valid;  // expert, this CTA's first row, the pair's first column, rows to store
};

// Map tile index t to (expert, this CTA's m0, n0); `s_mp_prefix[e]` counts m-tile pairs.
__device__ __forceinline__ bool pair_tile_of(int t, const int* s_mp_prefix, const int* s_mt, int E, int n_tiles,
                                             const int* offsets, uint32_t rank, PairTile& ti) {
    const int total = s_mp_prefix[E] * n_tiles;
    if (t >= total) return false;
    const int mp = t / n_tiles, nt = t % n_tiles;
    int lo = 0, hi = E - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (s_mp_prefix[mid] <= mp) lo = mid;
        else hi = mid - 1;
    }
    const int mt = 2 * (mp - s_mp_prefix[lo]) + (int)rank;
    ti.e = lo;
    ti.m0 = offsets[lo] + mt * kBM;
    ti.n0 = nt * kPBN;
    ti.valid = mt < s_mt[lo];
    return true;
}

__device__ __forceinline__ void mma_f8_pair(uint32_t tmem_d, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

}  // namespace

template <int kEpi>
__global__ void __launch_bounds__((2 + kEpi) * 32, 1) grouped_gemm_fp8_pair_kernel(const __grid_constant__ CUtensorMap map_a,
                                                                                const __grid_constant__ CUtensorMap map_b,
                                                                                GemmArgs a) {
    static_assert(kEpi == 8 || kEpi == 16, "8 or 16 epilogue warps");
    constexpr int kPCols = kPColsT<kEpi>;
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t s_full[kMaxGemmStages], s_empty[kMaxGemmStages];
    __shared__ __align__(8) uint64_t s_tfull[2], s_tempty[2];
    __shared__ uint32_t s_tmem_base;
    __shared__ int s_mp_prefix[kMaxGemmExperts + 1];
    __shared__ int s_mt[kMaxGemmExperts];

    const int warp = warp_id(), lane = lane_id();
    const int S = a.stages;
    const uint32_t rank = tc::cluster_ctarank();
    const int cluster = blockIdx.x >> 1, clusters = gridDim.x >> 1;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const int KB = a.k / kBK;
    const int n_tiles = a.n / kPBN;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&s_full[s], 1);   // leader: its own arrive.expect_tx (bytes of both CTAs)
            mbar_init(&s_empty[s], 1);  // one commit from the leader's MMA thread
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&s_tfull[b], 1);
            mbar_init(&s_tempty[b], 2 * kEpi);  // leader: the epilogue warps of both CTAs
        }
        fence_mbar_init();
        int acc = 0;
        s_mp_prefix[0] = 0;
        for (int e = 0; e < a.num_experts; ++e) {
            const int rows = a.expert_counts != nullptr ? a.expert_counts[e] : a.offsets[e + 1] - a.offsets[e];
            const int mt = (rows + kBM - 1) / kBM;
            s_mt[e] = mt;
            acc += (mt + 1) / 2;
            s_mp_prefix[e + 1] = acc;
        }
    }
    if (warp == 1) tc::tmem_alloc_pair(&s_tmem_base, 512);  // same warp in both CTAs
    tc_fence_before();
    __syncthreads();
    tc::cluster_sync();  // both CTAs' barriers exist before any cross-CTA arrive or load
    tc_fence_after();
    const uint32_t tmem_base = s_tmem_base;

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer (both CTAs)
        if (lane == 0) {
            uint32_t g = 0;
            bool ok = true;
            PairTile ti;
            for (int t = cluster; ok && pair_tile_of(t, s_mp_prefix, s_mt, a.num_experts, n_tiles, a.offsets, rank, ti);
                 t += clusters) {
                for (int kb = 0; kb < KB && ok; ++kb, ++g) {
                    const int s = g % S;
                    ok = wait_bar(&s_empty[s], ((g / S) & 1) ^ 1, a.st);
                    if (!ok) break;
                    uint8_t* sa_tile = smem + (size_t)s * kPStageBytes;
                    uint8_t* sb_tile = sa_tile + kBM * kBK;
                    if (rank == 0) mbar_arrive_expect_tx(&s_full[s], 2 * kPStageBytes);
                    const uint32_t full_leader = tc::mapa_shared(smem_u32(&s_full[s]), 0);
                    tc::tma_load_2d_pair(sa_tile, &map_a, kb * kBK, ti.m0, full_leader);
                    tc::tma_load_2d_pair(sb_tile, &map_b, kb * kBK, ti.e * a.n + ti.n0 + 128 * (int)rank, full_leader);
                }
            }
            // After an expired wait: the leader waits for the stages it expects before TMEM is freed.
            if (!ok && rank == 0) ring_drain(s_full, S, (int)g, a.st, kErrTimeoutTma);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer (leader only)
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = idesc_e4m3_f32(2 * kBM, kPBN);
            const uint32_t peer = 1;
            uint32_t g = 0;
            bool ok = true;
            PairTile ti;
            for (int t = cluster; ok && pair_tile_of(t, s_mp_prefix, s_mt, a.num_experts, n_tiles, a.offsets, 0, ti);
                 t += clusters) {
                for (int kb = 0; kb < KB && ok; ++kb, ++g) {
                    const int s = g % S, b = g & 1;
                    ok = wait_bar(&s_tempty[b], ((g >> 1) & 1) ^ 1, a.st) && wait_bar(&s_full[s], (g / S) & 1, a.st);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t sa_addr = smem_u32(smem + (size_t)s * kPStageBytes);
                    const uint32_t sb_addr = sa_addr + kBM * kBK;
                    const uint64_t da = smem_desc_sw128(sa_addr), db = smem_desc_sw128(sb_addr);
                    const uint32_t d_tmem = tmem_base + (uint32_t)(b * kPBN);
#pragma unroll
                    for (int k = 0; k < kBK / 32; ++k)
                        mma_f8_pair(d_tmem, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc, k > 0 ? 1u : 0u);
                    tc::mma_commit_pair(smem_u32(&s_empty[s]));
                    tc::mma_commit_pair(tc::mapa_shared(smem_u32(&s_empty[s]), peer));
                    tc::mma_commit_pair(smem_u32(&s_tfull[b]));
                    tc::mma_commit_pair(tc::mapa_shared(smem_u32(&s_tfull[b]), peer));
                }
            }
            if (!ok && g > 0) wait_bar(&s_empty[(g - 1) % S], ((g - 1) / S) & 1, a.st);
        }
    } else {
        // ---------------------------------------------------------------- epilogue / promotion (both CTAs)
        const int ew = warp - 2;
        const int q = warp & 3;
        const int h = ew >> 2;
        const int row = 32 * q + lane;
        uint32_t g = 0;
        bool ok = true;
        PairTile ti;
        for (int t = cluster; ok && pair_tile_of(t, s_mp_prefix, s_mt, a.num_experts, n_tiles, a.offsets, rank, ti);
             t += clusters) {
            float acc[kPCols];
#pragma unroll
            for (int i = 0; i < kPCols; ++i) acc[i] = 0.f;
            const int m = ti.m0 + row;
            // rows past this expert's tiles (the second half of an odd pair) compute but are not stored
            const float* sa_row = a.sa + (int64_t)min(m, a.rows - 1) * KB;
            const float* sb_blk = a.sb + ((int64_t)ti.e * (a.n / 128) + (ti.n0 + kPCols * h) / 128) * KB;
            float pa = sa_row[0], pb = sb_blk[0];
            for (int kb = 0; kb < KB; ++kb) {
                const int b = g & 1;
                const float scale = pa * pb;
                if (kb + 1 < KB) {
                    pa = sa_row[kb + 1];
                    pb = sb_blk[kb + 1];
                }
                int good = 1;
                if (lane == 0) good = wait_bar(&s_tfull[b], (g >> 1) & 1, a.st) ? 1 : 0;
                if (!__shfl_sync(0xffffffffu, good, 0)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t taddr = tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(b * kPBN + kPCols * h);
                if constexpr (kEpi == 16) {
#pragma unroll
                    for (int c = 0; c < kPCols; c += 8) {  // 8 staged values: the register budget of 18 warps
                        float v[8];
                        tc::tmem_ld_8(taddr + c, v);
                        tc::tmem_wait_ld_8(v);
#pragma unroll
                        for (int i = 0; i < 8; ++i) acc[c + i] = fmaf(scale, v[i], acc[c + i]);
                    }
                } else {
                    tc::tmem_promote<kPCols>(taddr, scale, acc);  // the next 8 columns in flight
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive_cluster(tc::mapa_shared(smem_u32(&s_tempty[b]), 0));
                ++g;
            }
            if (!ok) break;
            if (ti.valid && m < a.rows) {
                __nv_bfloat16* d = static_cast<__nv_bfloat16*>(a.d) + (int64_t)m * a.n + ti.n0 + kPCols * h;
#pragma unroll
                for (int c = 0; c < kPCols; c += 8) {
                    int4 o;
                    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
                    for (int i = 0; i < 4; ++i) o2[i] = __floats2bfloat162_rn(acc[c + 2 * i], acc[c + 2 * i + 1]);
                    *reinterpret_cast<int4*>(d + c) = o;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc::cluster_sync();  // no CTA frees TMEM or exits while the other may still signal it
    if (warp == 1) {
        tc_fence_after();
        tc::tmem_dealloc_pair(tmem_base, 512);
    }
}

// ------------------------------------------------------------------------------------------------
// Block-scaled variant (`kind::mxf8f6f4.block_scale`): with power-of-two scales (exact as UE8M0) the
// tensor core applies the 1x128 activation and 128x128 weight scales itself, per 32-deep K step, so
// the accumulator stays in TMEM over the whole K range and the epilogue runs once per tile instead of
// promoting every K block. Per stage, warp 0 writes the tile's scale factors next to the TMA tiles in
// the 128 x 4 UE8M0 atom the tensor core reads (byte (r % 32) * 16 + (r / 32) * 4 + j holds row r's
// scale for the j-th 32-deep K step; every step of a 128 block has the same scale here); the MMA
// thread copies them into TMEM (`tcgen05.cp ... 32x128b.warpx4`) and issues the four MMAs of the K
// block, each naming its K step through the scale-factor byte id. The scale-factor columns are one
// region, rewritten every K block: the copies and MMAs of the one issuing thread run in order.
// ------------------------------------------------------------------------------------------------
namespace {

constexpr int kBsBN = 128;
constexpr int kBsEpiWarps = 4;                       // one per TMEM lane quarter
constexpr int kBsThreads = (2 + kBsEpiWarps) * 32;   // warp 0: TMA + scale factors, warp 1: MMA
constexpr int kSfBytes = 512;                        // one 128-row x 4-step UE8M0 atom
constexpr int kBsStageBytes = (kBM + kBsBN) * kBK + 2 * kSfBytes;  // A, B, SFA, SFB (33 KiB, 1 KiB multiple)
constexpr uint32_t kBsSfaCol = 2 * kBsBN, kBsSfbCol = 2 * kBsBN + 4;  // after the two accumulators

// Instruction descriptor, kind::mxf8f6f4.block_scale: E4M3 x E4M3 (formats 0), both K-major, UE8M0
// scale factors (bit 23), N >> 3 at bit 17, M >> 4 at bit 24; the scale-factor byte ids of A (bits
// 29-30) and B (bits 4-5) are or-ed in per K step.
__host__ __device__ constexpr uint32_t idesc_mxf8_ue8m0(int m, int n) {
    return (1u << 23) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_mxf8_bs(uint32_t tmem_d, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t tmem_sfa, uint32_t tmem_sfb, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %6, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%4], [%5], p;\n\t}" ::"r"(tmem_d),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(tmem_sfa), "r"(tmem_sfb), "r"(accumulate)
        : "memory");
}

// Shared-memory -> TMEM copy of one 32-row x 16-byte block, replicated into the four lane quarters.
__device__ __forceinline__ void tmem_cp_32x128b_x4(uint32_t tmem_addr, uint64_t sdesc) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(tmem_addr), "l"(sdesc) : "memory");
}

// No-swizzle K-major descriptor of a 32 x 16-byte block: 8-row core matrices of 128 bytes, 128 bytes apart.
__device__ __forceinline__ uint64_t smem_desc_sf(uint32_t addr) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3fffu);   // start address
    d |= (uint64_t)(128 >> 4) << 16;          // leading byte offset (a single 16-byte column: unused)
    d |= (uint64_t)(128 >> 4) << 32;          // stride byte offset: next 8-row core matrix
    d |= (uint64_t)1 << 46;                   // descriptor version (sm_100)
    return d;                                 // layout type 0: no swizzle
}

// UE8M0 code of a positive power-of-two fp32 scale: its exponent field, repeated in four bytes.
__device__ __forceinline__ uint32_t ue8m0_x4(float scale) {
    return ((__float_as_uint(scale) >> 23) & 0xffu) * 0x01010101u;
}

}  // namespace

__global__ void __launch_bounds__(kBsThreads, 1) grouped_gemm_fp8_bs_kernel(const __grid_constant__ CUtensorMap map_a,
                                                                          const __grid_constant__ CUtensorMap map_b,
                                                                          GemmArgs a) {
    constexpr uint32_t kTmemCols = 512;
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t s_full[kMaxGemmStages], s_empty[kMaxGemmStages];
    __shared__ __align__(8) uint64_t s_tfull[2], s_tempty[2];
    __shared__ uint32_t s_tmem_base;
    __shared__ int s_mt_prefix[kMaxGemmExperts + 1];

    const int warp = warp_id(), lane = lane_id();
    const int S = a.stages;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const int KB = a.k / kBK;
    const int n_tiles = a.n / kBsBN;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&s_full[s], 1);
            mbar_init(&s_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&s_tfull[b], 1);
            mbar_init(&s_tempty[b], kBsEpiWarps);
        }
        fence_mbar_init();
        int acc = 0;
        s_mt_prefix[0] = 0;
        for (int e = 0; e < a.num_experts; ++e) {
            const int rows = a.expert_counts != nullptr ? a.expert_counts[e] : a.offsets[e + 1] - a.offsets[e];
            acc += (rows + kBM - 1) / kBM;
            s_mt_prefix[e + 1] = acc;
        }
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem_base)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = s_tmem_base;

    if (warp == 0) {
        // ---------------------------------------------------------------- scale factors + TMA producer
        // The scales of K block kb + 2 are loaded while block kb is written, so their global-load
        // latency overlaps two stages of the ring instead of stalling every TMA issue.
        uint32_t g = 0;
        int ok = 1;
        TileInfo ti;
        for (int t = blockIdx.x; ok && tile_of<kBsBN>(t, s_mt_prefix, a.num_experts, n_tiles, a.offsets, ti); t += gridDim.x) {
            const float* sb_blk = a.sb + ((int64_t)ti.e * (a.n / 128) + ti.n0 / 128) * KB;
            // lane l covers the rows l, l + 32, l + 64, l + 96 of the tile (row group l of the atom)
            auto fetch = [&](int kb, float (&va)[4], float& vb) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int m = ti.m0 + lane + 32 * j;
                    va[j] = m < a.rows ? a.sa[(int64_t)m * KB + kb] : 1.f;  // 2^0 past the rows
                }
                vb = sb_blk[kb];
            };
            auto step = [&](int kb, float (&va)[4], float& vb) {
                const int s = g % S;
                if (lane == 0) ok = wait_bar(&s_empty[s], ((g / S) & 1) ^ 1, a.st) ? 1 : 0;
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) return;
                uint8_t* st_a = smem + (size_t)s * kBsStageBytes;
                uint8_t* st_b = st_a + kBM * kBK;
                uint8_t* st_sfa = st_b + kBsBN * kBK;
                uint8_t* st_sfb = st_sfa + kSfBytes;
                // SFA: lane l writes the 16 bytes of row group l (rows l, l+32, l+64, l+96).
                *reinterpret_cast<uint4*>(st_sfa + lane * 16) = make_uint4(ue8m0_x4(va[0]), ue8m0_x4(va[1]), ue8m0_x4(va[2]), ue8m0_x4(va[3]));
                // SFB: the tile lies in one 128x128 weight block, so every byte is that block's scale.
                const uint32_t wb = ue8m0_x4(vb);
                *reinterpret_cast<uint4*>(st_sfb + lane * 16) = make_uint4(wb, wb, wb, wb);
                fence_proxy_async_smem();  // generic writes -> the tensor core's reads (async proxy)
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive_expect_tx(&s_full[s], (kBM + kBsBN) * kBK);
                    tma_load_2d(st_a, &map_a, kb * kBK, ti.m0, &s_full[s]);
                    tma_load_2d(st_b, &map_b, kb * kBK, ti.e * a.n + ti.n0, &s_full[s]);
                }
                ++g;
                if (kb + 2 < KB) fetch(kb + 2, va, vb);
            };
            float a0[4], a1[4], b0 = 1.f, b1 = 1.f;
            fetch(0, a0, b0);
            if (KB > 1) fetch(1, a1, b1);
            for (int kb = 0; kb < KB && ok; kb += 2) {
                step(kb, a0, b0);
                if (ok && kb + 1 < KB) step(kb + 1, a1, b1);
            }
        }
        // After an expired wait: the loads already issued land before the CTA exits.
        if (!ok && lane == 0) ring_drain(s_full, S, (int)g, a.st, kErrTimeoutTma);
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_mxf8_ue8m0(kBM, kBsBN);
            uint32_t g = 0, j = 0;
            bool ok = true;
            TileInfo ti;
            for (int t = blockIdx.x; ok && tile_of<kBsBN>(t, s_mt_prefix, a.num_experts, n_tiles, a.offsets, ti);
                 t += gridDim.x, ++j) {
                const int b = j & 1;
                ok = wait_bar(&s_tempty[b], ((j >> 1) & 1) ^ 1, a.st);
                if (!ok) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(b * kBsBN);
                for (int kb = 0; kb < KB && ok; ++kb, ++g) {
                    const int s = g % S;
                    ok = wait_bar(&s_full[s], (g / S) & 1, a.st);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t sa_addr = smem_u32(smem + (size_t)s * kBsStageBytes);
                    const uint32_t sb_addr = sa_addr + kBM * kBK;
                    const uint32_t sfa_addr = sb_addr + kBsBN * kBK;
                    tmem_cp_32x128b_x4(tmem_base + kBsSfaCol, smem_desc_sf(sfa_addr));
                    tmem_cp_32x128b_x4(tmem_base + kBsSfbCol, smem_desc_sf(sfa_addr + kSfBytes));
                    const uint64_t da = smem_desc_sw128(sa_addr), db = smem_desc_sw128(sb_addr);
#pragma unroll
                    for (int k = 0; k < kBK / 32; ++k)  // 32-deep steps; the scale-factor byte id is the step
                        mma_mxf8_bs(d_tmem, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k),
                                    idesc | ((uint32_t)k << 29) | ((uint32_t)k << 4),
                                    (tmem_base + kBsSfaCol) | ((uint32_t)k << 30),
                                    (tmem_base + kBsSfbCol) | ((uint32_t)k << 30), (kb > 0 || k > 0) ? 1u : 0u);
                    mma_commit(&s_empty[s]);
                }
                if (!ok) break;
                mma_commit(&s_tfull[b]);
            }
            // After an expired wait: the MMAs already issued complete before the TMEM is freed.
            if (!ok && g > 0) wait_bar(&s_empty[(g - 1) % S], ((g - 1) / S) & 1, a.st);
        }
    } else {
        // ---------------------------------------------------------------- epilogue (once per tile)
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        uint32_t j = 0;
        TileInfo ti;
        for (int t = blockIdx.x; tile_of<kBsBN>(t, s_mt_prefix, a.num_experts, n_tiles, a.offsets, ti); t += gridDim.x, ++j) {
            const int b = j & 1;
            int good = 1;
            if (lane == 0) good = wait_bar(&s_tfull[b], (j >> 1) & 1, a.st) ? 1 : 0;
            if (!__shfl_sync(0xffffffffu, good, 0)) break;
            tc_fence_after();
            const int m = ti.m0 + 32 * q + lane;
            __nv_bfloat16* d = static_cast<__nv_bfloat16*>(a.d) + (int64_t)m * a.n + ti.n0;
            const uint32_t taddr = tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(b * kBsBN);
#pragma unroll
            for (int c = 0; c < kBsBN; c += 32) {
                float v[32];
                tmem_ld_32(taddr + c, v);
                tmem_wait_ld();
                if (m < a.rows) {
#pragma unroll
                    for (int i = 0; i < 32; i += 8) {
                        int4 o;
                        __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
                        for (int u = 0; u < 4; ++u) o2[u] = __floats2bfloat162_rn(v[i + 2 * u], v[i + 2 * u + 1]);
                        *reinterpret_cast<int4*>(d + c + i) = o;
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_tempty[b]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols) : "memory");
    }
}

// ------------------------------------------------------------------------------------------------
// Host side: tensor maps through the driver entry point (no libcuda link), launch.
// ------------------------------------------------------------------------------------------------
namespace {

// 2D uint8 map over [rows][cols] (row-major), box 128 bytes x `box_rows` rows, 128-byte swizzle.
bool make_map_u8(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows = 128) {
    return tc::make_map_2d_box(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, base, rows, cols, 128, box_rows);
}

// Tile width: 256 when n allows (measured 187 vs 264 us on 4 x 1024 x 4096 x 7168: half the
// promotion round trips per FLOP); DEEPEP_B200_GEMM_BN=128 forces 128-wide tiles.
int tile_width(int n) {
    static const int requested = [] {
        const char* v = std::getenv("DEEPEP_B200_GEMM_BN");
        return v != nullptr ? std::atoi(v) : 256;
    }();
    return requested == 256 && n % 256 == 0 ? 256 : 128;
}

template <int kBN, bool kSend>
int launch_tiles(const GemmArgs& args_in, int num_sms, cudaStream_t stream) {
    constexpr int kStageBytes = kStageBytesT<kBN>;
    GemmArgs a = args_in;
    CUtensorMap map_a, map_b;
    if (!make_map_u8(&map_a, a.a, (uint64_t)a.rows, (uint64_t)a.k)) return 2;
    if (!make_map_u8(&map_b, a.b, (uint64_t)a.num_experts * a.n, (uint64_t)a.k, (uint32_t)kBN)) return 2;
    // Stages that fit the 227 KiB a CTA may use next to the static shared memory.
    const int max_stages = (int)((220 * 1024 - 1024) / kStageBytes);
    if (a.stages <= 0) a.stages = 6;
    if (a.stages > kMaxGemmStages) a.stages = kMaxGemmStages;
    if (a.stages > max_stages) a.stages = max_stages;
    const size_t smem = (size_t)a.stages * kStageBytes + 1024;
    cudaFuncSetAttribute(grouped_gemm_fp8_kernel<kBN, kSend>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    grouped_gemm_fp8_kernel<kBN, kSend><<<num_sms, kThreads, smem, stream>>>(map_a, map_b, a);
    return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

// CTA pairs: DEEPEP_B200_GEMM_PAIR=1 selects the cta_group::2 kernel (256 x 256 tiles) with 16
// epilogue warps, =2 the one with 8 epilogue warps and the pipelined promotion, when n allows.
int pair_epilogue_warps(int n) {
    static const int requested = [] {
        const char* v = std::getenv("DEEPEP_B200_GEMM_PAIR");
        if (v == nullptr) return 0;
        const std::string s(v);
        return s == "1" ? 16 : s == "2" ? 8 : 0;
    }();
    return n % kPBN == 0 ? requested : 0;
}

template <int kEpi>
int launch_pairs(const GemmArgs& args_in, int num_sms, cudaStream_t stream) {
    GemmArgs a = args_in;
    CUtensorMap map_a, map_b;
    if (!make_map_u8(&map_a, a.a, (uint64_t)a.rows, (uint64_t)a.k)) return 2;
    if (!make_map_u8(&map_b, a.b, (uint64_t)a.num_experts * a.n, (uint64_t)a.k, 128)) return 2;
    const int max_stages = (int)((218 * 1024 - 1024) / kPStageBytes);
    if (a.stages <= 0) a.stages = 6;
    if (a.stages > kMaxGemmStages) a.stages = kMaxGemmStages;
    if (a.stages > max_stages) a.stages = max_stages;
    const size_t smem = (size_t)a.stages * kPStageBytes + 1024;
    if (cudaFuncSetAttribute(grouped_gemm_fp8_pair_kernel<kEpi>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
        return 3;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)std::max(2, num_sms / 2 * 2));
    cfg.blockDim = dim3((2 + kEpi) * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, grouped_gemm_fp8_pair_kernel<kEpi>, map_a, map_b, a) == cudaSuccess ? 0 : 3;
}

}  // namespace

int launch_grouped_gemm_fp8(const GemmArgs& args_in, int num_sms, cudaStream_t stream) {
    if (args_in.k % kBK != 0 || args_in.n % 128 != 0 || args_in.num_experts > kMaxGemmExperts || args_in.rows <= 0) return 1;
    if (args_in.row_dest != nullptr) {
        // Combine send epilogue: the one-CTA fp32-scale kernel only.
        const GemmArgs& a = args_in;
        if (a.block_scaled || a.gc_num_ranks <= 0 || a.gc_num_ranks > kMaxRanks || a.gc_rank < 0 ||
            a.gc_rank >= a.gc_num_ranks || a.gc_slots <= 0 || a.gc_slots > kGcMaxSlots || a.gc_epoch <= 0)
            return 1;
        return tile_width(a.n) == 256 ? launch_tiles<256, true>(a, num_sms, stream) : launch_tiles<128, true>(a, num_sms, stream);
    }
    if (args_in.block_scaled) {
        GemmArgs a = args_in;
        CUtensorMap map_a, map_b;
        if (!make_map_u8(&map_a, a.a, (uint64_t)a.rows, (uint64_t)a.k)) return 2;
        if (!make_map_u8(&map_b, a.b, (uint64_t)a.num_experts * a.n, (uint64_t)a.k, (uint32_t)kBsBN)) return 2;
        const int max_stages = (int)((220 * 1024 - 1024) / kBsStageBytes);
        if (a.stages <= 0) a.stages = 6;
        if (a.stages > kMaxGemmStages) a.stages = kMaxGemmStages;
        if (a.stages > max_stages) a.stages = max_stages;
        const size_t smem = (size_t)a.stages * kBsStageBytes + 1024;
        cudaFuncSetAttribute(grouped_gemm_fp8_bs_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        grouped_gemm_fp8_bs_kernel<<<num_sms, kBsThreads, smem, stream>>>(map_a, map_b, a);
        return cudaGetLastError() == cudaSuccess ? 0 : 3;
    }
    const int pair_epi = pair_epilogue_warps(args_in.n);
    if (pair_epi == 16) return launch_pairs<16>(args_in, num_sms, stream);
    if (pair_epi == 8) return launch_pairs<8>(args_in, num_sms, stream);
    return tile_width(args_in.n) == 256 ? launch_tiles<256, false>(args_in, num_sms, stream)
                                        : launch_tiles<128, false>(args_in, num_sms, stream);
}

}  // namespace ep
