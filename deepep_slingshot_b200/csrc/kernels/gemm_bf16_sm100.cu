// Grouped bf16 GEMMs on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a: the backward
// ("dgrad" and "wgrad") GEMMs of the MoE expert FFN. Operands are K-major by default ("NT"):
//
//   mode 0, M-grouped: D[r, n] = sum_k A[r, k] * B[e*N + n, k] for rows r of expert e
//                      (A: [rows, K], rows of expert e at [offsets[e], offsets[e] + counts[e]),
//                       128-aligned; B: [E*N, K]; D: [rows, N])
//   mode 1, K-grouped: D[e, m, n] = sum_{k in [offsets[e], offsets[e+1])} A[m, k] * B[n, k]
//                      (A: [M, Ktot]; B: [N, Ktot]; D: [E, M, N]; an expert with no rows gets zeros)
//
// MN-major operands (the tensor as it lies in memory, no transpose copy): with `b_mn_major` B is
// [E*K, N] in mode 0 (the expert weights [E, K, N] of the forward) or [Ktot, N] in mode 1; with
// `a_mn_major` (mode 1) A is [Ktot, M]. An MN-major tile is loaded as two TMA boxes of 64 K rows x
// 64 MN elements (128-byte swizzle) 8 KiB apart and described to the MMA with the MN-major
// descriptor (LBO = 8 KiB between MN atoms, SBO = 1 KiB between 8-row K groups) and the
// instruction descriptor's transpose bit; each K = 16 instruction advances 2 KiB.
//
// Structure (same roles as the FP8 kernel, without the per-block scale promotion):
//  * one persistent CTA per SM walks output tiles of 128 x 128;
//  * warp 0, one thread: TMA 2D loads (128-byte swizzle, no multicast) of 64-wide K blocks of the A
//    and B tiles into an S-stage shared-memory ring;
//  * warp 1, one thread: four `tcgen05.mma.cta_group::1.kind::f16` (bf16 x bf16 -> fp32, M=128,
//    N=128, K=16) per K block, accumulating the whole K range of a tile in one TMEM buffer; two
//    buffers alternate between tiles so the epilogue of one tile overlaps the MMAs of the next;
//  * warps 2..9: `tcgen05.ld` the finished accumulator, release it, write the warp's 32 x 64 bf16
//    block into its shared-memory buffer in the 128-byte swizzle pattern and hand it to one TMA 2D
//    store (the tile leaves as bulk copies while the warp moves on; the buffer is rewritten only
//    after the store has read it).
// Every mbarrier wait is bounded (a status is reported, the kernel returns).
#include <cuda.h>
#include <cuda_bf16.h>

#include "../include/ep/device.cuh"
#include "gemm.h"
#include "tcgen05_common.cuh"

namespace ep {

namespace {

using tc::mma_commit;
using tc::smem_desc_sw128;
using tc::tma_load_2d;
using tc::tmem_ld_32;
using tc::tmem_wait_ld;
__device__ __forceinline__ void tc_fence_before() { tc::fence_before(); }
__device__ __forceinline__ void tc_fence_after() { tc::fence_after(); }

constexpr int kBM = 128, kBN = 128, kBK = 64;          // BK = 64 bf16 = one 128-byte swizzle row
constexpr int kStageBytes = (kBM + kBN) * kBK * 2;       // 32 KiB
constexpr int kMNAtomBytes = kBK * 128;                   // one MN-major box: 64 K rows x 128 bytes
constexpr int kEpiWarps = 8;
constexpr int kThreads = (2 + kEpiWarps) * 32;
constexpr int kEpiStageBytes = 32 * 128;                  // one epilogue warp's 32 rows x 64 bf16 store buffer
constexpr uint32_t kTmemCols = 2 * kBN;

// Instruction descriptor, kind::f16: BF16 x BF16 -> F32 (D format bit 4, A/B formats = 1 at bits
// 7 and 10), both K-major, M = 128, N = kBN.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int m, int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
struct Tile {
    int e, m0, n0;     // expert, first output row, first output column
    int k0, kblocks;   // first K element and number of 64-wide K blocks
    int64_t d_row0;    // first row of D (mode 1: e * M + m0)
    int b_row0;        // first row of the B tile in its tensor map (K-major B)
    int b_k_base;      // first K row of this expert in an MN-major B map (mode 0: e * K)
};

// Tile t of the launch (n innermost). Mode 0 uses the per-expert m-tile prefix in shared memory.
__device__ __forceinline__ bool tile_of(int t, const Bf16GemmArgs& a, const int* s_prefix, Tile& ti) {
    const int n_tiles = a.n / kBN;
    if (a.mode == 0) {
        const int total = s_prefix[a.num_experts] * n_tiles;
        if (t >= total) return false;
        const int mt = t / n_tiles, nt = t % n_tiles;
        int lo = 0, hi = a.num_experts - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (s_prefix[mid] <= mt) lo = mid;
            else hi = mid - 1;
        }
        ti.e = lo;
        ti.m0 = a.offsets[lo] + (mt - s_prefix[lo]) * kBM;
        ti.n0 = nt * kBN;
        ti.k0 = 0;
        ti.kblocks = a.k / kBK;
        ti.d_row0 = ti.m0;
        ti.b_row0 = lo * a.n + ti.n0;
        ti.b_k_base = lo * a.k;
        return true;
    }
    const int m_tiles = a.m / kBM;
    const int per_e = m_tiles * n_tiles;
    if (t >= a.num_experts * per_e) return false;
    ti.e = t / per_e;
    const int r = t % per_e;
    ti.m0 = (r / n_tiles) * kBM;
    ti.n0 = (r % n_tiles) * kBN;
    ti.k0 = a.offsets[ti.e];
    ti.kblocks = (a.offsets[ti.e + 1] - a.offsets[ti.e]) / kBK;
    ti.d_row0 = (int64_t)ti.e * a.m + ti.m0;
    ti.b_row0 = ti.n0;
    ti.b_k_base = 0;
    return true;
}

// Operand tile of one K block into shared memory: K-major, one box of 128 rows x 64 K; MN-major,
// two boxes of 64 K rows x 64 MN elements.
template <bool kMN>
__device__ __forceinline__ void load_operand(uint8_t* dst, const CUtensorMap* map, int k_row, int mn0, int kmajor_row0,
                                             int k_elem, uint64_t* bar) {
    if constexpr (kMN) {
        tma_load_2d(dst, map, mn0, k_row, bar);
        tma_load_2d(dst + kMNAtomBytes, map, mn0 + 64, k_row, bar);
    } else {
        tma_load_2d(dst, map, k_elem, kmajor_row0, bar);
    }
}

template <bool kMN>
__device__ __forceinline__ uint64_t operand_desc(uint32_t addr) {
    if constexpr (kMN) return tc::smem_desc_mn_sw128(addr, kMNAtomBytes);
    else return smem_desc_sw128(addr);
}

// Descriptor advance per K = 16 instruction, in 16-byte units: 32 bytes inside the K-major swizzle
// row, or two 8-row K groups (2 KiB) of an MN-major tile.
template <bool kMN>
constexpr uint64_t kStep = kMN ? (16 * 128) / 16 : 2;

}  // namespace

template <bool kAMN, bool kBMN>
__global__ void __launch_bounds__(kThreads, 1) grouped_gemm_bf16_kernel(const __grid_constant__ CUtensorMap map_a,
                                                                      const __grid_constant__ CUtensorMap map_b,
                                                                      const __grid_constant__ CUtensorMap map_d,
                                                                      Bf16GemmArgs a) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t s_full[kMaxGemmStages], s_empty[kMaxGemmStages];
    __shared__ __align__(8) uint64_t s_tfull[2], s_tempty[2];
    __shared__ uint32_t s_tmem_base;
    __shared__ int s_prefix[kMaxGemmExperts + 1];

    const int warp = warp_id(), lane = lane_id();
    const int S = a.stages;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&s_full[s], 1);
            mbar_init(&s_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&s_tfull[b], 1);
            mbar_init(&s_tempty[b], kEpiWarps);
        }
        fence_mbar_init();
        if (a.mode == 0) {
            int acc = 0;
            s_prefix[0] = 0;
            for (int e = 0; e < a.num_experts; ++e) {
                const int rows = a.expert_counts != nullptr ? a.expert_counts[e] : a.offsets[e + 1] - a.offsets[e];
                acc += (rows + kBM - 1) / kBM;
                s_prefix[e + 1] = acc;
            }
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
        // ---------------------------------------------------------------- TMA producer
        if (lane == 0) {
            uint32_t g = 0;
            bool ok = true;
            Tile ti;
            for (int t = blockIdx.x; ok && tile_of(t, a, s_prefix, ti); t += gridDim.x) {
                for (int kb = 0; kb < ti.kblocks && ok; ++kb, ++g) {
                    const int s = g % S;
                    ok = mbar_wait(&s_empty[s], ((g / S) & 1) ^ 1, a.st, kErrTimeoutTma);
                    if (!ok) break;
                    uint8_t* sa_tile = smem + (size_t)s * kStageBytes;
                    uint8_t* sb_tile = sa_tile + kBM * kBK * 2;
                    const int kx = ti.k0 + kb * kBK;
                    mbar_arrive_expect_tx(&s_full[s], kStageBytes);
                    load_operand<kAMN>(sa_tile, &map_a, kx, ti.m0, ti.m0, kx, &s_full[s]);
                    load_operand<kBMN>(sb_tile, &map_b, ti.b_k_base + kx, ti.n0, ti.b_row0, kx, &s_full[s]);
                }
            }
            // After an expired wait: the loads already issued land before the CTA exits.
            if (!ok) ring_drain(s_full, S, (int)g, a.st, kErrTimeoutTma);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16_f32(kBM, kBN) | (kAMN ? 1u << 15 : 0u) | (kBMN ? 1u << 16 : 0u);
            uint32_t g = 0, j = 0;  // g: K-block stages consumed, j: non-empty tiles (TMEM buffer index)
            bool ok = true;
            Tile ti;
            for (int t = blockIdx.x; ok && tile_of(t, a, s_prefix, ti); t += gridDim.x) {
                if (ti.kblocks == 0) continue;
                const int b = j & 1;
                ok = mbar_wait(&s_tempty[b], ((j >> 1) & 1) ^ 1, a.st, kErrTimeoutTma);
                if (!ok) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(b * kBN);
                for (int kb = 0; kb < ti.kblocks && ok; ++kb, ++g) {
                    const int s = g % S;
                    ok = mbar_wait(&s_full[s], (g / S) & 1, a.st, kErrTimeoutTma);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t sa_addr = smem_u32(smem + (size_t)s * kStageBytes);
                    const uint32_t sb_addr = sa_addr + kBM * kBK * 2;
                    const uint64_t da = operand_desc<kAMN>(sa_addr), db = operand_desc<kBMN>(sb_addr);
#pragma unroll
                    for (int k = 0; k < kBK / 16; ++k)  // K = 16 bf16 per instruction
                        mma_bf16(d_tmem, da + kStep<kAMN> * k, db + kStep<kBMN> * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
                    mma_commit(&s_empty[s]);
                }
                if (!ok) break;
                mma_commit(&s_tfull[b]);
                ++j;
            }
            // After an expired wait: issued MMAs complete before the TMEM is freed.
            if (!ok && g > 0) mbar_wait(&s_empty[(g - 1) % S], ((g - 1) / S) & 1, a.st, kErrTimeoutTma);
        }
    } else {
        // ---------------------------------------------------------------- epilogue
        const int ew = warp - 2;
        const int q = warp & 3;   // TMEM lane quarter of this warp
        const int h = ew >> 2;    // column half [64h, 64h + 64)
        const int row = 32 * q + lane;
        uint8_t* stg = smem + (size_t)a.stages * kStageBytes + (size_t)ew * kEpiStageBytes;  // this warp's store buffer
        uint32_t j = 0;
        Tile ti;
        for (int t = blockIdx.x; tile_of(t, a, s_prefix, ti); t += gridDim.x) {
            __nv_bfloat16* d = static_cast<__nv_bfloat16*>(a.d) + (ti.d_row0 + row) * (int64_t)a.n + ti.n0 + 64 * h;
            if (ti.kblocks == 0) {  // empty K range (mode 1): the result is zero
#pragma unroll
                for (int c = 0; c < 64; c += 8) *reinterpret_cast<int4*>(d + c) = make_int4(0, 0, 0, 0);
                continue;
            }
            const int b = j & 1;
            int good = 1;
            if (lane == 0) good = mbar_wait(&s_tfull[b], (j >> 1) & 1, a.st, kErrTimeoutTma) ? 1 : 0;
            if (!__shfl_sync(0xffffffffu, good, 0)) break;
            tc_fence_after();
            float v[64];
            const uint32_t taddr = tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(b * kBN + 64 * h);
            tmem_ld_32(taddr, v);
            tmem_ld_32(taddr + 32, v + 32);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_tempty[b]);
            ++j;
            // Each lane holds one row's 64 values. The warp's 32 x 64 block goes into its shared-memory
            // buffer in the 128-byte swizzle pattern (16-byte chunk c of row l at chunk c ^ (l & 7),
            // conflict-free), which the output tensor map also uses, and one TMA store writes it out.
            if (lane == 0) bulk_wait_read<0>();  // the previous tile's store has read the buffer
            __syncwarp();
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                int4 o;
                __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
                for (int i = 0; i < 4; ++i) o2[i] = __floats2bfloat162_rn(v[8 * c + 2 * i], v[8 * c + 2 * i + 1]);
                *reinterpret_cast<int4*>(stg + lane * 128 + ((c ^ (lane & 7)) << 4)) = o;
            }
            fence_proxy_async_smem();  // each lane's generic writes before the async-proxy read
            __syncwarp();
            if (lane == 0) {
                tc::tma_store_2d(&map_d, ti.n0 + 64 * h, (int)(ti.d_row0 + 32 * q), stg);
                bulk_commit();
            }
        }
    }
    if (warp >= 2 && lane_id() == 0) bulk_wait<0>();  // every TMA store of this warp has completed
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols) : "memory");
    }
}

// ------------------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------------------
namespace {

// 2D bf16 map over [rows][cols] (row-major), 128-byte swizzle. K-major operand tiles: box 64 x 128
// elements (K x rows); MN-major: box 64 x 64 (MN x K rows).
bool make_map_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, bool mn_major = false) {
    return tc::make_map_2d_box(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, rows, cols, (uint32_t)kBK,
                               mn_major ? (uint32_t)kBK : 128u);
}

template <bool kAMN, bool kBMN>
int launch_instance(const CUtensorMap& map_a, const CUtensorMap& map_b, const CUtensorMap& map_d, const Bf16GemmArgs& a,
                    int num_sms, cudaStream_t stream) {
    const size_t smem = (size_t)a.stages * kStageBytes + (size_t)kEpiWarps * kEpiStageBytes + 1024;
    cudaFuncSetAttribute(grouped_gemm_bf16_kernel<kAMN, kBMN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    grouped_gemm_bf16_kernel<kAMN, kBMN><<<num_sms, kThreads, smem, stream>>>(map_a, map_b, map_d, a);
    return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

}  // namespace

int launch_grouped_gemm_bf16(const Bf16GemmArgs& args_in, int num_sms, cudaStream_t stream) {
    Bf16GemmArgs a = args_in;
    if (a.n % kBN != 0 || a.num_experts <= 0 || a.num_experts > kMaxGemmExperts) return 1;
    const bool amn = a.a_mn_major != 0, bmn = a.b_mn_major != 0;
    CUtensorMap map_a, map_b;
    if (a.mode == 0) {
        if (a.k % kBK != 0 || a.rows <= 0 || amn) return 1;  // M-grouped rows are always K-major
        if (!make_map_bf16(&map_a, a.a, (uint64_t)a.rows, (uint64_t)a.k)) return 2;
        if (bmn) {
            if (!make_map_bf16(&map_b, a.b, (uint64_t)a.num_experts * a.k, (uint64_t)a.n, true)) return 2;
        } else if (!make_map_bf16(&map_b, a.b, (uint64_t)a.num_experts * a.n, (uint64_t)a.k)) {
            return 2;
        }
    } else {
        if (a.m % kBM != 0 || a.k % kBK != 0 || a.k <= 0) return 1;  // k = Ktot, offsets multiples of 64
        if (amn ? !make_map_bf16(&map_a, a.a, (uint64_t)a.k, (uint64_t)a.m, true)
                : !make_map_bf16(&map_a, a.a, (uint64_t)a.m, (uint64_t)a.k))
            return 2;
        if (bmn ? !make_map_bf16(&map_b, a.b, (uint64_t)a.k, (uint64_t)a.n, true)
                : !make_map_bf16(&map_b, a.b, (uint64_t)a.n, (uint64_t)a.k))
            return 2;
    }
    // Output map: D [rows, n] bf16 (mode 0) or [E * m, n] (mode 1), boxes of 32 rows x 64 columns
    // (128 bytes, the 128-byte swizzle of the epilogue buffers).
    CUtensorMap map_d;
    const uint64_t d_rows = a.mode == 0 ? (uint64_t)a.rows : (uint64_t)a.num_experts * a.m;
    if (!tc::make_map_2d_box(&map_d, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.d, d_rows, (uint64_t)a.n, 64, 32)) return 2;
    if (a.stages <= 0) a.stages = 5;  // 5 x 32 KiB ring + 32 KiB of epilogue store buffers
    if (a.stages > kMaxGemmStages) a.stages = kMaxGemmStages;
    if (a.stages > 5) a.stages = 5;
    if (amn) return bmn ? launch_instance<true, true>(map_a, map_b, map_d, a, num_sms, stream)
                        : launch_instance<true, false>(map_a, map_b, map_d, a, num_sms, stream);
    return bmn ? launch_instance<false, true>(map_a, map_b, map_d, a, num_sms, stream)
               : launch_instance<false, false>(map_a, map_b, map_d, a, num_sms, stream);
}

}  // namespace ep
