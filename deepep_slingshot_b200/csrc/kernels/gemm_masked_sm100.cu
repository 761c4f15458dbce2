// Masked grouped FP8 GEMM on tcgen05 / TMEM (sm_100a), optionally fused with the receive phase of
// the low-latency dispatch.
//
//   D[e, m, n] = sum_kb  sa(e, m, kb) * sb[e, n/128, kb] * sum_{k in block kb} A[e, m, k] * B[e, n, k]
//   for m < count[e]; rows at or beyond count[e] are not written.
//
// A: [E][slots][K] e4m3, the per-expert padded layout the low-latency dispatch receives into
//    (valid rows of expert e are [0, count[e])); sa: fp32 1x128 scales at sa[e*sa_e + kb*sa_k + m*sa_m]
//    (the dispatch writes them column-major per expert: sa_k = slots, sa_m = 1).
// B: [E][N][K] e4m3 K-major weights; sb: [E][N/128][K/128] fp32 128x128 scales. D: [E][slots][N] bf16.
//
// The reference hands the low-latency receive buffer to DeepGEMM's masked grouped GEMM through
// SGLang (backend/tests/sglang_dispatcher_smoke.py:107-124); this kernel is new. Structure:
//  * one persistent CTA per SM; tiles (m-tile, expert, n-tile) in that order, so the first pass of
//    the grid covers every expert's first m-tile (the only one a decode batch usually fills) and
//    the CTAs stay balanced; tiles with m0 >= count[e] are skipped by every role alike;
//  * warp 0 (one thread): TMA 2D tile loads (128-byte swizzle, no multicast) into an S-stage ring;
//  * warp 1 (one thread): tcgen05.mma.kind::f8f6f4 M128 N128 K32 x4 per K block into one of two
//    TMEM accumulators, tcgen05.commit frees the stage and publishes the accumulator;
//  * warps 2..9: tcgen05.ld each K-block partial, release the accumulator, promote with sa*sb in
//    fp32 registers, write the valid bf16 rows.
// Fused receive (`ll` set): the producer first prefetches into L2 the weights of the tiles its CTA
// will compute first (cp.async.bulk.prefetch.L2, local memory), then waits (bounded) for every
// rank's `dispatch_done` flag of this half, reads the per-expert slot counters as the counts and
// publishes them to the CTA through an mbarrier. The weights stream from HBM while the tokens are
// still crossing NVLink. The last CTA to read the counters does the receive bookkeeping of the
// low-latency dispatch hook: recv_count, cumulative statistics, and the reset of the flags and
// slot counters for the next use of the half. Fused combine send (`combine`): the epilogue stores
// each finished row straight into its source rank's combine slot over NVLink (the down projection's
// output never lands locally) and the last CTA releases the combine's flags; the receive hook of
// `low_latency_combine` then does the weighted reduction. All waits are bounded; an expired wait
// reports and the kernel returns.
#include <cuda.h>
#include <cuda_bf16.h>

#include "../include/ep/device.cuh"
#include "../include/ep/schedule.cuh"
#include "gemm.h"
#include "tcgen05_common.cuh"

namespace ep {

namespace {

constexpr int kBM = 128, kBN = 128, kBK = 128;
constexpr int kABytes = kBM * kBK, kBBytes = kBN * kBK;
constexpr int kStageBytes = kABytes + kBBytes;  // 32 KiB
constexpr int kEpiWarps = 8;
constexpr int kThreads = (2 + kEpiWarps) * 32;
constexpr uint32_t kTmemCols = 2 * kBN;
constexpr uint32_t kPrefetchChunk = 32 * 1024;

__host__ __device__ constexpr uint32_t idesc_e4m3_f32(int m, int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_f8(uint32_t tmem_d, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

struct MTile {
    int e, m0, n0;
};

// Tile t of the (m-tile, expert, n-tile) order (schedule.cuh); false past the last potential tile.
__device__ __forceinline__ bool masked_tile(int t, int E, int n_tiles, int m_tiles, MTile& ti) {
    int mt, nt;
    if (!masked_gemm_tile(t, E, n_tiles, m_tiles, mt, ti.e, nt)) return false;
    ti.m0 = mt * kBM;
    ti.n0 = nt * kBN;
    return true;
}

// Producer thread: counts of every expert into shared memory (after the fused receive wait).
// Returns false if a wait expired (the counts are then all zero).
__device__ bool load_counts(const MaskedGemmArgs& a, int* s_count) {
    const int E = a.num_experts;
    if (a.ll == nullptr) {
        for (int e = 0; e < E; ++e) s_count[e] = min(max(a.counts[e], 0), a.slots);
        return true;
    }
    const uint64_t t0 = trace_begin(a.st);
    bool ok = true;
    for (int r = 0; r < a.num_ranks && ok; ++r) ok = wait_ge(&a.ll->dispatch_done[r], 1, a.st, kErrTimeoutLLDispatch, r);
    for (int e = 0; e < E; ++e) s_count[e] = ok ? min(ld_volatile(&a.ll->slot_counter[e]), a.slots) : 0;
    // The rows were written by peers' bulk copies; order this thread's later TMA (async proxy) reads
    // after the acquire of their flags.
    fence_proxy_async_global();
    trace_end(a.st, kTraceLLDispatchRecvGemm, t0, ok ? 1 : 0);
    if (!ok) return false;
    // The last CTA that has read the counters does the receive bookkeeping and resets the half.
    const int old = atom_add_acq_rel_gpu(&a.ll->recv_finished_blocks, 1);
    if (old == (int)gridDim.x - 1) {
        a.ll->recv_finished_blocks = 0;
        for (int r = 0; r < a.num_ranks; ++r) a.ll->dispatch_done[r] = 0;
        for (int e = 0; e < E; ++e) {
            a.recv_count[e] = s_count[e];
            if (a.cumulative_stats != nullptr) a.cumulative_stats[e] += s_count[e];
            a.ll->slot_counter[e] = 0;
        }
        fence_gpu();
    }
    return true;
}

}  // namespace

__global__ void __launch_bounds__(kThreads, 1) masked_gemm_fp8_kernel(const __grid_constant__ CUtensorMap map_a,
                                                                    const __grid_constant__ CUtensorMap map_b, MaskedGemmArgs a) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t s_full[kMaxGemmStages], s_empty[kMaxGemmStages];
    __shared__ __align__(8) uint64_t s_tfull[2], s_tempty[2];
    __shared__ __align__(8) uint64_t s_ready;
    __shared__ uint32_t s_tmem_base;
    __shared__ int s_count[kMaxLocalExperts];

    const int warp = warp_id(), lane = lane_id();
    const int S = a.stages;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const int KB = a.k / kBK;
    const int n_tiles = a.n / kBN;
    const int m_tiles = (a.slots + kBM - 1) / kBM;
    const int E = a.num_experts;
    // The other roles wait for the counts as long as the producer may wait for the peers, and more.
    KernelStatus st_ready = a.st;
    st_ready.timeout_ns = 2 * a.st.timeout_ns + 1000000000ull;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&s_full[s], 1);
            mbar_init(&s_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&s_tfull[b], 1);
            mbar_init(&s_tempty[b], kEpiWarps);
        }
        mbar_init(&s_ready, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem_base)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem_base = s_tmem_base;

    if (warp == 0) {
        // ---------------------------------------------------------------- counts + TMA producer
        if (lane == 0) {
            if (a.ll != nullptr && a.l2_prefetch_bytes > 0) {
                // Weights of this CTA's first-pass tiles (m-tile 0) into L2 while the tokens arrive.
                int64_t budget = a.l2_prefetch_bytes;
                MTile ti;
                for (int t = blockIdx.x; budget > 0 && t < E * n_tiles && masked_tile(t, E, n_tiles, m_tiles, ti);
                     t += gridDim.x) {
                    const uint8_t* w = static_cast<const uint8_t*>(a.b) + ((int64_t)ti.e * a.n + ti.n0) * a.k;
                    const int64_t tile_bytes = (int64_t)kBN * a.k;
                    for (int64_t off = 0; off < tile_bytes && budget > 0; off += kPrefetchChunk) {
                        const uint32_t bytes = (uint32_t)min((int64_t)kPrefetchChunk, min(tile_bytes - off, budget)) & ~15u;
                        if (bytes == 0) break;
                        prefetch_l2(w + off, bytes);
                        budget -= bytes;
                    }
                }
            }
            const bool ok = load_counts(a, s_count);
            mbar_arrive(&s_ready);  // release: the counts are visible to every waiting role
            uint32_t g = 0;
            MTile ti;
            for (int t = blockIdx.x; ok && masked_tile(t, E, n_tiles, m_tiles, ti); t += gridDim.x) {
                if (ti.m0 >= s_count[ti.e]) continue;
                bool good = true;
                for (int kb = 0; kb < KB; ++kb, ++g) {
                    const int s = g % S;
                    good = mbar_wait(&s_empty[s], ((g / S) & 1) ^ 1, a.st, kErrTimeoutTma);
                    if (!good) break;
                    uint8_t* sa_tile = smem + (size_t)s * kStageBytes;
                    mbar_arrive_expect_tx(&s_full[s], kStageBytes);
                    tc::tma_load_2d(sa_tile, &map_a, kb * kBK, ti.e * a.slots + ti.m0, &s_full[s]);
                    tc::tma_load_2d(sa_tile + kABytes, &map_b, kb * kBK, ti.e * a.n + ti.n0, &s_full[s]);
                }
                if (!good) {
                    ring_drain(s_full, S, (int)g, a.st, kErrTimeoutTma);  // issued loads land before exit
                    break;
                }
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0 && mbar_wait(&s_ready, 0, st_ready, kErrTimeoutLLDispatch)) {
            constexpr uint32_t idesc = idesc_e4m3_f32(kBM, kBN);
            uint32_t g = 0;
            bool ok = true;
            MTile ti;
            for (int t = blockIdx.x; ok && masked_tile(t, E, n_tiles, m_tiles, ti); t += gridDim.x) {
                if (ti.m0 >= s_count[ti.e]) continue;
                for (int kb = 0; kb < KB && ok; ++kb, ++g) {
                    const int s = g % S, b = g & 1;
                    ok = mbar_wait(&s_tempty[b], ((g >> 1) & 1) ^ 1, a.st, kErrTimeoutTma) &&
                         mbar_wait(&s_full[s], (g / S) & 1, a.st, kErrTimeoutTma);
                    if (!ok) break;
                    tc::fence_after();
                    const uint32_t sa_addr = smem_u32(smem + (size_t)s * kStageBytes);
                    const uint64_t da = tc::smem_desc_sw128(sa_addr), db = tc::smem_desc_sw128(sa_addr + kABytes);
                    const uint32_t d_tmem = tmem_base + (uint32_t)(b * kBN);
#pragma unroll
                    for (int k = 0; k < kBK / 32; ++k)  // K = 32 fp8 = 32 bytes per instruction: +2 in 16-byte units
                        mma_f8(d_tmem, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc, k > 0 ? 1u : 0u);
                    tc::mma_commit(&s_empty[s]);
                    tc::mma_commit(&s_tfull[b]);
                }
            }
            // After an expired wait: issued MMAs complete before the TMEM is freed.
            if (!ok && g > 0) mbar_wait(&s_empty[(g - 1) % S], ((g - 1) / S) & 1, a.st, kErrTimeoutTma);
        }
    } else {
        // ---------------------------------------------------------------- epilogue / scale promotion
        const int ew = warp - 2;
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        const int h = ew >> 2;   // column half: [64h, 64h + 64)
        const int row = 32 * q + lane;
        int ready = 1;
        if (lane == 0) ready = mbar_wait(&s_ready, 0, st_ready, kErrTimeoutLLDispatch) ? 1 : 0;
        bool ok = __shfl_sync(0xffffffffu, ready, 0) != 0;
        uint32_t g = 0;
        MTile ti;
        for (int t = blockIdx.x; ok && masked_tile(t, E, n_tiles, m_tiles, ti); t += gridDim.x) {
            const int count = s_count[ti.e];
            if (ti.m0 >= count) continue;
            float acc[64];
#pragma unroll
            for (int i = 0; i < 64; ++i) acc[i] = 0.f;
            const int m = ti.m0 + row;
            const int m_clamped = min(m, a.slots - 1);
            const float* sa_row = a.sa + (int64_t)ti.e * a.sa_e + (int64_t)m_clamped * a.sa_m;
            const float* sb_blk = a.sb + ((int64_t)ti.e * (a.n / 128) + ti.n0 / 128) * KB;
            // the scales of K block kb + 1 load while block kb is waited for and promoted
            float pa = sa_row[0], pb = sb_blk[0];
            for (int kb = 0; kb < KB; ++kb, ++g) {
                const int b = g & 1;
                const float scale = pa * pb;
                if (kb + 1 < KB) {
                    pa = sa_row[(int64_t)(kb + 1) * a.sa_k];
                    pb = sb_blk[kb + 1];
                }
                int good = 1;
                if (lane == 0) good = mbar_wait(&s_tfull[b], (g >> 1) & 1, a.st, kErrTimeoutTma) ? 1 : 0;
                if (!__shfl_sync(0xffffffffu, good, 0)) {
                    ok = false;
                    break;
                }
                tc::fence_after();
                float v[64];
                const uint32_t taddr = tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(b * kBN + 64 * h);
                tc::tmem_ld_32(taddr, v);
                tc::tmem_ld_32(taddr + 32, v + 32);
                tc::tmem_wait_ld();
                tc::fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&s_tempty[b]);
#pragma unroll
                for (int i = 0; i < 64; ++i) acc[i] = fmaf(scale, v[i], acc[i]);
            }
            if (!ok) break;
            if (m < count) {
                __nv_bfloat16* d = nullptr;
                if (!a.combine) {
                    d = static_cast<__nv_bfloat16*>(a.d) + ((int64_t)ti.e * a.slots + m) * a.n + ti.n0 + 64 * h;
                } else {
                    // The row's combine slot on its source rank (peer store over NVLink).
                    const LLLayout& L = a.ll_layout;
                    const uint8_t* dsp = static_cast<const uint8_t*>(a.ll_peers.base[a.rank]) + (int64_t)a.dispatch_half * L.half_bytes;
                    const int64_t idx = (int64_t)ti.e * a.slots + m;
                    const int meta = reinterpret_cast<const int*>(dsp + L.recv_src_meta_off)[idx];
                    const int tok = reinterpret_cast<const int*>(dsp + L.recv_src_info_off)[idx];
                    const int src = meta / L.num_topk, k = meta % L.num_topk;
                    if (!in_window(src, 1, L.num_ranks) || !in_window(tok, 1, L.max_tokens)) {
                        report_error(a.st, kErrBounds, src, tok);
                        continue;
                    }
                    uint8_t* dst = static_cast<uint8_t*>(a.ll_peers.base[src]) + (int64_t)a.combine_half * L.half_bytes +
                                   L.combine_recv_off;
                    d = reinterpret_cast<__nv_bfloat16*>(dst) + ((int64_t)tok * L.num_topk + k) * L.hidden + ti.n0 + 64 * h;
                }
#pragma unroll
                for (int c = 0; c < 64; c += 8) {
                    int4 o;
                    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
                    for (int i = 0; i < 4; ++i) o2[i] = __floats2bfloat162_rn(acc[c + 2 * i], acc[c + 2 * i + 1]);
                    *reinterpret_cast<int4*>(d + c) = o;
                }
            }
        }
    }
    tc::fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols) : "memory");
    }
    if (a.combine && threadIdx.x == 0) {
        // Every thread's peer stores precede the barrier above; the system fence orders them before
        // the counter, and the last CTA releases this rank's flag in every rank's combine half.
        const LLLayout& L = a.ll_layout;
        uint8_t* mine = static_cast<uint8_t*>(a.ll_peers.base[a.rank]) + (int64_t)a.combine_half * L.half_bytes;
        LLCtrl* ctrl = reinterpret_cast<LLCtrl*>(mine + L.ctrl_off);
        fence_sys();
        const int old = atom_add_acq_rel_gpu(&ctrl->csend_finished_blocks, 1);
        if (old == (int)gridDim.x - 1) {
            ctrl->csend_finished_blocks = 0;
            fence_sys();
            for (int d = 0; d < L.num_ranks; ++d) {
                uint8_t* peer = static_cast<uint8_t*>(a.ll_peers.base[d]) + (int64_t)a.combine_half * L.half_bytes;
                st_release_sys(&reinterpret_cast<LLCtrl*>(peer + L.ctrl_off)->combine_done[a.rank], 1);
            }
        }
    }
}

int launch_masked_gemm_fp8(const MaskedGemmArgs& args_in, int num_sms, cudaStream_t stream) {
    MaskedGemmArgs a = args_in;
    if (a.k % kBK != 0 || a.n % kBN != 0 || a.num_experts <= 0 || a.num_experts > kMaxLocalExperts || a.slots <= 0 ||
        num_sms <= 0)
        return 1;
    if ((a.ll == nullptr) == (a.counts == nullptr)) return 1;  // exactly one source of counts
    if (a.combine && (a.n != a.ll_layout.hidden || a.ll_layout.num_ranks <= 0 || a.rank < 0 || a.rank >= a.ll_layout.num_ranks))
        return 1;
    if (a.ll != nullptr && (a.recv_count == nullptr || a.num_ranks <= 0 || a.num_ranks > kMaxRanks)) return 1;
    CUtensorMap map_a, map_b;
    if (!tc::make_map_2d(&map_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.a, (uint64_t)a.num_experts * a.slots, (uint64_t)a.k, 128))
        return 2;
    if (!tc::make_map_2d(&map_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.b, (uint64_t)a.num_experts * a.n, (uint64_t)a.k, 128))
        return 2;
    // 6 stages of 32 KiB + the static shared memory fit the 227 KiB a CTA may use.
    if (a.stages <= 0 || a.stages > 6) a.stages = 6;
    const size_t smem = (size_t)a.stages * kStageBytes + 1024;
    cudaFuncSetAttribute(masked_gemm_fp8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    masked_gemm_fp8_kernel<<<num_sms, kThreads, smem, stream>>>(map_a, map_b, a);
    return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

}  // namespace ep
