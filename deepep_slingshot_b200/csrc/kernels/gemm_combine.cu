// Normal-mode down projection -> combine: the steps around the grouped FP8 GEMM whose epilogue sends
// every expert row into its source rank's combine slot (gemm_sm100.cu, `kSend` instance).
//
// The reference's combine sends rows that a separate expert GEMM wrote to memory
// ([DE]csrc/kernels/legacy/intranode.cu:705, combine; the low-latency path's weighted receive is
// [DE]csrc/kernels/legacy/internode_ll.cu:715-1230). Here the GEMM's epilogue stores each finished
// bf16 row over NVLink straight into slot (t, k) of token t's source rank, so the transfer overlaps
// the remaining GEMM tiles, and the source rank sums its own slots with its own top-k weights:
//   1. `gc_row_dest_kernel` (receiver, before the GEMM): the destination word of every operand row
//      from the dispatch handle (source rank by the rank prefix, source token from recv_src_idx) and
//      the permute's (received token, k) -> row map;
//   2. the GEMM (receiver): rows to the slots; the last CTA publishes the epoch to every rank;
//   3. `gc_reduce_kernel` (source): waits for every rank's epoch (bounded), reduces
//      out[t] = bf16(sum_k w[t][k] * slot[t][k]) over k with topk_idx[t][k] >= 0 in fp32, then its
//      last block releases the slots to every rank (the next epoch's GEMM waits for that).
// Index rules: include/ep/gemm_combine.cuh. Every wait is bounded and reports into the region's
// error page.
#include <algorithm>

#include <cuda_bf16.h>

#include "../include/ep/device.cuh"
#include "../include/ep/gemm_combine.cuh"
#include "gemm.h"

namespace ep {

__global__ void __launch_bounds__(256) gc_row_dest_kernel(GcRowDestArgs a) {
    __shared__ int s_prefix[kMaxRanks + 1];
    if (threadIdx.x == 0) {
        s_prefix[0] = 0;
        for (int s = 0; s < a.num_ranks; ++s) s_prefix[s + 1] = a.rank_prefix_matrix[s * a.num_ranks + a.rank];
    }
    __syncthreads();
    const int64_t total = (int64_t)a.num_recv * a.num_topk;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int row = a.row_map[i];
        if (row < 0) continue;
        const int j = (int)(i / a.num_topk), k = (int)(i % a.num_topk);
        if (row >= a.rows) {
            report_error(a.st, kErrBounds, -1, row);
            continue;
        }
        const int s = gc_source_of(s_prefix, a.num_ranks, j);
        const int t = a.recv_src_idx[j];
        if (t < 0 || (int64_t)t * a.num_topk + k >= a.slots) {
            report_error(a.st, kErrBounds, s, t);
            continue;
        }
        a.row_dest[row] = gc_encode(s, t, k, a.num_topk);
    }
}

void launch_gc_row_dest(const GcRowDestArgs& a, cudaStream_t stream) {
    const int64_t total = (int64_t)a.num_recv * a.num_topk;
    if (total <= 0) return;
    const int blocks = (int)std::min<int64_t>((total + 255) / 256, 4096);
    gc_row_dest_kernel<<<blocks, 256, 0, stream>>>(a);
}

namespace {

__device__ __forceinline__ void bf16x8_fma(const int4& v, float w, float* acc) {
    const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(p[i]);
        acc[2 * i] = fmaf(w, f.x, acc[2 * i]);
        acc[2 * i + 1] = fmaf(w, f.y, acc[2 * i + 1]);
    }
}

constexpr int kReduceWarps = 8;
constexpr int kReduceBatch = 4;  // slot loads in flight per lane

}  // namespace

// One warp per token; each lane owns 16-byte column groups and sums the token's valid slots in
// batches of four independent loads (L1 bypassed: the slots were written by other GPUs).
__global__ void __launch_bounds__(kReduceWarps * 32) gc_reduce_kernel(GcReduceArgs a) {
    __shared__ int s_ok;
    SymCtrl* mine = static_cast<SymCtrl*>(a.regions.base[a.rank]);
    if (threadIdx.x == 0) s_ok = 1;
    __syncthreads();
    if ((int)threadIdx.x < a.num_ranks && !wait_ge(&mine->gc_done[threadIdx.x], a.epoch, a.st, kErrTimeoutCombineArrive, threadIdx.x))
        s_ok = 0;
    __syncthreads();
    if (s_ok) {
        const int lane = lane_id(), K = a.num_topk, units = a.hidden / 8;
        const __nv_bfloat16* slots =
            reinterpret_cast<const __nv_bfloat16*>(static_cast<const uint8_t*>(a.regions.base[a.rank]) + kSymCtrlBytes);
        for (int t = blockIdx.x * kReduceWarps + warp_id(); t < a.num_tokens; t += gridDim.x * kReduceWarps) {
            int64_t e = -1;
            float w = 0.f;
            if (lane < K) {
                e = a.topk_idx[(int64_t)t * K + lane];
                w = a.topk_weights != nullptr ? a.topk_weights[(int64_t)t * K + lane] : 1.f;
            }
            const uint32_t valid = __ballot_sync(0xffffffffu, lane < K && e >= 0);
            const int4* rows = reinterpret_cast<const int4*>(slots + (int64_t)t * K * a.hidden);
            int4* dst = reinterpret_cast<int4*>(static_cast<__nv_bfloat16*>(a.out) + (int64_t)t * a.hidden);
            for (int u = lane; u < units; u += 32) {
                float acc[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) acc[i] = 0.f;
                for (int k0 = 0; k0 < K; k0 += kReduceBatch) {
                    int4 v[kReduceBatch] = {};
                    float wk[kReduceBatch];
#pragma unroll
                    for (int b = 0; b < kReduceBatch; ++b) {
                        const int k = k0 + b;
                        wk[b] = __shfl_sync(0xffffffffu, w, k & 31);
                        if (k < K && ((valid >> k) & 1u)) v[b] = __ldcg(rows + (int64_t)k * units + u);
                    }
#pragma unroll
                    for (int b = 0; b < kReduceBatch; ++b) {
                        const int k = k0 + b;
                        if (k < K && ((valid >> k) & 1u)) bf16x8_fma(v[b], wk[b], acc);
                    }
                }
                int4 o;
                __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
                for (int i = 0; i < 4; ++i) o2[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
                dst[u] = o;
            }
        }
    }
    // Every block's slot reads are done (their values were consumed by the stores above) before the
    // last block releases the slots to every rank.
    __syncthreads();
    if (threadIdx.x == 0) {
        fence_sys();
        const int old = atom_add_acq_rel_gpu(&mine->gc_reduce_blocks, 1);
        if (old == (int)gridDim.x - 1) {
            mine->gc_reduce_blocks = 0;
            fence_sys();
            if (!aborted(a.st))
                for (int r = 0; r < a.num_ranks; ++r)
                    st_release_sys(&static_cast<SymCtrl*>(a.regions.base[r])->gc_free[a.rank], a.epoch);
        }
    }
}

void launch_gc_reduce(const GcReduceArgs& a, int num_sms, cudaStream_t stream) {
    // One launch even for zero tokens: its last block still releases the slots of this epoch.
    const int want = std::max(1, (a.num_tokens + kReduceWarps - 1) / kReduceWarps);
    const int blocks = std::max(1, std::min(want, std::max(1, num_sms) * 8));
    gc_reduce_kernel<<<blocks, kReduceWarps * 32, 0, stream>>>(a);
}

}  // namespace ep
