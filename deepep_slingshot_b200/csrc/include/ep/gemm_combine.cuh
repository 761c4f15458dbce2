// Index rules of the normal-mode down projection whose epilogue sends every expert row straight
// into its source rank's combine slot (gemm_sm100.cu `kSend` instance, gemm_combine.cu), shared by
// the kernels and the CPU host model of the protocol.
//
// Every rank owns a slot area of bf16 rows [max_tokens * num_topk][hidden] in its GEMM-combine
// region (after the region's control block): slot (t, k) holds the output row of expert
// topk_idx[t][k] for the rank's own token t, written by the rank that hosts that expert. A row of
// the expert-grouped GEMM operand carries one destination word,
//     (source rank << 24) | (t * num_topk + k),
// or -1 when it goes nowhere (alignment padding). The source rank then reduces its own slots with
// its own top-k weights: the selections with topk_idx[t][k] >= 0 are exactly the slots some rank
// wrote, since a receiver holds a row for (t, k) iff that expert is one of its local experts.
#pragma once

#include <cstdint>

#include <cuda_runtime.h>

namespace ep {

constexpr int kGcSlotBits = 24;
constexpr int kGcSlotMask = (1 << kGcSlotBits) - 1;
constexpr int64_t kGcMaxSlots = (int64_t)1 << kGcSlotBits;

__host__ __device__ __forceinline__ int gc_encode(int src_rank, int token, int k, int num_topk) {
    return (src_rank << kGcSlotBits) | (token * num_topk + k);
}
__host__ __device__ __forceinline__ int gc_rank_of(int dest) { return dest >> kGcSlotBits; }
__host__ __device__ __forceinline__ int gc_slot_of(int dest) { return dest & kGcSlotMask; }

// Source rank of received token j: prefix[0] = 0 and prefix[s + 1] = tokens received from ranks
// 0..s (received tokens are grouped by source rank, in rank order).
__host__ __device__ __forceinline__ int gc_source_of(const int* prefix, int num_ranks, int j) {
    int s = 0;
    while (s + 1 < num_ranks && prefix[s + 1] <= j) ++s;
    return s;
}

}  // namespace ep
