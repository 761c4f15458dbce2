// Launch API of the permute / unpermute kernels (see permute.cu).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace ep {

struct PermuteArgs {
    const void* x;               // [N][H] rows (bf16: 2-byte elements, FP8: 1-byte)
    int x_elem_bytes;
    const float* x_scales;       // [N][H/128] FP8 block scales or null
    const float* probs;          // [N][K] top-k weights or null
    const int64_t* topk_idx;     // [N][K] local expert ids, -1 = none
    int num_tokens, hidden, num_topk, num_experts, alignment;
    int* counts;                 // scratch [ceil(N/32)][E]
    int* bases;                  // scratch [ceil(N/32)][E]
    int* expert_offsets;         // [E+1] out: aligned exclusive prefix (offsets[E] = rows used)
    int* expert_counts;          // [E] out: unpadded counts (may be null)
    int* row_map;                // [N][K] out: grouped row of (t, k) or -1
    void* x_perm;                // [rows][H] out
    float* scales_perm;          // [rows][H/128] out (when x_scales)
    float* probs_perm;           // [rows] out (when probs)
    int zero_padding;            // zero the alignment padding rows of x_perm / scales_perm (grouped GEMMs over whole groups)
};

// Returns the first error of its own set-up calls (memset, function attribute), else
// cudaPeekAtLastError() after the launches (which does not clear it).
cudaError_t launch_permute(const PermuteArgs& a, cudaStream_t stream);
void launch_unpermute(const void* y, const int* row_map, const float* w, int N, int H, int K, void* out,
                      cudaStream_t stream);

}  // namespace ep
