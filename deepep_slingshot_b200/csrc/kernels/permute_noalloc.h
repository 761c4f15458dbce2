// Allocation-free C entry point of the expert-grouping permute.
//
// This entry point has no counterpart in the reference: it is an addition of this library.
//
// Who needs it: callers that must not allocate device memory at the moment they permute tokens.
// Examples are serving runtimes that reserve all GPU memory up front and forbid cudaMalloc on the
// request path, plain C/C++ hosts that have no caching allocator to hand out temporary buffers, and
// code that cannot afford the implicit device synchronization that cudaMalloc / cudaFree may cause.
// The regular `permute` op takes its two temporary count arrays from the PyTorch allocator; this
// variant keeps them in a fixed array that is part of the loaded library instead.
//
// Contract:
//  * The caller passes every input and output (device pointers) and a stream; the function calls no
//    cudaMalloc, cudaFree or other allocating routine.
//  * Its scratch is a file-scope `static __device__` array of EP_PERMUTE_NOALLOC_SCRATCH_INTS int32
//    per count table (two tables, 512 KiB in total). Every GPU that loads the library holds this
//    memory until the process exits.
//  * Size limit: ceil(num_tokens / 32) * num_experts must not exceed EP_PERMUTE_NOALLOC_SCRATCH_INTS
//    (for example 8192 tokens with 256 experts); larger requests are rejected with
//    EP_PERMUTE_NOALLOC_ERR_TOO_LARGE and nothing is launched.
//  * The first call on a device looks the scratch array up with cudaGetSymbolAddress (once per
//    device, with that device current). Make that first call before any CUDA-graph stream capture.
//  * All calls share the one scratch array and it keeps the last call's contents; the function clears
//    the part that must start at zero on the stream before using it. Calls whose work overlaps on
//    the GPU (different streams without ordering between them) race on the scratch and give wrong
//    results: order them on one stream or with events.
//  * Outputs are exactly those of the allocating `permute`: expert_offsets [E+1], expert_counts [E],
//    row_map [N][K], x_perm [rows][H], scales_perm [rows][H/128] (when x_scales), probs_perm [rows]
//    (when probs). `rows` must hold expert_offsets[E] rows (worst case N*K + E*(alignment-1)).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#define EP_PERMUTE_NOALLOC_SCRATCH_INTS 65536

#define EP_PERMUTE_NOALLOC_OK 0
#define EP_PERMUTE_NOALLOC_ERR_BAD_ARGS 1
#define EP_PERMUTE_NOALLOC_ERR_TOO_LARGE 2
#define EP_PERMUTE_NOALLOC_ERR_SYMBOL 3
#define EP_PERMUTE_NOALLOC_ERR_LAUNCH 4
#define EP_PERMUTE_NOALLOC_ERR_PENDING 5

extern "C" {

int ep_permute_noalloc(const void* x, int x_elem_bytes, const float* x_scales, const float* probs, const int64_t* topk_idx,
                       int num_tokens, int hidden, int num_topk, int num_experts, int alignment, int* expert_offsets,
                       int* expert_counts, int* row_map, void* x_perm, float* scales_perm, float* probs_perm,
                       cudaStream_t stream);

// Human-readable text of a return code of ep_permute_noalloc (static storage, never freed).
const char* ep_permute_noalloc_strerror(int code);
}
