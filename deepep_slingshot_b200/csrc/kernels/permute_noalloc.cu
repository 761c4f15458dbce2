// Allocation-free variant of the permute entry point. See permute_noalloc.h for who needs it and
// for the contract; this entry point has no counterpart in the reference.
#include <mutex>

#include "permute.h"
#include "permute_noalloc.h"

namespace {

// The scratch of every call: [0, N_INTS) per-(chunk, expert) counts, [N_INTS, 2*N_INTS) bases.
static __device__ __align__(256) int g_permute_noalloc_scratch[2 * EP_PERMUTE_NOALLOC_SCRATCH_INTS];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
int* g_scratch_ptr[kMaxDevices] = {};

// Once per device, with that device current: host code may not use the array's name as a device
// address, so look the address up and keep it.
int scratch_for_current_device(int** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return EP_PERMUTE_NOALLOC_ERR_SYMBOL;
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (g_scratch_ptr[dev] == nullptr) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_permute_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) return EP_PERMUTE_NOALLOC_ERR_SYMBOL;
        g_scratch_ptr[dev] = static_cast<int*>(p);
    }
    *out = g_scratch_ptr[dev];
    return EP_PERMUTE_NOALLOC_OK;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int ep_permute_noalloc(
    const void* x, int x_elem_bytes, const float* x_scales, const float* probs, const int64_t* topk_idx, int num_tokens,
    int hidden, int num_topk, int num_experts, int alignment, int* expert_offsets, int* expert_counts, int* row_map,
    void* x_perm, float* scales_perm, float* probs_perm, cudaStream_t stream) {
    if (x == nullptr || topk_idx == nullptr || expert_offsets == nullptr || row_map == nullptr || x_perm == nullptr ||
        num_tokens < 0 || hidden <= 0 || num_topk <= 0 || num_topk > 16 || num_experts <= 0 || alignment < 1 ||
        (x_elem_bytes != 1 && x_elem_bytes != 2) || ((int64_t)hidden * x_elem_bytes) % 16 != 0 ||
        (x_scales != nullptr && (hidden % 128 != 0 || scales_perm == nullptr)) || (probs != nullptr && probs_perm == nullptr))
        return EP_PERMUTE_NOALLOC_ERR_BAD_ARGS;
    const int64_t chunks = (num_tokens + 31) / 32;
    if (chunks * num_experts > EP_PERMUTE_NOALLOC_SCRATCH_INTS || num_experts > 4096) return EP_PERMUTE_NOALLOC_ERR_TOO_LARGE;
    // An error left pending by earlier work is reported as such, not taken for this call's launch
    // failure (and not cleared: it belongs to the caller).
    if (cudaPeekAtLastError() != cudaSuccess) return EP_PERMUTE_NOALLOC_ERR_PENDING;
    int* scratch = nullptr;
    const int rc = scratch_for_current_device(&scratch);
    if (rc != EP_PERMUTE_NOALLOC_OK) return rc;

    ep::PermuteArgs a{};
    a.x = x;
    a.x_elem_bytes = x_elem_bytes;
    a.x_scales = x_scales;
    a.probs = probs;
    a.topk_idx = topk_idx;
    a.num_tokens = num_tokens;
    a.hidden = hidden;
    a.num_topk = num_topk;
    a.num_experts = num_experts;
    a.alignment = alignment;
    a.counts = scratch;  // cleared on `stream` by launch_permute before use
    a.bases = scratch + EP_PERMUTE_NOALLOC_SCRATCH_INTS;
    a.expert_offsets = expert_offsets;
    a.expert_counts = expert_counts;
    a.row_map = row_map;
    a.x_perm = x_perm;
    a.scales_perm = scales_perm;
    a.probs_perm = probs_perm;
    // No error was pending at entry, so what is pending now comes from this call's own set-up or
    // launches; clear it and report it.
    const cudaError_t err = ep::launch_permute(a, stream);
    const cudaError_t last = cudaGetLastError();
    return (err == cudaSuccess && last == cudaSuccess) ? EP_PERMUTE_NOALLOC_OK : EP_PERMUTE_NOALLOC_ERR_LAUNCH;
}

extern "C" __attribute__((visibility("default"))) const char* ep_permute_noalloc_strerror(int code) {
    switch (code) {
        case EP_PERMUTE_NOALLOC_OK: return "ok";
        case EP_PERMUTE_NOALLOC_ERR_BAD_ARGS: return "bad arguments (null pointer, non-positive size, or misaligned row bytes)";
        case EP_PERMUTE_NOALLOC_ERR_TOO_LARGE:
            return "too large: ceil(num_tokens/32) * num_experts exceeds the fixed scratch of 65536 entries";
        case EP_PERMUTE_NOALLOC_ERR_SYMBOL: return "could not look up the device scratch array (cudaGetSymbolAddress failed)";
        case EP_PERMUTE_NOALLOC_ERR_LAUNCH: return "kernel launch or its set-up (memset, function attribute) failed";
        case EP_PERMUTE_NOALLOC_ERR_PENDING:
            return "a CUDA error from earlier work was already pending (left in place; nothing was launched)";
        default: return "unknown error";
    }
}
