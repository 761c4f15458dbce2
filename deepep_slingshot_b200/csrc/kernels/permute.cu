// Permute / unpermute between the dispatch receive layout ([tokens][hidden], top-k local expert ids
// per token) and the expert-grouped layout consumed by the grouped GEMMs ([rows][hidden], rows of
// expert e at [offset[e], offset[e] + count[e]), every count padded to `alignment`).
//
// The reference has no permute (SGLang/DeepGEMM do it downstream of DeepEP,
// backend/tests/sglang_dispatcher_smoke.py:107-124); the v2 `do_expand` layout
// ([DE]deep_ep/buffers/elastic.py:830-855) is the closest. Here it is three sm_100a kernels with a
// deterministic row order (chunk of 32 tokens, then top-k slot, then lane):
//   count   : one warp per 32-token chunk adds its per-expert counts into scratch[chunk][expert];
//   scan    : one CTA turns the counts into per-(chunk, expert) bases and aligned expert offsets;
//   scatter : one warp per chunk ranks equal experts with __match_any_sync, writes row_map and
//             copies rows (and FP8 scales / top-k probabilities) into the grouped layout.
// Scratch: 2 * num_chunks * num_experts int32 (counts, bases), zeroed by the count launch.
#include <cuda_bf16.h>

#include "../include/ep/device.cuh"
#include "permute.h"

namespace ep {

namespace {

__device__ __forceinline__ uint32_t lanemask_lt() {
    uint32_t m;
    asm volatile("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

}  // namespace

__global__ void __launch_bounds__(256) permute_count_kernel(const int64_t* __restrict__ topk_idx, int N, int K, int E,
                                                            int* __restrict__ counts) {
    const int lane = lane_id();
    const int chunk = blockIdx.x * (blockDim.x / 32) + warp_id();
    const int t = chunk * 32 + lane;
    if (chunk * 32 >= N) return;
    for (int k = 0; k < K; ++k) {
        int e = -1;
        if (t < N) {
            const int64_t v = topk_idx[(int64_t)t * K + k];
            e = (v >= 0 && v < E) ? (int)v : -1;
        }
        const uint32_t same = __match_any_sync(0xffffffffu, e);
        if (e >= 0 && (same & lanemask_lt()) == 0) atomicAdd(&counts[(int64_t)chunk * E + e], __popc(same));
    }
}

// One CTA: bases[c][e] = offset[e] + sum_{c' < c} counts[c'][e]; offsets = aligned exclusive prefix.
__global__ void __launch_bounds__(1024) permute_scan_kernel(const int* __restrict__ counts, int num_chunks, int E,
                                                            int alignment, int* __restrict__ bases,
                                                            int* __restrict__ expert_offsets, int* __restrict__ expert_counts) {
    __shared__ int s_warp[33];
    const int tid = threadIdx.x;
    // Pass 1: per-expert totals (thread per expert; E <= 1024 per pass, loop otherwise).
    int carry = 0;
    for (int e0 = 0; e0 < E; e0 += blockDim.x) {
        const int e = e0 + tid;
        int tot = 0;
        if (e < E)
            for (int c = 0; c < num_chunks; ++c) tot += counts[(int64_t)c * E + e];
        if (e < E && expert_counts != nullptr) expert_counts[e] = tot;
        const int al = e < E ? (alignment > 1 ? (tot + alignment - 1) / alignment * alignment : tot) : 0;
        // block exclusive scan of `al`
        int incl = al;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int n = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane_id() >= o) incl += n;
        }
        if (lane_id() == 31) s_warp[warp_id()] = incl;
        __syncthreads();
        if (warp_id() == 0) {
            const int nw = blockDim.x / 32;
            int w = lane_id() < nw ? s_warp[lane_id()] : 0;
            int wi = w;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int n = __shfl_up_sync(0xffffffffu, wi, o);
                if (lane_id() >= o) wi += n;
            }
            if (lane_id() < nw) s_warp[lane_id()] = wi - w;
            if (lane_id() == nw - 1) s_warp[32] = wi;
        }
        __syncthreads();
        const int excl = carry + s_warp[warp_id()] + incl - al;
        if (e < E) expert_offsets[e] = excl;
        const int block_total = s_warp[32];
        __syncthreads();
        if (e < E) {
            int run = excl;
            for (int c = 0; c < num_chunks; ++c) {
                bases[(int64_t)c * E + e] = run;
                run += counts[(int64_t)c * E + e];
            }
        }
        carry += block_total;
        __syncthreads();
    }
    if (tid == 0) expert_offsets[E] = carry;
}

__global__ void __launch_bounds__(256) permute_scatter_kernel(PermuteArgs a) {
    extern __shared__ int s_cnt[];  // [warps][E] running counts of this chunk
    const int lane = lane_id(), warp = warp_id();
    const int chunk = blockIdx.x * (blockDim.x / 32) + warp;
    int* my = s_cnt + warp * a.num_experts;
    for (int i = lane; i < a.num_experts; i += 32) my[i] = 0;
    __syncwarp();
    if (chunk * 32 >= a.num_tokens) return;
    const int t = chunk * 32 + lane;
    const int row_bytes = a.hidden * a.x_elem_bytes;
    const int nb = a.hidden / 128;
    for (int k = 0; k < a.num_topk; ++k) {
        int e = -1;
        if (t < a.num_tokens) {
            const int64_t v = a.topk_idx[(int64_t)t * a.num_topk + k];
            e = (v >= 0 && v < a.num_experts) ? (int)v : -1;
        }
        const uint32_t same = __match_any_sync(0xffffffffu, e);
        int pos = -1;
        if (e >= 0) {
            const int rank = __popc(same & lanemask_lt());
            pos = a.bases[(int64_t)chunk * a.num_experts + e] + my[e] + rank;
        }
        __syncwarp();
        if (e >= 0 && (same & lanemask_lt()) == 0) my[e] += __popc(same);
        __syncwarp();
        if (t < a.num_tokens) a.row_map[(int64_t)t * a.num_topk + k] = pos;
        if (a.probs != nullptr && pos >= 0) a.probs_perm[pos] = a.probs[(int64_t)t * a.num_topk + k];
        // Copy the rows of this k-slice: the warp moves one row at a time with 16-byte vectors.
        uint32_t todo = __ballot_sync(0xffffffffu, pos >= 0);
        while (todo) {
            const int src_lane = __ffs(todo) - 1;
            todo &= todo - 1;
            const int st = chunk * 32 + src_lane;
            const int dp = __shfl_sync(0xffffffffu, pos, src_lane);
            const uint8_t* s = static_cast<const uint8_t*>(a.x) + (int64_t)st * row_bytes;
            uint8_t* d = static_cast<uint8_t*>(a.x_perm) + (int64_t)dp * row_bytes;
            for (int o = lane * 16; o < row_bytes; o += 512)
                *reinterpret_cast<int4*>(d + o) = ld_nc_v4(reinterpret_cast<const int4*>(s + o));
            if (a.x_scales != nullptr)
                for (int b = lane; b < nb; b += 32) a.scales_perm[(int64_t)dp * nb + b] = a.x_scales[(int64_t)st * nb + b];
        }
    }
}

void launch_permute(const PermuteArgs& a, cudaStream_t stream) {
    const int num_chunks = (a.num_tokens + 31) / 32;
    cudaMemsetAsync(a.counts, 0, sizeof(int) * (size_t)num_chunks * a.num_experts, stream);
    const int blocks = (num_chunks + 7) / 8;
    if (num_chunks > 0)
        permute_count_kernel<<<blocks, 256, 0, stream>>>(a.topk_idx, a.num_tokens, a.num_topk, a.num_experts, a.counts);
    permute_scan_kernel<<<1, 1024, 0, stream>>>(a.counts, num_chunks, a.num_experts, a.alignment, a.bases,
                                                a.expert_offsets, a.expert_counts);
    if (num_chunks > 0) {
        const size_t smem = sizeof(int) * 8 * (size_t)a.num_experts;
        if (smem > 48 * 1024) cudaFuncSetAttribute(permute_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        permute_scatter_kernel<<<blocks, 256, smem, stream>>>(a);
    }
}

// out[t] = sum_k w[t][k] * y[row_map[t][k]] (fp32 accumulation, bf16 out). One warp per token.
__global__ void __launch_bounds__(256) unpermute_kernel(const __nv_bfloat16* __restrict__ y, const int* __restrict__ row_map,
                                                        const float* __restrict__ w, int N, int H, int K,
                                                        __nv_bfloat16* __restrict__ out) {
    const int lane = lane_id();
    const int warps = blockDim.x / 32;
    for (int t = blockIdx.x * warps + warp_id(); t < N; t += gridDim.x * warps) {
        int rows[kMaxTopk];
        float ws[kMaxTopk];
        int n = 0;
        for (int k = 0; k < K; ++k) {
            const int r = row_map[(int64_t)t * K + k];
            if (r >= 0) {
                rows[n] = r;
                ws[n] = w != nullptr ? w[(int64_t)t * K + k] : 1.f;
                ++n;
            }
        }
        for (int e0 = lane * 8; e0 < H; e0 += 256) {
            int4 v[kMaxTopk];
#pragma unroll
            for (int q = 0; q < kMaxTopk; ++q)
                if (q < n) v[q] = *reinterpret_cast<const int4*>(y + (int64_t)rows[q] * H + e0);
            float acc[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll
            for (int q = 0; q < kMaxTopk; ++q) {
                if (q >= n) break;
                const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&v[q]);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float2 f = __bfloat1622float2(h2[i]);
                    acc[2 * i] = fmaf(ws[q], f.x, acc[2 * i]);
                    acc[2 * i + 1] = fmaf(ws[q], f.y, acc[2 * i + 1]);
                }
            }
            int4 o;
            __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
            for (int i = 0; i < 4; ++i) o2[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
            *reinterpret_cast<int4*>(out + (int64_t)t * H + e0) = o;
        }
    }
}

void launch_unpermute(const void* y, const int* row_map, const float* w, int N, int H, int K, void* out, cudaStream_t stream) {
    if (N == 0) return;
    const int blocks = (N + 7) / 8;
    unpermute_kernel<<<blocks, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(y), row_map, w, N, H, K,
                                                 static_cast<__nv_bfloat16*>(out));
}

}  // namespace ep
