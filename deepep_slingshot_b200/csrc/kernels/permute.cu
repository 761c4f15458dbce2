// Permute / unpermute between the dispatch receive layout ([tokens][hidden], top-k local expert ids
// per token) and the expert-grouped layout consumed by the grouped GEMMs ([rows][hidden], rows of
// expert e at [offset[e], offset[e] + count[e]), every count padded to `alignment`).
//
// The reference has no permute (SGLang/DeepGEMM do it downstream of DeepEP,
// backend/tests/sglang_dispatcher_smoke.py:107-124); the v2 `do_expand` layout
// ([DE]deep_ep/buffers/elastic.py:830-855) is the closest. Here it is three sm_100a kernels with a
// deterministic row order (chunk of 32 tokens, then top-k slot, then lane), in four launches:
//   count   : one warp per 32-token chunk adds its per-expert counts into scratch[chunk][expert];
//   scan    : one CTA turns the counts into per-(chunk, expert) bases and aligned expert offsets;
//   rowmap  : one warp per chunk ranks equal experts with __match_any_sync and writes row_map (and
//             the permuted top-k probabilities);
//   copy    : one warp per (token, row segment) reads the segment once and writes its K copies
//             (and the FP8 scales) into the grouped layout.
// Scratch: 2 * num_chunks * num_experts int32 (counts, bases), zeroed by the count launch.
#include <algorithm>

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
// Experts are processed 1024 at a time; when fewer, the chunk range is split among `1024 / E` thread
// groups so each thread walks C / groups chunks instead of all of them.
__global__ void __launch_bounds__(1024) permute_scan_kernel(const int* __restrict__ counts, int num_chunks, int E,
                                                            int alignment, int* __restrict__ bases,
                                                            int* __restrict__ expert_offsets, int* __restrict__ expert_counts) {
    __shared__ int s_part[1024];  // [group][expert of this pass]: partial sums, then group prefixes
    __shared__ int s_off[1024];
    __shared__ int s_warp[33];
    const int tid = threadIdx.x;
    int carry = 0;
    for (int e0 = 0; e0 < E; e0 += 1024) {
        const int eb = min(1024, E - e0);
        const int ng = 1024 / eb;
        const int g = tid / eb, el = tid % eb, e = e0 + el;
        const bool act = g < ng;
        const int c0 = act ? (int)((int64_t)num_chunks * g / ng) : 0;
        const int c1 = act ? (int)((int64_t)num_chunks * (g + 1) / ng) : 0;
        int part = 0;
#pragma unroll 8
        for (int c = c0; c < c1; ++c) part += counts[(int64_t)c * E + e];
        if (act) s_part[g * eb + el] = part;
        __syncthreads();
        int tot = 0;
        if (tid < eb) {
            for (int gg = 0; gg < ng; ++gg) {
                const int v = s_part[gg * eb + tid];
                s_part[gg * eb + tid] = tot;
                tot += v;
            }
            if (expert_counts != nullptr) expert_counts[e0 + tid] = tot;
        }
        const int al = tid < eb ? (alignment > 1 ? (tot + alignment - 1) / alignment * alignment : tot) : 0;
        int incl = al;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int n = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane_id() >= o) incl += n;
        }
        if (lane_id() == 31) s_warp[warp_id()] = incl;
        __syncthreads();
        if (warp_id() == 0) {
            const int w = s_warp[lane_id()];
            int wi = w;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int n = __shfl_up_sync(0xffffffffu, wi, o);
                if (lane_id() >= o) wi += n;
            }
            s_warp[lane_id()] = wi - w;
            if (lane_id() == 31) s_warp[32] = wi;
        }
        __syncthreads();
        if (tid < eb) {
            const int excl = carry + s_warp[warp_id()] + incl - al;
            expert_offsets[e0 + tid] = excl;
            s_off[tid] = excl;
        }
        const int block_total = s_warp[32];
        __syncthreads();
        if (act) {
            int run = s_off[el] + s_part[g * eb + el];
#pragma unroll 4
            for (int c = c0; c < c1; ++c) {
                bases[(int64_t)c * E + e] = run;
                run += counts[(int64_t)c * E + e];
            }
        }
        carry += block_total;
        __syncthreads();
    }
    if (tid == 0) expert_offsets[E] = carry;
}

// One warp per 32-token chunk: grouped row of every (token, k) and the permuted top-k probability.
__global__ void __launch_bounds__(256) permute_rowmap_kernel(PermuteArgs a) {
    extern __shared__ int s_cnt[];  // [warps][E] running counts of this chunk
    const int lane = lane_id(), warp = warp_id();
    const int chunk = blockIdx.x * (blockDim.x / 32) + warp;
    int* my = s_cnt + warp * a.num_experts;
    for (int i = lane; i < a.num_experts; i += 32) my[i] = 0;
    __syncwarp();
    if (chunk * 32 >= a.num_tokens) return;
    const int t = chunk * 32 + lane;
    for (int k = 0; k < a.num_topk; ++k) {
        int e = -1;
        if (t < a.num_tokens) {
            const int64_t v = a.topk_idx[(int64_t)t * a.num_topk + k];
            e = (v >= 0 && v < a.num_experts) ? (int)v : -1;
        }
        const uint32_t same = __match_any_sync(0xffffffffu, e);
        int pos = -1;
        if (e >= 0) pos = a.bases[(int64_t)chunk * a.num_experts + e] + my[e] + __popc(same & lanemask_lt());
        __syncwarp();
        if (e >= 0 && (same & lanemask_lt()) == 0) my[e] += __popc(same);
        __syncwarp();
        if (t < a.num_tokens) a.row_map[(int64_t)t * a.num_topk + k] = pos;
        if (a.probs != nullptr && pos >= 0) a.probs_perm[pos] = a.probs[(int64_t)t * a.num_topk + k];
    }
}

// Token-major row copy: one warp per (token, 2 KB segment of the row) reads the segment once and
// writes it to each of the token's grouped rows (K destinations). Segment 0 also copies the scales.
constexpr int kPermuteCopyUnroll = 4;
constexpr int kPermuteSegBytes = 32 * 16 * kPermuteCopyUnroll;

__global__ void __launch_bounds__(512) permute_copy_kernel(PermuteArgs a) {
    const int lane = lane_id();
    const int warps = blockDim.x / 32;
    const int row_bytes = a.hidden * a.x_elem_bytes;
    const int segs = (row_bytes + kPermuteSegBytes - 1) / kPermuteSegBytes;
    const int nb = a.hidden / 128;
    const int64_t items = (int64_t)a.num_tokens * segs;
    for (int64_t it = (int64_t)blockIdx.x * warps + warp_id(); it < items; it += (int64_t)gridDim.x * warps) {
        const int t = (int)(it / segs), seg = (int)(it % segs);
        const int pos = lane < a.num_topk ? a.row_map[(int64_t)t * a.num_topk + lane] : -1;
        const uint32_t valid = __ballot_sync(0xffffffffu, pos >= 0);
        if (valid == 0) continue;
        const uint8_t* src = static_cast<const uint8_t*>(a.x) + (int64_t)t * row_bytes;
        const int o0 = seg * kPermuteSegBytes + lane * 16;
        int4 v[kPermuteCopyUnroll];
#pragma unroll
        for (int u = 0; u < kPermuteCopyUnroll; ++u)
            if (o0 + u * 512 < row_bytes) v[u] = ld_nc_v4(reinterpret_cast<const int4*>(src + o0 + u * 512));
        float sv[2];
        const bool do_scales = a.x_scales != nullptr && seg == 0;
        if (do_scales) {
#pragma unroll
            for (int j = 0; j < 2; ++j) sv[j] = lane + 32 * j < nb ? a.x_scales[(int64_t)t * nb + lane + 32 * j] : 0.f;
        }
        uint32_t m = valid;
        while (m) {
            const int k = __ffs(m) - 1;
            m &= m - 1;
            const int dp = __shfl_sync(0xffffffffu, pos, k);
            uint8_t* dst = static_cast<uint8_t*>(a.x_perm) + (int64_t)dp * row_bytes;
#pragma unroll
            for (int u = 0; u < kPermuteCopyUnroll; ++u)
                if (o0 + u * 512 < row_bytes) *reinterpret_cast<int4*>(dst + o0 + u * 512) = v[u];
            if (do_scales) {
#pragma unroll
                for (int j = 0; j < 2; ++j)
                    if (lane + 32 * j < nb) a.scales_perm[(int64_t)dp * nb + lane + 32 * j] = sv[j];
                for (int b = lane + 64; b < nb; b += 32) a.scales_perm[(int64_t)dp * nb + b] = a.x_scales[(int64_t)t * nb + b];
            }
        }
    }
}

// One CTA per expert: zero rows [offset[e] + count[e], offset[e + 1]) of x_perm (and their scales
// and probabilities).
__global__ void __launch_bounds__(256) permute_zero_padding_kernel(PermuteArgs a) {
    const int e = blockIdx.x;
    const int r0 = a.expert_offsets[e] + a.expert_counts[e], r1 = a.expert_offsets[e + 1];
    const int row_bytes = a.hidden * a.x_elem_bytes;
    const int nb = a.hidden / 128;
    for (int r = r0; r < r1; ++r) {
        int4* d = reinterpret_cast<int4*>(static_cast<uint8_t*>(a.x_perm) + (int64_t)r * row_bytes);
        for (int o = threadIdx.x; o < row_bytes / 16; o += blockDim.x) d[o] = make_int4(0, 0, 0, 0);
        if (a.scales_perm != nullptr)
            for (int b = threadIdx.x; b < nb; b += blockDim.x) a.scales_perm[(int64_t)r * nb + b] = 0.f;
        if (a.probs_perm != nullptr && threadIdx.x == 0) a.probs_perm[r] = 0.f;
    }
}

cudaError_t launch_permute(const PermuteArgs& a, cudaStream_t stream) {
    const int num_chunks = (a.num_tokens + 31) / 32;
    cudaError_t err = cudaMemsetAsync(a.counts, 0, sizeof(int) * (size_t)num_chunks * a.num_experts, stream);
    if (err != cudaSuccess) return err;
    const int blocks = (num_chunks + 7) / 8;
    if (num_chunks > 0)
        permute_count_kernel<<<blocks, 256, 0, stream>>>(a.topk_idx, a.num_tokens, a.num_topk, a.num_experts, a.counts);
    permute_scan_kernel<<<1, 1024, 0, stream>>>(a.counts, num_chunks, a.num_experts, a.alignment, a.bases,
                                                a.expert_offsets, a.expert_counts);
    if (num_chunks > 0) {
        const size_t smem = sizeof(int) * 8 * (size_t)a.num_experts;
        if (smem > 48 * 1024) {
            err = cudaFuncSetAttribute(permute_rowmap_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (err != cudaSuccess) return err;
        }
        permute_rowmap_kernel<<<blocks, 256, smem, stream>>>(a);
        const int row_bytes = a.hidden * a.x_elem_bytes;
        const int64_t items = (int64_t)a.num_tokens * ((row_bytes + kPermuteSegBytes - 1) / kPermuteSegBytes);
        const int copy_blocks = (int)std::min<int64_t>((items + 15) / 16, 148 * 4);
        permute_copy_kernel<<<copy_blocks, 512, 0, stream>>>(a);
    }
    if (a.zero_padding && a.alignment > 1 && a.expert_counts != nullptr)
        permute_zero_padding_kernel<<<a.num_experts, 256, 0, stream>>>(a);
    return cudaPeekAtLastError();
}

// out[t] = sum_k w[t][k] * y[row_map[t][k]] (fp32 accumulation in k order, bf16 out).
// One warp per (token, 512-column segment); lane k holds the row and weight of slot k, the warp
// walks the slots four at a time so 8 independent 16-byte loads per lane are in flight.
constexpr int kUnpermuteSeg = 512;

__global__ void __launch_bounds__(256, 3) unpermute_kernel(const __nv_bfloat16* __restrict__ y, const int* __restrict__ row_map,
                                                           const float* __restrict__ w, int N, int H, int K,
                                                           __nv_bfloat16* __restrict__ out) {
    const int lane = lane_id();
    const int warps = blockDim.x / 32;
    const int segs = (H + kUnpermuteSeg - 1) / kUnpermuteSeg;
    const int64_t items = (int64_t)N * segs;
    for (int64_t it = (int64_t)blockIdx.x * warps + warp_id(); it < items; it += (int64_t)gridDim.x * warps) {
        const int t = (int)(it / segs), seg = (int)(it % segs);
        const int my_row = lane < K ? row_map[(int64_t)t * K + lane] : -1;
        const float my_w = (lane < K && w != nullptr) ? w[(int64_t)t * K + lane] : 1.f;
        const int c0 = seg * kUnpermuteSeg + lane * 8;
        const bool in0 = c0 < H, in1 = c0 + 256 < H;
        float acc[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[i] = 0.f;
        for (int q0 = 0; q0 < K; q0 += 4) {
            int4 v[4][2];
            int r[4];
            float ws[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                r[j] = __shfl_sync(0xffffffffu, my_row, (q0 + j) & 31);
                ws[j] = __shfl_sync(0xffffffffu, my_w, (q0 + j) & 31);
                if (q0 + j >= K) r[j] = -1;
                if (r[j] >= 0) {
                    const __nv_bfloat16* p = y + (int64_t)r[j] * H + c0;
                    if (in0) v[j][0] = ld_nc_v4(reinterpret_cast<const int4*>(p));
                    if (in1) v[j][1] = ld_nc_v4(reinterpret_cast<const int4*>(p + 256));
                }
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (r[j] < 0) continue;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&v[j][h]);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float2 f = __bfloat1622float2(h2[i]);
                        acc[8 * h + 2 * i] = fmaf(ws[j], f.x, acc[8 * h + 2 * i]);
                        acc[8 * h + 2 * i + 1] = fmaf(ws[j], f.y, acc[8 * h + 2 * i + 1]);
                    }
                }
            }
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            if (!(h == 0 ? in0 : in1)) continue;
            int4 o;
            __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
            for (int i = 0; i < 4; ++i) o2[i] = __floats2bfloat162_rn(acc[8 * h + 2 * i], acc[8 * h + 2 * i + 1]);
            *reinterpret_cast<int4*>(out + (int64_t)t * H + c0 + 256 * h) = o;
        }
    }
}

void launch_unpermute(const void* y, const int* row_map, const float* w, int N, int H, int K, void* out, cudaStream_t stream) {
    if (N == 0) return;
    const int64_t items = (int64_t)N * ((H + kUnpermuteSeg - 1) / kUnpermuteSeg);
    const int blocks = (int)std::min<int64_t>((items + 7) / 8, 148 * 3 * 4);
    unpermute_kernel<<<blocks, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(y), row_map, w, N, H, K,
                                                 static_cast<__nv_bfloat16*>(out));
}

}  // namespace ep
