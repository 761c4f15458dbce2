// Elementwise and gather kernels of the MoE layer's backward pass, sm_100a.
//
// The reference has no model layer (its expert compute is SGLang + DeepGEMM); these kernels serve
// this library's `models.MoEFFN` backward, around the grouped GEMMs:
//  * unpermute_backward_kernel: the transpose of the weighted unpermute. For every received token j
//    and top-k slot k with a grouped row r = row_map[j][k]:
//        g_y[r]   = bf16(g_tok[j] * w[j][k])            (the expert output's gradient)
//        g_w[j][k] = sum_h g_tok[j][h] * y[r][h]        (the routing weight's gradient, fp32)
//    and g_w[j][k] = 0 for slots without a local expert. One warp per token reads g_tok[j] once.
//  * swiglu_backward_kernel: with a = silu(gate) * up, s = sigmoid(gate):
//        g_gate = g_a * up * s * (1 + gate * (1 - s)),  g_up = g_a * gate * s   (fp32 math, bf16 out)
//  * zero_group_padding_kernel: zero the rows [offsets[e] + counts[e], offsets[e + 1]) of up to three
//    grouped tensors (the alignment padding that grouped GEMMs read as whole groups).
#include <cuda_bf16.h>

#include "../include/ep/device.cuh"
#include "api.h"

namespace ep {

// kMaxRows: an upper bound on the local rows per token (8 covers top-8 routing, 16 any top-k <= 16).
template <int kMaxRows>
__global__ void __launch_bounds__(256) unpermute_backward_kernel(const __nv_bfloat16* __restrict__ g_tok,
                                                                 const int* __restrict__ row_map,
                                                                 const float* __restrict__ w,
                                                                 const __nv_bfloat16* __restrict__ y, int N, int H, int K,
                                                                 int y_rows, __nv_bfloat16* __restrict__ g_y,
                                                                 float* __restrict__ g_w, KernelStatus st) {
    const int lane = lane_id();
    const int warps = blockDim.x / 32;
    for (int j = blockIdx.x * warps + warp_id(); j < N; j += gridDim.x * warps) {
        int r = -1;
        float wk = 0.f;
        if (lane < K) {
            r = row_map[(int64_t)j * K + lane];
            wk = w[(int64_t)j * K + lane];
            if (r >= 0 && !in_window(r, 1, y_rows)) {
                report_error(st, kErrBounds, j, r);
                r = -1;
            }
        }
        const uint32_t valid = __ballot_sync(0xffffffffu, r >= 0);
        const int n = __popc(valid);
        int rows[kMaxRows];
        float ws[kMaxRows], dot[kMaxRows];
        uint32_t m = valid;
#pragma unroll
        for (int q = 0; q < kMaxRows; ++q) {
            const int src = m ? __ffs(m) - 1 : 0;
            rows[q] = __shfl_sync(0xffffffffu, r, src);
            ws[q] = __shfl_sync(0xffffffffu, wk, src);
            dot[q] = 0.f;
            if (m) m &= m - 1;
        }
        for (int e = lane * 8; e - lane * 8 < H; e += 256) {
            if (e >= H) continue;
            const int4 gv = ld_nc_v4(reinterpret_cast<const int4*>(g_tok + (int64_t)j * H + e));
            const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gv);
            float gf[8];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 f = __bfloat1622float2(g2[i]);
                gf[2 * i] = f.x;
                gf[2 * i + 1] = f.y;
            }
#pragma unroll
            for (int q = 0; q < kMaxRows; ++q) {
                if (q >= n) break;
                const int4 yv = ld_nc_v4(reinterpret_cast<const int4*>(y + (int64_t)rows[q] * H + e));
                const __nv_bfloat162* y2 = reinterpret_cast<const __nv_bfloat162*>(&yv);
                int4 ov;
                __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&ov);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float2 yf = __bfloat1622float2(y2[i]);
                    dot[q] = fmaf(gf[2 * i], yf.x, dot[q]);
                    dot[q] = fmaf(gf[2 * i + 1], yf.y, dot[q]);
                    o2[i] = __floats2bfloat162_rn(gf[2 * i] * ws[q], gf[2 * i + 1] * ws[q]);
                }
                *reinterpret_cast<int4*>(g_y + (int64_t)rows[q] * H + e) = ov;
            }
        }
        // Each slot's dot product: reduce over the warp, then the lane of the slot writes it.
        float mine = 0.f;
        uint32_t mm = valid;
#pragma unroll
        for (int q = 0; q < kMaxRows; ++q) {
            if (q >= n) break;
            const float total = warp_reduce_sum(dot[q]);
            const int src = __ffs(mm) - 1;
            mm &= mm - 1;
            if (lane == src) mine = total;
        }
        if (lane < K) g_w[(int64_t)j * K + lane] = mine;  // 0 for slots without a local expert
    }
}

void launch_unpermute_backward(const void* g_tok, const int* row_map, const float* w, const void* y, int N, int H, int K,
                               int y_rows, void* g_y, float* g_w, KernelStatus st, cudaStream_t stream) {
    if (N == 0) return;
    int blocks = (N + 7) / 8;
    if (blocks > 148 * 8) blocks = 148 * 8;
    auto* gt = static_cast<const __nv_bfloat16*>(g_tok);
    auto* yy = static_cast<const __nv_bfloat16*>(y);
    auto* gy = static_cast<__nv_bfloat16*>(g_y);
    if (K <= 8) unpermute_backward_kernel<8><<<blocks, 256, 0, stream>>>(gt, row_map, w, yy, N, H, K, y_rows, gy, g_w, st);
    else unpermute_backward_kernel<16><<<blocks, 256, 0, stream>>>(gt, row_map, w, yy, N, H, K, y_rows, gy, g_w, st);
}

__global__ void __launch_bounds__(256) swiglu_backward_kernel(const __nv_bfloat16* __restrict__ h,
                                                              const __nv_bfloat16* __restrict__ g_a, int64_t rows, int inter,
                                                              __nv_bfloat16* __restrict__ g_h) {
    const int64_t vecs_per_row = inter / 8;
    const int64_t total = rows * vecs_per_row;
    for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < total; v += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = v / vecs_per_row;
        const int c = (int)(v % vecs_per_row) * 8;
        const __nv_bfloat16* hr = h + r * 2 * inter;
        const int4 gv = ld_nc_v4(reinterpret_cast<const int4*>(hr + c));
        const int4 uv = ld_nc_v4(reinterpret_cast<const int4*>(hr + inter + c));
        const int4 av = ld_nc_v4(reinterpret_cast<const int4*>(g_a + r * inter + c));
        const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gv);
        const __nv_bfloat162* u2 = reinterpret_cast<const __nv_bfloat162*>(&uv);
        const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&av);
        int4 og, ou;
        __nv_bfloat162* og2 = reinterpret_cast<__nv_bfloat162*>(&og);
        __nv_bfloat162* ou2 = reinterpret_cast<__nv_bfloat162*>(&ou);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 gate = __bfloat1622float2(g2[i]), up = __bfloat1622float2(u2[i]), ga = __bfloat1622float2(a2[i]);
            const float s0 = 1.0f / (1.0f + __expf(-gate.x)), s1 = 1.0f / (1.0f + __expf(-gate.y));
            og2[i] = __floats2bfloat162_rn(ga.x * up.x * s0 * (1.0f + gate.x * (1.0f - s0)),
                                           ga.y * up.y * s1 * (1.0f + gate.y * (1.0f - s1)));
            ou2[i] = __floats2bfloat162_rn(ga.x * gate.x * s0, ga.y * gate.y * s1);
        }
        __nv_bfloat16* out = g_h + r * 2 * inter;
        *reinterpret_cast<int4*>(out + c) = og;
        *reinterpret_cast<int4*>(out + inter + c) = ou;
    }
}

void launch_swiglu_backward(const void* h, const void* g_a, int64_t rows, int inter, void* g_h, cudaStream_t stream) {
    const int64_t total = rows * (inter / 8);
    if (total == 0) return;
    int64_t blocks = (total + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    swiglu_backward_kernel<<<(int)blocks, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(h),
                                                            static_cast<const __nv_bfloat16*>(g_a), rows, inter,
                                                            static_cast<__nv_bfloat16*>(g_h));
}

__global__ void __launch_bounds__(256) zero_group_padding_kernel(ZeroPaddingArgs a) {
    const int e = blockIdx.x;
    const int r0 = a.offsets[e] + a.counts[e], r1 = a.offsets[e + 1];
    for (int t = 0; t < a.num_tensors; ++t) {
        uint8_t* base = static_cast<uint8_t*>(a.ptr[t]);
        const int64_t row_bytes = a.row_bytes[t];
        for (int r = r0; r < r1; ++r) {
            int4* d = reinterpret_cast<int4*>(base + (int64_t)r * row_bytes);
            for (int64_t o = threadIdx.x; o < row_bytes / 16; o += blockDim.x) d[o] = make_int4(0, 0, 0, 0);
        }
    }
}

void launch_zero_group_padding(const ZeroPaddingArgs& a, int num_groups, cudaStream_t stream) {
    if (num_groups == 0 || a.num_tensors == 0) return;
    zero_group_padding_kernel<<<num_groups, 256, 0, stream>>>(a);
}

}  // namespace ep
