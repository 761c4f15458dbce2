// Standalone per-token FP8 cast kernels (the reference's Python/torch.compile helpers
// `per_token_cast_to_fp8` / `per_token_cast_back`, [DE]deep_ep/utils/math.py:36-61), as sm_100a
// kernels: one warp per row, 16-byte vector loads, scales fp32 [N][H/128].
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include "../include/ep/device.cuh"
#include "../include/ep/quant.cuh"
#include "api.h"

namespace ep {

__global__ void __launch_bounds__(256) per_token_cast_to_fp8_kernel(const __nv_bfloat16* __restrict__ x, int num_tokens,
                                                                    int hidden, uint8_t* __restrict__ out,
                                                                    float* __restrict__ scales, int round_scale) {
    const int warps = blockDim.x / 32;
    for (int t = blockIdx.x * warps + warp_id(); t < num_tokens; t += gridDim.x * warps)
        quantize_row_to_fp8(x + (int64_t)t * hidden, out + (int64_t)t * hidden, scales + (int64_t)t * (hidden / 128), hidden,
                            round_scale != 0);
}

__global__ void __launch_bounds__(256) per_token_cast_back_kernel(const uint8_t* __restrict__ x, const float* __restrict__ scales,
                                                                  int num_tokens, int hidden, __nv_bfloat16* __restrict__ out) {
    const int64_t n_vec = (int64_t)num_tokens * hidden / 8;
    for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < n_vec; v += (int64_t)gridDim.x * blockDim.x) {
        const int64_t e = v * 8;
        const int64_t t = e / hidden;
        const int64_t c = e % hidden;
        const float s = scales[t * (hidden / 128) + c / 128];
        const uint2 q = *reinterpret_cast<const uint2*>(x + e);
        const __nv_fp8x2_storage_t* p = reinterpret_cast<const __nv_fp8x2_storage_t*>(&q);
        int4 o;
        __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(p[i], __NV_E4M3);
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hr));
            o2[i] = __floats2bfloat162_rn(f.x * s, f.y * s);
        }
        *reinterpret_cast<int4*>(out + e) = o;
    }
}

// SwiGLU + per-token FP8 requantization, one warp per row:
//   a = silu(h[:, :I]) * h[:, I:]  (fp32 math, rounded to bf16 and stored for the backward pass),
//   (a_q, a_s) = 1x128 FP8 quantization of the bf16 `a` (the input of the down projection).
// With `counts` the rows are the masked per-expert layout [E][slots]: row r belongs to expert
// r / slots and is skipped unless r % slots < counts[r / slots].
__global__ void __launch_bounds__(256) swiglu_quant_kernel(const __nv_bfloat16* __restrict__ h, int rows, int inter,
                                                           __nv_bfloat16* __restrict__ a, uint8_t* __restrict__ a_q,
                                                           float* __restrict__ a_s, int round_scale,
                                                           const int* __restrict__ counts, int slots) {
    const int lane = lane_id();
    const int warps = blockDim.x / 32;
    for (int r = blockIdx.x * warps + warp_id(); r < rows; r += gridDim.x * warps) {
        if (counts != nullptr && r % slots >= __ldg(counts + r / slots)) continue;
        const __nv_bfloat16* gate = h + (int64_t)r * 2 * inter;
        const __nv_bfloat16* up = gate + inter;
        for (int base = 0; base < inter; base += 256) {
            const int e = base + lane * 8;
            const bool valid = e < inter;
            int4 gv = make_int4(0, 0, 0, 0), uv = make_int4(0, 0, 0, 0);
            if (valid) {
                gv = ld_nc_v4(reinterpret_cast<const int4*>(gate + e));
                uv = ld_nc_v4(reinterpret_cast<const int4*>(up + e));
            }
            const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gv);
            const __nv_bfloat162* u2 = reinterpret_cast<const __nv_bfloat162*>(&uv);
            int4 ov;
            __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&ov);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 gf = __bfloat1622float2(g2[i]), uf = __bfloat1622float2(u2[i]);
                const float s0 = gf.x / (1.0f + __expf(-gf.x)), s1 = gf.y / (1.0f + __expf(-gf.y));
                o2[i] = __floats2bfloat162_rn(s0 * uf.x, s1 * uf.y);
            }
            float scale;
            const uint2 qv = quantize_8(ov, round_scale != 0, &scale);
            if (valid) {
                *reinterpret_cast<int4*>(a + (int64_t)r * inter + e) = ov;
                *reinterpret_cast<uint2*>(a_q + (int64_t)r * inter + e) = qv;
                if ((lane & 15) == 0) a_s[(int64_t)r * (inter / 128) + e / 128] = scale;
            }
        }
    }
}

void launch_swiglu_quant(const void* h, int rows, int inter, void* a, void* a_q, float* a_s, int round_scale, cudaStream_t stream,
                         const int* counts, int slots) {
    if (rows == 0) return;
    int blocks = (rows + 7) / 8;
    if (blocks > 4736) blocks = 4736;
    swiglu_quant_kernel<<<blocks, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(h), rows, inter,
                                                    static_cast<__nv_bfloat16*>(a), static_cast<uint8_t*>(a_q), a_s, round_scale,
                                                    counts, counts != nullptr ? slots : 1);
}

void launch_per_token_cast_to_fp8(const void* x, int num_tokens, int hidden, void* out_fp8, float* out_scales,
                                  int round_scale, cudaStream_t stream) {
    if (num_tokens == 0) return;
    int blocks = (num_tokens + 7) / 8;
    if (blocks > 1184) blocks = 1184;
    per_token_cast_to_fp8_kernel<<<blocks, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), num_tokens, hidden,
                                                             static_cast<uint8_t*>(out_fp8), out_scales, round_scale);
}

void launch_per_token_cast_back(const void* x_fp8, const float* scales, int num_tokens, int hidden, void* out_bf16,
                                cudaStream_t stream) {
    if (num_tokens == 0) return;
    const int64_t n_vec = (int64_t)num_tokens * hidden / 8;
    int64_t blocks = (n_vec + 255) / 256;
    if (blocks > 4736) blocks = 4736;
    per_token_cast_back_kernel<<<(int)blocks, 256, 0, stream>>>(static_cast<const uint8_t*>(x_fp8), scales, num_tokens, hidden,
                                                                static_cast<__nv_bfloat16*>(out_bf16));
}

// 128x128 block FP8 quantization of expert weights [E][n][k] (bf16): one CTA per block, each thread
// owns 8 rows x 8 columns (eight 16-byte loads in flight). Numerics of the torch definition used as
// the oracle: amax clamped at 1e-4, scale = amax / 448, q = saturate(v / scale) (true division,
// round-to-nearest-even into e4m3).
__global__ void __launch_bounds__(256) quantize_weights_fp8_kernel(const __nv_bfloat16* __restrict__ w, int n, int k,
                                                                    uint8_t* __restrict__ q, float* __restrict__ scales,
                                                                    int round_scale) {
    __shared__ float s_red[8];
    const int kb = k / 128, nb = n / 128;
    const int64_t blk = blockIdx.x;
    const int e = (int)(blk / ((int64_t)nb * kb));
    const int rem = (int)(blk % ((int64_t)nb * kb));
    const int bn = rem / kb, bk = rem % kb;
    const int tid = threadIdx.x;
    const int c = (tid & 15) * 8;
    const int r0 = tid >> 4;  // rows r0, r0 + 16, ..., r0 + 112
    const int64_t base = ((int64_t)e * n + (int64_t)bn * 128) * k + (int64_t)bk * 128 + c;
    int4 v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = ld_nc_v4(reinterpret_cast<const int4*>(w + base + (int64_t)(r0 + 16 * i) * k));
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&v[i]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 f = __bfloat1622float2(h2[j]);
            amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
        }
    }
    amax = warp_reduce_max(amax);
    if (lane_id() == 0) s_red[warp_id()] = amax;
    __syncthreads();
    amax = s_red[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) amax = fmaxf(amax, s_red[i]);
    // amax / 448 (clamped), or that rounded up to a power of two with round_scale (UE8M0-exact); the
    // values are multiplied by one per-block factor (448 / amax, or the exact inverse of the power of
    // two) instead of divided by the scale element by element.
    amax = fmaxf(amax, 1e-4f);
    const float scale = fp8_scale_from_amax(amax, round_scale != 0);
    const float mult = round_scale != 0 ? 1.0f / scale : 448.0f / amax;
    if (tid == 0) scales[blk] = scale;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&v[i]);
        uint32_t packed[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const float2 a = __bfloat1622float2(h2[2 * j]), b = __bfloat1622float2(h2[2 * j + 1]);
            const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a.x * mult, a.y * mult), __NV_SATFINITE, __NV_E4M3);
            const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(make_float2(b.x * mult, b.y * mult), __NV_SATFINITE, __NV_E4M3);
            packed[j] = (uint32_t)lo | ((uint32_t)hi << 16);
        }
        *reinterpret_cast<uint2*>(q + base + (int64_t)(r0 + 16 * i) * k) = make_uint2(packed[0], packed[1]);
    }
}

void launch_quantize_weights_fp8(const void* w, int num_experts, int n, int k, void* q, float* scales, cudaStream_t stream,
                                 int round_scale) {
    const int64_t blocks = (int64_t)num_experts * (n / 128) * (k / 128);
    if (blocks == 0) return;
    quantize_weights_fp8_kernel<<<(unsigned)blocks, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(w), n, k,
                                                                       static_cast<uint8_t*>(q), scales, round_scale);
}

}  // namespace ep
