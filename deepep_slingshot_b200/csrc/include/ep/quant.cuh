// FP8 e4m3 1x128 per-token quantization of one row by one warp (device helper shared by the
// normal-mode stage kernel, the LL dispatch kernel and the standalone cast op).
// Numerics follow the reference's `per_token_cast_to_fp8` ([DE]deep_ep/utils/math.py:36-44):
// amax over each 128-element block, clamped at 1e-4; values scaled by 448/amax and cast with
// saturation; scale = amax/448. With `round_scale` the scale is a power of two (UE8M0-exact).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include "device.cuh"

namespace ep {

// Quantize 8 bf16 values held by one lane; 16 consecutive lanes form one 128-element block.
__device__ __forceinline__ uint2 quantize_8(const int4& v, bool round_scale, float* scale_out) {
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&v);
    float f[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 p = __bfloat1622float2(h2[i]);
        f[2 * i] = p.x;
        f[2 * i + 1] = p.y;
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(f[i]));
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float scale = fp8_scale_from_amax(amax, round_scale);
    const float mult = round_scale ? (1.0f / scale) : (448.0f / fmaxf(amax, 1e-4f));
    uint32_t packed[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const __nv_fp8x2_storage_t lo =
            __nv_cvt_float2_to_fp8x2(make_float2(f[4 * i] * mult, f[4 * i + 1] * mult), __NV_SATFINITE, __NV_E4M3);
        const __nv_fp8x2_storage_t hi =
            __nv_cvt_float2_to_fp8x2(make_float2(f[4 * i + 2] * mult, f[4 * i + 3] * mult), __NV_SATFINITE, __NV_E4M3);
        packed[i] = (uint32_t)lo | ((uint32_t)hi << 16);
    }
    *scale_out = scale;
    return make_uint2(packed[0], packed[1]);
}

// `out_x` and `out_scales` may point to global or shared memory. `hidden` % 128 == 0.
// Loads are batched four 256-element slices at a time so each lane keeps 4 x 16 B in flight.
// With kSmemSource the row is read from shared memory (plain loads) instead of global memory.
// kUnroll: 256-column groups loaded before any is quantized (16-byte loads in flight per lane).
template <bool kSmemSource = false, int kUnroll = 4>
__device__ __forceinline__ void quantize_row_to_fp8(const __nv_bfloat16* __restrict__ xr, uint8_t* __restrict__ out_x,
                                                    float* __restrict__ out_scales, int hidden, bool round_scale) {
    const int lane = lane_id();
    for (int base = 0; base < hidden; base += 256 * kUnroll) {
        int4 v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int e = base + u * 256 + lane * 8;
            if constexpr (kSmemSource)
                v[u] = e < hidden ? *reinterpret_cast<const int4*>(xr + e) : make_int4(0, 0, 0, 0);
            else
                v[u] = e < hidden ? ld_nc_v4(reinterpret_cast<const int4*>(xr + e)) : make_int4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int e = base + u * 256 + lane * 8;
            if (base + u * 256 >= hidden) break;  // warp-uniform
            float scale;
            const uint2 q = quantize_8(v[u], round_scale, &scale);
            if (e < hidden) {
                *reinterpret_cast<uint2*>(out_x + e) = q;
                if ((lane & 15) == 0) out_scales[e / 128] = scale;
            }
        }
    }
}

}  // namespace ep
