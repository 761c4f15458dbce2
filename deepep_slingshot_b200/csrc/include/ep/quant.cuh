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

// `out_x` and `out_scales` may point to global or shared memory. `hidden` % 128 == 0.
__device__ __forceinline__ void quantize_row_to_fp8(const __nv_bfloat16* __restrict__ xr, uint8_t* __restrict__ out_x,
                                                    float* __restrict__ out_scales, int hidden, bool round_scale) {
    const int lane = lane_id();
    for (int base = 0; base < hidden; base += 256) {
        const int e = base + lane * 8;
        const bool valid = e < hidden;
        int4 v = make_int4(0, 0, 0, 0);
        if (valid) v = ld_nc_v4(reinterpret_cast<const int4*>(xr + e));
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&v);
        float f[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float2 p = __bfloat1622float2(h2[i]);
            f[2 * i] = p.x;
            f[2 * i + 1] = p.y;
        }
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(f[i]));
        // 16 lanes cover one 128-element block
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float scale = fp8_scale_from_amax(amax, round_scale);
        const float mult = round_scale ? (1.0f / scale) : (448.0f / fmaxf(amax, 1e-4f));
        uint32_t packed[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(make_float2(f[4 * i] * mult, f[4 * i + 1] * mult),
                                                               __NV_SATFINITE, __NV_E4M3);
            __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(make_float2(f[4 * i + 2] * mult, f[4 * i + 3] * mult),
                                                               __NV_SATFINITE, __NV_E4M3);
            packed[i] = (uint32_t)lo | ((uint32_t)hi << 16);
        }
        if (valid) {
            *reinterpret_cast<uint2*>(out_x + e) = make_uint2(packed[0], packed[1]);
            if ((lane & 15) == 0) out_scales[e / 128] = scale;
        }
    }
}

}  // namespace ep
