// LogFMT-10: the 10-bit logarithmic wire format of the low-latency combine (the reference's
// `use_logfmt`, [DE]csrc/kernels/legacy/internode_ll.cu:556-712). The number format is the same
// (it decides what a receiver reconstructs); the packing, the in-place compaction and the warp
// mapping are this library's own.
//
// Per group of 128 values (one row has hidden / 128 groups):
//   amax / amin = max / min of |x| (bf16, exact); log_amax = log2(amax),
//   log_amin = max(log2(amin), log_amax - 32). The group is encoded only when log_amax < 0 and
//   log_amin < log_amax (values below 1 with some spread); otherwise it travels as raw bf16.
//   Encoded value: sign bit << 9 | magnitude code m in [0, 511]; m = 0 is zero, m >= 1 decodes to
//   2^((m - 1) * step + log_amin) with step = (log_amax - log_amin) / 510. A value is rounded to
//   the nearer level in linear space: with t = (log2|x| - log_amin) / step, the level above
//   floor(t) is chosen when frac(t) >= log2((1 + 2^step) / 2) / step.
// Group metadata (u32): bf16 bits of amax | bf16 bits of amin << 16; bit 15 (amax's sign, unused
// by an absolute value) marks an encoded group.
// Wire layout of a row: groups in order, 160 bytes per encoded group (lane l of the encoding warp
// owns elements 4l..4l+3 and writes their four 10-bit codes as 5 bytes at 5l), 256 bytes per raw
// group; a group's offset is 160 x (encoded groups before it) + 256 x (raw groups before it).
#pragma once

#include <cstring>

#include <cuda_bf16.h>

#include "device.cuh"

namespace ep {

constexpr int kLogFmtMaxGroupsPerLane = 4;  // hidden <= 32 * 4 * 128 = 16384

__device__ __forceinline__ uint32_t bf16_bits(float v) {
    const __nv_bfloat16 b = __float2bfloat16_rn(v);
    return (uint32_t)(*reinterpret_cast<const uint16_t*>(&b));
}
__device__ __forceinline__ float bf16_bits_to_float(uint32_t bits) {
    return __uint_as_float((bits & 0xffffu) << 16);
}

struct LogFmtGroup {
    float log_amin, step;
    bool cast;
};

// Derive the group parameters from amax / amin exactly as both sides must.
__host__ __device__ __forceinline__ LogFmtGroup logfmt_params(float amax, float amin) {
    LogFmtGroup g;
    const float log_amax = log2f(amax);
    g.log_amin = fmaxf(log2f(amin), log_amax - 32.0f);
    g.cast = (log_amax < 0.0f) && (g.log_amin < log_amax);
    g.step = (log_amax - g.log_amin) / 510.0f;
    return g;
}

// 10-bit code of one value of an encoded group: sign << 9 | magnitude level (0 = zero).
// `inv` = 1 / step, `up` = log2((1 + 2^step) / 2) / step (the linear-space rounding point).
__host__ __device__ __forceinline__ uint32_t logfmt_code(float v, const LogFmtGroup& p, float inv, float up) {
    int code = 0;
    if (v != 0.f) {
        const float t = (log2f(fabsf(v)) - p.log_amin) * inv;
        const float f = floorf(t + 2.0f - up);
        code = f < 0.f ? 0 : (f > 511.f ? 511 : (int)f);
    }
    uint32_t sign;
    memcpy(&sign, &v, sizeof(sign));
    return (uint32_t)code | ((sign >> 31) << 9);
}

// Four 10-bit codes -> 5 bytes (little-endian 40-bit word).
__host__ __device__ __forceinline__ void logfmt_pack4(const uint32_t* c, uint8_t* d) {
    const uint32_t lo = c[0] | (c[1] << 10) | (c[2] << 20) | (c[3] << 30);
    const uint32_t hi = c[3] >> 2;
    d[0] = (uint8_t)lo;
    d[1] = (uint8_t)(lo >> 8);
    d[2] = (uint8_t)(lo >> 16);
    d[3] = (uint8_t)(lo >> 24);
    d[4] = (uint8_t)hi;
}

// 10 bytes read as five little-endian 16-bit words (two encoder lanes x 40 bits) -> 8 codes. Each
// 40-bit half is assembled in its own 64-bit word.
__host__ __device__ __forceinline__ void logfmt_unpack8(const uint16_t* s, uint32_t* codes) {
    const uint64_t half0 = (uint64_t)s[0] | ((uint64_t)s[1] << 16) | ((uint64_t)(s[2] & 0xffu) << 32);
    const uint64_t half1 = (uint64_t)(s[2] >> 8) | ((uint64_t)s[3] << 8) | ((uint64_t)s[4] << 24);
    for (int i = 0; i < 8; ++i) codes[i] = (uint32_t)((i < 4 ? half0 : half1) >> (10 * (i & 3))) & 0x3ffu;
}

// Value of a 10-bit code of an encoded group.
__host__ __device__ __forceinline__ float logfmt_value(uint32_t code, const LogFmtGroup& p) {
    const uint32_t mag = code & 511u;
    const float val = mag == 0 ? 0.f : exp2f((float)(mag - 1) * p.step + p.log_amin);
    return (code >> 9) ? -val : val;
}

// Encode a bf16 row held in shared memory IN PLACE (one warp); returns the compacted byte count
// and writes each group's metadata to `meta[g]` (global, may be a peer's memory).
__device__ __forceinline__ int logfmt_encode_row(uint8_t* buf, int hidden, uint32_t* meta) {
    const int lane = lane_id();
    const int groups = hidden / 128;
    uint32_t my_meta[kLogFmtMaxGroupsPerLane];
#pragma unroll
    for (int i = 0; i < kLogFmtMaxGroupsPerLane; ++i) my_meta[i] = 0;
    int off = 0;
    for (int g = 0; g < groups; ++g) {
        const uint2 raw = *reinterpret_cast<const uint2*>(buf + g * 256 + lane * 8);
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
        float v[4];
        const float2 p0 = __bfloat1622float2(h2[0]), p1 = __bfloat1622float2(h2[1]);
        v[0] = p0.x, v[1] = p0.y, v[2] = p1.x, v[3] = p1.y;
        float amax = 0.f, amin = INFINITY;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            amax = fmaxf(amax, fabsf(v[i]));
            amin = fminf(amin, fabsf(v[i]));
        }
        amax = warp_reduce_max(amax);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amin = fminf(amin, __shfl_xor_sync(0xffffffffu, amin, o));
        const LogFmtGroup p = logfmt_params(amax, amin);
        const uint32_t m = bf16_bits(amax) | (bf16_bits(amin) << 16) | (p.cast ? 0x8000u : 0u);
#pragma unroll
        for (int i = 0; i < kLogFmtMaxGroupsPerLane; ++i)
            if (g == i * 32 + lane) my_meta[i] = m;
        __syncwarp();  // every lane has read group g before any lane overwrites bytes below 256 * (g + 1)
        if (p.cast) {
            const float inv = 1.0f / p.step;
            const float up = log2f((1.0f + exp2f(p.step)) * 0.5f) * inv;
            uint32_t c[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) c[i] = logfmt_code(v[i], p, inv, up);
            logfmt_pack4(c, buf + off + lane * 5);
            off += 160;
        } else {
            *reinterpret_cast<uint2*>(buf + off + lane * 8) = raw;
            off += 256;
        }
        __syncwarp();
    }
#pragma unroll
    for (int i = 0; i < kLogFmtMaxGroupsPerLane; ++i)
        if (i * 32 + lane < groups) meta[i * 32 + lane] = my_meta[i];
    return off;
}

// Decode 8 consecutive values [p, p + 8) (p % 8 == 0) of group `g` of an encoded row and add
// `w * value` to acc. `row` is the row's wire base, `cast_before` the encoded groups before g.
__device__ __forceinline__ void logfmt_accumulate8(const uint8_t* row, int g, int p, int cast_before, uint32_t meta,
                                                   float w, float* acc) {
    const int off = 160 * cast_before + 256 * (g - cast_before);
    if (meta & 0x8000u) {
        const LogFmtGroup prm = logfmt_params(bf16_bits_to_float(meta & 0x7fffu), bf16_bits_to_float(meta >> 16));
        uint32_t codes[8];
        logfmt_unpack8(reinterpret_cast<const uint16_t*>(row + off + (p / 8) * 10), codes);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = fmaf(w, logfmt_value(codes[i], prm), acc[i]);
    } else {
        const int4 v = *reinterpret_cast<const int4*>(row + off + p * 2);
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(h2[i]);
            acc[2 * i] = fmaf(w, f.x, acc[2 * i]);
            acc[2 * i + 1] = fmaf(w, f.y, acc[2 * i + 1]);
        }
    }
}

}  // namespace ep
