// Shared pieces of the tcgen05 GEMM kernels (gemm_sm100.cu, gemm_bf16_sm100.cu): 2D TMA tile loads
// (no multicast), tcgen05 fences / commit / TMEM loads, the K-major 128-byte-swizzle shared-memory
// descriptor, and host-side tensor-map encoding through the driver entry point (no libcuda link).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include "../include/ep/device.cuh"

namespace ep {
namespace tc {

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// 2D tile from this CTA's shared memory to global memory (bulk group; the caller commits and waits).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int x, int y, const void* smem_src) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y), "r"(smem_u32(smem_src))
                 : "memory");
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major tile, 128-byte swizzle, 8-row core groups 1024 B apart (each tile row is 128 bytes).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3fffu);          // start address
    d |= (uint64_t)1 << 16;                           // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;                 // stride byte offset: next 8-row group
    d |= (uint64_t)1 << 46;                           // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;                           // layout: 128-byte swizzle
    return d;
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// 8 consecutive fp32 columns of this warp's 32 TMEM lanes (one value per thread per column).
__device__ __forceinline__ void tmem_ld_8(uint32_t taddr, float* v) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
// Waits for this thread's outstanding tcgen05.ld and ties `v` (8 values loaded by tmem_ld_8) to the
// wait, so no use of them can be scheduled before it.
__device__ __forceinline__ void tmem_wait_ld_8(float* v) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+f"(v[0]), "+f"(v[1]), "+f"(v[2]), "+f"(v[3]), "+f"(v[4]), "+f"(v[5]), "+f"(v[6]), "+f"(v[7])
                 :
                 : "memory");
}
// acc[0..kCols) += scale * (kCols fp32 TMEM columns from taddr), 8 columns per load with the next
// load in flight while the current 8 are accumulated (one TMEM round trip exposed per call instead
// of one per chunk).
template <int kCols>
__device__ __forceinline__ void tmem_promote(uint32_t taddr, float scale, float* acc) {
    static_assert(kCols % 16 == 0, "pairs of 8-column chunks");
    float va[8], vb[8];
    tmem_ld_8(taddr, va);
    tmem_wait_ld_8(va);
#pragma unroll
    for (int c = 0; c < kCols; c += 16) {
        tmem_ld_8(taddr + c + 8, vb);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[c + i] = fmaf(scale, va[i], acc[c + i]);
        tmem_wait_ld_8(vb);
        if (c + 16 < kCols) tmem_ld_8(taddr + c + 16, va);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[c + 8 + i] = fmaf(scale, vb[i], acc[c + 8 + i]);
        if (c + 16 < kCols) tmem_wait_ld_8(va);
    }
}
// 16 consecutive fp32 columns of this warp's 32 TMEM lanes (one value per thread per column).
__device__ __forceinline__ void tmem_ld_16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld_32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%"
        "22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                                   const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (fn == nullptr) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// K-major-in-memory operands read as MN-major (the contiguous dimension is M or N): 128-byte swizzle,
// 8-row K groups 1024 B apart (stride byte offset), 64-element (128-byte) MN atoms `lbo_bytes` apart
// (leading byte offset). One MMA of K = 16 16-bit elements covers two K groups: advance the start
// address by 2048 bytes per instruction.
__device__ __forceinline__ uint64_t smem_desc_mn_sw128(uint32_t addr, uint32_t lbo_bytes) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3fffu);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3fffu) << 16;  // leading byte offset: next MN atom
    d |= (uint64_t)(1024 >> 4) << 32;                   // stride byte offset: next 8-row K group
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// 2D map over a row-major [rows][cols] tensor of `type` (`elem_bytes` each), box `box_cols` x
// `box_rows` (box_cols * elem_bytes = 128 bytes), 128-byte swizzle.
inline bool make_map_2d_box(CUtensorMap* map, CUtensorMapDataType type, int elem_bytes, const void* base, uint64_t rows,
                            uint64_t cols, uint32_t box_cols, uint32_t box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (fn == nullptr) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * (uint64_t)elem_bytes};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t elem[2] = {1, 1};
    return fn(map, type, 2, const_cast<void*>(base), dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Box of 128 rows (the K-major tiles of the GEMM kernels).
inline bool make_map_2d(CUtensorMap* map, CUtensorMapDataType type, int elem_bytes, const void* base, uint64_t rows,
                        uint64_t cols, uint32_t box_cols) {
    return make_map_2d_box(map, type, elem_bytes, base, rows, cols, box_cols, 128);
}

}  // namespace tc
}  // namespace ep

// ------------------------------------------------------------------------------------------------
// CTA pairs (`cta_group::2`): two CTAs of a cluster of two share one MMA of M = 256. Every shared
// memory address below is a CTA-local offset, identical in both CTAs of the pair; `mapa` turns it
// into the cluster address of the same object in the other CTA. No multicast form is used.
// ------------------------------------------------------------------------------------------------
namespace ep {
namespace tc {

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// Cluster address of the shared-memory object at CTA-local address `addr` in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t out;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(addr), "r"(rank));
    return out;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// 2D tile into this CTA's shared memory; the bytes complete on the barrier at cluster address
// `bar_cluster` (the pair's leader CTA holds the stage's full barrier).
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, int x, int y, uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster)
        : "memory");
}
// Completion of this thread's earlier tcgen05 operations arrives once on the barrier at cluster
// address `bar_cluster` (either CTA of the pair).
__device__ __forceinline__ void mma_commit_pair(uint32_t bar_cluster) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster) : "memory");
}
// Arrive (release, cluster scope) on the barrier at cluster address `bar_cluster`.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(cols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t base, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(cols) : "memory");
}

}  // namespace tc
}  // namespace ep
