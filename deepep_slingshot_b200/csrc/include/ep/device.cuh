// Device-side transport primitives for the NVLink 5 / NVSwitch expert-parallel kernels (sm_100a).
//
// This file is the B200 restatement of the transport contract the reference builds on its NIC
// (put, signal after payload visibility, flush before source reuse, bounded wait):
//   * put    -> plain `st.global` or a TMA bulk store `cp.async.bulk.global.shared::cta` into a peer
//               GPU's buffer (the peer address comes from the CUDA-IPC peer table);
//   * signal -> `st.release.sys` / `red.release.sys.add` on a flag that lives in the WAITER's memory;
//   * flush  -> `cp.async.bulk.wait_group 0` + proxy fence before the release;
//   * wait   -> `ld.acquire.sys` spin with a %globaltimer limit that RETURNS a status instead of
//               trapping (reference: backend/device/cxi_primitives.cuh:39 default_timeout and
//               backend/device/gin_cxi.cuh:9 `require` trap; DeepEP `timeout_while`
//               [DE]deep_ep/include/deep_ep/common/comm.cuh:30-53 prints and traps).
// No cluster-multicast form of any TMA copy is used here: these kernels run on 2..8 GPUs.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include "abi.h"

namespace ep {

// ------------------------------------------------------------------------------------------------
// Window rule of every indexed peer access: the range [index, index + count) must lie inside
// [0, window). Written without forming index + count, so huge or negative values cannot wrap.
// Kernels report kErrBounds and skip the access when it fails (the address is never formed).
// ------------------------------------------------------------------------------------------------
__host__ __device__ __forceinline__ bool in_window(int64_t index, int64_t count, int64_t window) {
    return index >= 0 && count >= 0 && window >= 0 && count <= window && index <= window - count;
}

// ------------------------------------------------------------------------------------------------
// Scalar memory-model helpers
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
    int v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ int ld_relaxed_sys(const int* p) {
    int v;
    asm volatile("ld.relaxed.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ int ld_volatile(const int* p) {
    int v;
    asm volatile("ld.volatile.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t ld_volatile_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(int* p, int v) {
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys(int* p, int v) {
    asm volatile("st.relaxed.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_add_release_sys(int* p, int v) {
    asm volatile("red.release.sys.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int atom_add_relaxed_sys(int* p, int v) {
    int old;
    asm volatile("atom.relaxed.sys.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ int atom_add_acq_rel_sys(int* p, int v) {
    int old;
    asm volatile("atom.acq_rel.sys.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ int atom_add_acq_rel_gpu(int* p, int v) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ void fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ void fence_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
// Orders this thread's async-proxy (TMA) global accesses with its generic-proxy accesses.
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }
__device__ __forceinline__ int warp_id() { return threadIdx.x >> 5; }

// ------------------------------------------------------------------------------------------------
// Error reporting. `ErrorState` lives in host-mapped memory (the host reads it without a sync) and
// `abort_flag` in device memory (cheap to poll from spinning warps).
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ void report_error(const KernelStatus& st, int code, int peer, int detail) {
    if (st.host_error != nullptr) {
        if (atomicCAS(&st.host_error->code, 0, code) == 0) {
            st.host_error->peer = peer;
            st.host_error->detail = detail;
            st.host_error->rank = st.rank;
            __threadfence_system();
        }
    }
    if (st.abort_flag != nullptr) atomicExch(st.abort_flag, 1);
}

__device__ __forceinline__ bool aborted(const KernelStatus& st) {
    return st.abort_flag != nullptr && ld_volatile(st.abort_flag) != 0;
}

// ------------------------------------------------------------------------------------------------
// Device trace ring (see TraceRing): `trace_begin` reads the clock only when tracing is on.
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint64_t trace_begin(const KernelStatus& st) {
    return st.trace != nullptr ? globaltimer_ns() : 0;
}
__device__ __forceinline__ void trace_end(const KernelStatus& st, int event, uint64_t start, int a = 0, int b = 0) {
    if (st.trace == nullptr) return;
    TraceRing* tr = st.trace;
    const unsigned long long i = atomicAdd(tr->cursor, 1ull);
    if (i >= tr->capacity) return;
    uint32_t sm;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
    TraceRecord r;
    r.start_ns = start;
    r.end_ns = globaltimer_ns();
    r.event = event;
    r.block = (int)blockIdx.x;
    r.smid = (int)sm;
    r.rank = st.rank;
    r.a = a;
    r.b = b;
    tr->records[i] = r;
}

// Spin until `*flag >= target` (signed comparison over a monotonic epoch) with a time limit.
// Returns true on success. On timeout it reports `code` and returns false; it also gives up early
// when another block of this launch has already set the abort flag.
__device__ __forceinline__ bool wait_ge(const int* flag, int target, const KernelStatus& st, int code, int peer) {
    if (ld_acquire_sys(flag) - target >= 0) return true;
    const uint64_t start = globaltimer_ns();
    uint32_t iter = 0;
    while (true) {
        if (ld_acquire_sys(flag) - target >= 0) return true;
        if ((++iter & 255u) == 0) {
            if (globaltimer_ns() - start > st.timeout_ns) {
                report_error(st, code, peer, target);
                return false;
            }
            if (aborted(st)) return false;
        }
    }
}

// Same as wait_ge, but waits for equality (used for counters that are reset after use).
__device__ __forceinline__ bool wait_eq(const int* flag, int target, const KernelStatus& st, int code, int peer) {
    if (ld_acquire_sys(flag) == target) return true;
    const uint64_t start = globaltimer_ns();
    uint32_t iter = 0;
    while (true) {
        if (ld_acquire_sys(flag) == target) return true;
        if ((++iter & 255u) == 0) {
            if (globaltimer_ns() - start > st.timeout_ns) {
                report_error(st, code, peer, target);
                return false;
            }
            if (aborted(st)) return false;
        }
    }
}

// ------------------------------------------------------------------------------------------------
// mbarrier + TMA bulk copies (non-tensor, 1D). Sizes and addresses must be multiples of 16 bytes.
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded mbarrier wait. A TMA load from a peer that never completes would otherwise spin forever.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, const KernelStatus& st, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = globaltimer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - start > st.timeout_ns) {
            report_error(st, code, -1, 0);
            return false;
        }
    }
}

// Bounded wait until the loads a ring producer issued into its last min(S, issued) slots have
// landed (the last use of each slot; earlier uses completed before their slot was refilled). The
// producer calls it before its CTA exits or reuses the ring's shared memory, so that no copy into
// shared memory is still in flight after a consumer stopped early. Costs nothing once the consumer
// has taken every row (those phases are complete).
__device__ __forceinline__ void ring_drain(uint64_t* full, int S, int issued, const KernelStatus& st, int code) {
    for (int i = issued > S ? issued - S : 0; i < issued; ++i)
        if (!mbar_wait(&full[i % S], (uint32_t)((i / S) & 1), st, code)) return;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// global (local or peer, no multicast) -> shared memory of this CTA, completion on `bar`.
__device__ __forceinline__ void tma_load_1d(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(smem_dst)),
        "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// shared memory -> global (local or peer), tracked by the bulk-group mechanism.
__device__ __forceinline__ void tma_store_1d(void* gdst, const void* smem_src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem_u32(smem_src)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait() {
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// ------------------------------------------------------------------------------------------------
// Vector helpers
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ int4 ld_nc_v4(const int4* p) {
    int4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ int4 ld_v4(const int4* p) { return *p; }
__device__ __forceinline__ void st_na_v4(int4* p, const int4& v) {
    asm volatile("st.global.L1::no_allocate.v4.s32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

template <typename T>
__device__ __forceinline__ T warp_reduce_max(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
template <typename T>
__device__ __forceinline__ T warp_reduce_sum(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
// Inclusive warp scan.
__device__ __forceinline__ int warp_inclusive_scan(int v) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane_id() >= o) v += n;
    }
    return v;
}

// Per-128-element FP8 e4m3 block scale: amax / 448, amax clamped at 1e-4 (the reference's
// `per_token_cast_to_fp8`, [DE]deep_ep/utils/math.py:36-44). With `round_scale` the scale is rounded
// up to a power of two (exponent-only, UE8M0-representable).
__device__ __forceinline__ float fp8_scale_from_amax(float amax, bool round_scale) {
    amax = fmaxf(amax, 1e-4f);
    float scale = amax / 448.0f;
    if (round_scale) {
        // ceil to power of two on the exponent field; the value is positive and normal here
        uint32_t bits = __float_as_uint(scale);
        uint32_t exp = (bits >> 23) & 0xffu;
        if ((bits & 0x7fffffu) != 0) exp += 1;
        scale = __uint_as_float(exp << 23);
    }
    return scale;
}

}  // namespace ep
