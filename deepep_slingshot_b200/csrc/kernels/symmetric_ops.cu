// Kernels of the symmetric side regions: pipeline send/recv between ring neighbours, the flag
// signal/wait used by AGRS sessions and region barriers, and Engram row fetch.
//
// Reference behaviour: PP ring with in-flight slots and credits ([DE]deep_ep/include/deep_ep/impls/
// pp_send_recv.cuh:113-213, runtime [DE]csrc/elastic/buffer.hpp:297-339), AGRS write-and-wait
// signals ([DE]csrc/elastic/buffer.hpp:365-470, [DE]csrc/kernels/backend/cuda_driver.cu) and Engram
// GET of rows owned by `index / entries_per_rank` ([DE]deep_ep/include/deep_ep/impls/engram_fetch.cuh:11-87).
//
// B200 design: the sender TMA-stores its tensor straight into the neighbour's receive slot over
// NVLink (there is no send staging copy, the reference needs one for the NIC put), the last CTA
// to finish bumps the neighbour's arrival counter with a system-scope release, and the receiver
// releases the slot with the same mechanism. Engram rows are read by the fetching GPU with plain
// 16-byte loads from the owner's storage (peer memory, no multicast). Every wait is bounded.
#include <algorithm>

#include "../include/ep/device.cuh"
#include "symmetric_ops.h"

namespace ep {

namespace {

constexpr int kCopyStages = 8;
constexpr int kCopyLag = 4;            // TMA stores kept in flight before a stage is refilled
constexpr int kCopyStageBytes = 16384;

// Copy src[0, n) -> dst[0, n) (n a multiple of 16, both 16-byte aligned) with TMA through
// kCopyStages shared-memory stages. Called by ONE thread; returns false if a load never completed.
__device__ bool tma_copy(const uint8_t* src, uint8_t* dst, int64_t n, uint8_t* smem, uint64_t* bars,
                         const KernelStatus& st, int code) {
    if (n <= 0) return true;
    const int64_t iters = (n + kCopyStageBytes - 1) / kCopyStageBytes;
    auto len = [&](int64_t i) { const int64_t r = n - i * kCopyStageBytes; return (uint32_t)(r < kCopyStageBytes ? r : kCopyStageBytes); };
    int64_t issued = 0;  // loads issued so far (in index order)
    auto issue_load = [&](int64_t i) {
        issued = i + 1;
        const int s = (int)(i % kCopyStages);
        mbar_arrive_expect_tx(&bars[s], len(i));
        tma_load_1d(smem + s * kCopyStageBytes, src + i * kCopyStageBytes, len(i), &bars[s]);
    };
    for (int64_t i = 0; i < iters && i < kCopyStages; ++i) issue_load(i);
    for (int64_t i = 0; i < iters; ++i) {
        const int s = (int)(i % kCopyStages);
        if (!mbar_wait(&bars[s], (uint32_t)((i / kCopyStages) & 1), st, code)) {
            bulk_wait<0>();
            ring_drain(bars, kCopyStages, (int)issued, st, code);  // loads in flight land before the return
            return false;
        }
        tma_store_1d(dst + i * kCopyStageBytes, smem + s * kCopyStageBytes, len(i));
        bulk_commit();
        // The store issued kCopyLag iterations ago has read its stage: refill that stage.
        const int64_t j = i - kCopyLag;
        if (j >= 0 && j + kCopyStages < iters) {
            bulk_wait_read<kCopyLag>();
            issue_load(j + kCopyStages);
        }
    }
    bulk_wait<0>();
    return true;
}

}  // namespace

// Grid: num_blocks CTAs of 32 threads; lane 0 of each CTA copies one contiguous 16-byte-aligned
// share of the tensor, the CTA that arrives last on the ticket signals the neighbour.
__global__ void __launch_bounds__(32, 1) pp_copy_kernel(PPArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    if (threadIdx.x != 0) return;
    const uint64_t t_start = trace_begin(a.st);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kCopyStages * kCopyStageBytes);
    const int c = ld_volatile(a.count);
    // send: the slot is free once the neighbour released tensor c - inflight; recv: tensor c arrived
    const int target = a.is_send ? c + 1 - a.inflight : c + 1;
    bool ok = wait_ge(a.wait_flag, target, a.st, kErrTimeoutPP, a.peer);
    if (ok) fence_proxy_async_global();  // order the acquire before the async-proxy reads below
    uint8_t* slot = a.slots + (int64_t)((unsigned)c % (unsigned)a.inflight) * a.slot_bytes;
    const uint8_t* src = a.is_send ? a.x : slot;
    uint8_t* dst = a.is_send ? slot : a.x;
    const int64_t body = a.bytes & ~int64_t(15);
    const int64_t per = ((body / 16 + gridDim.x - 1) / gridDim.x) * 16;
    const int64_t b0 = ::min(body, (int64_t)blockIdx.x * per);
    const int64_t b1 = ::min(body, b0 + per);
    if (ok) {
        for (int s = 0; s < kCopyStages; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
        ok = tma_copy(src + b0, dst + b0, b1 - b0, smem, bars, a.st, kErrTimeoutTma);
        if (ok && blockIdx.x == 0)
            for (int64_t i = body; i < a.bytes; ++i) dst[i] = src[i];
    }
    trace_end(a.st, kTracePP, t_start, a.is_send, (int)::min(a.bytes, (int64_t)0x7fffffff));
    fence_proxy_async_global();
    __threadfence_system();
    const int t = atomicAdd(a.ticket, 1);
    if (t == (int)gridDim.x - 1) {
        *a.ticket = 0;
        __threadfence_system();
        if (!aborted(a.st)) red_add_release_sys(a.signal_flag, 1);
        *a.count = c + 1;
    }
}

int pp_copy_smem_bytes() { return kCopyStages * kCopyStageBytes + kCopyStages * 8; }

void launch_pp_copy(const PPArgs& a, int num_blocks, cudaStream_t stream) {
    const int smem = pp_copy_smem_bytes();
    cudaFuncSetAttribute(pp_copy_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    pp_copy_kernel<<<std::max(1, num_blocks), 32, smem, stream>>>(a);
}

__global__ void __launch_bounds__(32, 1) signal_wait_kernel(SignalWaitArgs a) {
    if (threadIdx.x != 0) return;
    __threadfence_system();
    for (int i = 0; i < a.num_writes; ++i) st_release_sys(a.write[i], a.value);
    for (int i = 0; i < a.num_waits; ++i)
        if (!wait_ge(a.wait[i], a.value, a.st, a.code, a.wait_peer[i])) return;
}

void launch_signal_wait(const SignalWaitArgs& a, cudaStream_t stream) {
    signal_wait_kernel<<<1, 32, 0, stream>>>(a);
}

// One warp per fetched row, 16-byte loads from the owner's storage, four in flight per lane.
__global__ void __launch_bounds__(256) engram_fetch_kernel(EngramFetchArgs a) {
    const int lane = lane_id();
    const int warps = blockDim.x / 32;
    const int units = a.row_bytes / 16;
    const int64_t total = (int64_t)a.entries_per_rank * a.num_ranks;
    for (int t = blockIdx.x * warps + warp_id(); t < a.num_tokens; t += gridDim.x * warps) {
        const int idx = a.indices[t];
        int4* dst = reinterpret_cast<int4*>(a.out + (int64_t)t * a.row_bytes);
        if (!in_window(idx, 1, total)) {
            for (int u = lane; u < units; u += 32) dst[u] = make_int4(0, 0, 0, 0);
            if (lane == 0) report_error(a.st, kErrBounds, -1, idx);
            continue;
        }
        const int owner = idx / a.entries_per_rank;
        const int entry = idx % a.entries_per_rank;
        const int4* src = reinterpret_cast<const int4*>(static_cast<const uint8_t*>(a.storage.base[owner]) +
                                                        (int64_t)entry * a.row_bytes);
        for (int u0 = lane; u0 < units; u0 += 128) {
            int4 v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (u0 + 32 * j < units) v[j] = ld_nc_v4(src + u0 + 32 * j);
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (u0 + 32 * j < units) dst[u0 + 32 * j] = v[j];
        }
    }
}

void launch_engram_fetch(const EngramFetchArgs& a, int num_blocks, cudaStream_t stream) {
    if (a.num_tokens == 0) return;
    const int blocks = std::max(1, std::min(num_blocks, (a.num_tokens + 7) / 8));
    engram_fetch_kernel<<<blocks, 256, 0, stream>>>(a);
}

}  // namespace ep
