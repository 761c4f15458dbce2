// Transport-contract checks over NVLink peer memory, sm_100a.
//
// The reference qualifies its GPU-initiated transport with device tests of the contract the EP
// kernels rely on (backend/tests/gin_producer_stress.cu:10-63: many producers signal one counter and
// the waiter sees the exact total; backend/tests/gin_bounds.cu:9-28: out-of-window puts are rejected
// with a diagnostic code). The same contract, restated for this library's NVLink primitives:
//  * signal_stress_kernel: every warp of the producer blocks adds 1 to the next rank's self-test
//    flag `rounds` times with `red.release.sys`; the last block waits (bounded) until its own flag
//    reaches the exact total the previous rank's producers send, records overshoot, and resets it.
//    Producers and the waiter are one launch, so on one GPU the waiter only waits for co-resident
//    blocks of its own grid.
//  * window_check_kernel: the window rule of every indexed peer access (`in_window`), evaluated on
//    a table of cases; no access is made, in or out of range.
#include "../include/ep/device.cuh"
#include "api.h"

namespace ep {

__global__ void signal_stress_kernel(int* peer_flag, int* my_flag, int rounds, int expected, int* status, KernelStatus st) {
    if (blockIdx.x + 1 < gridDim.x) {
        if (lane_id() == 0)
            for (int i = 0; i < rounds; ++i) red_add_release_sys(peer_flag, 1);
        return;
    }
    if (threadIdx.x != 0) return;
    const bool ok = wait_ge(my_flag, expected, st, kErrTimeoutTest, -1);
    const int seen = ld_acquire_sys(my_flag);
    // 0: exact total, 1: more adds than sent, 2: the wait expired
    *status = !ok ? 2 : (seen == expected ? 0 : 1);
    status[1] = seen;
    st_relaxed_sys(my_flag, 0);
}

void launch_signal_stress(int* peer_flag, int* my_flag, int producer_blocks, int warps, int rounds, int expected,
                          int* status, KernelStatus st, cudaStream_t stream) {
    signal_stress_kernel<<<producer_blocks + 1, warps * 32, 0, stream>>>(peer_flag, my_flag, rounds, expected, status, st);
}

__global__ void window_check_kernel(const int64_t* cases, int n, int* codes) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        codes[i] = in_window(cases[3 * i], cases[3 * i + 1], cases[3 * i + 2]) ? kOk : kErrBounds;
}

void launch_window_check(const int64_t* cases, int n, int* codes, cudaStream_t stream) {
    window_check_kernel<<<(n + 255) / 256 > 0 ? (n + 255) / 256 : 1, 256, 0, stream>>>(cases, n, codes);
}

}  // namespace ep
