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
//  * flag_pingpong_kernel: NVLink micro-probe of the signalling latency the protocols pay per flag
//    (the reference's NIC offset/latency probes, harness/pipeline_1101/offset_probe.cu, answer the
//    same question for its fabric). One thread writes the peer's flag with `st.release.sys` and
//    waits (bounded) for the answer on its own flag; the responder mirrors it. Between two GPUs
//    each side is one single-block launch on its own GPU; on one GPU both sides are the two blocks of
//    one launch (co-resident), never two launches that wait on each other.
//  * probe_copy_kernel: copy bandwidth between local memory and a peer's mapped memory (peer
//    stores or peer loads) at a chosen vector width, for the size / alignment sweep.
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

__global__ void flag_pingpong_kernel(int* peer_flag, int* my_flag, int iters, int role, long long* out_ns,
                                     KernelStatus st) {
    if (threadIdx.x != 0) return;
    // role 0: initiator, 1: responder; role 2: one GPU, block 0 initiates and block 1 answers
    const bool initiator = role == 2 ? blockIdx.x == 0 : role == 0;
    int* to = role == 2 ? (blockIdx.x == 0 ? peer_flag : my_flag) : peer_flag;
    const int* from = role == 2 ? (blockIdx.x == 0 ? my_flag : peer_flag) : my_flag;
    const uint64_t t0 = globaltimer_ns();
    for (int i = 1; i <= iters; ++i) {
        if (initiator) {
            st_release_sys(to, i);
            if (!wait_ge(from, i, st, kErrTimeoutTest, -1)) {
                out_ns[blockIdx.x] = -1;
                return;
            }
        } else {
            if (!wait_ge(from, i, st, kErrTimeoutTest, -1)) {
                out_ns[blockIdx.x] = -1;
                return;
            }
            st_release_sys(to, i);
        }
    }
    out_ns[blockIdx.x] = (long long)(globaltimer_ns() - t0);
}

void launch_flag_pingpong(int* peer_flag, int* my_flag, int iters, int role, long long* out_ns, KernelStatus st,
                          cudaStream_t stream) {
    flag_pingpong_kernel<<<role == 2 ? 2 : 1, 32, 0, stream>>>(peer_flag, my_flag, iters, role, out_ns, st);
}

template <typename T>
__device__ __forceinline__ void copy_vec(uint8_t* dst, const uint8_t* src, int64_t n, int64_t tid, int64_t nth) {
    T* d = reinterpret_cast<T*>(dst);
    const T* s = reinterpret_cast<const T*>(src);
    int64_t i = tid;
    for (; i + 3 * nth < n; i += 4 * nth) {  // four independent accesses in flight per thread
        const T a = s[i], b = s[i + nth], c = s[i + 2 * nth], e = s[i + 3 * nth];
        d[i] = a;
        d[i + nth] = b;
        d[i + 2 * nth] = c;
        d[i + 3 * nth] = e;
    }
    for (; i < n; i += nth) d[i] = s[i];
}

// dst and src share the same alignment (the host passes vec = the largest power of two, at most 16,
// dividing both addresses); the bytes past the last whole vector are copied one by one.
__global__ void probe_copy_kernel(uint8_t* dst, const uint8_t* src, int64_t bytes, int vec) {
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, nth = (int64_t)gridDim.x * blockDim.x;
    const int64_t n = bytes / vec;
    if (vec == 16) copy_vec<int4>(dst, src, n, tid, nth);
    else if (vec == 8) copy_vec<int2>(dst, src, n, tid, nth);
    else if (vec == 4) copy_vec<int>(dst, src, n, tid, nth);
    else if (vec == 2) copy_vec<short>(dst, src, n, tid, nth);
    else copy_vec<uint8_t>(dst, src, n, tid, nth);
    for (int64_t i = n * vec + tid; i < bytes; i += nth) dst[i] = src[i];
}

void launch_probe_copy(void* dst, const void* src, int64_t bytes, int vec, int blocks, cudaStream_t stream) {
    probe_copy_kernel<<<blocks, 512, 0, stream>>>(static_cast<uint8_t*>(dst), static_cast<const uint8_t*>(src), bytes, vec);
}

void launch_window_check(const int64_t* cases, int n, int* codes, cudaStream_t stream) {
    window_check_kernel<<<(n + 255) / 256 > 0 ? (n + 255) / 256 : 1, 256, 0, stream>>>(cases, n, codes);
}

}  // namespace ep
