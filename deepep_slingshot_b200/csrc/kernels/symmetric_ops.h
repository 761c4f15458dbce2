// Launch API of the kernels that serve the symmetric side regions (symmetric_ops.cu): pipeline
// send/recv, the flag signal/wait used by AGRS sessions and region barriers, Engram row fetch.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../include/ep/abi.h"

namespace ep {

// One pipeline transfer. Send: x -> the neighbour's slot (peer memory). Recv: my slot -> x.
struct PPArgs {
    uint8_t* x;              // local tensor (source for send, destination for recv)
    uint8_t* slots;          // slot set of this direction: send -> peer's, recv -> mine
    int64_t bytes;
    int64_t slot_bytes;
    int inflight;
    int is_send;
    int peer;                // neighbour rank (for error reports)
    int* count;              // local pp_send_count[d] / pp_recv_count[d]
    const int* wait_flag;    // local: send waits pp_release[d] (credit), recv waits pp_arrival[d]
    int* signal_flag;        // peer: send bumps its pp_arrival[d'], recv bumps its pp_release[d']
    int* ticket;             // local CTA ticket
    KernelStatus st;
};
void launch_pp_copy(const PPArgs& a, int num_blocks, cudaStream_t stream);
int pp_copy_smem_bytes();

// Write `value` into each of `num_writes` peer flags, then wait until each of the `num_waits` local
// flags has reached `value` (one thread, bounded). Region barriers and AGRS arrivals use it.
struct SignalWaitArgs {
    int* write[kMaxRanks];
    const int* wait[kMaxRanks];
    int wait_peer[kMaxRanks];
    int num_writes;
    int num_waits;
    int value;
    int code;
    KernelStatus st;
};
void launch_signal_wait(const SignalWaitArgs& a, cudaStream_t stream);

// Engram fetch: out[t] = storage of rank (idx / entries_per_rank), entry (idx % entries_per_rank).
// A bad index writes a zero row and reports kErrBounds.
struct EngramFetchArgs {
    PeerTable storage;       // base of every rank's storage (data area of its region)
    const int* indices;
    uint8_t* out;
    int num_tokens;
    int entries_per_rank;
    int row_bytes;           // multiple of 16
    int num_ranks;
    KernelStatus st;
};
void launch_engram_fetch(const EngramFetchArgs& a, int num_blocks, cudaStream_t stream);

}  // namespace ep
