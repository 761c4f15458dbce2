// Launch API of the tcgen05 grouped GEMM kernels (see gemm_sm100.cu).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../include/ep/abi.h"

namespace ep {

constexpr int kMaxGemmStages = 8;
constexpr int kMaxGemmExperts = 1024;

struct GemmArgs {
    const void* a;            // [rows][k] e4m3, grouped by expert
    const float* sa;          // [rows][k/128]
    const void* b;            // [E][n][k] e4m3
    const float* sb;          // [E][n/128][k/128]
    const int* offsets;       // [E+1] 128-aligned row offsets of the experts
    const int* expert_counts; // [E] valid rows per expert (null: use the aligned block)
    void* d;                  // [rows][n] bf16
    int rows, n, k, num_experts;
    int stages;
    int block_scaled;         // 1: scales are powers of two, applied by the block-scaled MMA (UE8M0)
    // Combine send as the epilogue (row_dest != null; fp32-scale kernel only): row m also goes, bf16,
    // to slot gc_slot_of(row_dest[m]) of rank gc_rank_of(row_dest[m]) (negative: nowhere) in the
    // slot area of that rank's GEMM-combine region, and `d` may be null (rows not kept locally).
    // Before its first store every CTA waits until each rank released its slots of epoch
    // gc_epoch - 1; the last CTA to finish publishes gc_epoch in gc_done[gc_rank] of every rank.
    const int* row_dest;      // [rows]
    PeerTable gc_regions;     // region bases ([SymCtrl | slots]) of every rank
    int gc_rank, gc_num_ranks, gc_epoch;
    int64_t gc_slots;         // slots per rank
    KernelStatus st;
};

// Returns 0 on success, 1 bad shapes, 2 tensor-map encode failure, 3 launch failure.
int launch_grouped_gemm_fp8(const GemmArgs& a, int num_sms, cudaStream_t stream);

// Down projection -> combine (gemm_combine.cu), the two steps around the sending GEMM:
// the destination word of every operand row from the dispatch handle and the permute's row map,
// and the source rank's reduction of its slots once every rank's rows have landed.
struct GcRowDestArgs {
    const int* row_map;             // [num_recv][num_topk] operand row of (received token, k), -1 none
    const int* recv_src_idx;        // [num_recv] token index on its source rank
    const int* rank_prefix_matrix;  // [R][R] from the dispatch
    int* row_dest;                  // [rows] out, preset to -1
    int num_recv, num_topk, rows, rank, num_ranks;
    int64_t slots;                  // slots per rank
    KernelStatus st;
};
void launch_gc_row_dest(const GcRowDestArgs& a, cudaStream_t stream);

struct GcReduceArgs {
    PeerTable regions;              // region bases of every rank (flags are released into them)
    int rank, num_ranks, epoch;
    const int64_t* topk_idx;        // [num_tokens][num_topk] this rank's own routing (-1: none)
    const float* topk_weights;      // [num_tokens][num_topk] (null: weight 1)
    void* out;                      // [num_tokens][hidden] bf16
    int num_tokens, num_topk, hidden;
    int64_t slots;
    KernelStatus st;
};
void launch_gc_reduce(const GcReduceArgs& a, int num_sms, cudaStream_t stream);

// bf16 grouped GEMMs with both operands K-major (gemm_bf16_sm100.cu).
//   mode 0 (M-grouped): a [rows][k], b [E*n][k], d [rows][n]; rows of expert e at offsets[e], 128-aligned
//   mode 1 (K-grouped): a [m][k], b [n][k], d [E][m][n]; expert e contracts k in [offsets[e], offsets[e+1])
// MN-major operands: b_mn_major makes b [E*k][n] (mode 0) or [k][n] (mode 1); a_mn_major (mode 1
// only) makes a [k][m].
struct Bf16GemmArgs {
    const void* a;
    const void* b;
    const int* offsets;       // [E+1] (mode 0: 128-aligned rows; mode 1: 64-aligned K offsets)
    const int* expert_counts; // mode 0: [E] valid rows per expert (null: the aligned block)
    void* d;
    int mode;
    int rows, m, n, k, num_experts;
    int stages;
    int a_mn_major, b_mn_major;
    KernelStatus st;
};
int launch_grouped_gemm_bf16(const Bf16GemmArgs& a, int num_sms, cudaStream_t stream);

// Masked grouped FP8 GEMM over the low-latency per-expert padded layout (gemm_masked_sm100.cu).
//   a [E][slots][k] e4m3; scale of (e, m, kb) at sa[e*sa_e + kb*sa_k + m*sa_m]; b [E][n][k] e4m3;
//   sb [E][n/128][k/128]; d [E][slots][n] bf16, rows m < count[e] written.
// Counts come either from `counts` (device, [E]) or, fused with the low-latency dispatch receive,
// from the slot counters of `ll` once every rank's dispatch_done flag is set (exactly one is set).
struct MaskedGemmArgs {
    const void* a;
    const float* sa;
    int64_t sa_e, sa_k, sa_m;
    const void* b;
    const float* sb;
    const int* counts;
    void* d;
    int num_experts, slots, n, k;
    int stages;
    LLCtrl* ll;                 // fused receive: this rank's control block of the dispatch half
    int num_ranks;
    int* recv_count;            // fused: [E] out
    int* cumulative_stats;      // fused: [E] += counts (optional)
    int64_t l2_prefetch_bytes;  // fused: weights each CTA prefetches into L2 while it waits
    // Fused low-latency combine send (combine != 0): row m of expert e goes to its source rank's
    // combine slot [token][k] of the combine half (from the dispatch half's source info) instead of
    // d; the last CTA then releases `combine_done` in every rank, as the combine's send phase does.
    int combine;
    PeerTable ll_peers;
    LLLayout ll_layout;
    int dispatch_half, combine_half, rank;
    KernelStatus st;
};
// Returns 0 on success, 1 bad arguments, 2 tensor-map encode failure, 3 launch failure.
int launch_masked_gemm_fp8(const MaskedGemmArgs& a, int num_sms, cudaStream_t stream);

// Normal-mode dispatch receive fused with the gate/up grouped FP8 GEMM (fused_dispatch_gemm.cu).
// Launched after the dispatch's stage and notify steps (expert alignment 128). Zeroed on entry:
// claim [E_l], landed [E_l * max_mtiles], tile_counter [1].
struct FusedDispatchGemmArgs {
    PeerTable peers;
    NormalLayout layout;
    RecordFormat rec;                // FP8 records (x_bytes == hidden)
    int rank, num_ranks, num_local_experts, num_topk;
    const int* rank_prefix_matrix;   // [R][R] from notify
    const int* dev_num_recv;         // received tokens (device, from notify)
    int num_out_rows;                // rows allocated in row_map / recv_* (>= received tokens)
    int pull_ctas;                   // CTAs that pull first, then join the GEMM
    int chunk;                       // row dealing of the pull pairs (as the plain pull)
    const int* num_recv_per_expert;  // [E_l] 128-aligned counts from notify
    const int* raw_counts;           // [E_l] received rows per expert (notify's statistics output)
    int* claim;                      // [E_l] slot counters
    int* landed;                     // [E_l][max_mtiles] rows landed per 128-row tile
    int max_mtiles;                  // m-tiles per expert the buffers allow
    uint8_t* a;                      // [rows_cap][hidden] e4m3, experts at 128-aligned offsets
    float* sa;                       // [rows_cap][hidden/128]
    int rows_cap;
    int* row_map;                    // [num_out_rows][K]: operand row of (received token, k), -1 if not local
    float* recv_topk_weights;        // [num_out_rows][K]: local weights (0 elsewhere)
    int* recv_src_idx;               // [num_out_rows]: source token of every received row
    HostCounters* host;              // host-mapped counts (null: none)
    int host_ticket;
    const void* b;                   // [E_l][n][hidden] e4m3 weights
    const float* sb;                 // [E_l][n/128][hidden/128]
    int n;
    void* d;                         // [rows_cap][n] bf16
    int* tile_counter;
    KernelStatus st;
};
// Returns 0 on success, 1 bad arguments, 2 tensor-map encode failure, 3 launch failure.
int launch_fused_dispatch_gemm(const FusedDispatchGemmArgs& a, int num_sms, cudaStream_t stream);

}  // namespace ep
