// Launch API of the sm_100a kernels. Plain C++ (no torch headers) so that the CUDA translation units
// compile fast and can also be driven from C (see the extern "C" entry points in the .cu files).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../include/ep/abi.h"

namespace ep {

// ---------------------------------------------------------------- layout (get_dispatch_layout)
void launch_dispatch_layout(const int64_t* topk_idx, int num_tokens, int num_topk, int num_experts, int num_ranks,
                            int* num_tokens_per_rank, int* num_tokens_per_expert, bool* is_token_in_rank,
                            cudaStream_t stream);

// ---------------------------------------------------------------- normal-mode dispatch
struct StageArgs {
    const void* x;               // [N][H] bf16 or fp8
    const float* x_scales;       // pre-quantized input scales, or null
    int64_t scale_stride_t;      // element stride between tokens
    int64_t scale_stride_b;      // element stride between 128-blocks
    const int64_t* topk_idx;     // [N][K] or null
    const float* topk_weights;   // [N][K] or null
    uint8_t* staging;            // local staging base (region base + staging_off)
    int num_tokens, hidden, num_topk, topk_pad;
    int in_elem_bytes;           // 2 = bf16 input, 1 = fp8 input
    int quantize;                // 1: fuse bf16 -> fp8 e4m3 1x128 quantization
    int round_scale;             // 1: power-of-two scales
    int tma_rows;                // 1 (set by the launcher): rows are TMA-loaded into shared memory before quantizing
    int regs_rows;               // 1: the standalone stage quantizes rows through registers (no TMA row loads)
    int chunk;                   // overlapped stage: tokens per staged-chunk flag (same on every rank)
    // Standalone stage only: wait until every receiver pulled the previous dispatch (pull_done[r] >=
    // epoch - 1; with epoch 0, >= *dispatch_epoch read before the count step advances it).
    const int* pull_done;
    const int* dispatch_epoch;
    int num_ranks;
    RecordFormat rec;
    int record_stride;
    // This dispatch's epoch (the count step's, known to the host), and the staged-chunk signalling:
    // with signal_chunks the standalone stage releases staged[rank][chunk] = epoch in every
    // receiver's control block as each chunk completes (stage warps of the pull always do).
    int epoch;
    int signal_chunks;
    // 1: the per-token chunk counter add is acquire-release at GPU scope (the counter is local); the
    // release of the staged flag to the receivers stays at system scope and, by cumulativity,
    // covers the writes of every warp whose add it observed. 0: system scope (default).
    int signal_gpu_scope;
    // 1 (default): the signalling lane orders the staged rows for the async proxy (fence.proxy.async)
    // before it counts them; 0: only the receivers' fence after they acquire the flag does.
    int writer_proxy_fence;
    int rank;
    PeerTable peers;
    NormalLayout layout;
    KernelStatus st;
};
// Standalone stage: before the count exchange (fused dispatch + GEMM), or concurrently with the
// count step with per-chunk signalling (normal dispatch). max_sms > 0 caps the SMs it occupies.
void launch_dispatch_stage(const StageArgs& a, int max_sms, cudaStream_t stream);

// Dispatch count step (multi-CTA): waits until every receiver has finished pulling the previous
// dispatch, builds the ordered per-destination token lists and send_head from the routing alone
// (each CTA adds up the per-destination counts of the CTAs before it), counts tokens per expert,
// then its last CTA exchanges the counts with every peer and computes the receive layout.
struct CountArgs {
    const int64_t* topk_idx;         // [N][K] or null
    const bool* is_token_in_rank;    // [N][R] or null (then derived from topk_idx)
    int num_tokens, num_topk, num_experts, num_local_experts;
    int num_ranks, rank;
    int cached;                      // 1: only wait for the previous pulls, reset, and exchange readiness
    int tokens_per_cta;              // multiple of the block size; grid = ceil(N / tokens_per_cta) <= kMaxCountCtas
    int expert_alignment;
    PeerTable peers;
    NormalLayout layout;
    int* send_head;                  // [N][R]
    int* rank_prefix_matrix;         // [R][R] inclusive prefix over sources
    int* send_prefix_matrix;         // [R][R] exclusive prefix over destinations
    int* recv_rank_prefix;           // [R+1]
    int* num_recv_per_expert;        // [E_l] aligned counts (device)
    int* dev_num_recv;               // [1]
    int* cumulative_stats;           // [E_l] optional
    int* expert_counts;              // scratch [E]: zero at entry, zero again at exit
    // Host-mapped counts for the CPU (null: none): the last CTA writes the received-token count and
    // the aligned per-expert counts, then `host_ticket`, as soon as the exchange is done, so a
    // CPU-synced dispatch returns while the stage and the pull still run.
    HostCounters* host;
    int host_ticket;
    KernelStatus st;
};
void launch_dispatch_count(const CountArgs& a, cudaStream_t stream);

struct PullArgs {
    PeerTable peers;
    NormalLayout layout;
    RecordFormat rec;
    int rank, num_ranks, num_local_experts, num_topk;
    const int* rank_prefix_matrix;   // [R][R]
    const int* dev_num_recv;         // device count or null
    int num_recv_host;               // used when dev_num_recv is null
    int num_out_rows;                // allocated output rows (>= num_recv)
    int fill_padding;                // 1: rows past num_recv get topk -1 / src -1 (worst-case mode)
    void* recv_x;
    float* recv_scales;              // null for bf16
    int scales_col_major;            // 1: [H/128][ld] layout
    int64_t scales_ld;
    int64_t* recv_topk_idx;          // null allowed
    float* recv_topk_weights;        // null allowed
    int* recv_src_idx;               // written for fresh dispatches (null in cached mode)
    const int* cached_src_idx;       // cached mode: source token of every receive row (handle)
    int stages;
    HostCounters* host;              // host-mapped counts for the CPU (null: none)
    const int* num_recv_per_expert;  // [E_l] aligned counts computed by notify
    int host_ticket;
    int chunk;                       // rows dealt to pipeline pairs in chunks of this size (0: contiguous)
    // Overlapped stage: with stage_warps > 0 the same launch also stages this rank's tokens (stage
    // warps next to the pull pairs). With stage_warps > 0 or wait_staged (the stage ran as its own
    // launch, concurrently with the count step) the pull waits per (source, chunk) for the staged
    // flags and takes rows in wavefront order; its last block resets this rank's chunk counters.
    int stage_warps;
    int wait_staged;
    // This dispatch's epoch when no count step ran before the pull (cached handle with the
    // concurrent stage): the pull uses it and its last block records it as the dispatch epoch.
    // 0: the count step set the dispatch epoch.
    int epoch;
    StageArgs stage;
    KernelStatus st;
};
void launch_dispatch_pull(const PullArgs& a, int num_sms, cudaStream_t stream);

// ---------------------------------------------------------------- normal-mode combine
struct CombineArgs {
    PeerTable peers;
    NormalLayout layout;
    int rank, num_ranks, num_topk;
    const void* x;                   // bf16 [num_recv][H] expert outputs (one row per received token)
    const float* topk_weights;       // [num_recv][K] or null
    int num_recv_max;                // rows available in x; the true count comes from the prefix matrix
    const int* rank_prefix_matrix;
    const int* send_prefix_matrix;
    const int* recv_src_idx;         // [num_recv] source token index of every received row (handle)
    const int* send_head;            // [N][R] position of my token t in rank r's block, -1 if not sent
    int num_tokens;
    int has_weights;
    const void* bias0;               // bf16 [N][H] or null
    const void* bias1;
    void* out;                       // bf16 [N][H]
    float* out_topk_weights;         // [N][K] or null
    int push_blocks;                 // set by the launcher
    int chunk;                       // push order: -1 wavefront over destinations, 0 contiguous, N chunks of N rows
    int stages;
    int announce_lagged;             // 1: announce a batch of rows one batch later, without draining the stores
    // Expanded mode (row_map != null): x holds one row per (received token, local expert) in any
    // order (the expert-grouped GEMM output) and the sender reduces each token's rows before the
    // push: slot = bf16(sum_k row_weights[j][k] * x[row_map[j][k]]), fp32 accumulation in k order.
    const int* row_map;              // [num_recv][row_map_k] row of x, -1 = not a local expert of the token
    const float* row_weights;        // [num_recv][row_map_k] fp32 factors, or null (plain sum)
    int row_map_k;
    int x_rows;                      // rows of x (bounds of row_map entries)
    KernelStatus st;
};
void launch_combine(const CombineArgs& a, int num_sms, cudaStream_t stream);

// ---------------------------------------------------------------- MoE backward helpers
// g_y[row_map[j][k]] = bf16(g_tok[j] * w[j][k]) and g_w[j][k] = <g_tok[j], y[row_map[j][k]]> (0 for
// row -1); K <= 16. g_y rows that no slot names are left as they are (the caller zeroes them).
void launch_unpermute_backward(const void* g_tok, const int* row_map, const float* w, const void* y, int N, int H, int K,
                               int y_rows, void* g_y, float* g_w, KernelStatus st, cudaStream_t stream);
// SwiGLU backward: h [rows][2I] (gate | up), g_a [rows][I] -> g_h [rows][2I], all bf16, I % 8 == 0.
void launch_swiglu_backward(const void* h, const void* g_a, int64_t rows, int inter, void* g_h, cudaStream_t stream);
// Zero the padding rows [offsets[e] + counts[e], offsets[e + 1]) of up to three grouped tensors.
struct ZeroPaddingArgs {
    void* ptr[3];
    int64_t row_bytes[3];  // multiples of 16
    int num_tensors;
    const int* offsets;    // [E + 1]
    const int* counts;     // [E]
};
void launch_zero_group_padding(const ZeroPaddingArgs& a, int num_groups, cudaStream_t stream);

// ---------------------------------------------------------------- transport-contract checks
// Multi-producer signalling: producer_blocks x warps warps each add 1 to *peer_flag `rounds` times
// (sys-scope release reductions); one more block waits (bounded) until *my_flag == expected and
// writes status[0] (0 exact, 1 overshoot, 2 wait expired) and status[1] (the value seen).
void launch_signal_stress(int* peer_flag, int* my_flag, int producer_blocks, int warps, int rounds, int expected,
                          int* status, KernelStatus st, cudaStream_t stream);
// The window rule of indexed peer accesses on a table of (index, count, window): kOk or kErrBounds.
// NVLink micro-probes (transport_checks.cu). role: 0 initiator, 1 responder (one block each, on
// two GPUs), 2 both sides as two blocks of one launch (one GPU). out_ns[block] = elapsed ns, -1 on
// an expired wait.
void launch_flag_pingpong(int* peer_flag, int* my_flag, int iters, int role, long long* out_ns, KernelStatus st,
                          cudaStream_t stream);
// vec: bytes per access (16, 8, 4, 2 or 1), dividing both addresses.
void launch_probe_copy(void* dst, const void* src, int64_t bytes, int vec, int blocks, cudaStream_t stream);
void launch_window_check(const int64_t* cases, int n, int* codes, cudaStream_t stream);

// ---------------------------------------------------------------- barrier
void launch_barrier(PeerTable peers, int64_t ctrl_off, int rank, int num_ranks, KernelStatus st, cudaStream_t stream);
// Writes the GPU's %globaltimer (ns) into `out` (trace clock alignment).
void launch_read_globaltimer(unsigned long long* out, cudaStream_t stream);

// ---------------------------------------------------------------- low-latency mode
struct LLDispatchArgs {
    PeerTable peers;                 // LL region bases
    LLLayout layout;
    int half;
    const void* x;                   // bf16 [N][H]
    const int64_t* topk_idx;         // [N][K]
    int num_tokens;
    int rank;
    int use_fp8, round_scale, use_ue8m0;
    int phases;                      // 1 send, 2 recv, 3 both
    int* mask;                       // [R] shrink-mode mask (1 = masked) or null
    int shrink;                      // 1: timeouts mask the rank instead of failing
    // recv outputs
    int* recv_count;                 // [E_l]
    int64_t* layout_range;           // [E_l][R]
    int* cumulative_stats;           // [E_l] optional
    int64_t* wait_stats;             // [R] optional
    KernelStatus st;
};
void launch_ll_dispatch(const LLDispatchArgs& a, cudaStream_t stream);

struct LLCombineArgs {
    PeerTable peers;
    LLLayout layout;
    int half;                        // combine half
    int dispatch_half;               // half whose src info / counts describe the rows
    const void* x;                   // bf16 [E_l][R*maxT][H]
    const int* recv_count;           // [E_l] from the dispatch
    const int64_t* topk_idx;         // [N][K]
    const float* topk_weights;       // [N][K]
    int num_tokens;
    int rank;
    int phases;
    int* mask;
    int shrink;
    void* out;                       // bf16 [N][H]
    int64_t* wait_stats;             // [R] optional
    int use_logfmt;                  // rows travel LogFMT-10 encoded where a 128-group qualifies
    KernelStatus st;
};
void launch_ll_combine(const LLCombineArgs& a, cudaStream_t stream);

void launch_ll_clean(PeerTable peers, LLLayout layout, int rank, KernelStatus st, cudaStream_t stream);

// ---------------------------------------------------------------- standalone ops
void launch_per_token_cast_to_fp8(const void* x, int num_tokens, int hidden, void* out_fp8, float* out_scales,
                                  int round_scale, cudaStream_t stream);
// `counts` (optional, device [E]) masks the per-expert layout [E][slots]: rows at or beyond counts[e]
// are skipped (their outputs are left unwritten).
void launch_swiglu_quant(const void* h, int rows, int inter, void* a, void* a_q, float* a_s, int round_scale,
                         cudaStream_t stream, const int* counts = nullptr, int slots = 0);
void launch_per_token_cast_back(const void* x_fp8, const float* scales, int num_tokens, int hidden, void* out_bf16,
                                cudaStream_t stream);
// round_scale: power-of-two block scales (exact as UE8M0, as the block-scaled MMA needs).
void launch_quantize_weights_fp8(const void* w, int num_experts, int n, int k, void* q, float* scales, cudaStream_t stream,
                                 int round_scale = 0);

}  // namespace ep
