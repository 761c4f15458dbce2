// C++ runtime of the B200 expert-parallel buffer (the reference's legacy `Buffer` runtime,
// [DE]csrc/legacy/buffer.hpp:84-1792, and its `Config`, [DE]csrc/legacy/config.hpp:24-188),
// re-designed for one NVLink 5 / NVSwitch domain:
//  * two symmetric regions per rank, each a cudaMalloc allocation shared through CUDA IPC handles
//    that Python all-gathers over torch.distributed: the normal-mode region (`num_nvl_bytes`) and the
//    low-latency region (`num_rdma_bytes`; on one box the LL traffic is NVLink peer stores too);
//  * peer tables passed by value to every kernel; no NIC, no NVSHMEM, no proxy thread;
//  * host-mapped counters for the CPU sync of received counts, a host-mapped error page and a device
//    abort flag: every kernel wait is bounded and reports, the host turns reports into exceptions.
#pragma once

#include <ATen/cuda/CUDAContext.h>
#include <ATen/cuda/CUDAEvent.h>
#include <c10/cuda/CUDAStream.h>
#include <pybind11/functional.h>
#include <pybind11/pybind11.h>
#include <torch/extension.h>

#include <functional>
#include <map>
#include <memory>
#include <optional>
#include <string>
#include <tuple>
#include <vector>

#include "../include/ep/abi.h"
#include "../kernels/api.h"

namespace ep {

// Tuning/config object kept for API parity ([DE]csrc/legacy/config.hpp:24-51). On NVLink with the
// pull/push design only `num_sms` drives the kernels; the chunk sizes are accepted and stored.
struct Config {
    int num_sms;
    int num_max_nvl_chunked_send_tokens;
    int num_max_nvl_chunked_recv_tokens;
    int num_max_rdma_chunked_send_tokens;
    int num_max_rdma_chunked_recv_tokens;
    Config(int num_sms, int nvl_send, int nvl_recv, int rdma_send, int rdma_recv)
        : num_sms(num_sms),
          num_max_nvl_chunked_send_tokens(nvl_send),
          num_max_nvl_chunked_recv_tokens(nvl_recv),
          num_max_rdma_chunked_send_tokens(rdma_send),
          num_max_rdma_chunked_recv_tokens(rdma_recv) {}
    // Size of the normal-mode region for `num_max_tokens` tokens per rank (default 4096, top-8).
    int64_t get_nvl_buffer_size_hint(int64_t hidden_bytes, int num_ranks, int num_max_tokens = 4096, int num_topk = 8) const;
    int64_t get_rdma_buffer_size_hint(int64_t hidden_bytes, int num_ranks) const;
};

struct EventHandle {
    std::shared_ptr<at::cuda::CUDAEvent> event;
    EventHandle();
    explicit EventHandle(const at::cuda::CUDAStream& stream);
    void current_stream_wait() const;
};

// Human-readable name of an ErrorCode (kernel error reports).
const char* error_name(int code);

NormalLayout compute_normal_layout(int64_t region_bytes, int hidden, int num_ranks);
int64_t normal_region_size_for(int num_max_tokens, int hidden, int num_ranks);
RecordFormat record_format(int hidden, int num_topk, bool fp8);
LLLayout compute_ll_layout(int64_t region_bytes, int max_tokens, int hidden, int num_experts, int num_ranks);
int64_t ll_region_size_for(int max_tokens, int hidden, int num_ranks, int num_experts);

class Buffer {
   public:
    Buffer(int rank, int num_ranks, int64_t num_nvl_bytes, int64_t num_rdma_bytes, bool low_latency_mode,
           bool explicitly_destroy, bool enable_shrink, double gpu_timeout_secs);
    ~Buffer() noexcept(false);

    bool is_available() const { return available_; }
    int get_num_rdma_ranks() const { return 1; }
    int get_rdma_rank() const { return 0; }
    int get_root_rdma_rank(bool global) const { return global ? 0 : 0; }
    int get_local_device_id() const { return device_id_; }
    pybind11::bytearray get_local_ipc_handle() const;
    pybind11::bytearray get_local_ll_ipc_handle() const;
    void sync(const std::vector<int>& device_ids, const std::vector<std::optional<pybind11::bytes>>& handles,
              const std::vector<std::optional<pybind11::bytes>>& ll_handles);
    void destroy();
    torch::Stream get_comm_stream() const;
    torch::Tensor get_local_buffer_tensor(const pybind11::object& dtype, int64_t offset, bool use_rdma_buffer) const;
    int64_t get_capacity(int hidden, int num_topk) const;

    void check_error() const;
    std::tuple<int, int, int, int> get_error_state() const;
    void clear_error();
    void set_timeout_secs(double secs);
    std::map<std::string, double> get_profile();

    // Device trace ring (off by default): every traced kernel appends per-block records.
    void enable_trace(int64_t capacity);
    void disable_trace();
    // (records [n, 40] uint8 on the CPU, appended count; count > capacity means records were dropped)
    std::tuple<torch::Tensor, int64_t> read_trace(bool reset);
    // (host CLOCK_MONOTONIC ns before, GPU %globaltimer ns, host ns after) for clock alignment.
    std::tuple<int64_t, int64_t, int64_t> sample_clock();

    // ---------------------------------------------------------------- normal mode
    std::tuple<torch::Tensor, std::optional<torch::Tensor>, torch::Tensor, torch::Tensor, std::optional<EventHandle>>
    get_dispatch_layout(const torch::Tensor& topk_idx, int num_experts, std::optional<EventHandle>& previous_event,
                        bool async, bool allocate_on_comm_stream);

    std::tuple<torch::Tensor, std::optional<torch::Tensor>, std::optional<torch::Tensor>, std::optional<torch::Tensor>,
               std::vector<int>, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor,
               std::optional<torch::Tensor>, std::optional<EventHandle>>
    intranode_dispatch(const torch::Tensor& x, const std::optional<torch::Tensor>& x_scales,
                       const std::optional<torch::Tensor>& topk_idx, const std::optional<torch::Tensor>& topk_weights,
                       const std::optional<torch::Tensor>& is_token_in_rank, int num_experts,
                       const std::optional<torch::Tensor>& cached_rank_prefix_matrix,
                       const std::optional<torch::Tensor>& cached_send_prefix_matrix,
                       const std::optional<torch::Tensor>& cached_recv_src_idx,
                       const std::optional<torch::Tensor>& cached_send_head, int expert_alignment,
                       int num_worst_tokens, bool quantize_fp8, bool round_scale, bool scales_col_major,
                       const std::optional<torch::Tensor>& cumulative_local_expert_recv_stats, int num_sms,
                       std::optional<EventHandle>& previous_event, bool async, bool allocate_on_comm_stream);

    std::tuple<torch::Tensor, std::optional<torch::Tensor>, std::optional<EventHandle>> intranode_combine(
        const torch::Tensor& x, const std::optional<torch::Tensor>& topk_weights, const std::optional<torch::Tensor>& bias_0,
        const std::optional<torch::Tensor>& bias_1, const torch::Tensor& rank_prefix_matrix,
        const torch::Tensor& send_prefix_matrix, const torch::Tensor& send_head, const torch::Tensor& recv_src_idx, int num_sms,
        std::optional<EventHandle>& previous_event, bool async, bool allocate_on_comm_stream,
        const std::optional<torch::Tensor>& row_map, const std::optional<torch::Tensor>& row_weights);

    void barrier(bool use_comm_stream, bool with_cpu_sync);
    // Transport self-test (multi-producer signalling into the next rank's control block); returns
    // {status, value seen} after synchronizing. Every rank must call it together.
    std::vector<int> selftest_signal_stress(int producer_blocks, int warps, int rounds);
    double probe_flag_latency(int peer, int iters);
    std::vector<double> probe_peer_copy(int shift, int64_t bytes, int64_t offset, bool store, int reps, int blocks,
                                        const torch::Tensor& local);

    // ---------------------------------------------------------------- low-latency mode
    void clean_low_latency_buffer(int num_max_dispatch_tokens_per_rank, int hidden, int num_experts);
    std::tuple<torch::Tensor, std::optional<torch::Tensor>, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, int,
               std::optional<EventHandle>, std::optional<std::function<void()>>>
    low_latency_dispatch(const torch::Tensor& x, const torch::Tensor& topk_idx,
                         const std::optional<torch::Tensor>& cumulative_local_expert_recv_stats,
                         const std::optional<torch::Tensor>& dispatch_wait_recv_cost_stats,
                         int num_max_dispatch_tokens_per_rank, int num_experts, bool use_fp8, bool round_scale,
                         bool use_ue8m0, bool async, bool return_recv_hook);
    // Normal-mode FP8 dispatch whose receive writes the expert-grouped GEMM operand and runs the
    // gate/up grouped GEMM in the same launch, tile by tile as rows land (fused_dispatch_gemm.cu).
    // Returns (h [rows, n] bf16, a [rows, hidden] e4m3, a_scales [rows, hidden/128], row_map
    // [num_recv, K], recv_topk_weights [num_recv, K], expert_offsets [E_l + 1], expert_counts [E_l],
    // recv_src_idx, aligned per-expert counts (host), rank_prefix_matrix, send_prefix_matrix,
    // recv_rank_prefix, send_head).
    std::tuple<torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor,
               torch::Tensor, std::vector<int>, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor>
    intranode_dispatch_gemm(const torch::Tensor& x, const torch::Tensor& topk_idx, const torch::Tensor& topk_weights,
                            int num_experts, const torch::Tensor& w, const torch::Tensor& w_scales, bool round_scale,
                            int num_sms, int pull_ctas);
    // FP8 low-latency dispatch whose receive runs inside the first expert GEMM (masked, tcgen05):
    // returns (gemm out [E_l, slots, n] bf16, recv_x, recv_scales, recv_count, src_info, src_meta, half).
    std::tuple<torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, int>
    low_latency_dispatch_gemm(const torch::Tensor& x, const torch::Tensor& topk_idx,
                              const std::optional<torch::Tensor>& cumulative_local_expert_recv_stats,
                              int num_max_dispatch_tokens_per_rank, int num_experts, const torch::Tensor& w,
                              const torch::Tensor& w_scales, bool round_scale, int num_sms);
    // Down projection (masked grouped FP8 GEMM) whose epilogue is the low-latency combine's send, then
    // the combine's receive (weighted reduction): returns the combined [num_tokens, hidden] bf16.
    torch::Tensor low_latency_gemm_combine(const torch::Tensor& a, const torch::Tensor& a_scales, const torch::Tensor& recv_count,
                                           const torch::Tensor& w, const torch::Tensor& w_scales, const torch::Tensor& topk_idx,
                                           const torch::Tensor& topk_weights, int dispatch_half,
                                           int num_max_dispatch_tokens_per_rank, int num_experts, int num_sms);
    std::tuple<torch::Tensor, std::optional<EventHandle>, std::optional<std::function<void()>>> low_latency_combine(
        const torch::Tensor& x, const torch::Tensor& topk_idx, const torch::Tensor& topk_weights,
        const torch::Tensor& recv_count, int dispatch_half, const std::optional<torch::Tensor>& combine_wait_recv_cost_stats,
        int num_max_dispatch_tokens_per_rank, int num_experts, bool use_logfmt, bool zero_copy, bool async,
        bool return_recv_hook, const std::optional<torch::Tensor>& out);
    torch::Tensor get_next_low_latency_combine_buffer(int num_max_dispatch_tokens_per_rank, int hidden, int num_experts);
    void low_latency_update_mask_buffer(int rank_to_mask, bool mask);
    void low_latency_query_mask_buffer(const torch::Tensor& mask_status);
    void low_latency_clean_mask_buffer();

    int rank() const { return rank_; }
    int num_ranks() const { return num_ranks_; }

   private:
    CountArgs count_args(const NormalLayout& L, int N, int K, int num_experts, bool cached, int expert_alignment);
    KernelStatus status() const;
    PeerTable nvl_peers() const;
    PeerTable ll_peers() const;
    void wait_host_counters(int ticket);
    void prof_mark(cudaStream_t stream, int point);
    bool profile_enabled_ = false;
    int row_chunk_ = 0;
    int combine_row_chunk_ = -1;
    bool combine_announce_lagged_ = false;
    bool poison_outputs_ = false;  // DEEPEP_B200_POISON_OUTPUTS=1: outputs start as 0xFF bytes
    std::vector<std::pair<int, cudaEvent_t>> prof_events_;

    int rank_, num_ranks_, device_id_;
    int64_t num_nvl_bytes_, num_rdma_bytes_;
    bool low_latency_mode_, explicitly_destroy_, enable_shrink_;
    bool available_ = false, destroyed_ = false;
    uint64_t timeout_ns_;

    void* nvl_base_ = nullptr;
    void* ll_base_ = nullptr;
    cudaIpcMemHandle_t nvl_ipc_{}, ll_ipc_{};
    void* nvl_peer_[kMaxRanks] = {};
    void* ll_peer_[kMaxRanks] = {};
    bool nvl_peer_opened_[kMaxRanks] = {};
    bool ll_peer_opened_[kMaxRanks] = {};

    // host-mapped error page and counters
    ErrorState* host_error_ = nullptr;
    ErrorState* host_error_dev_ = nullptr;
    HostCounters* host_counters_ = nullptr;
    HostCounters* host_counters_dev_ = nullptr;
    int* dev_workspace_ = nullptr;  // [0] abort flag, [1] num_recv, [2..] scratch
    int* mask_ = nullptr;           // [kMaxRanks] shrink-mode mask
    TraceRing* trace_dev_ = nullptr;
    TraceRecord* trace_records_ = nullptr;
    unsigned long long* trace_cursor_ = nullptr;
    int64_t trace_capacity_ = 0;

    at::cuda::CUDAStream comm_stream_;
    at::cuda::CUDAStream count_stream_;  // the dispatch count step, concurrent with the stage on comm_stream_
    bool stage_concurrent_ = true;       // stage as its own launch next to the count step (else: stage warps of the pull)
    bool stage_signal_gpu_scope_ = false;  // chunk counters at GPU scope (DEEPEP_B200_STAGE_SIGNAL_SCOPE=gpu)
    bool stage_writer_fence_ = true;       // writer-side async-proxy fence (DEEPEP_B200_STAGE_WRITER_FENCE=0 drops it)
    bool stage_regs_rows_ = false;         // stage rows through registers (DEEPEP_B200_STAGE_ROWS=regs)
    int dispatch_epoch_ = 0, combine_seq_ = 0, barrier_epoch_ = 0, ll_dispatch_seq_ = 0, ll_combine_seq_ = 0;
};

}  // namespace ep
