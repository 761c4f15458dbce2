// Symmetric side regions of the elastic (v2) API: pipeline send/recv between ring neighbours,
// all-gather sessions on the copy engines (AGRS) and Engram row storage/fetch.
//
// Reference: `ElasticBuffer::{pp_*, agrs_*, all_gather, engram_*}` ([DE]csrc/elastic/buffer.hpp:
// 212-470), which carve these out of one NCCL symmetric window and use GIN puts/gets and driver
// stream memory operations. Here every feature gets its own CUDA-IPC region ([SymCtrl | data]),
// allocated when the feature is configured (a collective call in the reference too), so features
// never alias each other's bytes. Transfers: PP = TMA stores into the neighbour's slot; AGRS = one
// cudaMemcpyAsync per (peer, tensor) on the region's copy stream; Engram = peer loads by the
// fetching GPU. Signals are bounded-wait kernels that report into a host-mapped error page.
#pragma once

#include <ATen/cuda/CUDAContext.h>
#include <ATen/cuda/CUDAEvent.h>
#include <c10/cuda/CUDAStream.h>
#include <pybind11/functional.h>
#include <pybind11/pybind11.h>
#include <torch/extension.h>

#include <functional>
#include <memory>
#include <optional>
#include <tuple>
#include <vector>

#include "../include/ep/abi.h"

namespace ep {

class SymmetricRegion {
public:
    // `data_bytes` of payload after the 64 KiB control block; `timeout_s` bounds every device wait.
    SymmetricRegion(int rank, int num_ranks, int64_t data_bytes, double timeout_s);
    ~SymmetricRegion();

    pybind11::bytes get_local_ipc_handle() const;
    int get_local_device_id() const { return device_id_; }
    // Open every peer's region (handles indexed by rank; the local entry is ignored).
    void sync(const std::vector<pybind11::bytes>& handles);
    bool is_available() const { return available_; }
    void destroy();
    int64_t data_bytes() const { return data_bytes_; }
    torch::Tensor local_data(int64_t offset, int64_t bytes) const;

    void check_error() const;
    std::tuple<int, int, int, int> get_error_state() const;
    void clear_error();
    // All ranks: write my epoch into every peer, wait for theirs (bounded, on the current stream).
    void barrier();

    // ---- pipeline ring (prev / next neighbour only)
    void pp_set_config(int64_t num_max_tensor_bytes, int num_max_inflight_tensors);
    void pp_send(const torch::Tensor& x, int dst_rank, int num_sms);
    void pp_recv(const torch::Tensor& x, int src_rank, int num_sms);

    // ---- all-gather sessions on the copy engines
    void agrs_set_config(int64_t num_max_session_bytes, int num_max_all_gathers_per_session);
    void create_agrs_session();
    void destroy_agrs_session();
    std::vector<torch::Tensor> agrs_get_inplace_tensor(const std::vector<int64_t>& num_bytes_list);
    std::pair<std::vector<torch::Tensor>, std::function<void()>> all_gather(const std::vector<torch::Tensor>& tensors);

    // ---- Engram storage (bf16 rows) and fetch by global entry index
    void engram_write(const torch::Tensor& storage);
    std::function<torch::Tensor()> engram_fetch(const torch::Tensor& indices, int num_sms);

    // ---- down projection with the combine send as its epilogue (normal-mode MoE layer)
    // Receiver side: the grouped FP8 GEMM y = a b_e^T (fp32 block scales) whose epilogue stores every
    // row of (received token j, k) into slot (recv_src_idx[j], k) of j's source rank over NVLink.
    // Returns y when `keep_local` (an empty tensor otherwise). Collective: every rank sends, then
    // every rank reduces, in the same order (epochs are host counters, so not graph-replayable).
    torch::Tensor gemm_combine_send(const torch::Tensor& a, const torch::Tensor& sa, const torch::Tensor& b,
                                    const torch::Tensor& sb, const torch::Tensor& offsets,
                                    const std::optional<torch::Tensor>& counts, const torch::Tensor& row_map,
                                    const torch::Tensor& recv_src_idx, const torch::Tensor& rank_prefix_matrix,
                                    bool keep_local, int num_sms);
    // Source side: out [tokens, hidden] bf16 = sum over k with topk_idx >= 0 of weight * slot (t, k),
    // in fp32, once every rank's rows of the last send have landed.
    torch::Tensor gemm_combine_reduce(const torch::Tensor& topk_idx, const std::optional<torch::Tensor>& topk_weights,
                                      int num_sms);

private:
    KernelStatus status() const;
    SymCtrl* ctrl_of(int r) const { return static_cast<SymCtrl*>(peer_[r]); }
    uint8_t* data_of(int r) const { return static_cast<uint8_t*>(peer_[r]) + kSymCtrlBytes; }
    void require_available() const;

    int rank_, num_ranks_, device_id_ = 0;
    int64_t data_bytes_;
    double timeout_s_;
    bool available_ = false, destroyed_ = false;
    void* base_ = nullptr;
    void* peer_[kMaxRanks] = {};
    bool peer_opened_[kMaxRanks] = {};
    cudaIpcMemHandle_t ipc_{};
    ErrorState* host_error_ = nullptr;
    ErrorState* host_error_dev_ = nullptr;
    int* abort_flag_ = nullptr;
    at::cuda::CUDAStream copy_stream_;
    int barrier_epoch_ = 0;
    int gc_epoch_ = 0, gc_hidden_ = 0, gc_topk_ = 0;
    bool gc_pending_ = false;  // a send awaits its reduce

    // pipeline
    int64_t pp_max_bytes_ = 0;
    int pp_inflight_ = 0;
    // AGRS (host-side session state; a session is driven by the host, it is not graph-replayable)
    int64_t agrs_session_bytes_ = 0;
    int agrs_max_per_session_ = 0;
    bool agrs_in_session_ = false;
    int64_t agrs_offset_ = 0;
    int agrs_slot_ = 0;
    int agrs_session_ = 0;
    // Engram
    int engram_entries_ = 0;
    int engram_hidden_ = 0;
};

}  // namespace ep
