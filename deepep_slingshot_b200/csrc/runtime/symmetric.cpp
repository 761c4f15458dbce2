// Symmetric side regions: pipeline send/recv, AGRS all-gather sessions, Engram storage/fetch.
// See symmetric.hpp for the design summary.
#include "symmetric.hpp"
#include "cuda_check.hpp"

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDACachingAllocator.h>

#include <algorithm>
#include <cstring>
#include <stdexcept>
#include <string>

#include "../include/ep/schedule.cuh"
#include "../kernels/gemm.h"
#include "../include/ep/gemm_combine.cuh"
#include "../kernels/symmetric_ops.h"
#include "buffer.hpp"

namespace ep {


namespace {

int64_t align_to(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

}  // namespace

SymmetricRegion::SymmetricRegion(int rank, int num_ranks, int64_t data_bytes, double timeout_s)
    : rank_(rank), num_ranks_(num_ranks), data_bytes_(align_to(std::max<int64_t>(data_bytes, 16), 128)),
      timeout_s_(timeout_s), copy_stream_(at::cuda::getStreamFromPool(true)) {
    TORCH_CHECK(num_ranks >= 1 && num_ranks <= kMaxRanks, "SymmetricRegion: 1..8 ranks on one NVLink domain");
    TORCH_CHECK(rank >= 0 && rank < num_ranks);
    EP_CUDA_CHECK(cudaGetDevice(&device_id_));
    const int64_t total = kSymCtrlBytes + data_bytes_;
    EP_CUDA_CHECK(cudaMalloc(&base_, total));
    EP_CUDA_CHECK(cudaMemset(base_, 0, total));
    EP_CUDA_CHECK(cudaIpcGetMemHandle(&ipc_, base_));
    EP_CUDA_CHECK(cudaHostAlloc(reinterpret_cast<void**>(&host_error_), sizeof(ErrorState), cudaHostAllocMapped));
    std::memset(host_error_, 0, sizeof(ErrorState));
    EP_CUDA_CHECK(cudaHostGetDevicePointer(reinterpret_cast<void**>(&host_error_dev_), host_error_, 0));
    EP_CUDA_CHECK(cudaMalloc(&abort_flag_, sizeof(int)));
    EP_CUDA_CHECK(cudaMemset(abort_flag_, 0, sizeof(int)));
    EP_CUDA_CHECK(cudaDeviceSynchronize());
    peer_[rank_] = base_;
}

SymmetricRegion::~SymmetricRegion() {
    try {
        destroy();
    } catch (...) {
    }
}

pybind11::bytes SymmetricRegion::get_local_ipc_handle() const {
    return pybind11::bytes(reinterpret_cast<const char*>(&ipc_), sizeof(ipc_));
}

void SymmetricRegion::sync(const std::vector<pybind11::bytes>& handles) {
    TORCH_CHECK((int)handles.size() == num_ranks_, "one IPC handle per rank");
    for (int r = 0; r < num_ranks_; ++r) {
        if (r == rank_) continue;
        const std::string h = handles[r];
        TORCH_CHECK(h.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
        cudaIpcMemHandle_t ipc;
        std::memcpy(&ipc, h.data(), sizeof(ipc));
        EP_CUDA_CHECK(cudaIpcOpenMemHandle(&peer_[r], ipc, cudaIpcMemLazyEnablePeerAccess));
        peer_opened_[r] = true;
    }
    available_ = true;
}

void SymmetricRegion::destroy() {
    if (destroyed_) return;
    destroyed_ = true;
    available_ = false;
    cudaDeviceSynchronize();
    for (int r = 0; r < num_ranks_; ++r)
        if (peer_opened_[r]) cudaIpcCloseMemHandle(peer_[r]);
    if (base_) cudaFree(base_);
    if (abort_flag_) cudaFree(abort_flag_);
    if (host_error_) cudaFreeHost(host_error_);
    base_ = nullptr;
    abort_flag_ = nullptr;
    host_error_ = nullptr;
}

void SymmetricRegion::require_available() const {
    TORCH_CHECK(available_, "SymmetricRegion is not synced (or was destroyed)");
}

torch::Tensor SymmetricRegion::local_data(int64_t offset, int64_t bytes) const {
    require_available();
    TORCH_CHECK(offset >= 0 && bytes >= 0 && offset + bytes <= data_bytes_);
    return torch::from_blob(data_of(rank_) + offset, {bytes}, torch::dtype(torch::kUInt8).device(torch::kCUDA, device_id_));
}

KernelStatus SymmetricRegion::status() const {
    KernelStatus s{};
    s.host_error = host_error_dev_;
    s.abort_flag = abort_flag_;
    s.timeout_ns = (uint64_t)(timeout_s_ * 1e9);
    s.rank = rank_;
    return s;
}

void SymmetricRegion::check_error() const {
    if (host_error_ == nullptr) return;
    const int code = *reinterpret_cast<volatile int*>(&host_error_->code);
    if (code != 0)
        throw std::runtime_error("B200 EP symmetric-region error on rank " + std::to_string(host_error_->rank) + ": " +
                                 error_name(code) + " (code " + std::to_string(code) + ", peer " +
                                 std::to_string(host_error_->peer) + ", detail " + std::to_string(host_error_->detail) + ")");
}

std::tuple<int, int, int, int> SymmetricRegion::get_error_state() const {
    if (host_error_ == nullptr) return {0, 0, 0, 0};
    return {host_error_->code, host_error_->peer, host_error_->detail, host_error_->rank};
}

void SymmetricRegion::clear_error() {
    EP_CUDA_CHECK(cudaDeviceSynchronize());
    if (host_error_) std::memset(host_error_, 0, sizeof(ErrorState));
    if (abort_flag_) EP_CUDA_CHECK(cudaMemset(abort_flag_, 0, sizeof(int)));
    EP_CUDA_CHECK(cudaDeviceSynchronize());
}

void SymmetricRegion::barrier() {
    require_available();
    SignalWaitArgs a{};
    a.value = ++barrier_epoch_;
    for (int r = 0; r < num_ranks_; ++r) {
        if (r == rank_) continue;
        a.write[a.num_writes++] = &ctrl_of(r)->barrier_signal[rank_];
        a.wait_peer[a.num_waits] = r;
        a.wait[a.num_waits++] = &ctrl_of(rank_)->barrier_signal[r];
    }
    a.code = kErrTimeoutAgrs;
    a.st = status();
    auto stream = at::cuda::getCurrentCUDAStream();
    launch_signal_wait(a, stream);
    EP_CUDA_CHECK(cudaGetLastError());
    EP_CUDA_CHECK(cudaStreamSynchronize(stream));
    check_error();
}

// ------------------------------------------------------------------------------------------------
// Pipeline ring
// ------------------------------------------------------------------------------------------------
void SymmetricRegion::pp_set_config(int64_t num_max_tensor_bytes, int num_max_inflight_tensors) {
    require_available();
    TORCH_CHECK(num_max_tensor_bytes > 0 && num_max_inflight_tensors > 0);
    const int64_t slot = align_to(num_max_tensor_bytes, 128);
    TORCH_CHECK(2 * slot * num_max_inflight_tensors <= data_bytes_, "pipeline slots exceed the region");
    barrier();
    pp_max_bytes_ = slot;
    pp_inflight_ = num_max_inflight_tensors;
}

void SymmetricRegion::pp_send(const torch::Tensor& x, int dst_rank, int num_sms) {
    require_available();
    check_error();
    TORCH_CHECK(pp_inflight_ > 0, "call pp_set_config first");
    TORCH_CHECK(x.is_cuda() && x.is_contiguous() && (int64_t)x.nbytes() <= pp_max_bytes_, "pp_send: tensor too large or not contiguous");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0, "pp_send: tensor must be 16-byte aligned");
    const int prev = (rank_ + num_ranks_ - 1) % num_ranks_, next = (rank_ + 1) % num_ranks_;
    TORCH_CHECK(dst_rank == prev || dst_rank == next, "pp_send: destination must be the previous or next rank");
    const int ds = ring_dir(rank_, dst_rank, num_ranks_), dr = ring_dir(dst_rank, rank_, num_ranks_);
    PPArgs a{};
    a.x = static_cast<uint8_t*>(x.data_ptr());
    a.slots = data_of(dst_rank) + (int64_t)dr * pp_inflight_ * pp_max_bytes_;
    a.bytes = (int64_t)x.nbytes();
    a.slot_bytes = pp_max_bytes_;
    a.inflight = pp_inflight_;
    a.is_send = 1;
    a.peer = dst_rank;
    a.count = &ctrl_of(rank_)->pp_send_count[ds];
    a.wait_flag = &ctrl_of(rank_)->pp_release[ds];
    a.signal_flag = &ctrl_of(dst_rank)->pp_arrival[dr];
    a.ticket = &ctrl_of(rank_)->pp_send_ticket[ds];
    a.st = status();
    const int blocks = (int)std::min<int64_t>(num_sms > 0 ? num_sms : 32, std::max<int64_t>(1, (a.bytes + 65535) / 65536));
    launch_pp_copy(a, blocks, at::cuda::getCurrentCUDAStream());
    EP_CUDA_CHECK(cudaGetLastError());
}

void SymmetricRegion::pp_recv(const torch::Tensor& x, int src_rank, int num_sms) {
    require_available();
    check_error();
    TORCH_CHECK(pp_inflight_ > 0, "call pp_set_config first");
    TORCH_CHECK(x.is_cuda() && x.is_contiguous() && (int64_t)x.nbytes() <= pp_max_bytes_, "pp_recv: tensor too large or not contiguous");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0, "pp_recv: tensor must be 16-byte aligned");
    const int prev = (rank_ + num_ranks_ - 1) % num_ranks_, next = (rank_ + 1) % num_ranks_;
    TORCH_CHECK(src_rank == prev || src_rank == next, "pp_recv: source must be the previous or next rank");
    const int dr = ring_dir(rank_, src_rank, num_ranks_), ds = ring_dir(src_rank, rank_, num_ranks_);
    PPArgs a{};
    a.x = static_cast<uint8_t*>(x.data_ptr());
    a.slots = data_of(rank_) + (int64_t)dr * pp_inflight_ * pp_max_bytes_;
    a.bytes = (int64_t)x.nbytes();
    a.slot_bytes = pp_max_bytes_;
    a.inflight = pp_inflight_;
    a.is_send = 0;
    a.peer = src_rank;
    a.count = &ctrl_of(rank_)->pp_recv_count[dr];
    a.wait_flag = &ctrl_of(rank_)->pp_arrival[dr];
    a.signal_flag = &ctrl_of(src_rank)->pp_release[ds];
    a.ticket = &ctrl_of(rank_)->pp_recv_ticket[dr];
    a.st = status();
    const int blocks = (int)std::min<int64_t>(num_sms > 0 ? num_sms : 32, std::max<int64_t>(1, (a.bytes + 65535) / 65536));
    launch_pp_copy(a, blocks, at::cuda::getCurrentCUDAStream());
    EP_CUDA_CHECK(cudaGetLastError());
}

// ------------------------------------------------------------------------------------------------
// AGRS: all-gather sessions on the copy engines
// ------------------------------------------------------------------------------------------------
void SymmetricRegion::agrs_set_config(int64_t num_max_session_bytes, int num_max_all_gathers_per_session) {
    require_available();
    TORCH_CHECK(num_max_session_bytes > 0 && num_max_all_gathers_per_session > 0);
    TORCH_CHECK(num_max_session_bytes <= data_bytes_, "AGRS session bytes exceed the region");
    TORCH_CHECK(num_max_all_gathers_per_session <= kMaxAgrsSlots, "at most 64 all-gathers per session");
    TORCH_CHECK(!agrs_in_session_, "agrs_set_config inside a session");
    barrier();
    agrs_session_bytes_ = align_to(num_max_session_bytes, 32);
    agrs_max_per_session_ = num_max_all_gathers_per_session;
}

void SymmetricRegion::create_agrs_session() {
    TORCH_CHECK(agrs_max_per_session_ > 0, "call agrs_set_config first");
    TORCH_CHECK(!agrs_in_session_, "an AGRS session is already open");
    agrs_in_session_ = true;
    agrs_offset_ = 0;
    agrs_slot_ = 0;
    agrs_session_ += 1;
}

void SymmetricRegion::destroy_agrs_session() {
    TORCH_CHECK(agrs_in_session_, "no AGRS session is open");
    agrs_in_session_ = false;
    // Everything the compute stream does with this session's buffer precedes the session-end signal;
    // a peer's next-session copies into my buffer wait for it on that peer's copy stream.
    auto compute = at::cuda::getCurrentCUDAStream();
    at::cuda::CUDAEvent ev;
    ev.record(compute);
    ev.block(copy_stream_);
    SignalWaitArgs a{};
    a.value = agrs_session_;
    for (int r = 0; r < num_ranks_; ++r) {
        if (r == rank_) continue;
        a.write[a.num_writes++] = &ctrl_of(r)->agrs_session_signal[rank_];
        a.wait_peer[a.num_waits] = r;
        a.wait[a.num_waits++] = &ctrl_of(rank_)->agrs_session_signal[r];
    }
    a.code = kErrTimeoutAgrs;
    a.st = status();
    launch_signal_wait(a, copy_stream_.stream());
    EP_CUDA_CHECK(cudaGetLastError());
}

std::vector<torch::Tensor> SymmetricRegion::agrs_get_inplace_tensor(const std::vector<int64_t>& num_bytes_list) {
    TORCH_CHECK(agrs_in_session_, "agrs_get_inplace_tensor needs an open AGRS session");
    TORCH_CHECK(!num_bytes_list.empty());
    std::vector<torch::Tensor> out;
    int64_t offset = agrs_offset_;
    for (const int64_t nb : num_bytes_list) {
        TORCH_CHECK(nb > 0 && offset + nb * num_ranks_ <= agrs_session_bytes_ && agrs_slot_ < agrs_max_per_session_,
                    "not enough AGRS session buffer (close the session to recycle it)");
        out.push_back(local_data(offset + nb * rank_, nb));
        offset += align_to(nb * num_ranks_, 32);
    }
    return out;
}

std::pair<std::vector<torch::Tensor>, std::function<void()>>
SymmetricRegion::all_gather(const std::vector<torch::Tensor>& tensors) {
    require_available();
    check_error();
    TORCH_CHECK(agrs_in_session_, "all_gather needs an open AGRS session");
    TORCH_CHECK(!tensors.empty());
    TORCH_CHECK(agrs_slot_ < agrs_max_per_session_, "too many all-gathers in this AGRS session");
    const int n = (int)tensors.size();
    std::vector<int64_t> offsets(n);
    int64_t cursor = agrs_offset_;
    for (int j = 0; j < n; ++j) {
        const auto& x = tensors[j];
        TORCH_CHECK(x.is_cuda() && x.is_contiguous() && x.nbytes() > 0, "all_gather: contiguous CUDA tensors");
        offsets[j] = cursor;
        cursor += align_to((int64_t)x.nbytes() * num_ranks_, 32);
        const uint8_t* p = static_cast<const uint8_t*>(x.data_ptr());
        const uint8_t* d0 = data_of(rank_);
        if (p >= d0 && p < d0 + agrs_session_bytes_)
            TORCH_CHECK(p == d0 + offsets[j] + (int64_t)x.nbytes() * rank_,
                        "an in-place AGRS tensor must be used by the all_gather that follows its allocation");
    }
    TORCH_CHECK(cursor <= agrs_session_bytes_, "not enough AGRS session buffer (close the session to recycle it)");
    agrs_offset_ = cursor;
    const int slot = agrs_slot_++;

    auto compute = at::cuda::getCurrentCUDAStream();
    at::cuda::CUDAEvent ready;
    ready.record(compute);
    ready.block(copy_stream_);
    // One copy-engine memcpy per (destination rank, tensor), starting with the next rank.
    for (int i = 0; i < num_ranks_; ++i) {
        const int r = (rank_ + i) % num_ranks_;
        for (int j = 0; j < n; ++j) {
            const auto& x = tensors[j];
            uint8_t* dst = data_of(r) + offsets[j] + (int64_t)x.nbytes() * rank_;
            if (dst == static_cast<const uint8_t*>(x.data_ptr())) continue;
            EP_CUDA_CHECK(cudaMemcpyAsync(dst, x.data_ptr(), x.nbytes(), cudaMemcpyDefault, copy_stream_.stream()));
        }
    }
    for (const auto& x : tensors) c10::cuda::CUDACachingAllocator::recordStream(x.storage().data_ptr(), copy_stream_);
    SignalWaitArgs a{};
    a.value = agrs_session_;
    for (int r = 0; r < num_ranks_; ++r) {
        if (r == rank_) continue;
        a.write[a.num_writes++] = &ctrl_of(r)->agrs_recv_signal[slot][rank_];
        a.wait_peer[a.num_waits] = r;
        a.wait[a.num_waits++] = &ctrl_of(rank_)->agrs_recv_signal[slot][r];
    }
    a.code = kErrTimeoutAgrs;
    a.st = status();
    launch_signal_wait(a, copy_stream_.stream());
    EP_CUDA_CHECK(cudaGetLastError());
    auto done = std::make_shared<at::cuda::CUDAEvent>();
    done->record(copy_stream_);

    std::vector<torch::Tensor> out;
    for (int j = 0; j < n; ++j) out.push_back(local_data(offsets[j], (int64_t)tensors[j].nbytes() * num_ranks_));
    auto hook = [done]() { done->block(at::cuda::getCurrentCUDAStream()); };
    return {out, hook};
}

// ------------------------------------------------------------------------------------------------
// Engram
// ------------------------------------------------------------------------------------------------
void SymmetricRegion::engram_write(const torch::Tensor& storage) {
    require_available();
    TORCH_CHECK(storage.is_cuda() && storage.is_contiguous() && storage.dim() == 2 && storage.scalar_type() == torch::kBFloat16,
                "engram storage: contiguous [num_entries, hidden] bf16 CUDA tensor");
    TORCH_CHECK((int64_t)storage.nbytes() <= data_bytes_, "engram storage exceeds the region");
    TORCH_CHECK((storage.size(1) * 2) % 16 == 0, "engram hidden * 2 bytes must be a multiple of 16");
    barrier();  // earlier fetches by peers have finished reading the old storage
    EP_CUDA_CHECK(cudaMemcpyAsync(data_of(rank_), storage.data_ptr(), storage.nbytes(), cudaMemcpyDeviceToDevice,
                                   at::cuda::getCurrentCUDAStream()));
    barrier();  // every rank's storage is in place
    engram_entries_ = (int)storage.size(0);
    engram_hidden_ = (int)storage.size(1);
}

std::function<torch::Tensor()> SymmetricRegion::engram_fetch(const torch::Tensor& indices, int num_sms) {
    require_available();
    check_error();
    TORCH_CHECK(engram_entries_ > 0, "call engram_write first");
    TORCH_CHECK(indices.is_cuda() && indices.is_contiguous() && indices.dim() == 1 && indices.scalar_type() == torch::kInt32,
                "engram indices: contiguous [num_tokens] int32 CUDA tensor");
    const int T = (int)indices.size(0);
    auto compute = at::cuda::getCurrentCUDAStream();
    auto out = torch::empty({T, engram_hidden_}, torch::dtype(torch::kBFloat16).device(torch::kCUDA, device_id_));
    at::cuda::CUDAEvent ready;
    ready.record(compute);
    ready.block(copy_stream_);
    EngramFetchArgs a{};
    for (int r = 0; r < num_ranks_; ++r) a.storage.base[r] = data_of(r);
    a.indices = indices.data_ptr<int>();
    a.out = static_cast<uint8_t*>(out.data_ptr());
    a.num_tokens = T;
    a.entries_per_rank = engram_entries_;
    a.row_bytes = engram_hidden_ * 2;
    a.num_ranks = num_ranks_;
    a.st = status();
    launch_engram_fetch(a, num_sms > 0 ? num_sms : 148, copy_stream_.stream());
    EP_CUDA_CHECK(cudaGetLastError());
    c10::cuda::CUDACachingAllocator::recordStream(indices.storage().data_ptr(), copy_stream_);
    c10::cuda::CUDACachingAllocator::recordStream(out.storage().data_ptr(), copy_stream_);
    auto done = std::make_shared<at::cuda::CUDAEvent>();
    done->record(copy_stream_);
    return [done, out]() {
        done->block(at::cuda::getCurrentCUDAStream());
        return out;
    };
}

// =================================================================================================
// Down projection -> combine
// =================================================================================================
torch::Tensor SymmetricRegion::gemm_combine_send(const torch::Tensor& a, const torch::Tensor& sa, const torch::Tensor& b,
                                                 const torch::Tensor& sb, const torch::Tensor& offsets,
                                                 const std::optional<torch::Tensor>& counts, const torch::Tensor& row_map,
                                                 const torch::Tensor& recv_src_idx, const torch::Tensor& rank_prefix_matrix,
                                                 bool keep_local, int num_sms) {
    require_available();
    check_error();
    TORCH_CHECK(!gc_pending_, "gemm_combine_send: the previous send has not been reduced (call gemm_combine_reduce)");
    TORCH_CHECK(a.is_cuda() && a.dim() == 2 && a.is_contiguous() && a.scalar_type() == torch::kFloat8_e4m3fn,
                "a must be a contiguous [rows, k] e4m3 CUDA tensor");
    TORCH_CHECK(b.is_cuda() && b.dim() == 3 && b.is_contiguous() && b.scalar_type() == torch::kFloat8_e4m3fn,
                "b must be a contiguous [experts, n, k] e4m3 CUDA tensor");
    const int rows = (int)a.size(0), k = (int)a.size(1), E = (int)b.size(0), n = (int)b.size(1);
    TORCH_CHECK(rows > 0 && b.size(2) == k && k % 128 == 0 && n % 128 == 0, "k and n must be multiples of 128");
    TORCH_CHECK(sa.scalar_type() == torch::kFloat32 && sa.is_contiguous() && sa.dim() == 2 && sa.size(0) == rows &&
                    sa.size(1) == k / 128,
                "sa must be contiguous [rows, k/128] fp32");
    TORCH_CHECK(sb.scalar_type() == torch::kFloat32 && sb.is_contiguous() && sb.dim() == 3 && sb.size(0) == E &&
                    sb.size(1) == n / 128 && sb.size(2) == k / 128,
                "sb must be contiguous [experts, n/128, k/128] fp32");
    TORCH_CHECK(offsets.scalar_type() == torch::kInt32 && offsets.is_contiguous() && offsets.numel() == E + 1,
                "offsets must be [experts + 1] int32");
    if (counts.has_value())
        TORCH_CHECK(counts->scalar_type() == torch::kInt32 && counts->is_contiguous() && counts->numel() == E,
                    "counts must be [experts] int32");
    TORCH_CHECK(row_map.is_cuda() && row_map.scalar_type() == torch::kInt32 && row_map.dim() == 2 && row_map.is_contiguous(),
                "row_map must be the permute's contiguous [received tokens, top-k] int32 map");
    const int num_recv = (int)row_map.size(0), K = (int)row_map.size(1);
    TORCH_CHECK(K >= 1 && K <= 32, "top-k must be 1..32");
    TORCH_CHECK(recv_src_idx.scalar_type() == torch::kInt32 && recv_src_idx.is_contiguous() && recv_src_idx.numel() == num_recv,
                "recv_src_idx must be the dispatch handle's [received tokens] int32 source indices");
    TORCH_CHECK(rank_prefix_matrix.scalar_type() == torch::kInt32 && rank_prefix_matrix.is_contiguous() &&
                    rank_prefix_matrix.numel() == (int64_t)num_ranks_ * num_ranks_,
                "rank_prefix_matrix must be the dispatch handle's [ranks, ranks] int32 matrix");
    const int64_t slots = std::min<int64_t>(data_bytes_ / ((int64_t)n * 2), kGcMaxSlots);
    TORCH_CHECK(slots > 0, "the region holds no row of this hidden size");
    if (num_sms <= 0) EP_CUDA_CHECK(cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, device_id_));

    auto stream = at::cuda::getCurrentCUDAStream();
    auto i32 = torch::dtype(torch::kInt32).device(torch::kCUDA, device_id_);
    auto row_dest = torch::full({rows}, -1, i32);
    GcRowDestArgs ra{};
    ra.row_map = row_map.data_ptr<int>();
    ra.recv_src_idx = recv_src_idx.data_ptr<int>();
    ra.rank_prefix_matrix = rank_prefix_matrix.data_ptr<int>();
    ra.row_dest = row_dest.data_ptr<int>();
    ra.num_recv = num_recv;
    ra.num_topk = K;
    ra.rows = rows;
    ra.rank = rank_;
    ra.num_ranks = num_ranks_;
    ra.slots = slots;
    ra.st = status();
    launch_gc_row_dest(ra, stream);
    EP_CUDA_CHECK(cudaGetLastError());

    torch::Tensor y = keep_local ? torch::empty({rows, n}, a.options().dtype(torch::kBFloat16))
                                 : torch::empty({0, n}, a.options().dtype(torch::kBFloat16));
    GemmArgs g{};
    g.a = a.data_ptr();
    g.sa = sa.data_ptr<float>();
    g.b = b.data_ptr();
    g.sb = sb.data_ptr<float>();
    g.offsets = offsets.data_ptr<int>();
    g.expert_counts = counts.has_value() ? counts->data_ptr<int>() : nullptr;
    g.d = keep_local ? y.data_ptr() : nullptr;
    g.rows = rows;
    g.n = n;
    g.k = k;
    g.num_experts = E;
    g.row_dest = row_dest.data_ptr<int>();
    for (int r = 0; r < num_ranks_; ++r) g.gc_regions.base[r] = peer_[r];
    g.gc_rank = rank_;
    g.gc_num_ranks = num_ranks_;
    g.gc_epoch = gc_epoch_ + 1;
    g.gc_slots = slots;
    g.st = status();
    const int rc = launch_grouped_gemm_fp8(g, num_sms, stream);
    TORCH_CHECK(rc == 0, "gemm_combine_send: GEMM launch failed (code " + std::to_string(rc) + ")");
    ++gc_epoch_;
    gc_hidden_ = n;
    gc_topk_ = K;
    gc_pending_ = true;
    return y;
}

torch::Tensor SymmetricRegion::gemm_combine_reduce(const torch::Tensor& topk_idx, const std::optional<torch::Tensor>& topk_weights,
                                                   int num_sms) {
    require_available();
    check_error();
    TORCH_CHECK(gc_pending_, "gemm_combine_reduce: no gemm_combine_send to reduce");
    TORCH_CHECK(topk_idx.is_cuda() && topk_idx.dim() == 2 && topk_idx.is_contiguous() && topk_idx.scalar_type() == torch::kInt64,
                "topk_idx must be this rank's contiguous [tokens, top-k] int64 routing");
    const int N = (int)topk_idx.size(0), K = (int)topk_idx.size(1);
    TORCH_CHECK(K == gc_topk_, "top-k differs from the send's row map");
    if (topk_weights.has_value())
        TORCH_CHECK(topk_weights->scalar_type() == torch::kFloat32 && topk_weights->is_contiguous() && topk_weights->dim() == 2 &&
                        topk_weights->size(0) == N && topk_weights->size(1) == K,
                    "topk_weights must be contiguous [tokens, top-k] fp32");
    const int64_t slots = std::min<int64_t>(data_bytes_ / ((int64_t)gc_hidden_ * 2), kGcMaxSlots);
    TORCH_CHECK((int64_t)N * K <= slots, "more tokens x top-k than the region's slots");
    if (num_sms <= 0) EP_CUDA_CHECK(cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, device_id_));
    auto out = torch::empty({N, gc_hidden_}, torch::dtype(torch::kBFloat16).device(torch::kCUDA, device_id_));
    GcReduceArgs r{};
    for (int q = 0; q < num_ranks_; ++q) r.regions.base[q] = peer_[q];
    r.rank = rank_;
    r.num_ranks = num_ranks_;
    r.epoch = gc_epoch_;
    r.topk_idx = topk_idx.data_ptr<int64_t>();
    r.topk_weights = topk_weights.has_value() ? topk_weights->data_ptr<float>() : nullptr;
    r.out = out.data_ptr();
    r.num_tokens = N;
    r.num_topk = K;
    r.hidden = gc_hidden_;
    r.slots = slots;
    r.st = status();
    launch_gc_reduce(r, num_sms, at::cuda::getCurrentCUDAStream());
    EP_CUDA_CHECK(cudaGetLastError());
    gc_pending_ = false;
    return out;
}

}  // namespace ep
