// C++ runtime of the B200 expert-parallel buffer. See buffer.hpp for the design summary.
#include "buffer.hpp"
#include "cuda_check.hpp"
#include "../kernels/gemm.h"

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/python.h>

#include <chrono>
#include <cstring>
#include <stdexcept>
#include <thread>
#include <cstdlib>

namespace ep {


namespace {

constexpr int64_t kAlign = 128;
constexpr int64_t kCtrlRegionMin = 2 << 20;  // control block always present (barriers)

int64_t align_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

void stream_wait(const at::cuda::CUDAStream& waiter, const at::cuda::CUDAStream& signaler) {
    if (waiter == signaler) return;
    at::cuda::CUDAEvent ev;
    ev.record(signaler);
    ev.block(waiter);
}

// The reference's stream discipline ([DE]csrc/legacy/buffer.hpp:337-404): kernels run on the comm
// stream, which first waits for `previous_event` (or the current stream); outputs may be allocated
// on the comm stream; with `async` an event is returned and tensors are recorded on the comm stream,
// otherwise the current stream waits for the comm stream.
struct StreamScope {
    at::cuda::CUDAStream compute;
    at::cuda::CUDAStream comm;
    bool alloc_on_comm;
    StreamScope(const at::cuda::CUDAStream& comm_stream, std::optional<EventHandle>& previous_event, bool allocate_on_comm_stream)
        : compute(at::cuda::getCurrentCUDAStream()), comm(comm_stream), alloc_on_comm(allocate_on_comm_stream) {
        if (previous_event.has_value()) previous_event->event->block(comm);
        else stream_wait(comm, compute);
        if (alloc_on_comm) at::cuda::setCurrentCUDAStream(comm);
    }
    std::optional<EventHandle> finish(bool async, std::initializer_list<std::optional<torch::Tensor>> tensors) {
        std::optional<EventHandle> event;
        if (async) {
            event = EventHandle(comm);
            for (const auto& t : tensors)
                if (t.has_value() && t->defined()) t->record_stream(comm);
        } else {
            stream_wait(compute, comm);
        }
        if (alloc_on_comm) at::cuda::setCurrentCUDAStream(compute);
        return event;
    }
};

// Fill a tensor's bytes with 0xFF on `stream` (the poison of DEEPEP_B200_POISON_OUTPUTS).
void poison(const torch::Tensor& t, cudaStream_t stream) {
    if (t.numel() > 0) EP_CUDA_CHECK(cudaMemsetAsync(t.data_ptr(), 0xFF, t.numel() * t.element_size(), stream));
}

}  // namespace

const char* error_name(int code) {
    switch (code) {
        case kErrTimeoutNotify: return "timeout waiting for a peer's dispatch counts (count step)";
        case kErrTimeoutStaged: return "timeout waiting for a source to stage the tokens being pulled";
        case kErrTimeoutPullDone: return "timeout waiting for receivers to finish reading the staging area";
        case kErrTimeoutCombineReady: return "timeout waiting for a destination to finish its previous combine";
        case kErrTimeoutCombineArrive: return "timeout waiting for combine contributions to arrive";
        case kErrTimeoutBarrier: return "timeout in the NVLink barrier";
        case kErrTimeoutLLDispatch: return "timeout in low-latency dispatch receive";
        case kErrTimeoutLLCombine: return "timeout in low-latency combine receive";
        case kErrTimeoutTma: return "timeout waiting for a TMA bulk copy";
        case kErrCapacity: return "receive capacity exceeded";
        case kErrBounds: return "index out of bounds in a peer window";
        case kErrBadArgs: return "bad kernel arguments";
        case kErrTimeoutPP: return "timeout in pipeline-parallel send/recv";
        case kErrTimeoutAgrs: return "timeout waiting for a peer's AGRS signal or region barrier";
        case kErrTimeoutTest: return "transport self-test wait expired";
        default: return "unknown error";
    }
}


// =================================================================================================
// Config / layouts
// =================================================================================================
RecordFormat record_format(int hidden, int num_topk, bool fp8) {
    RecordFormat r{};
    const int topk_pad = (int)align_up(num_topk, 4);
    r.x_bytes = fp8 ? hidden : hidden * 2;
    r.scale_off = r.x_bytes;
    r.scale_bytes = fp8 ? (int)align_up((int64_t)(hidden / 128) * 4, 16) : 0;
    r.idx_off = r.scale_off + r.scale_bytes;
    r.w_off = r.idx_off + topk_pad * 4;
    r.bytes = r.w_off + topk_pad * 4;
    return r;
}

static int64_t normal_bytes_per_token(int hidden, int num_ranks, int* record_stride) {
    const RecordFormat bf = record_format(hidden, kMaxTopk, false);
    const RecordFormat f8 = record_format(hidden, kMaxTopk, true);
    const int rec = (int)align_up(std::max(bf.bytes, f8.bytes), kAlign);
    if (record_stride) *record_stride = rec;
    return (int64_t)num_ranks * 4 + rec + (int64_t)num_ranks * hidden * 2 + (int64_t)num_ranks * kMaxTopk * 4 + 1 + 4;
}

NormalLayout compute_normal_layout(int64_t region_bytes, int hidden, int num_ranks) {
    NormalLayout l{};
    int rec = 0;
    const int64_t per_token = normal_bytes_per_token(hidden, num_ranks, &rec);
    const int64_t ctrl = align_up(sizeof(NormalCtrl), 4096);
    const int64_t slack = 8 * kAlign + (int64_t)kMaxExperts * 4;
    int64_t cap = region_bytes > ctrl + slack ? (region_bytes - ctrl - slack) / per_token : 0;
    cap = cap / 32 * 32;
    l.capacity = (int32_t)std::min<int64_t>(cap, 1 << 24);
    l.hidden = hidden;
    l.num_topk = kMaxTopk;
    l.topk_pad = kMaxTopk;
    l.record_bytes = rec;
    l.num_ranks = num_ranks;
    l.ctrl_off = 0;
    l.list_off = ctrl;
    l.staging_off = align_up(l.list_off + (int64_t)num_ranks * l.capacity * 4, kAlign);
    l.combine_off = align_up(l.staging_off + (int64_t)l.capacity * rec, kAlign);
    l.combine_w_off = align_up(l.combine_off + (int64_t)l.capacity * num_ranks * hidden * 2, kAlign);
    l.scratch_off = align_up(l.combine_w_off + (int64_t)l.capacity * num_ranks * kMaxTopk * 4, kAlign);
    l.arrival_off = align_up(l.scratch_off + align_up(l.capacity, kAlign) + (int64_t)kMaxExperts * 4, kAlign);
    l.total_bytes = align_up(l.arrival_off + (int64_t)l.capacity * 4, kAlign);
    return l;
}

int64_t normal_region_size_for(int num_max_tokens, int hidden, int num_ranks) {
    const int64_t per_token = normal_bytes_per_token(hidden, num_ranks, nullptr);
    const int64_t ctrl = align_up(sizeof(NormalCtrl), 4096);
    const int64_t tokens = align_up(num_max_tokens, 32);
    return align_up(ctrl + 8 * kAlign + tokens * per_token + 16 * kAlign + (int64_t)kMaxExperts * 4, 2 << 20);
}

LLLayout compute_ll_layout(int64_t region_bytes, int max_tokens, int hidden, int num_experts, int num_ranks) {
    LLLayout l{};
    const int64_t E_l = num_experts / num_ranks;
    const int64_t slots = (int64_t)num_ranks * max_tokens;
    const int64_t nb = hidden / 128;
    l.max_tokens = max_tokens;
    l.hidden = hidden;
    l.num_experts = num_experts;
    l.num_local_experts = (int)E_l;
    l.num_ranks = num_ranks;
    l.num_topk = kMaxTopk;
    int64_t off = 0;
    l.ctrl_off = off;
    off = align_up(off + sizeof(LLCtrl), kAlign);
    l.recv_x_off = off;
    off = align_up(off + E_l * slots * hidden * 2, kAlign);
    l.recv_scales_off = off;
    off = align_up(off + E_l * nb * slots * 4, kAlign);
    l.recv_src_info_off = off;
    off = align_up(off + E_l * slots * 4, kAlign);
    l.recv_src_meta_off = off;
    off = align_up(off + E_l * slots * 4, kAlign);
    l.combine_recv_off = off;
    off = align_up(off + (int64_t)max_tokens * kMaxTopk * hidden * 2, kAlign);
    l.combine_send_off = off;
    off = align_up(off + E_l * slots * hidden * 2, kAlign);
    l.combine_meta_off = off;
    off = align_up(off + (int64_t)max_tokens * kMaxTopk * nb * 4, kAlign);
    l.half_bytes = align_up(off, 4096);
    (void)region_bytes;
    return l;
}

int64_t ll_region_size_for(int max_tokens, int hidden, int num_ranks, int num_experts) {
    const LLLayout l = compute_ll_layout(0, max_tokens, hidden, num_experts, num_ranks);
    return align_up(2 * l.half_bytes, 2 << 20);
}

int64_t Config::get_nvl_buffer_size_hint(int64_t hidden_bytes, int num_ranks, int num_max_tokens, int num_topk) const {
    (void)num_topk;
    const int hidden = (int)(hidden_bytes / 2);  // sized for bf16 rows (covers FP8 records too)
    return normal_region_size_for(num_max_tokens, std::max(hidden, 128), num_ranks);
}

int64_t Config::get_rdma_buffer_size_hint(int64_t hidden_bytes, int num_ranks) const {
    (void)hidden_bytes;
    (void)num_ranks;
    return 0;  // no RDMA domain on one NVLink box
}

// =================================================================================================
// EventHandle
// =================================================================================================
EventHandle::EventHandle() {
    event = std::make_shared<at::cuda::CUDAEvent>();
    event->record(at::cuda::getCurrentCUDAStream());
}
EventHandle::EventHandle(const at::cuda::CUDAStream& stream) {
    event = std::make_shared<at::cuda::CUDAEvent>();
    event->record(stream);
}
void EventHandle::current_stream_wait() const { event->block(at::cuda::getCurrentCUDAStream()); }

// =================================================================================================
// Buffer: construction, IPC exchange, teardown
// =================================================================================================
Buffer::Buffer(int rank, int num_ranks, int64_t num_nvl_bytes, int64_t num_rdma_bytes, bool low_latency_mode,
               bool explicitly_destroy, bool enable_shrink, double gpu_timeout_secs)
    : rank_(rank),
      num_ranks_(num_ranks),
      num_nvl_bytes_(std::max<int64_t>(num_nvl_bytes, kCtrlRegionMin)),
      num_rdma_bytes_(num_rdma_bytes),
      low_latency_mode_(low_latency_mode),
      explicitly_destroy_(explicitly_destroy),
      enable_shrink_(enable_shrink),
      comm_stream_(at::cuda::getStreamFromPool(true)),
      count_stream_(at::cuda::getStreamFromPool(true)) {
    if (num_ranks < 1 || num_ranks > kMaxRanks)
        throw std::runtime_error("B200 EP buffer: the group must be one NVLink domain of 1..8 ranks (got " +
                                 std::to_string(num_ranks) + "); internode RDMA is not available on a single box");
    if (rank < 0 || rank >= num_ranks) throw std::runtime_error("bad rank");
    EP_CUDA_CHECK(cudaGetDevice(&device_id_));
    set_timeout_secs(gpu_timeout_secs);
    const char* prof = std::getenv("DEEPEP_B200_PROFILE");
    profile_enabled_ = prof != nullptr && std::string(prof) == "1";
    // Row dealing of the pull/push pipelines: chunks of N rows round-robin over pairs (0: contiguous).
    const char* chunk = std::getenv("DEEPEP_B200_ROW_CHUNK");
    row_chunk_ = chunk != nullptr ? std::max(0, std::atoi(chunk)) : 0;
    // Combine push order: -1 = wavefront over destinations in token order (default), >= 0 as above.
    const char* cchunk = std::getenv("DEEPEP_B200_COMBINE_ROW_CHUNK");
    combine_row_chunk_ = cchunk != nullptr ? std::max(-1, std::atoi(cchunk)) : -1;
    // Combine arrival announcements: "drain" (default) waits for a batch's stores before announcing
    // it; "lagged" announces each batch one batch later and keeps the newer stores in flight.
    const char* poison_env = std::getenv("DEEPEP_B200_POISON_OUTPUTS");
    poison_outputs_ = poison_env != nullptr && std::string(poison_env) == "1";
    const char* announce = std::getenv("DEEPEP_B200_COMBINE_ANNOUNCE");
    combine_announce_lagged_ = announce != nullptr && std::string(announce) == "lagged";
    // Dispatch staging: "concurrent" (default) runs the stage as its own launch on the comm stream
    // while the count step runs on a second stream, the pull after both; "warps" stages inside the
    // pull launch (stage warps beside the pull pairs, after the count step).
    const char* stage_mode = std::getenv("DEEPEP_B200_DISPATCH_STAGE");
    stage_concurrent_ = stage_mode == nullptr || std::string(stage_mode) != "warps";
    // Scope of the stage's per-token chunk-counter add: "sys" (default) or "gpu" (the flag release
    // to the receivers stays at system scope either way).
    const char* scope_env = std::getenv("DEEPEP_B200_STAGE_SIGNAL_SCOPE");
    stage_signal_gpu_scope_ = scope_env != nullptr && std::string(scope_env) == "gpu";
    const char* fence_env = std::getenv("DEEPEP_B200_STAGE_WRITER_FENCE");
    stage_writer_fence_ = fence_env == nullptr || std::string(fence_env) != "0";
    // Row path of the standalone stage: "tma" (default: each warp TMA-loads a whole row into shared
    // memory, then quantizes it) or "regs" (rows through registers, six column groups in flight).
    const char* rows_env = std::getenv("DEEPEP_B200_STAGE_ROWS");
    stage_regs_rows_ = rows_env != nullptr && std::string(rows_env) == "regs";

    num_nvl_bytes_ = align_up(num_nvl_bytes_, 2 << 20);
    EP_CUDA_CHECK(cudaMalloc(&nvl_base_, num_nvl_bytes_));
    EP_CUDA_CHECK(cudaMemset(nvl_base_, 0, num_nvl_bytes_));
    EP_CUDA_CHECK(cudaIpcGetMemHandle(&nvl_ipc_, nvl_base_));
    if (num_rdma_bytes_ > 0) {
        num_rdma_bytes_ = align_up(num_rdma_bytes_, 2 << 20);
        EP_CUDA_CHECK(cudaMalloc(&ll_base_, num_rdma_bytes_));
        EP_CUDA_CHECK(cudaMemset(ll_base_, 0, num_rdma_bytes_));
        EP_CUDA_CHECK(cudaIpcGetMemHandle(&ll_ipc_, ll_base_));
    }
    EP_CUDA_CHECK(cudaHostAlloc(reinterpret_cast<void**>(&host_error_), sizeof(ErrorState), cudaHostAllocMapped));
    std::memset(host_error_, 0, sizeof(ErrorState));
    EP_CUDA_CHECK(cudaHostGetDevicePointer(reinterpret_cast<void**>(&host_error_dev_), host_error_, 0));
    EP_CUDA_CHECK(cudaHostAlloc(reinterpret_cast<void**>(&host_counters_), sizeof(HostCounters), cudaHostAllocMapped));
    std::memset(host_counters_, 0, sizeof(HostCounters));
    EP_CUDA_CHECK(cudaHostGetDevicePointer(reinterpret_cast<void**>(&host_counters_dev_), host_counters_, 0));
    EP_CUDA_CHECK(cudaMalloc(reinterpret_cast<void**>(&dev_workspace_), 4096));
    EP_CUDA_CHECK(cudaMemset(dev_workspace_, 0, 4096));
    EP_CUDA_CHECK(cudaMalloc(reinterpret_cast<void**>(&mask_), sizeof(int) * kMaxRanks));
    EP_CUDA_CHECK(cudaMemset(mask_, 0, sizeof(int) * kMaxRanks));
    EP_CUDA_CHECK(cudaDeviceSynchronize());
}

Buffer::~Buffer() noexcept(false) {
    if (!explicitly_destroy_) {
        destroy();
    } else if (!destroyed_) {
        fprintf(stderr, "B200 EP buffer: explicitly_destroy is set but destroy() was never called; resources leak\n");
    }
}

pybind11::bytearray Buffer::get_local_ipc_handle() const {
    return {nvl_ipc_.reserved, CUDA_IPC_HANDLE_SIZE};
}
pybind11::bytearray Buffer::get_local_ll_ipc_handle() const {
    if (ll_base_ == nullptr) return {"", 0};
    return {ll_ipc_.reserved, CUDA_IPC_HANDLE_SIZE};
}

void Buffer::sync(const std::vector<int>& device_ids, const std::vector<std::optional<pybind11::bytes>>& handles,
                  const std::vector<std::optional<pybind11::bytes>>& ll_handles) {
    if (available_) throw std::runtime_error("buffer already synced");
    if ((int)device_ids.size() != num_ranks_ || (int)handles.size() != num_ranks_)
        throw std::runtime_error("sync: wrong number of peers");
    for (int r = 0; r < num_ranks_; ++r) {
        if (r == rank_) {
            nvl_peer_[r] = nvl_base_;
            ll_peer_[r] = ll_base_;
            continue;
        }
        if (device_ids[r] == device_id_)
            throw std::runtime_error("sync: two ranks share one GPU; kernels that wait on one another cannot share a device");
        int can = 0;
        EP_CUDA_CHECK(cudaDeviceCanAccessPeer(&can, device_id_, device_ids[r]));
        if (!can) throw std::runtime_error("sync: no peer access to device " + std::to_string(device_ids[r]));
        auto h = std::string(handles[r].value());
        if (h.size() != CUDA_IPC_HANDLE_SIZE) throw std::runtime_error("sync: bad IPC handle size");
        cudaIpcMemHandle_t ipc;
        std::memcpy(ipc.reserved, h.data(), CUDA_IPC_HANDLE_SIZE);
        EP_CUDA_CHECK(cudaIpcOpenMemHandle(&nvl_peer_[r], ipc, cudaIpcMemLazyEnablePeerAccess));
        nvl_peer_opened_[r] = true;
        if (ll_base_ != nullptr) {
            if ((int)ll_handles.size() != num_ranks_ || !ll_handles[r].has_value())
                throw std::runtime_error("sync: missing low-latency IPC handle");
            auto lh = std::string(ll_handles[r].value());
            if (lh.size() != CUDA_IPC_HANDLE_SIZE) throw std::runtime_error("sync: bad LL IPC handle size");
            cudaIpcMemHandle_t lipc;
            std::memcpy(lipc.reserved, lh.data(), CUDA_IPC_HANDLE_SIZE);
            EP_CUDA_CHECK(cudaIpcOpenMemHandle(&ll_peer_[r], lipc, cudaIpcMemLazyEnablePeerAccess));
            ll_peer_opened_[r] = true;
        }
    }
    EP_CUDA_CHECK(cudaDeviceSynchronize());
    available_ = true;
}

void Buffer::destroy() {
    if (destroyed_) return;
    destroyed_ = true;
    cudaDeviceSynchronize();
    for (int r = 0; r < kMaxRanks; ++r) {
        if (nvl_peer_opened_[r]) cudaIpcCloseMemHandle(nvl_peer_[r]);
        if (ll_peer_opened_[r]) cudaIpcCloseMemHandle(ll_peer_[r]);
        nvl_peer_opened_[r] = ll_peer_opened_[r] = false;
    }
    if (nvl_base_) cudaFree(nvl_base_);
    if (ll_base_) cudaFree(ll_base_);
    if (dev_workspace_) cudaFree(dev_workspace_);
    if (mask_) cudaFree(mask_);
    if (trace_dev_) {
        cudaFree(trace_dev_);
        cudaFree(trace_records_);
        cudaFree(trace_cursor_);
        trace_dev_ = nullptr;
    }
    if (host_error_) cudaFreeHost(host_error_);
    if (host_counters_) cudaFreeHost(host_counters_);
    for (auto& pe : prof_events_) cudaEventDestroy(pe.second);  // profile points never collected
    prof_events_.clear();
    nvl_base_ = ll_base_ = nullptr;
    dev_workspace_ = mask_ = nullptr;
    host_error_ = nullptr;
    host_counters_ = nullptr;
    available_ = false;
}

torch::Stream Buffer::get_comm_stream() const { return comm_stream_; }

torch::Tensor Buffer::get_local_buffer_tensor(const pybind11::object& dtype, int64_t offset, bool use_rdma_buffer) const {
    const auto scalar = torch::python::detail::py_object_to_dtype(dtype);
    const int64_t esize = c10::elementSize(scalar);
    void* base = use_rdma_buffer ? ll_base_ : nvl_base_;
    const int64_t bytes = use_rdma_buffer ? num_rdma_bytes_ : num_nvl_bytes_;
    if (base == nullptr) throw std::runtime_error("requested region is not allocated");
    const int64_t n = bytes / esize - offset;
    return torch::from_blob(static_cast<uint8_t*>(base) + offset * esize, {n},
                            torch::TensorOptions().dtype(scalar).device(torch::kCUDA, device_id_));
}

int64_t Buffer::get_capacity(int hidden, int num_topk) const {
    (void)num_topk;
    return compute_normal_layout(num_nvl_bytes_, hidden, num_ranks_).capacity;
}

// =================================================================================================
// Errors
// =================================================================================================
void Buffer::set_timeout_secs(double secs) {
    if (secs <= 0) secs = 100.0;
    timeout_ns_ = (uint64_t)(secs * 1e9);
}

KernelStatus Buffer::status() const {
    KernelStatus s{};
    s.host_error = host_error_dev_;
    s.abort_flag = dev_workspace_;
    s.timeout_ns = timeout_ns_;
    s.rank = rank_;
    s.trace = trace_dev_;
    return s;
}

void Buffer::enable_trace(int64_t capacity) {
    TORCH_CHECK(capacity > 0, "trace capacity must be positive");
    disable_trace();
    EP_CUDA_CHECK(cudaMalloc(&trace_records_, sizeof(TraceRecord) * capacity));
    EP_CUDA_CHECK(cudaMalloc(&trace_cursor_, sizeof(unsigned long long)));
    EP_CUDA_CHECK(cudaMemset(trace_cursor_, 0, sizeof(unsigned long long)));
    EP_CUDA_CHECK(cudaMalloc(&trace_dev_, sizeof(TraceRing)));
    TraceRing ring{trace_records_, trace_cursor_, (uint64_t)capacity};
    EP_CUDA_CHECK(cudaMemcpy(trace_dev_, &ring, sizeof(ring), cudaMemcpyHostToDevice));
    trace_capacity_ = capacity;
}

void Buffer::disable_trace() {
    if (trace_dev_ == nullptr) return;
    EP_CUDA_CHECK(cudaDeviceSynchronize());
    cudaFree(trace_dev_);
    cudaFree(trace_records_);
    cudaFree(trace_cursor_);
    trace_dev_ = nullptr;
    trace_records_ = nullptr;
    trace_cursor_ = nullptr;
    trace_capacity_ = 0;
}

std::tuple<torch::Tensor, int64_t> Buffer::read_trace(bool reset) {
    TORCH_CHECK(trace_dev_ != nullptr, "tracing is not enabled");
    EP_CUDA_CHECK(cudaDeviceSynchronize());
    unsigned long long n = 0;
    EP_CUDA_CHECK(cudaMemcpy(&n, trace_cursor_, sizeof(n), cudaMemcpyDeviceToHost));
    const int64_t kept = std::min<int64_t>((int64_t)n, trace_capacity_);
    auto out = torch::empty({kept, (int64_t)sizeof(TraceRecord)}, torch::dtype(torch::kUInt8));
    if (kept > 0)
        EP_CUDA_CHECK(cudaMemcpy(out.data_ptr(), trace_records_, sizeof(TraceRecord) * kept, cudaMemcpyDeviceToHost));
    if (reset) EP_CUDA_CHECK(cudaMemset(trace_cursor_, 0, sizeof(unsigned long long)));
    return {out, (int64_t)n};
}

std::tuple<int64_t, int64_t, int64_t> Buffer::sample_clock() {
    auto stream = at::cuda::getCurrentCUDAStream();
    EP_CUDA_CHECK(cudaStreamSynchronize(stream));
    auto mono = []() {
        return (int64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
                   std::chrono::steady_clock::now().time_since_epoch()).count();
    };
    auto cell = torch::zeros({1}, torch::dtype(torch::kInt64).device(torch::kCUDA, device_id_));
    EP_CUDA_CHECK(cudaStreamSynchronize(stream));
    const int64_t before = mono();
    launch_read_globaltimer(reinterpret_cast<unsigned long long*>(cell.data_ptr<int64_t>()), stream.stream());
    EP_CUDA_CHECK(cudaStreamSynchronize(stream));
    const int64_t after = mono();
    return {before, cell.cpu().item<int64_t>(), after};
}

void Buffer::check_error() const {
    if (host_error_ == nullptr) return;
    const int code = *reinterpret_cast<volatile int*>(&host_error_->code);
    if (code != 0) {
        throw std::runtime_error("B200 EP kernel error on rank " + std::to_string(host_error_->rank) + ": " +
                                 error_name(code) + " (code " + std::to_string(code) + ", peer " +
                                 std::to_string(host_error_->peer) + ", detail " + std::to_string(host_error_->detail) + ")");
    }
}

std::tuple<int, int, int, int> Buffer::get_error_state() const {
    if (host_error_ == nullptr) return {0, 0, 0, 0};
    return {host_error_->code, host_error_->peer, host_error_->detail, host_error_->rank};
}

void Buffer::clear_error() {
    EP_CUDA_CHECK(cudaDeviceSynchronize());
    if (host_error_) std::memset(host_error_, 0, sizeof(ErrorState));
    if (dev_workspace_) EP_CUDA_CHECK(cudaMemset(dev_workspace_, 0, sizeof(int)));
    EP_CUDA_CHECK(cudaDeviceSynchronize());
}

PeerTable Buffer::nvl_peers() const {
    PeerTable p{};
    for (int r = 0; r < num_ranks_; ++r) p.base[r] = nvl_peer_[r];
    return p;
}
PeerTable Buffer::ll_peers() const {
    PeerTable p{};
    for (int r = 0; r < num_ranks_; ++r) p.base[r] = ll_peer_[r];
    return p;
}

// Opt-in kernel timing (env DEEPEP_B200_PROFILE=1): events at fixed points of every dispatch /
// combine; `get_profile()` synchronizes and returns the mean milliseconds between marks.
// Points: 0 count, 1 output allocation, 2 stage + pull, 3 dispatch end, 4 combine, 5 combine end.
void Buffer::prof_mark(cudaStream_t stream, int point) {
    if (!profile_enabled_) return;
    cudaEvent_t e;
    cudaEventCreate(&e);
    cudaEventRecord(e, stream);
    prof_events_.push_back({point, e});
}

std::map<std::string, double> Buffer::get_profile() {
    std::map<std::string, double> out;
    cudaDeviceSynchronize();
    // count: the count step; count_to_pull: its end to the pull launch (the rest of the concurrent stage
    // launch, or the output set-up); pull: the pull launch (with stage warps in the "warps" mode)
    const char* names[] = {"count", "count_to_pull", "pull", "dispatch_end", "combine", "combine_end"};
    std::map<std::string, std::pair<double, int>> acc;
    for (size_t i = 0; i + 1 < prof_events_.size(); ++i) {
        const int a = prof_events_[i].first, b = prof_events_[i + 1].first;
        if (b != a + 1 || a == 3) continue;
        float ms = 0;
        cudaEventElapsedTime(&ms, prof_events_[i].second, prof_events_[i + 1].second);
        const std::string key = names[a];
        acc[key].first += ms;
        acc[key].second += 1;
    }
    for (auto& kv : acc) out[kv.first + "_ms"] = kv.second.first / std::max(1, kv.second.second);
    for (auto& pe : prof_events_) cudaEventDestroy(pe.second);
    prof_events_.clear();
    return out;
}

void Buffer::wait_host_counters(int ticket) {
    const auto start = std::chrono::steady_clock::now();
    const double limit = (double)timeout_ns_ * 1e-9;
    uint64_t it = 0;
    while (*reinterpret_cast<volatile int*>(&host_counters_->ready_ticket) != ticket) {
        if ((++it & 1023) == 0) {
            check_error();
            // A faulted context never completes the notify kernel: surface the CUDA error at once.
            const cudaError_t q = cudaStreamQuery(comm_stream_.stream());
            if (q != cudaSuccess && q != cudaErrorNotReady)
                throw std::runtime_error(std::string("B200 EP: CUDA error while waiting for received token counts: ") +
                                         cudaGetErrorString(q));
            const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count();
            if (el > limit)
                throw std::runtime_error("B200 EP: CPU timeout waiting for received token counts (rank " + std::to_string(rank_) + ")");
        }
    }
    std::atomic_thread_fence(std::memory_order_acquire);
    check_error();
}

// =================================================================================================
// Normal mode
// =================================================================================================
std::tuple<torch::Tensor, std::optional<torch::Tensor>, torch::Tensor, torch::Tensor, std::optional<EventHandle>>
Buffer::get_dispatch_layout(const torch::Tensor& topk_idx, int num_experts, std::optional<EventHandle>& previous_event,
                            bool async, bool allocate_on_comm_stream) {
    check_error();
    TORCH_CHECK(topk_idx.dim() == 2 && topk_idx.is_contiguous() && topk_idx.scalar_type() == torch::kInt64);
    TORCH_CHECK(num_experts % num_ranks_ == 0, "num_experts must be a multiple of the group size");
    StreamScope scope(comm_stream_, previous_event, allocate_on_comm_stream);
    const int N = (int)topk_idx.size(0), K = (int)topk_idx.size(1);
    auto i32 = torch::dtype(torch::kInt32).device(torch::kCUDA);
    auto num_tokens_per_rank = torch::empty({num_ranks_}, i32);
    auto num_tokens_per_expert = torch::empty({num_experts}, i32);
    auto is_token_in_rank = torch::empty({N, num_ranks_}, torch::dtype(torch::kBool).device(torch::kCUDA));
    launch_dispatch_layout(topk_idx.data_ptr<int64_t>(), N, K, num_experts, num_ranks_, num_tokens_per_rank.data_ptr<int>(),
                           num_tokens_per_expert.data_ptr<int>(), is_token_in_rank.data_ptr<bool>(), scope.comm.stream());
    auto event = scope.finish(async, {topk_idx, num_tokens_per_rank, num_tokens_per_expert, is_token_in_rank});
    return {num_tokens_per_rank, std::nullopt, num_tokens_per_expert, is_token_in_rank, event};
}

// Tokens per staged-chunk flag: the same on every rank (a function of the common capacity), with at
// most kMaxStageChunks chunks per rank and at least 128 tokens per chunk.
static int stage_chunk_tokens(int capacity) {
    return std::max(128, (capacity + kMaxStageChunks - 1) / kMaxStageChunks);
}

// Count-step arguments shared by dispatch() and dispatch_gemm(); the caller fills the routing
// inputs and the output tensors.
CountArgs Buffer::count_args(const NormalLayout& L, int N, int K, int num_experts, bool cached, int expert_alignment) {
    CountArgs na{};
    na.num_tokens = N;
    na.num_topk = K;
    na.num_experts = num_experts;
    na.num_local_experts = cached ? 0 : num_experts / num_ranks_;
    na.num_ranks = num_ranks_;
    na.rank = rank_;
    na.cached = cached ? 1 : 0;
    // at most kMaxCountCtas CTAs, each a multiple of the 256-thread block in tokens
    const int per_cta = (N + kMaxCountCtas - 1) / kMaxCountCtas;
    na.tokens_per_cta = std::max(1, (per_cta + 255) / 256) * 256;
    na.expert_alignment = std::max(1, expert_alignment);
    na.peers = nvl_peers();
    na.layout = L;
    na.dev_num_recv = dev_workspace_ + 1;
    na.expert_counts = reinterpret_cast<int*>(static_cast<uint8_t*>(nvl_base_) + L.scratch_off + align_up(L.capacity, kAlign));
    na.st = status();
    return na;
}

std::tuple<torch::Tensor, std::optional<torch::Tensor>, std::optional<torch::Tensor>, std::optional<torch::Tensor>,
           std::vector<int>, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor,
           std::optional<torch::Tensor>, std::optional<EventHandle>>
Buffer::intranode_dispatch(const torch::Tensor& x, const std::optional<torch::Tensor>& x_scales,
                           const std::optional<torch::Tensor>& topk_idx, const std::optional<torch::Tensor>& topk_weights,
                           const std::optional<torch::Tensor>& is_token_in_rank, int num_experts,
                           const std::optional<torch::Tensor>& cached_rank_prefix_matrix,
                           const std::optional<torch::Tensor>& cached_send_prefix_matrix,
                           const std::optional<torch::Tensor>& cached_recv_src_idx,
                           const std::optional<torch::Tensor>& cached_send_head, int expert_alignment,
                           int num_worst_tokens, bool quantize_fp8, bool round_scale, bool scales_col_major,
                           const std::optional<torch::Tensor>& cumulative_local_expert_recv_stats, int num_sms,
                           std::optional<EventHandle>& previous_event, bool async, bool allocate_on_comm_stream) {
    check_error();
    TORCH_CHECK(available_, "buffer not synced");
    const bool cached = cached_rank_prefix_matrix.has_value();
    TORCH_CHECK(x.dim() == 2 && x.is_contiguous(), "x must be a contiguous [num_tokens, hidden] tensor");
    const bool fp8_in = x.scalar_type() == torch::kFloat8_e4m3fn;
    TORCH_CHECK(fp8_in || x.scalar_type() == torch::kBFloat16, "x must be bf16 or float8_e4m3fn");
    TORCH_CHECK(fp8_in == x_scales.has_value(), "FP8 input needs scales (and only FP8 input takes them)");
    TORCH_CHECK(!(fp8_in && quantize_fp8), "input is already FP8");
    const bool out_fp8 = fp8_in || quantize_fp8;
    const int N = (int)x.size(0), H = (int)x.size(1), R = num_ranks_;
    TORCH_CHECK(H % 128 == 0, "hidden must be a multiple of 128");
    const int K = (!cached && topk_idx.has_value()) ? (int)topk_idx->size(1) : 0;
    TORCH_CHECK(K <= kMaxTopk, "top-k larger than 16 is not supported");
    if (!cached) {
        TORCH_CHECK(topk_idx.has_value() || is_token_in_rank.has_value(), "need topk_idx or is_token_in_rank");
        TORCH_CHECK(num_experts > 0 && num_experts % R == 0, "num_experts must be a positive multiple of the group size");
        TORCH_CHECK(num_experts / R <= kMaxLocalExperts, "too many local experts");
        if (topk_idx.has_value())
            TORCH_CHECK(topk_idx->scalar_type() == torch::kInt64 && topk_idx->is_contiguous() && topk_idx->size(0) == N);
        if (topk_weights.has_value())
            TORCH_CHECK(topk_weights->scalar_type() == torch::kFloat32 && topk_weights->is_contiguous() &&
                        topk_weights->size(0) == N && topk_weights->size(1) == K);
        if (is_token_in_rank.has_value())
            TORCH_CHECK(is_token_in_rank->scalar_type() == torch::kBool && is_token_in_rank->is_contiguous() &&
                        is_token_in_rank->size(0) == N && is_token_in_rank->size(1) == R);
    } else {
        TORCH_CHECK(cached_send_prefix_matrix.has_value() && cached_recv_src_idx.has_value() && cached_send_head.has_value());
        TORCH_CHECK(cached_send_head->size(0) == N, "cached handle was built for a different token count");
    }
    const NormalLayout L = compute_normal_layout(num_nvl_bytes_, H, R);
    TORCH_CHECK(N <= L.capacity, "num_tokens (" + std::to_string(N) + ") exceeds the buffer capacity (" +
                                     std::to_string(L.capacity) + "); allocate num_nvl_bytes >= Buffer.get_nvl_buffer_size_hint(...)");
    const RecordFormat rec = record_format(H, K, out_fp8);
    const int E_l = cached ? 0 : num_experts / R;
    if (num_sms <= 0) num_sms = 32;

    const int ticket = ++dispatch_epoch_;
    StreamScope scope(comm_stream_, previous_event, allocate_on_comm_stream);
    auto stream = scope.comm.stream();
    auto i32 = torch::dtype(torch::kInt32).device(torch::kCUDA);
    const KernelStatus st = status();
    const PeerTable peers = nvl_peers();
    uint8_t* my_base = static_cast<uint8_t*>(nvl_base_);

    // 1) count: lists, send_head and per-expert counts from the routing alone, then the count
    //    exchange and the receive layout. It does not wait for any quantization.
    torch::Tensor send_head, rpm, spm, recv_rank_prefix;
    std::optional<torch::Tensor> num_recv_per_expert;
    if (cached) {
        rpm = *cached_rank_prefix_matrix;
        spm = *cached_send_prefix_matrix;
        send_head = *cached_send_head;
        recv_rank_prefix = torch::empty({0}, i32);
    } else {
        send_head = torch::empty({N, R}, i32);
        rpm = torch::empty({R, R}, i32);
        spm = torch::empty({R, R}, i32);
        recv_rank_prefix = torch::empty({R + 1}, i32);
        num_recv_per_expert = torch::empty({E_l}, i32);
    }
    const int stage_chunk = stage_chunk_tokens(L.capacity);
    CountArgs na = count_args(L, N, K, cached ? 0 : num_experts, cached, expert_alignment);
    na.topk_idx = (!cached && topk_idx.has_value()) ? topk_idx->data_ptr<int64_t>() : nullptr;
    na.is_token_in_rank = (!cached && is_token_in_rank.has_value()) ? is_token_in_rank->data_ptr<bool>() : nullptr;
    na.send_head = send_head.data_ptr<int>();
    na.rank_prefix_matrix = rpm.data_ptr<int>();
    na.send_prefix_matrix = spm.data_ptr<int>();
    na.recv_rank_prefix = cached ? nullptr : recv_rank_prefix.data_ptr<int>();
    na.num_recv_per_expert = cached ? nullptr : num_recv_per_expert->data_ptr<int>();
    na.cumulative_stats = cumulative_local_expert_recv_stats.has_value() ? cumulative_local_expert_recv_stats->data_ptr<int>() : nullptr;
    // the counts reach the CPU from the count step itself (a synced dispatch returns before the pull ends)
    na.host = cached ? nullptr : host_counters_dev_;
    na.host_ticket = ticket;
    // 2) the stage: its own launch concurrent with the count step (default), or stage warps of the
    //    pull launch; either way every chunk's completion is signalled to the receivers
    StageArgs sa{};
    sa.x = x.data_ptr();
    if (fp8_in) {
        TORCH_CHECK(x_scales->scalar_type() == torch::kFloat32 && x_scales->dim() == 2 && x_scales->size(0) == N &&
                        x_scales->size(1) == H / 128,
                    "x scales must be float32 [num_tokens, hidden / 128]");
        sa.x_scales = x_scales->data_ptr<float>();
        sa.scale_stride_t = x_scales->stride(0);
        sa.scale_stride_b = x_scales->stride(1);
    }
    sa.topk_idx = (!cached && topk_idx.has_value()) ? topk_idx->data_ptr<int64_t>() : nullptr;
    sa.topk_weights = (!cached && topk_weights.has_value()) ? topk_weights->data_ptr<float>() : nullptr;
    sa.staging = my_base + L.staging_off;
    sa.num_tokens = N;
    sa.hidden = H;
    sa.num_topk = K;
    sa.topk_pad = (int)align_up(K, 4);
    sa.in_elem_bytes = fp8_in ? 1 : 2;
    sa.quantize = quantize_fp8 ? 1 : 0;
    sa.round_scale = round_scale ? 1 : 0;
    sa.chunk = stage_chunk;
    sa.num_ranks = R;
    sa.rec = rec;
    sa.record_stride = L.record_bytes;
    sa.epoch = ticket;
    sa.signal_gpu_scope = stage_signal_gpu_scope_ ? 1 : 0;
    sa.regs_rows = stage_regs_rows_ ? 1 : 0;
    sa.writer_proxy_fence = stage_writer_fence_ ? 1 : 0;
    sa.rank = rank_;
    sa.peers = peers;
    sa.layout = L;
    sa.st = st;
    NormalCtrl* my_ctrl = reinterpret_cast<NormalCtrl*>(my_base + L.ctrl_off);
    sa.pull_done = my_ctrl->pull_done;
    sa.dispatch_epoch = &my_ctrl->dispatch_epoch;
    const bool skip_count = stage_concurrent_ && cached;
    if (skip_count) {
        // Cached handle: the counts and lists are known, so no count step runs. The stage waits for
        // the receivers' previous pulls (staging reuse) and releases each chunk with this dispatch's
        // epoch; the pull waits for every source's chunks and records the epoch when it ends.
        sa.signal_chunks = 1;
        launch_dispatch_stage(sa, 0, stream);
    } else if (stage_concurrent_) {
        // The count step starts on its own stream once every earlier comm-stream kernel is done (the
        // flags it waits on for this GPU are then already set), launched first so that its CTAs take
        // SMs before the stage's; the stage leaves a few SMs free for them. Neither waits on the
        // other; the pull waits for both through the streams.
        sa.signal_chunks = 1;
        stream_wait(count_stream_, scope.comm);
        prof_mark(count_stream_.stream(), 0);
        launch_dispatch_count(na, count_stream_.stream());
        prof_mark(count_stream_.stream(), 1);
        int sm_count = 148;
        EP_CUDA_CHECK(cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, device_id_));
        launch_dispatch_stage(sa, std::max(1, sm_count - 8), stream);
        stream_wait(scope.comm, count_stream_);
    } else {
        prof_mark(stream, 0);
        launch_dispatch_count(na, stream);
        prof_mark(stream, 1);
    }

    // 3) receive size. Cached: known. Worst case (`num_worst_tokens`): no CPU sync at all. Otherwise
    //    the pull is launched at once into outputs sized for the largest possible receive
    //    (num_ranks * capacity rows; the kernel reads the true count on the device) and the host
    //    waits for the mapped counts while the pull runs, then returns exact-size views.
    int num_recv = -1, num_out_rows = 0;
    const bool cpu_sync = !cached && num_worst_tokens <= 0;
    if (cached) {
        num_recv = (int)cached_recv_src_idx->size(0);
        num_out_rows = num_recv;
    } else if (num_worst_tokens > 0) {
        num_out_rows = num_worst_tokens;
    } else {
        num_out_rows = R * L.capacity;
    }

    // 4) outputs + pull
    auto recv_x = torch::empty({num_out_rows, H}, x.options().dtype(out_fp8 ? torch::kFloat8_e4m3fn : torch::kBFloat16));
    std::optional<torch::Tensor> recv_scales, scales_storage;
    int64_t scales_ld = 0;
    if (out_fp8) {
        if (scales_col_major) {
            scales_ld = align_up(std::max(num_out_rows, 1), 4);
            scales_storage = torch::empty({H / 128, scales_ld}, torch::dtype(torch::kFloat32).device(torch::kCUDA));
            recv_scales = scales_storage->narrow(1, 0, num_out_rows).t();
        } else {
            recv_scales = torch::empty({num_out_rows, H / 128}, torch::dtype(torch::kFloat32).device(torch::kCUDA));
        }
    }
    std::optional<torch::Tensor> recv_topk_idx, recv_topk_weights;
    if (!cached && topk_idx.has_value())
        recv_topk_idx = torch::empty({num_out_rows, K}, torch::dtype(torch::kInt64).device(torch::kCUDA));
    if (!cached && topk_weights.has_value())
        recv_topk_weights = torch::empty({num_out_rows, K}, torch::dtype(torch::kFloat32).device(torch::kCUDA));
    torch::Tensor recv_src_idx = cached ? *cached_recv_src_idx : torch::empty({num_out_rows}, i32);
    if (poison_outputs_) {
        // Debug: every output byte starts as 0xFF (NaN for the float types, -1 for ids), so a row the
        // kernels should have written but did not shows up in the caller's checks.
        poison(recv_x, stream);
        if (recv_scales.has_value()) poison(scales_storage.has_value() ? *scales_storage : *recv_scales, stream);
        if (recv_topk_idx.has_value()) poison(*recv_topk_idx, stream);
        if (recv_topk_weights.has_value()) poison(*recv_topk_weights, stream);
        if (!cached) poison(recv_src_idx, stream);
    }

    PullArgs pa{};
    pa.peers = peers;
    pa.layout = L;
    pa.rec = rec;
    pa.rank = rank_;
    pa.num_ranks = R;
    pa.num_local_experts = E_l;
    pa.num_topk = K;
    pa.rank_prefix_matrix = rpm.data_ptr<int>();
    pa.dev_num_recv = cached ? nullptr : dev_workspace_ + 1;
    pa.num_recv_host = num_recv;
    pa.num_out_rows = num_out_rows;
    pa.fill_padding = num_worst_tokens > 0 ? 1 : 0;
    pa.recv_x = recv_x.data_ptr();
    pa.recv_scales = recv_scales.has_value() ? recv_scales->data_ptr<float>() : nullptr;
    pa.scales_col_major = scales_col_major ? 1 : 0;
    pa.scales_ld = scales_ld;
    pa.recv_topk_idx = recv_topk_idx.has_value() ? recv_topk_idx->data_ptr<int64_t>() : nullptr;
    pa.recv_topk_weights = recv_topk_weights.has_value() ? recv_topk_weights->data_ptr<float>() : nullptr;
    pa.recv_src_idx = cached ? nullptr : recv_src_idx.data_ptr<int>();
    pa.cached_src_idx = cached ? cached_recv_src_idx->data_ptr<int>() : nullptr;
    pa.stages = 0;
    pa.host = nullptr;  // the count step wrote the host counters
    pa.num_recv_per_expert = cached ? nullptr : num_recv_per_expert->data_ptr<int>();
    pa.host_ticket = ticket;
    pa.chunk = row_chunk_;
    pa.stage_warps = stage_concurrent_ ? 0 : 1;
    pa.wait_staged = stage_concurrent_ ? 1 : 0;
    pa.epoch = skip_count ? ticket : 0;
    pa.stage = sa;
    pa.st = st;
    prof_mark(stream, 2);
    launch_dispatch_pull(pa, num_sms, stream);
    prof_mark(stream, 3);
    EP_CUDA_CHECK(cudaGetLastError());

    std::vector<int> per_expert_list;
    if (cpu_sync) {
        wait_host_counters(ticket);
        num_recv = host_counters_->num_recv_tokens;
        per_expert_list.assign(host_counters_->num_recv_tokens_per_expert, host_counters_->num_recv_tokens_per_expert + E_l);
        recv_x = recv_x.narrow(0, 0, num_recv);
        if (recv_scales.has_value())
            recv_scales = scales_col_major ? scales_storage->narrow(1, 0, num_recv).t() : recv_scales->narrow(0, 0, num_recv);
        if (recv_topk_idx.has_value()) recv_topk_idx = recv_topk_idx->narrow(0, 0, num_recv);
        if (recv_topk_weights.has_value()) recv_topk_weights = recv_topk_weights->narrow(0, 0, num_recv);
        recv_src_idx = recv_src_idx.narrow(0, 0, num_recv);
    }

    auto event = scope.finish(async, {x, x_scales, topk_idx, topk_weights, is_token_in_rank, recv_x, recv_scales, recv_topk_idx,
                                      recv_topk_weights, recv_src_idx, send_head, rpm, spm, recv_rank_prefix,
                                      num_recv_per_expert, cumulative_local_expert_recv_stats});
    return {recv_x, recv_scales, recv_topk_idx, recv_topk_weights, per_expert_list, rpm, spm, recv_rank_prefix,
            recv_src_idx, send_head, num_recv_per_expert, event};
}

std::tuple<torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor,
           torch::Tensor, std::vector<int>, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor>
Buffer::intranode_dispatch_gemm(const torch::Tensor& x, const torch::Tensor& topk_idx, const torch::Tensor& topk_weights,
                                int num_experts, const torch::Tensor& w, const torch::Tensor& w_scales, bool round_scale,
                                int num_sms, int pull_ctas) {
    check_error();
    TORCH_CHECK(available_, "buffer not synced");
    TORCH_CHECK(x.dim() == 2 && x.is_contiguous() && x.scalar_type() == torch::kBFloat16, "x must be contiguous bf16 [tokens, hidden]");
    const int N = (int)x.size(0), H = (int)x.size(1), R = num_ranks_;
    TORCH_CHECK(H % 128 == 0, "hidden must be a multiple of 128");
    TORCH_CHECK(topk_idx.scalar_type() == torch::kInt64 && topk_idx.is_contiguous() && topk_idx.dim() == 2 && topk_idx.size(0) == N);
    const int K = (int)topk_idx.size(1);
    TORCH_CHECK(K <= kMaxTopk, "top-k larger than 16 is not supported");
    TORCH_CHECK(topk_weights.scalar_type() == torch::kFloat32 && topk_weights.is_contiguous() && topk_weights.size(0) == N &&
                topk_weights.size(1) == K);
    TORCH_CHECK(num_experts > 0 && num_experts % R == 0 && num_experts / R <= kMaxLocalExperts);
    const int E_l = num_experts / R;
    TORCH_CHECK(w.is_cuda() && w.dim() == 3 && w.is_contiguous() && w.scalar_type() == torch::kFloat8_e4m3fn && w.size(0) == E_l &&
                    w.size(2) == H && w.size(1) % 128 == 0,
                "weights must be contiguous [num_local_experts, n, hidden] e4m3 with n % 128 == 0");
    const int n = (int)w.size(1);
    TORCH_CHECK(w_scales.scalar_type() == torch::kFloat32 && w_scales.is_contiguous() && w_scales.dim() == 3 &&
                w_scales.size(0) == E_l && w_scales.size(1) == n / 128 && w_scales.size(2) == H / 128);
    const NormalLayout L = compute_normal_layout(num_nvl_bytes_, H, R);
    TORCH_CHECK(N <= L.capacity, "num_tokens exceeds the buffer capacity");
    const RecordFormat rec = record_format(H, K, /*fp8=*/true);
    int sm_count = 148;
    EP_CUDA_CHECK(cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, device_id_));
    if (num_sms <= 0 || num_sms > sm_count) num_sms = sm_count;
    if (pull_ctas <= 0) pull_ctas = std::min(32, num_sms);
    TORCH_CHECK(pull_ctas <= num_sms, "pull_ctas must not exceed num_sms");
    const int num_out_rows = R * L.capacity;  // received tokens, worst case
    const int max_mtiles = (num_out_rows + 127) / 128;
    TORCH_CHECK(max_mtiles <= 512, "the fused dispatch supports at most 65536 received rows per expert; use dispatch()");
    const int64_t rows_cap = (int64_t)num_out_rows * std::min(K, E_l) + (int64_t)E_l * 127;
    TORCH_CHECK(rows_cap < (int64_t)1 << 31);

    auto i32 = torch::dtype(torch::kInt32).device(torch::kCUDA);
    // Zeroed on the compute stream before the comm stream waits for it.
    auto raw_counts = torch::zeros({E_l}, i32);
    auto counters = torch::zeros({E_l + (int64_t)E_l * max_mtiles + 1}, i32);  // claim | landed | tile counter

    const int ticket = ++dispatch_epoch_;
    std::optional<EventHandle> no_event;
    StreamScope scope(comm_stream_, no_event, false);
    auto stream = scope.comm.stream();
    const KernelStatus st = status();
    const PeerTable peers = nvl_peers();
    uint8_t* my_base = static_cast<uint8_t*>(nvl_base_);

    // 1) stage (bf16 -> FP8 records) as a kernel of its own: the count exchange below is then a
    //    barrier after every rank's staging, which the fused receive relies on (it has no staged flags).
    NormalCtrl* my_ctrl = reinterpret_cast<NormalCtrl*>(my_base + L.ctrl_off);
    StageArgs sa{};
    sa.x = x.data_ptr();
    sa.topk_idx = topk_idx.data_ptr<int64_t>();
    sa.topk_weights = topk_weights.data_ptr<float>();
    sa.staging = my_base + L.staging_off;
    sa.pull_done = my_ctrl->pull_done;
    sa.dispatch_epoch = &my_ctrl->dispatch_epoch;
    sa.num_ranks = R;
    sa.num_tokens = N;
    sa.hidden = H;
    sa.num_topk = K;
    sa.topk_pad = (int)align_up(K, 4);
    sa.in_elem_bytes = 2;
    sa.quantize = 1;
    sa.round_scale = round_scale ? 1 : 0;
    sa.rec = rec;
    sa.record_stride = L.record_bytes;
    sa.epoch = ticket;
    sa.st = st;
    launch_dispatch_stage(sa, 0, stream);

    // 2) count: lists, counts, 128-aligned per-expert rows, raw per-expert rows (statistics output)
    auto send_head = torch::empty({N, R}, i32);
    auto rpm = torch::empty({R, R}, i32);
    auto spm = torch::empty({R, R}, i32);
    auto recv_rank_prefix = torch::empty({R + 1}, i32);
    auto aligned_counts = torch::empty({E_l}, i32);
    CountArgs na = count_args(L, N, K, num_experts, false, 128);
    na.topk_idx = topk_idx.data_ptr<int64_t>();
    na.send_head = send_head.data_ptr<int>();
    na.rank_prefix_matrix = rpm.data_ptr<int>();
    na.send_prefix_matrix = spm.data_ptr<int>();
    na.recv_rank_prefix = recv_rank_prefix.data_ptr<int>();
    na.num_recv_per_expert = aligned_counts.data_ptr<int>();
    na.cumulative_stats = raw_counts.data_ptr<int>();
    launch_dispatch_count(na, stream);

    // 3) outputs (worst-case rows; exact views after the CPU sync) + the fused receive / GEMM
    auto a_rows = torch::empty({rows_cap, H}, x.options().dtype(torch::kFloat8_e4m3fn));
    auto a_scales = torch::empty({rows_cap, H / 128}, torch::dtype(torch::kFloat32).device(torch::kCUDA));
    auto h = torch::empty({rows_cap, n}, x.options());
    auto row_map = torch::empty({num_out_rows, K}, i32);
    auto recv_w = torch::empty({num_out_rows, K}, torch::dtype(torch::kFloat32).device(torch::kCUDA));
    auto recv_src_idx = torch::empty({num_out_rows}, i32);

    FusedDispatchGemmArgs fa{};
    fa.peers = peers;
    fa.layout = L;
    fa.rec = rec;
    fa.rank = rank_;
    fa.num_ranks = R;
    fa.num_local_experts = E_l;
    fa.num_topk = K;
    fa.rank_prefix_matrix = rpm.data_ptr<int>();
    fa.dev_num_recv = dev_workspace_ + 1;
    fa.num_out_rows = num_out_rows;
    fa.pull_ctas = pull_ctas;
    fa.chunk = row_chunk_;
    fa.num_recv_per_expert = aligned_counts.data_ptr<int>();
    fa.raw_counts = raw_counts.data_ptr<int>();
    fa.claim = counters.data_ptr<int>();
    fa.landed = fa.claim + E_l;
    fa.max_mtiles = max_mtiles;
    fa.tile_counter = fa.landed + (int64_t)E_l * max_mtiles;
    fa.a = static_cast<uint8_t*>(a_rows.data_ptr());
    fa.sa = a_scales.data_ptr<float>();
    fa.rows_cap = (int)rows_cap;
    fa.row_map = row_map.data_ptr<int>();
    fa.recv_topk_weights = recv_w.data_ptr<float>();
    fa.recv_src_idx = recv_src_idx.data_ptr<int>();
    fa.host = host_counters_dev_;
    fa.host_ticket = ticket;
    fa.b = w.data_ptr();
    fa.sb = w_scales.data_ptr<float>();
    fa.n = n;
    fa.d = h.data_ptr();
    fa.st = st;
    const int rc = launch_fused_dispatch_gemm(fa, num_sms, stream);
    TORCH_CHECK(rc == 0, "fused dispatch + GEMM launch failed (code " + std::to_string(rc) + ")");
    EP_CUDA_CHECK(cudaGetLastError());

    wait_host_counters(ticket);
    const int num_recv = host_counters_->num_recv_tokens;
    std::vector<int> per_expert_list(host_counters_->num_recv_tokens_per_expert,
                                     host_counters_->num_recv_tokens_per_expert + E_l);
    int64_t rows = 0;
    for (int c : per_expert_list) rows += c;
    scope.finish(false, {});
    auto offsets = torch::zeros({E_l + 1}, i32);
    offsets.narrow(0, 1, E_l).copy_(aligned_counts.cumsum(0));
    return {h.narrow(0, 0, rows), a_rows.narrow(0, 0, rows), a_scales.narrow(0, 0, rows), row_map.narrow(0, 0, num_recv),
            recv_w.narrow(0, 0, num_recv), offsets, raw_counts, recv_src_idx.narrow(0, 0, num_recv), per_expert_list, rpm, spm,
            recv_rank_prefix, send_head};
}

std::tuple<torch::Tensor, std::optional<torch::Tensor>, std::optional<EventHandle>> Buffer::intranode_combine(
    const torch::Tensor& x, const std::optional<torch::Tensor>& topk_weights, const std::optional<torch::Tensor>& bias_0,
    const std::optional<torch::Tensor>& bias_1, const torch::Tensor& rank_prefix_matrix,
    const torch::Tensor& send_prefix_matrix, const torch::Tensor& send_head, const torch::Tensor& recv_src_idx, int num_sms,
    std::optional<EventHandle>& previous_event, bool async, bool allocate_on_comm_stream,
    const std::optional<torch::Tensor>& row_map, const std::optional<torch::Tensor>& row_weights) {
    check_error();
    // Expanded mode: x has one row per (received token, local expert); row_map [num_recv][K] names
    // each token's rows, row_weights [num_recv][K] (optional) their fp32 factors.
    const bool expanded = row_map.has_value();
    const int64_t num_recv_rows = expanded ? row_map->size(0) : x.size(0);
    if (expanded) {
        TORCH_CHECK(row_map->dim() == 2 && row_map->scalar_type() == torch::kInt32 && row_map->is_contiguous() &&
                        row_map->size(1) >= 1 && row_map->size(1) <= 32,
                    "row_map must be contiguous int32 [num_recv, K] with 1 <= K <= 32");
        if (row_weights.has_value())
            TORCH_CHECK(row_weights->scalar_type() == torch::kFloat32 && row_weights->is_contiguous() &&
                            row_weights->sizes() == row_map->sizes(),
                        "row_weights must be contiguous fp32 with row_map's shape");
    } else {
        TORCH_CHECK(!row_weights.has_value(), "row_weights needs row_map");
    }
    TORCH_CHECK(recv_src_idx.scalar_type() == torch::kInt32 && recv_src_idx.is_contiguous() && recv_src_idx.size(0) >= num_recv_rows,
                "handle's recv_src_idx must cover every received token");
    TORCH_CHECK(available_, "buffer not synced");
    TORCH_CHECK(x.dim() == 2 && x.is_contiguous() && x.scalar_type() == torch::kBFloat16, "x must be contiguous bf16 [rows, hidden]");
    const int H = (int)x.size(1), R = num_ranks_;
    const int N = (int)send_head.size(0);
    TORCH_CHECK(H % 8 == 0, "hidden must be a multiple of 8");
    const int K = topk_weights.has_value() ? (int)topk_weights->size(1) : 0;
    if (topk_weights.has_value())
        TORCH_CHECK(topk_weights->scalar_type() == torch::kFloat32 && topk_weights->is_contiguous() &&
                    topk_weights->size(0) == num_recv_rows);
    for (const auto* b : {&bias_0, &bias_1})
        if (b->has_value())
            TORCH_CHECK((*b)->scalar_type() == torch::kBFloat16 && (*b)->is_contiguous() && (*b)->size(0) == N && (*b)->size(1) == H);
    const NormalLayout L = compute_normal_layout(num_nvl_bytes_, H, R);
    TORCH_CHECK(N <= L.capacity, "num_tokens exceeds the buffer capacity");
    if (num_sms <= 0) num_sms = 32;
    StreamScope scope(comm_stream_, previous_event, allocate_on_comm_stream);
    auto stream = scope.comm.stream();
    auto out = torch::empty({N, H}, x.options());
    std::optional<torch::Tensor> out_w;
    if (topk_weights.has_value()) out_w = torch::empty({N, K}, torch::dtype(torch::kFloat32).device(torch::kCUDA));
    if (poison_outputs_) {
        poison(out, stream);
        if (out_w.has_value()) poison(*out_w, stream);
    }
    const KernelStatus st = status();
    const PeerTable peers = nvl_peers();

    CombineArgs ca{};
    ca.peers = peers;
    ca.layout = L;
    ca.rank = rank_;
    ca.num_ranks = R;
    ca.num_topk = K;
    ca.x = x.data_ptr();
    ca.topk_weights = topk_weights.has_value() ? topk_weights->data_ptr<float>() : nullptr;
    ca.num_recv_max = (int)num_recv_rows;
    ca.row_map = expanded ? row_map->data_ptr<int>() : nullptr;
    ca.row_weights = row_weights.has_value() ? row_weights->data_ptr<float>() : nullptr;
    ca.row_map_k = expanded ? (int)row_map->size(1) : 0;
    ca.x_rows = (int)x.size(0);
    ca.rank_prefix_matrix = rank_prefix_matrix.data_ptr<int>();
    ca.send_prefix_matrix = send_prefix_matrix.data_ptr<int>();
    ca.recv_src_idx = recv_src_idx.data_ptr<int>();
    ca.send_head = send_head.data_ptr<int>();
    ca.num_tokens = N;
    ca.has_weights = topk_weights.has_value() ? 1 : 0;
    ca.bias0 = bias_0.has_value() ? bias_0->data_ptr() : nullptr;
    ca.bias1 = bias_1.has_value() ? bias_1->data_ptr() : nullptr;
    ca.out = out.data_ptr();
    ca.out_topk_weights = out_w.has_value() ? out_w->data_ptr<float>() : nullptr;
    ca.stages = 0;
    ca.chunk = combine_row_chunk_;
    ca.announce_lagged = combine_announce_lagged_ ? 1 : 0;
    ca.st = st;
    prof_mark(stream, 4);
    launch_combine(ca, num_sms, stream);
    prof_mark(stream, 5);
    EP_CUDA_CHECK(cudaGetLastError());
    auto event = scope.finish(async, {x, topk_weights, bias_0, bias_1, rank_prefix_matrix, send_prefix_matrix, send_head, out, out_w,
                                      row_map, row_weights});
    return {out, out_w, event};
}

std::vector<int> Buffer::selftest_signal_stress(int producer_blocks, int warps, int rounds) {
    check_error();
    TORCH_CHECK(available_, "buffer not synced");
    TORCH_CHECK(producer_blocks >= 1 && producer_blocks <= 1024 && warps >= 1 && warps <= 32 && rounds >= 1,
                "producer_blocks in [1, 1024], warps in [1, 32], rounds >= 1");
    const int64_t total = (int64_t)producer_blocks * warps * rounds;
    TORCH_CHECK(total < (int64_t)1 << 30, "too many signals for an int counter");
    const NormalLayout L = compute_normal_layout(num_nvl_bytes_, 128, num_ranks_);
    const int next = (rank_ + 1) % num_ranks_;
    auto* mine = reinterpret_cast<NormalCtrl*>(static_cast<uint8_t*>(nvl_base_) + L.ctrl_off);
    auto* peer = reinterpret_cast<NormalCtrl*>(static_cast<uint8_t*>(nvl_peer_[next]) + L.ctrl_off);
    auto result = torch::full({2}, -1, torch::dtype(torch::kInt32).device(torch::kCUDA));
    auto stream = at::cuda::getCurrentCUDAStream();
    // every rank's flag starts at zero before any rank's producers run
    EP_CUDA_CHECK(cudaMemsetAsync(&mine->selftest_flag, 0, sizeof(int), stream));
    barrier(false, true);
    launch_signal_stress(&peer->selftest_flag, &mine->selftest_flag, producer_blocks, warps, rounds, (int)total,
                         result.data_ptr<int>(), status(), stream);
    EP_CUDA_CHECK(cudaGetLastError());
    auto host = result.cpu();
    barrier(false, true);
    return {host[0].item<int>(), host[1].item<int>()};
}

// NVLink micro-probes. Every rank calls them together, with no dispatch or combine in flight.
// Flag round trip between rank 0 and `peer` (one GPU: between the two blocks of one launch): mean
// round-trip ns on rank 0 and on `peer`, 0 on the other ranks; an expired wait raises.
double Buffer::probe_flag_latency(int peer, int iters) {
    check_error();
    TORCH_CHECK(available_, "buffer not synced");
    TORCH_CHECK(iters >= 1 && iters <= (1 << 20), "iters in [1, 2^20]");
    TORCH_CHECK(num_ranks_ == 1 ? peer == 0 : (peer >= 1 && peer < num_ranks_), "peer must be another rank (0 on one GPU)");
    const NormalLayout L = compute_normal_layout(num_nvl_bytes_, 128, num_ranks_);
    auto ctrl_of = [&](void* base) { return reinterpret_cast<NormalCtrl*>(static_cast<uint8_t*>(base) + L.ctrl_off); };
    NormalCtrl* mine = ctrl_of(nvl_base_);
    auto out = torch::zeros({2}, torch::dtype(torch::kInt64).device(torch::kCUDA));
    auto stream = at::cuda::getCurrentCUDAStream();
    EP_CUDA_CHECK(cudaMemsetAsync(&mine->probe_flag, 0, sizeof(int), stream));
    EP_CUDA_CHECK(cudaMemsetAsync(&mine->selftest_flag, 0, sizeof(int), stream));
    barrier(false, true);  // every flag is zero before either side writes
    auto* ns = reinterpret_cast<long long*>(out.data_ptr<int64_t>());
    const bool active = num_ranks_ == 1 || rank_ == 0 || rank_ == peer;
    if (num_ranks_ == 1) launch_flag_pingpong(&mine->selftest_flag, &mine->probe_flag, iters, 2, ns, status(), stream);
    else if (rank_ == 0) launch_flag_pingpong(&ctrl_of(nvl_peer_[peer])->probe_flag, &mine->probe_flag, iters, 0, ns, status(), stream);
    else if (rank_ == peer) launch_flag_pingpong(&ctrl_of(nvl_peer_[0])->probe_flag, &mine->probe_flag, iters, 1, ns, status(), stream);
    EP_CUDA_CHECK(cudaGetLastError());
    const int64_t elapsed = out.cpu()[0].item<int64_t>();
    barrier(false, true);  // raises if a wait expired
    return active ? (double)elapsed / iters : 0.0;
}

// Copy `bytes` between `local` and the normal-mode region of rank (rank + shift) % R (past its
// control block; dispatch / combine data there is overwritten), `offset` bytes in on both sides:
// peer stores (`store`) or peer loads. Every rank copies at the same time, after a barrier. Returns
// the `reps` CUDA-event timings of this rank's copy in milliseconds, then the access width used.
std::vector<double> Buffer::probe_peer_copy(int shift, int64_t bytes, int64_t offset, bool store, int reps, int blocks,
                                            const torch::Tensor& local) {
    check_error();
    TORCH_CHECK(available_, "buffer not synced");
    TORCH_CHECK(shift >= 0 && shift < num_ranks_ && reps >= 1 && reps <= 1000 && blocks >= 1 && blocks <= 4096, "bad probe arguments");
    TORCH_CHECK(local.is_cuda() && local.is_contiguous() && local.scalar_type() == torch::kUInt8, "local must be a contiguous uint8 CUDA tensor");
    TORCH_CHECK(bytes >= 1 && offset >= 0 && offset + bytes <= local.numel(), "local tensor smaller than offset + bytes");
    const int64_t data_off = align_up(sizeof(NormalCtrl), 4096);  // everything past the control block
    TORCH_CHECK(offset + bytes <= num_nvl_bytes_ - data_off, "offset + bytes exceed the peer's normal-mode region");
    uint8_t* remote = static_cast<uint8_t*>(nvl_peer_[(rank_ + shift) % num_ranks_]) + data_off + offset;
    uint8_t* here = local.data_ptr<uint8_t>() + offset;
    const uintptr_t both = reinterpret_cast<uintptr_t>(remote) | reinterpret_cast<uintptr_t>(here);
    int vec = 16;
    while (vec > 1 && (both % vec) != 0) vec >>= 1;
    auto stream = at::cuda::getCurrentCUDAStream();
    barrier(false, true);
    std::vector<double> ms;
    cudaEvent_t e0, e1;
    EP_CUDA_CHECK(cudaEventCreate(&e0));
    EP_CUDA_CHECK(cudaEventCreate(&e1));
    for (int r = 0; r < reps; ++r) {
        EP_CUDA_CHECK(cudaEventRecord(e0, stream));
        if (store) launch_probe_copy(remote, here, bytes, vec, blocks, stream);
        else launch_probe_copy(here, remote, bytes, vec, blocks, stream);
        EP_CUDA_CHECK(cudaEventRecord(e1, stream));
        EP_CUDA_CHECK(cudaEventSynchronize(e1));
        float t = 0.f;
        EP_CUDA_CHECK(cudaEventElapsedTime(&t, e0, e1));
        ms.push_back(t);
    }
    EP_CUDA_CHECK(cudaEventDestroy(e0));
    EP_CUDA_CHECK(cudaEventDestroy(e1));
    barrier(false, true);
    ms.push_back((double)vec);  // last entry: the access width used
    return ms;
}

void Buffer::barrier(bool use_comm_stream, bool with_cpu_sync) {
    check_error();
    if (with_cpu_sync) EP_CUDA_CHECK(cudaDeviceSynchronize());
    auto compute = at::cuda::getCurrentCUDAStream();
    auto stream = use_comm_stream ? comm_stream_ : compute;
    if (use_comm_stream) stream_wait(comm_stream_, compute);
    launch_barrier(nvl_peers(), 0, rank_, num_ranks_, status(), stream.stream());
    if (use_comm_stream) stream_wait(compute, comm_stream_);
    if (with_cpu_sync) {
        EP_CUDA_CHECK(cudaDeviceSynchronize());
        check_error();
    }
}

// =================================================================================================
// Low-latency mode
// =================================================================================================
void Buffer::clean_low_latency_buffer(int num_max_dispatch_tokens_per_rank, int hidden, int num_experts) {
    TORCH_CHECK(ll_base_ != nullptr, "no low-latency region (num_rdma_bytes == 0)");
    const LLLayout L = compute_ll_layout(num_rdma_bytes_, num_max_dispatch_tokens_per_rank, hidden, num_experts, num_ranks_);
    TORCH_CHECK(2 * L.half_bytes <= num_rdma_bytes_, "low-latency region too small");
    barrier(true, true);
    launch_ll_clean(ll_peers(), L, rank_, status(), comm_stream_.stream());
    barrier(true, true);
}

std::tuple<torch::Tensor, std::optional<torch::Tensor>, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, int,
           std::optional<EventHandle>, std::optional<std::function<void()>>>
Buffer::low_latency_dispatch(const torch::Tensor& x, const torch::Tensor& topk_idx,
                             const std::optional<torch::Tensor>& cumulative_local_expert_recv_stats,
                             const std::optional<torch::Tensor>& dispatch_wait_recv_cost_stats,
                             int num_max_dispatch_tokens_per_rank, int num_experts, bool use_fp8, bool round_scale,
                             bool use_ue8m0, bool async, bool return_recv_hook) {
    check_error();
    TORCH_CHECK(available_ && ll_base_ != nullptr, "low-latency mode needs num_rdma_bytes > 0");
    TORCH_CHECK(x.dim() == 2 && x.is_contiguous() && x.scalar_type() == torch::kBFloat16, "x must be contiguous bf16");
    TORCH_CHECK(topk_idx.dim() == 2 && topk_idx.is_contiguous() && topk_idx.scalar_type() == torch::kInt64);
    TORCH_CHECK(!use_ue8m0 || round_scale, "use_ue8m0 requires round_scale");
    const int N = (int)x.size(0), H = (int)x.size(1), K = (int)topk_idx.size(1), R = num_ranks_;
    const int maxT = num_max_dispatch_tokens_per_rank;
    TORCH_CHECK(N <= maxT, "num_tokens exceeds num_max_dispatch_tokens_per_rank");
    TORCH_CHECK(H % 128 == 0 && K <= kMaxTopk && num_experts % R == 0);
    LLLayout L = compute_ll_layout(num_rdma_bytes_, maxT, H, num_experts, R);
    TORCH_CHECK(2 * L.half_bytes <= num_rdma_bytes_, "low-latency region too small: need " + std::to_string(2 * L.half_bytes) +
                                                         " bytes (Buffer.get_low_latency_rdma_size_hint)");
    TORCH_CHECK(L.num_local_experts <= kMaxLocalExperts);
    L.num_topk = K;
    const int half = (++ll_dispatch_seq_) & 1;
    const int E_l = L.num_local_experts, slots = R * maxT;

    auto compute = at::cuda::getCurrentCUDAStream();
    auto launch_stream = return_recv_hook ? compute : comm_stream_;
    if (!return_recv_hook) stream_wait(comm_stream_, compute);
    auto i32 = torch::dtype(torch::kInt32).device(torch::kCUDA);
    auto recv_count = torch::empty({E_l}, i32);
    auto layout_range = torch::empty({E_l, R}, torch::dtype(torch::kInt64).device(torch::kCUDA));
    if (return_recv_hook || async) {
        recv_count.record_stream(launch_stream);
        layout_range.record_stream(launch_stream);
    }

    LLDispatchArgs a{};
    a.peers = ll_peers();
    a.layout = L;
    a.half = half;
    a.x = x.data_ptr();
    a.topk_idx = topk_idx.data_ptr<int64_t>();
    a.num_tokens = N;
    a.rank = rank_;
    a.use_fp8 = use_fp8 ? 1 : 0;
    a.round_scale = round_scale ? 1 : 0;
    a.use_ue8m0 = use_ue8m0 ? 1 : 0;
    a.mask = mask_;
    a.shrink = enable_shrink_ ? 1 : 0;
    a.recv_count = recv_count.data_ptr<int>();
    a.layout_range = layout_range.data_ptr<int64_t>();
    a.cumulative_stats = cumulative_local_expert_recv_stats.has_value() ? cumulative_local_expert_recv_stats->data_ptr<int>() : nullptr;
    a.wait_stats = dispatch_wait_recv_cost_stats.has_value() ? dispatch_wait_recv_cost_stats->data_ptr<int64_t>() : nullptr;
    a.st = status();
    a.phases = return_recv_hook ? 1 : 3;
    launch_ll_dispatch(a, launch_stream.stream());
    EP_CUDA_CHECK(cudaGetLastError());

    uint8_t* half_base = static_cast<uint8_t*>(ll_base_) + (int64_t)half * L.half_bytes;
    auto dev = torch::TensorOptions().device(torch::kCUDA, device_id_);
    auto recv_x = torch::from_blob(half_base + L.recv_x_off, {E_l, slots, H}, dev.dtype(use_fp8 ? torch::kFloat8_e4m3fn : torch::kBFloat16));
    std::optional<torch::Tensor> recv_scales;
    if (use_fp8) {
        const int nb = H / 128;
        recv_scales = torch::from_blob(half_base + L.recv_scales_off, {E_l, slots, nb}, {(int64_t)nb * slots, 1, slots},
                                       dev.dtype(torch::kFloat32));
    }
    auto src_info = torch::from_blob(half_base + L.recv_src_info_off, {E_l, slots}, dev.dtype(torch::kInt32));
    auto src_meta = torch::from_blob(half_base + L.recv_src_meta_off, {E_l, slots}, dev.dtype(torch::kInt32));

    std::optional<EventHandle> event;
    std::optional<std::function<void()>> hook;
    if (return_recv_hook) {
        LLDispatchArgs ra = a;
        ra.phases = 2;
        hook = [ra, recv_count, layout_range, this]() mutable {
            check_error();
            launch_ll_dispatch(ra, at::cuda::getCurrentCUDAStream().stream());
        };
    } else if (async) {
        event = EventHandle(comm_stream_);
        x.record_stream(comm_stream_);
        topk_idx.record_stream(comm_stream_);
    } else {
        stream_wait(compute, comm_stream_);
    }
    return {recv_x, recv_scales, recv_count, src_info, src_meta, layout_range, half, event, hook};
}

std::tuple<torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, int>
Buffer::low_latency_dispatch_gemm(const torch::Tensor& x, const torch::Tensor& topk_idx,
                                  const std::optional<torch::Tensor>& cumulative_local_expert_recv_stats,
                                  int num_max_dispatch_tokens_per_rank, int num_experts, const torch::Tensor& w,
                                  const torch::Tensor& w_scales, bool round_scale, int num_sms) {
    TORCH_CHECK(!enable_shrink_, "the fused receive does not support shrink mode");
    const int R = num_ranks_, maxT = num_max_dispatch_tokens_per_rank, H = (int)x.size(1);
    // Send phase only (on the compute stream); the hook is dropped: the GEMM kernel below receives.
    auto sent = low_latency_dispatch(x, topk_idx, std::nullopt, std::nullopt, maxT, num_experts, /*use_fp8=*/true,
                                     round_scale, /*use_ue8m0=*/false, /*async=*/false, /*return_recv_hook=*/true);
    torch::Tensor recv_x = std::get<0>(sent), recv_count = std::get<2>(sent);
    torch::Tensor recv_scales = std::get<1>(sent).value();
    const int half = std::get<6>(sent);
    const LLLayout L = compute_ll_layout(num_rdma_bytes_, maxT, H, num_experts, R);
    const int E_l = L.num_local_experts, slots = R * maxT;
    TORCH_CHECK(w.is_cuda() && w.dim() == 3 && w.is_contiguous() && w.scalar_type() == torch::kFloat8_e4m3fn && w.size(0) == E_l &&
                    w.size(2) == H && w.size(1) % 128 == 0,
                "weights must be contiguous [num_local_experts, n, hidden] e4m3 with n % 128 == 0");
    const int n = (int)w.size(1);
    TORCH_CHECK(w_scales.scalar_type() == torch::kFloat32 && w_scales.is_contiguous() && w_scales.dim() == 3 &&
                    w_scales.size(0) == E_l && w_scales.size(1) == n / 128 && w_scales.size(2) == H / 128,
                "weight scales must be [num_local_experts, n/128, hidden/128] fp32");
    if (cumulative_local_expert_recv_stats.has_value())
        TORCH_CHECK(cumulative_local_expert_recv_stats->scalar_type() == torch::kInt32 &&
                    cumulative_local_expert_recv_stats->numel() == E_l);
    if (num_sms <= 0) EP_CUDA_CHECK(cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, device_id_));
    auto out = torch::empty({E_l, slots, n}, x.options());
    MaskedGemmArgs g{};
    g.a = recv_x.data_ptr();
    g.sa = recv_scales.data_ptr<float>();
    g.sa_e = recv_scales.stride(0);
    g.sa_m = recv_scales.stride(1);
    g.sa_k = recv_scales.stride(2);
    g.b = w.data_ptr();
    g.sb = w_scales.data_ptr<float>();
    g.counts = nullptr;
    g.d = out.data_ptr();
    g.num_experts = E_l;
    g.slots = slots;
    g.n = n;
    g.k = H;
    uint8_t* half_base = static_cast<uint8_t*>(ll_base_) + (int64_t)half * L.half_bytes;
    g.ll = reinterpret_cast<LLCtrl*>(half_base + L.ctrl_off);
    g.num_ranks = R;
    g.recv_count = recv_count.data_ptr<int>();
    g.cumulative_stats =
        cumulative_local_expert_recv_stats.has_value() ? cumulative_local_expert_recv_stats->data_ptr<int>() : nullptr;
    // About 3/4 of the 126 MB L2 for weights fetched while the peers' tokens are in flight.
    g.l2_prefetch_bytes = ((int64_t)(96 << 20) / num_sms) & ~(int64_t)15;
    g.st = status();
    const int rc = launch_masked_gemm_fp8(g, num_sms, at::cuda::getCurrentCUDAStream().stream());
    TORCH_CHECK(rc == 0, "fused low-latency receive + masked GEMM launch failed (code " + std::to_string(rc) + ")");
    return {out, recv_x, recv_scales, recv_count, std::get<3>(sent), std::get<4>(sent), half};
}

torch::Tensor Buffer::low_latency_gemm_combine(const torch::Tensor& a, const torch::Tensor& a_scales,
                                              const torch::Tensor& recv_count, const torch::Tensor& w, const torch::Tensor& w_scales,
                                              const torch::Tensor& topk_idx, const torch::Tensor& topk_weights, int dispatch_half,
                                              int num_max_dispatch_tokens_per_rank, int num_experts, int num_sms) {
    check_error();
    TORCH_CHECK(available_ && ll_base_ != nullptr, "low-latency mode needs num_rdma_bytes > 0");
    TORCH_CHECK(!enable_shrink_, "the fused combine does not support shrink mode");
    const int R = num_ranks_, maxT = num_max_dispatch_tokens_per_rank;
    TORCH_CHECK(a.is_cuda() && a.dim() == 3 && a.is_contiguous() && a.scalar_type() == torch::kFloat8_e4m3fn,
                "a must be a contiguous [num_local_experts, slots, k] e4m3 tensor");
    TORCH_CHECK(w.dim() == 3 && w.is_contiguous() && w.scalar_type() == torch::kFloat8_e4m3fn, "w must be [E_l, hidden, k] e4m3");
    const int E_l = (int)a.size(0), slots = (int)a.size(1), k = (int)a.size(2), H = (int)w.size(1);
    TORCH_CHECK(slots == R * maxT && w.size(0) == E_l && w.size(2) == k && k % 128 == 0 && H % 128 == 0);
    TORCH_CHECK(a_scales.scalar_type() == torch::kFloat32 && a_scales.dim() == 3 && a_scales.size(0) == E_l &&
                a_scales.size(1) == slots && a_scales.size(2) == k / 128);
    TORCH_CHECK(w_scales.scalar_type() == torch::kFloat32 && w_scales.is_contiguous() && w_scales.size(0) == E_l &&
                w_scales.size(1) == H / 128 && w_scales.size(2) == k / 128);
    TORCH_CHECK(recv_count.scalar_type() == torch::kInt32 && recv_count.is_contiguous() && recv_count.numel() == E_l);
    const int N = (int)topk_idx.size(0), K = (int)topk_idx.size(1);
    TORCH_CHECK(topk_idx.scalar_type() == torch::kInt64 && topk_idx.is_contiguous() && N <= maxT && K <= kMaxTopk);
    TORCH_CHECK(topk_weights.scalar_type() == torch::kFloat32 && topk_weights.is_contiguous() && topk_weights.size(0) == N);
    LLLayout L = compute_ll_layout(num_rdma_bytes_, maxT, H, num_experts, R);
    TORCH_CHECK(2 * L.half_bytes <= num_rdma_bytes_, "low-latency region too small");
    TORCH_CHECK(L.num_local_experts == E_l, "a must hold every local expert");
    L.num_topk = K;
    const int half = (++ll_combine_seq_) & 1;
    auto compute = at::cuda::getCurrentCUDAStream();
    if (num_sms <= 0) EP_CUDA_CHECK(cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, device_id_));

    // 1) down projection whose epilogue stores rows into the sources' combine slots (send phase)
    MaskedGemmArgs g{};
    g.a = a.data_ptr();
    g.sa = a_scales.data_ptr<float>();
    g.sa_e = a_scales.stride(0);
    g.sa_m = a_scales.stride(1);
    g.sa_k = a_scales.stride(2);
    g.b = w.data_ptr();
    g.sb = w_scales.data_ptr<float>();
    g.counts = recv_count.data_ptr<int>();
    g.d = nullptr;
    g.num_experts = E_l;
    g.slots = slots;
    g.n = H;
    g.k = k;
    g.combine = 1;
    g.ll_peers = ll_peers();
    g.ll_layout = L;
    g.dispatch_half = dispatch_half;
    g.combine_half = half;
    g.rank = rank_;
    g.st = status();
    const int rc = launch_masked_gemm_fp8(g, num_sms, compute.stream());
    TORCH_CHECK(rc == 0, "fused masked GEMM + combine send launch failed (code " + std::to_string(rc) + ")");

    // 2) the combine's receive phase: weighted top-k reduction
    auto combined = torch::empty({N, H}, topk_weights.options().dtype(torch::kBFloat16));
    LLCombineArgs ca{};
    ca.peers = ll_peers();
    ca.layout = L;
    ca.half = half;
    ca.dispatch_half = dispatch_half;
    ca.x = nullptr;
    ca.recv_count = recv_count.data_ptr<int>();
    ca.topk_idx = topk_idx.data_ptr<int64_t>();
    ca.topk_weights = topk_weights.data_ptr<float>();
    ca.num_tokens = N;
    ca.rank = rank_;
    ca.mask = mask_;
    ca.shrink = 0;
    ca.out = combined.data_ptr();
    ca.st = status();
    ca.phases = 2;
    launch_ll_combine(ca, compute.stream());
    EP_CUDA_CHECK(cudaGetLastError());
    return combined;
}

std::tuple<torch::Tensor, std::optional<EventHandle>, std::optional<std::function<void()>>> Buffer::low_latency_combine(
    const torch::Tensor& x, const torch::Tensor& topk_idx, const torch::Tensor& topk_weights, const torch::Tensor& recv_count,
    int dispatch_half, const std::optional<torch::Tensor>& combine_wait_recv_cost_stats, int num_max_dispatch_tokens_per_rank,
    int num_experts, bool use_logfmt, bool zero_copy, bool async, bool return_recv_hook, const std::optional<torch::Tensor>& out) {
    check_error();
    TORCH_CHECK(available_ && ll_base_ != nullptr, "low-latency mode needs num_rdma_bytes > 0");
    TORCH_CHECK(!(use_logfmt && zero_copy), "LogFMT combine encodes from the caller's tensor: zero_copy is not allowed");
    const int R = num_ranks_, maxT = num_max_dispatch_tokens_per_rank;
    TORCH_CHECK(x.dim() == 3 && x.scalar_type() == torch::kBFloat16 && x.is_contiguous());
    const int H = (int)x.size(2), N = (int)topk_idx.size(0), K = (int)topk_idx.size(1);
    TORCH_CHECK(topk_weights.scalar_type() == torch::kFloat32 && topk_weights.is_contiguous() && topk_weights.size(0) == N);
    TORCH_CHECK(N <= maxT && K <= kMaxTopk);
    LLLayout L = compute_ll_layout(num_rdma_bytes_, maxT, H, num_experts, R);
    TORCH_CHECK(2 * L.half_bytes <= num_rdma_bytes_, "low-latency region too small");
    TORCH_CHECK(x.size(0) == L.num_local_experts && x.size(1) == (int64_t)R * maxT, "x must be [num_local_experts, num_ranks * max_tokens, hidden]");
    L.num_topk = K;
    const int half = (++ll_combine_seq_) & 1;
    auto compute = at::cuda::getCurrentCUDAStream();
    auto launch_stream = return_recv_hook ? compute : comm_stream_;
    if (!return_recv_hook) stream_wait(comm_stream_, compute);
    torch::Tensor combined = out.has_value() ? *out : torch::empty({N, H}, x.options());
    TORCH_CHECK(combined.is_contiguous() && combined.size(0) == N && combined.size(1) == H && combined.scalar_type() == torch::kBFloat16);

    LLCombineArgs a{};
    a.peers = ll_peers();
    a.layout = L;
    a.half = half;
    a.dispatch_half = dispatch_half;
    const void* src = x.data_ptr();
    if (zero_copy) {
        // The caller filled the registered send buffer of this combine's half.
        src = static_cast<uint8_t*>(ll_base_) + (int64_t)half * L.half_bytes + L.combine_send_off;
    }
    a.x = src;
    a.recv_count = recv_count.data_ptr<int>();
    a.topk_idx = topk_idx.data_ptr<int64_t>();
    a.topk_weights = topk_weights.data_ptr<float>();
    a.num_tokens = N;
    a.rank = rank_;
    a.mask = mask_;
    a.shrink = enable_shrink_ ? 1 : 0;
    a.out = combined.data_ptr();
    a.wait_stats = combine_wait_recv_cost_stats.has_value() ? combine_wait_recv_cost_stats->data_ptr<int64_t>() : nullptr;
    a.st = status();
    a.phases = return_recv_hook ? 1 : 3;
    a.use_logfmt = use_logfmt ? 1 : 0;
    TORCH_CHECK(!use_logfmt || H <= 128 * 128, "LogFMT combine supports hidden <= 16384");
    launch_ll_combine(a, launch_stream.stream());
    EP_CUDA_CHECK(cudaGetLastError());

    std::optional<EventHandle> event;
    std::optional<std::function<void()>> hook;
    if (return_recv_hook) {
        LLCombineArgs ra = a;
        ra.phases = 2;
        hook = [ra, combined, topk_idx, topk_weights, this]() mutable {
            check_error();
            launch_ll_combine(ra, at::cuda::getCurrentCUDAStream().stream());
        };
    } else if (async) {
        event = EventHandle(comm_stream_);
        for (auto t : {x, topk_idx, topk_weights, recv_count, combined}) t.record_stream(comm_stream_);
    } else {
        stream_wait(compute, comm_stream_);
    }
    return {combined, event, hook};
}

torch::Tensor Buffer::get_next_low_latency_combine_buffer(int num_max_dispatch_tokens_per_rank, int hidden, int num_experts) {
    TORCH_CHECK(ll_base_ != nullptr, "no low-latency region");
    const LLLayout L = compute_ll_layout(num_rdma_bytes_, num_max_dispatch_tokens_per_rank, hidden, num_experts, num_ranks_);
    const int half = (ll_combine_seq_ + 1) & 1;
    uint8_t* base = static_cast<uint8_t*>(ll_base_) + (int64_t)half * L.half_bytes + L.combine_send_off;
    return torch::from_blob(base, {L.num_local_experts, (int64_t)num_ranks_ * num_max_dispatch_tokens_per_rank, hidden},
                            torch::TensorOptions().dtype(torch::kBFloat16).device(torch::kCUDA, device_id_));
}

void Buffer::low_latency_update_mask_buffer(int rank_to_mask, bool mask) {
    TORCH_CHECK(enable_shrink_, "mask APIs need enable_shrink=True");
    TORCH_CHECK(rank_to_mask >= 0 && rank_to_mask < num_ranks_);
    const int v = mask ? 1 : 0;
    EP_CUDA_CHECK(cudaMemcpyAsync(mask_ + rank_to_mask, &v, sizeof(int), cudaMemcpyHostToDevice, at::cuda::getCurrentCUDAStream()));
    EP_CUDA_CHECK(cudaStreamSynchronize(at::cuda::getCurrentCUDAStream()));
}

void Buffer::low_latency_query_mask_buffer(const torch::Tensor& mask_status) {
    TORCH_CHECK(enable_shrink_, "mask APIs need enable_shrink=True");
    TORCH_CHECK(mask_status.numel() == num_ranks_ && mask_status.scalar_type() == torch::kInt32 && mask_status.is_cuda());
    EP_CUDA_CHECK(cudaMemcpyAsync(mask_status.data_ptr(), mask_, sizeof(int) * num_ranks_, cudaMemcpyDeviceToDevice,
                                  at::cuda::getCurrentCUDAStream()));
}

void Buffer::low_latency_clean_mask_buffer() {
    TORCH_CHECK(enable_shrink_, "mask APIs need enable_shrink=True");
    EP_CUDA_CHECK(cudaMemsetAsync(mask_, 0, sizeof(int) * kMaxRanks, at::cuda::getCurrentCUDAStream()));
}

}  // namespace ep
