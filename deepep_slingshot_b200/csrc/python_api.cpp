// pybind11 module `deepep_slingshot_b200._C`: the runtime classes (Buffer, Config, EventHandle) and
// the standalone sm_100a ops. Mirrors the reference's module surface ([DE]csrc/python_api.cpp:1-39,
// pybind section [DE]csrc/legacy/buffer.hpp:1751-1792).
#include <ATen/cuda/CUDAContext.h>
#include <pybind11/functional.h>
#include <pybind11/stl.h>
#include <torch/extension.h>

#include "kernels/api.h"
#include "runtime/buffer.hpp"
#include "runtime/host_segment.hpp"
#include "runtime/ops.hpp"
#include "runtime/symmetric.hpp"

namespace py = pybind11;

PYBIND11_MODULE(_C, m) {
    m.doc() = "B200-native expert-parallel communication runtime (NVLink 5 / NVSwitch, sm_100a)";
    m.attr("abi_version") = ep::kAbiVersion;
    m.attr("max_ranks") = ep::kMaxRanks;
    m.attr("max_topk") = ep::kMaxTopk;

    py::class_<ep::Config>(m, "Config")
        .def(py::init<int, int, int, int, int>(), py::arg("num_sms") = 20, py::arg("num_max_nvl_chunked_send_tokens") = 6,
             py::arg("num_max_nvl_chunked_recv_tokens") = 256, py::arg("num_max_rdma_chunked_send_tokens") = 6,
             py::arg("num_max_rdma_chunked_recv_tokens") = 256)
        .def_readwrite("num_sms", &ep::Config::num_sms)
        .def_readwrite("num_max_nvl_chunked_send_tokens", &ep::Config::num_max_nvl_chunked_send_tokens)
        .def_readwrite("num_max_nvl_chunked_recv_tokens", &ep::Config::num_max_nvl_chunked_recv_tokens)
        .def_readwrite("num_max_rdma_chunked_send_tokens", &ep::Config::num_max_rdma_chunked_send_tokens)
        .def_readwrite("num_max_rdma_chunked_recv_tokens", &ep::Config::num_max_rdma_chunked_recv_tokens)
        .def("get_nvl_buffer_size_hint", &ep::Config::get_nvl_buffer_size_hint, py::arg("hidden_bytes"), py::arg("num_ranks"),
             py::arg("num_max_tokens") = 4096, py::arg("num_topk") = 8)
        .def("get_rdma_buffer_size_hint", &ep::Config::get_rdma_buffer_size_hint);

    py::class_<ep::EventHandle>(m, "EventHandle")
        .def(py::init<>())
        .def("current_stream_wait", &ep::EventHandle::current_stream_wait);

    m.def("normal_region_size_for", &ep::normal_region_size_for);
    m.def("ll_region_size_for", &ep::ll_region_size_for);
    m.def("normal_layout_capacity", [](int64_t region_bytes, int hidden, int num_ranks) {
        return ep::compute_normal_layout(region_bytes, hidden, num_ranks).capacity;
    });
    m.def("window_check", [](const torch::Tensor& cases) {
        TORCH_CHECK(cases.is_cuda() && cases.scalar_type() == torch::kInt64 && cases.dim() == 2 && cases.size(1) == 3 &&
                        cases.is_contiguous(),
                    "cases must be a contiguous int64 CUDA tensor [n, 3] of (index, count, window)");
        auto codes = torch::empty({cases.size(0)}, cases.options().dtype(torch::kInt32));
        ep::launch_window_check(cases.data_ptr<int64_t>(), (int)cases.size(0), codes.data_ptr<int>(),
                                at::cuda::getCurrentCUDAStream());
        return codes;
    });
    m.def("normal_layout", [](int64_t region_bytes, int hidden, int num_ranks) {
        const ep::NormalLayout l = ep::compute_normal_layout(region_bytes, hidden, num_ranks);
        py::dict d;
        d["ctrl_off"] = l.ctrl_off;
        d["list_off"] = l.list_off;
        d["staging_off"] = l.staging_off;
        d["combine_off"] = l.combine_off;
        d["combine_w_off"] = l.combine_w_off;
        d["scratch_off"] = l.scratch_off;
        d["arrival_off"] = l.arrival_off;
        d["total_bytes"] = l.total_bytes;
        d["capacity"] = l.capacity;
        d["record_bytes"] = l.record_bytes;
        return d;
    });
    m.def("ll_layout", [](int max_tokens, int hidden, int num_ranks, int num_experts) {
        const ep::LLLayout l = ep::compute_ll_layout(0, max_tokens, hidden, num_experts, num_ranks);
        py::dict d;
        d["half_bytes"] = l.half_bytes;
        d["ctrl_off"] = l.ctrl_off;
        d["recv_x_off"] = l.recv_x_off;
        d["recv_scales_off"] = l.recv_scales_off;
        d["recv_src_info_off"] = l.recv_src_info_off;
        d["recv_src_meta_off"] = l.recv_src_meta_off;
        d["combine_recv_off"] = l.combine_recv_off;
        d["combine_send_off"] = l.combine_send_off;
        d["combine_meta_off"] = l.combine_meta_off;
        return d;
    });
    m.attr("sym_ctrl_bytes") = ep::kSymCtrlBytes;
    m.attr("sym_ctrl_struct_bytes") = (int64_t)sizeof(ep::SymCtrl);

    py::class_<ep::Buffer>(m, "Buffer")
        .def(py::init<int, int, int64_t, int64_t, bool, bool, bool, double>())
        .def("is_available", &ep::Buffer::is_available)
        .def("get_num_rdma_ranks", &ep::Buffer::get_num_rdma_ranks)
        .def("get_rdma_rank", &ep::Buffer::get_rdma_rank)
        .def("get_root_rdma_rank", &ep::Buffer::get_root_rdma_rank)
        .def("get_local_device_id", &ep::Buffer::get_local_device_id)
        .def("get_local_ipc_handle", &ep::Buffer::get_local_ipc_handle)
        .def("get_local_ll_ipc_handle", &ep::Buffer::get_local_ll_ipc_handle)
        .def("sync", &ep::Buffer::sync)
        .def("destroy", &ep::Buffer::destroy)
        .def("get_comm_stream", &ep::Buffer::get_comm_stream)
        .def("get_local_buffer_tensor", &ep::Buffer::get_local_buffer_tensor)
        .def("get_capacity", &ep::Buffer::get_capacity)
        .def("check_error", &ep::Buffer::check_error)
        .def("get_error_state", &ep::Buffer::get_error_state)
        .def("clear_error", &ep::Buffer::clear_error)
        .def("set_timeout_secs", &ep::Buffer::set_timeout_secs)
        .def("get_profile", &ep::Buffer::get_profile)
        .def("enable_trace", &ep::Buffer::enable_trace)
        .def("disable_trace", &ep::Buffer::disable_trace)
        .def("read_trace", &ep::Buffer::read_trace)
        .def("sample_clock", &ep::Buffer::sample_clock)
        .def("get_dispatch_layout", &ep::Buffer::get_dispatch_layout)
        .def("intranode_dispatch", &ep::Buffer::intranode_dispatch)
        .def("intranode_dispatch_gemm", &ep::Buffer::intranode_dispatch_gemm)
        .def("intranode_combine", &ep::Buffer::intranode_combine)
        .def("barrier", &ep::Buffer::barrier)
        .def("selftest_signal_stress", &ep::Buffer::selftest_signal_stress)
        .def("probe_flag_latency", &ep::Buffer::probe_flag_latency)
        .def("probe_peer_copy", &ep::Buffer::probe_peer_copy)
        .def("clean_low_latency_buffer", &ep::Buffer::clean_low_latency_buffer)
        .def("low_latency_dispatch", &ep::Buffer::low_latency_dispatch)
        .def("low_latency_dispatch_gemm", &ep::Buffer::low_latency_dispatch_gemm)
        .def("low_latency_gemm_combine", &ep::Buffer::low_latency_gemm_combine)
        .def("low_latency_combine", &ep::Buffer::low_latency_combine)
        .def("get_next_low_latency_combine_buffer", &ep::Buffer::get_next_low_latency_combine_buffer)
        .def("low_latency_update_mask_buffer", &ep::Buffer::low_latency_update_mask_buffer)
        .def("low_latency_query_mask_buffer", &ep::Buffer::low_latency_query_mask_buffer)
        .def("low_latency_clean_mask_buffer", &ep::Buffer::low_latency_clean_mask_buffer);

    py::class_<ep::SymmetricRegion>(m, "SymmetricRegion")
        .def(py::init<int, int, int64_t, double>())
        .def("get_local_ipc_handle", &ep::SymmetricRegion::get_local_ipc_handle)
        .def("get_local_device_id", &ep::SymmetricRegion::get_local_device_id)
        .def("sync", &ep::SymmetricRegion::sync)
        .def("is_available", &ep::SymmetricRegion::is_available)
        .def("destroy", &ep::SymmetricRegion::destroy)
        .def("data_bytes", &ep::SymmetricRegion::data_bytes)
        .def("local_data", &ep::SymmetricRegion::local_data)
        .def("check_error", &ep::SymmetricRegion::check_error)
        .def("get_error_state", &ep::SymmetricRegion::get_error_state)
        .def("clear_error", &ep::SymmetricRegion::clear_error)
        .def("barrier", &ep::SymmetricRegion::barrier)
        .def("pp_set_config", &ep::SymmetricRegion::pp_set_config)
        .def("pp_send", &ep::SymmetricRegion::pp_send)
        .def("pp_recv", &ep::SymmetricRegion::pp_recv)
        .def("agrs_set_config", &ep::SymmetricRegion::agrs_set_config)
        .def("create_agrs_session", &ep::SymmetricRegion::create_agrs_session)
        .def("destroy_agrs_session", &ep::SymmetricRegion::destroy_agrs_session)
        .def("agrs_get_inplace_tensor", &ep::SymmetricRegion::agrs_get_inplace_tensor)
        .def("all_gather", &ep::SymmetricRegion::all_gather)
        .def("engram_write", &ep::SymmetricRegion::engram_write)
        .def("engram_fetch", &ep::SymmetricRegion::engram_fetch)
        .def("gemm_combine_send", &ep::SymmetricRegion::gemm_combine_send)
        .def("gemm_combine_reduce", &ep::SymmetricRegion::gemm_combine_reduce);

    py::class_<ep::HostSegment>(m, "HostSegment")
        .def(py::init<const std::string&, int64_t, bool>())
        .def("name", &ep::HostSegment::name)
        .def("bytes", &ep::HostSegment::bytes)
        .def("is_owner", &ep::HostSegment::is_owner)
        .def("host_ptr", &ep::HostSegment::host_ptr)
        .def("device_ptr", &ep::HostSegment::device_ptr)
        .def("host_view", &ep::HostSegment::host_view)
        .def("destroy", &ep::HostSegment::destroy);

    ep::register_ops(m);
}
