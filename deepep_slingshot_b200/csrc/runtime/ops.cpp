// Torch bindings of the standalone sm_100a ops.
#include "ops.hpp"

#include <ATen/cuda/CUDAContext.h>
#include <pybind11/stl.h>
#include <torch/extension.h>

#include "../kernels/api.h"
#include "../kernels/permute.h"

namespace ep {

namespace {

std::tuple<torch::Tensor, torch::Tensor> per_token_cast_to_fp8(const torch::Tensor& x, bool round_scale) {
    TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous() && x.scalar_type() == torch::kBFloat16,
                "x must be a contiguous CUDA bf16 [tokens, hidden] tensor");
    const int N = (int)x.size(0), H = (int)x.size(1);
    TORCH_CHECK(H % 128 == 0, "hidden must be a multiple of 128");
    auto out = torch::empty({N, H}, x.options().dtype(torch::kFloat8_e4m3fn));
    auto scales = torch::empty({N, H / 128}, x.options().dtype(torch::kFloat32));
    launch_per_token_cast_to_fp8(x.data_ptr(), N, H, out.data_ptr(), scales.data_ptr<float>(), round_scale ? 1 : 0,
                                 at::cuda::getCurrentCUDAStream());
    return {out, scales};
}

torch::Tensor per_token_cast_back(const torch::Tensor& x, const torch::Tensor& scales) {
    TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous() && x.scalar_type() == torch::kFloat8_e4m3fn);
    const int N = (int)x.size(0), H = (int)x.size(1);
    TORCH_CHECK(H % 128 == 0 && scales.scalar_type() == torch::kFloat32 && scales.size(0) == N && scales.size(1) == H / 128);
    auto s = scales.contiguous();
    auto out = torch::empty({N, H}, x.options().dtype(torch::kBFloat16));
    launch_per_token_cast_back(x.data_ptr(), s.data_ptr<float>(), N, H, out.data_ptr(), at::cuda::getCurrentCUDAStream());
    return out;
}

// Grouped-by-expert permutation of dispatched tokens. Output rows are allocated for the worst case
// (`num_out_rows`, default N*K + E*(alignment-1)); rows past expert_offsets[E] are unused.
std::tuple<torch::Tensor, std::optional<torch::Tensor>, std::optional<torch::Tensor>, torch::Tensor, torch::Tensor, torch::Tensor>
permute(const torch::Tensor& x, const std::optional<torch::Tensor>& x_scales, const torch::Tensor& topk_idx,
        const std::optional<torch::Tensor>& probs, int num_experts, int alignment, int64_t num_out_rows) {
    TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous());
    TORCH_CHECK(x.scalar_type() == torch::kBFloat16 || x.scalar_type() == torch::kFloat8_e4m3fn);
    TORCH_CHECK(topk_idx.scalar_type() == torch::kInt64 && topk_idx.is_contiguous() && topk_idx.size(0) == x.size(0));
    TORCH_CHECK(num_experts > 0 && num_experts <= 4096 && alignment >= 1);
    const int N = (int)x.size(0), H = (int)x.size(1), K = (int)topk_idx.size(1);
    TORCH_CHECK((H * x.element_size()) % 16 == 0, "row bytes must be a multiple of 16");
    if (num_out_rows <= 0) num_out_rows = (int64_t)N * K + (int64_t)num_experts * (alignment - 1);
    auto i32 = x.options().dtype(torch::kInt32);
    const int chunks = (N + 31) / 32;
    auto counts = torch::empty({std::max(chunks, 1), num_experts}, i32);
    auto bases = torch::empty({std::max(chunks, 1), num_experts}, i32);
    auto offsets = torch::empty({num_experts + 1}, i32);
    auto ecounts = torch::empty({num_experts}, i32);
    auto row_map = torch::empty({N, K}, i32);
    auto x_perm = torch::empty({num_out_rows, H}, x.options());
    std::optional<torch::Tensor> sp, pp;
    PermuteArgs a{};
    if (x_scales.has_value()) {
        TORCH_CHECK(x_scales->scalar_type() == torch::kFloat32 && x_scales->is_contiguous() && x_scales->size(1) == H / 128);
        sp = torch::empty({num_out_rows, H / 128}, x.options().dtype(torch::kFloat32));
        a.x_scales = x_scales->data_ptr<float>();
        a.scales_perm = sp->data_ptr<float>();
    }
    if (probs.has_value()) {
        TORCH_CHECK(probs->scalar_type() == torch::kFloat32 && probs->is_contiguous() && probs->size(1) == K);
        pp = torch::zeros({num_out_rows}, x.options().dtype(torch::kFloat32));
        a.probs = probs->data_ptr<float>();
        a.probs_perm = pp->data_ptr<float>();
    }
    a.x = x.data_ptr();
    a.x_elem_bytes = (int)x.element_size();
    a.topk_idx = topk_idx.data_ptr<int64_t>();
    a.num_tokens = N;
    a.hidden = H;
    a.num_topk = K;
    a.num_experts = num_experts;
    a.alignment = alignment;
    a.counts = counts.data_ptr<int>();
    a.bases = bases.data_ptr<int>();
    a.expert_offsets = offsets.data_ptr<int>();
    a.expert_counts = ecounts.data_ptr<int>();
    a.row_map = row_map.data_ptr<int>();
    a.x_perm = x_perm.data_ptr();
    launch_permute(a, at::cuda::getCurrentCUDAStream());
    return {x_perm, sp, pp, row_map, offsets, ecounts};
}

torch::Tensor unpermute(const torch::Tensor& y, const torch::Tensor& row_map, const std::optional<torch::Tensor>& weights) {
    TORCH_CHECK(y.is_cuda() && y.dim() == 2 && y.is_contiguous() && y.scalar_type() == torch::kBFloat16);
    TORCH_CHECK(row_map.scalar_type() == torch::kInt32 && row_map.is_contiguous());
    const int N = (int)row_map.size(0), K = (int)row_map.size(1), H = (int)y.size(1);
    TORCH_CHECK(H % 8 == 0 && K <= kMaxTopk);
    if (weights.has_value())
        TORCH_CHECK(weights->scalar_type() == torch::kFloat32 && weights->is_contiguous() && weights->size(0) == N && weights->size(1) == K);
    auto out = torch::empty({N, H}, y.options());
    launch_unpermute(y.data_ptr(), row_map.data_ptr<int>(), weights.has_value() ? weights->data_ptr<float>() : nullptr, N, H, K,
                     out.data_ptr(), at::cuda::getCurrentCUDAStream());
    return out;
}

}  // namespace

void register_ops(pybind11::module_& m) {
    m.def("permute", &permute, pybind11::arg("x"), pybind11::arg("x_scales"), pybind11::arg("topk_idx"), pybind11::arg("probs"),
          pybind11::arg("num_experts"), pybind11::arg("alignment") = 1, pybind11::arg("num_out_rows") = 0);
    m.def("unpermute", &unpermute);
    m.def("per_token_cast_to_fp8", &per_token_cast_to_fp8, pybind11::arg("x"), pybind11::arg("round_scale") = false);
    m.def("per_token_cast_back", &per_token_cast_back);
}

}  // namespace ep
