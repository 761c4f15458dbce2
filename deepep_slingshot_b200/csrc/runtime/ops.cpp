// Torch bindings of the standalone sm_100a ops.
#include "ops.hpp"

#include <ATen/cuda/CUDAContext.h>
#include <pybind11/stl.h>
#include <torch/extension.h>

#include "../kernels/api.h"

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

}  // namespace

void register_ops(pybind11::module_& m) {
    m.def("per_token_cast_to_fp8", &per_token_cast_to_fp8, pybind11::arg("x"), pybind11::arg("round_scale") = false);
    m.def("per_token_cast_back", &per_token_cast_back);
}

}  // namespace ep
