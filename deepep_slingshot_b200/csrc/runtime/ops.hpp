// Standalone sm_100a ops exposed to Python (quantization, permute/unpermute, grouped GEMM).
#pragma once
#include <pybind11/pybind11.h>

namespace ep {
void register_ops(pybind11::module_& m);
}
