// Host-side CUDA error check: throws std::runtime_error with the call site (surfaced in Python).
#pragma once

#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

#define EP_CUDA_CHECK(cmd)                                                                                   \
    do {                                                                                                     \
        cudaError_t e_ = (cmd);                                                                              \
        if (e_ != cudaSuccess)                                                                               \
            throw std::runtime_error(std::string("CUDA error: ") + cudaGetErrorString(e_) + " at " __FILE__ ":" + \
                                     std::to_string(__LINE__));                                              \
    } while (0)
