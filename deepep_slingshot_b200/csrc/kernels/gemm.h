// Launch API of the tcgen05 grouped GEMM kernels (see gemm_sm100.cu).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../include/ep/abi.h"

namespace ep {

constexpr int kMaxGemmStages = 8;
constexpr int kMaxGemmExperts = 1024;

struct GemmArgs {
    const void* a;            // [rows][k] e4m3, grouped by expert
    const float* sa;          // [rows][k/128]
    const void* b;            // [E][n][k] e4m3
    const float* sb;          // [E][n/128][k/128]
    const int* offsets;       // [E+1] 128-aligned row offsets of the experts
    const int* expert_counts; // [E] valid rows per expert (null: use the aligned block)
    void* d;                  // [rows][n] bf16
    int rows, n, k, num_experts;
    int stages;
    KernelStatus st;
};

// Returns 0 on success, 1 bad shapes, 2 tensor-map encode failure, 3 launch failure.
int launch_grouped_gemm_fp8(const GemmArgs& a, int num_sms, cudaStream_t stream);

}  // namespace ep
