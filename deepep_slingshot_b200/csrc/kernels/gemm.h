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

// bf16 grouped GEMMs with both operands K-major (gemm_bf16_sm100.cu).
//   mode 0 (M-grouped): a [rows][k], b [E*n][k], d [rows][n]; rows of expert e at offsets[e], 128-aligned
//   mode 1 (K-grouped): a [m][k], b [n][k], d [E][m][n]; expert e contracts k in [offsets[e], offsets[e+1])
struct Bf16GemmArgs {
    const void* a;
    const void* b;
    const int* offsets;       // [E+1] (mode 0: 128-aligned rows; mode 1: 64-aligned K offsets)
    const int* expert_counts; // mode 0: [E] valid rows per expert (null: the aligned block)
    void* d;
    int mode;
    int rows, m, n, k, num_experts;
    int stages;
    KernelStatus st;
};
int launch_grouped_gemm_bf16(const Bf16GemmArgs& a, int num_sms, cudaStream_t stream);

}  // namespace ep
