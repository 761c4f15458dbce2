// Normal-mode (throughput) expert-parallel kernels for one NVLink 5 / NVSwitch domain, sm_100a.
//
// Capability parity with the reference's intranode path ([DE]csrc/kernels/legacy/layout.cu:10-150,
// [DE]csrc/kernels/legacy/intranode.cu:25-1117, v2 [DE]deep_ep/include/deep_ep/impls/dispatch.cuh,
// combine.cuh, combine_reduce_epilogue.cuh), re-designed for B200:
//
//  dispatch = stage -> notify -> pull
//    * stage  (many CTAs): each source rank writes one 16-byte-aligned RECORD per token into its own
//               staging area: the row (bf16, or FP8 e4m3 with the 1x128 quantization fused here),
//               its fp32 block scales and its top-k ids/weights. Local HBM traffic only.
//    * notify (one CTA): builds the per-destination token lists and `send_head`, pushes the count
//               row and the per-expert counts into every peer's control block, releases a flag, waits
//               for every peer's flag and computes the receive layout (prefix matrices, aligned
//               per-expert counts) into device memory and into host-mapped counters.
//    * pull   (num_sms CTAs): every receiver pulls the records it needs straight out of the
//               sources' staging with TMA bulk loads over NVLink (no multicast) into a shared-memory
//               ring and TMA-stores them into its own output tensors. There is no receive ring and
//               no copy epilogue: the output tensors are written once.
//  combine = push -> reduce
//    * push   : each rank TMA-stores its expert-output rows into the source rank's combine slots
//               (slot = send_prefix + position, known from the dispatch layout) and adds the row count
//               to a counter in the source's memory with a sys-scope release.
//    * reduce : the source waits for all rows, sums them in fp32 (+ bias), casts to bf16, sums the
//               top-k weights, and releases `combine_ready` so peers may reuse its slots.
// Every wait is bounded and reports an error code instead of trapping.
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include "../include/ep/device.cuh"
#include "../include/ep/quant.cuh"
#include "api.h"

namespace ep {

namespace {

__device__ __forceinline__ NormalCtrl* ctrl_of(const PeerTable& p, const NormalLayout& l, int r) {
    return reinterpret_cast<NormalCtrl*>(static_cast<uint8_t*>(p.base[r]) + l.ctrl_off);
}

// Block-wide exclusive scan over all threads of the block (blockDim.x <= 1024). Returns the
// exclusive prefix of `v`; `*total` receives the block sum. `ws` must hold 33 ints.
__device__ int block_exclusive_scan(int v, int* total, int* ws) {
    const int lane = lane_id(), warp = warp_id(), nwarps = (blockDim.x + 31) / 32;
    int incl = warp_inclusive_scan(v);
    if (lane == 31) ws[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int w = lane < nwarps ? ws[lane] : 0;
        int wincl = warp_inclusive_scan(w);
        if (lane < nwarps) ws[lane] = wincl - w;
        if (lane == nwarps - 1) ws[32] = wincl;
    }
    __syncthreads();
    int result = ws[warp] + incl - v;
    *total = ws[32];
    __syncthreads();
    return result;
}

}  // namespace

// =================================================================================================
// get_dispatch_layout: per-rank / per-expert token counts and is_token_in_rank[N][R].
// =================================================================================================
__global__ void __launch_bounds__(256) dispatch_layout_kernel(const int64_t* __restrict__ topk_idx, int num_tokens,
                                                              int num_topk, int num_experts, int num_ranks,
                                                              int* __restrict__ num_tokens_per_rank,
                                                              int* __restrict__ num_tokens_per_expert,
                                                              bool* __restrict__ is_token_in_rank) {
    extern __shared__ int s_cnt[];  // [num_experts + num_ranks]
    for (int i = threadIdx.x; i < num_experts + num_ranks; i += blockDim.x) s_cnt[i] = 0;
    __syncthreads();
    const int experts_per_rank = num_experts / num_ranks;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < num_tokens; t += gridDim.x * blockDim.x) {
        uint32_t mask = 0;
        for (int k = 0; k < num_topk; ++k) {
            const int64_t e = topk_idx[(int64_t)t * num_topk + k];
            if (e >= 0 && e < num_experts) {
                atomicAdd(&s_cnt[e], 1);
                mask |= 1u << (int)(e / experts_per_rank);
            }
        }
        for (int r = 0; r < num_ranks; ++r) {
            const bool in = (mask >> r) & 1u;
            is_token_in_rank[(int64_t)t * num_ranks + r] = in;
            if (in) atomicAdd(&s_cnt[num_experts + r], 1);
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < num_experts; i += blockDim.x)
        if (s_cnt[i]) atomicAdd(&num_tokens_per_expert[i], s_cnt[i]);
    for (int r = threadIdx.x; r < num_ranks; r += blockDim.x)
        if (s_cnt[num_experts + r]) atomicAdd(&num_tokens_per_rank[r], s_cnt[num_experts + r]);
}

void launch_dispatch_layout(const int64_t* topk_idx, int num_tokens, int num_topk, int num_experts, int num_ranks,
                            int* num_tokens_per_rank, int* num_tokens_per_expert, bool* is_token_in_rank,
                            cudaStream_t stream) {
    cudaMemsetAsync(num_tokens_per_rank, 0, sizeof(int) * num_ranks, stream);
    cudaMemsetAsync(num_tokens_per_expert, 0, sizeof(int) * num_experts, stream);
    if (num_tokens == 0) return;
    const int threads = 256;
    int blocks = (num_tokens + threads - 1) / threads;
    blocks = blocks > 296 ? 296 : blocks;
    const size_t smem = sizeof(int) * (num_experts + num_ranks);
    dispatch_layout_kernel<<<blocks, threads, smem, stream>>>(topk_idx, num_tokens, num_topk, num_experts, num_ranks,
                                                              num_tokens_per_rank, num_tokens_per_expert,
                                                              is_token_in_rank);
}

// =================================================================================================
// stage: one record per token into the local staging area, FP8 quantization fused.
// =================================================================================================
__global__ void __launch_bounds__(256) dispatch_stage_kernel(StageArgs a) {
    if (a.wait_epoch > 0 && (int)threadIdx.x < a.num_ranks)
        wait_ge(&a.pull_done[threadIdx.x], a.wait_epoch, a.st, kErrTimeoutPullDone, threadIdx.x);
    __syncthreads();
    if (aborted(a.st)) return;

    const int lane = lane_id();
    const int warps = blockDim.x / 32;
    const int total_warps = gridDim.x * warps;
    for (int t = blockIdx.x * warps + warp_id(); t < a.num_tokens; t += total_warps) {
        uint8_t* rec = a.staging + (int64_t)t * a.record_stride;
        if (a.quantize) {
            quantize_row_to_fp8(static_cast<const __nv_bfloat16*>(a.x) + (int64_t)t * a.hidden, rec,
                                reinterpret_cast<float*>(rec + a.rec.scale_off), a.hidden, a.round_scale != 0);
        } else {
            const int x_bytes = a.hidden * a.in_elem_bytes;
            const uint8_t* src = static_cast<const uint8_t*>(a.x) + (int64_t)t * x_bytes;
            for (int o = lane * 16; o < x_bytes; o += 512)
                *reinterpret_cast<int4*>(rec + o) = ld_nc_v4(reinterpret_cast<const int4*>(src + o));
            if (a.x_scales != nullptr) {
                float* dst = reinterpret_cast<float*>(rec + a.rec.scale_off);
                const int nb = a.hidden / 128;
                for (int b = lane; b < nb; b += 32) dst[b] = a.x_scales[t * a.scale_stride_t + b * a.scale_stride_b];
            }
        }
        if (lane < a.topk_pad) {
            int idx = -1;
            float w = 0.f;
            if (lane < a.num_topk) {
                if (a.topk_idx != nullptr) idx = (int)a.topk_idx[(int64_t)t * a.num_topk + lane];
                if (a.topk_weights != nullptr) w = a.topk_weights[(int64_t)t * a.num_topk + lane];
            }
            reinterpret_cast<int*>(rec + a.rec.idx_off)[lane] = idx;
            reinterpret_cast<float*>(rec + a.rec.w_off)[lane] = w;
        }
    }
}

void launch_dispatch_stage(const StageArgs& a, int num_sms, cudaStream_t stream) {
    int blocks = (a.num_tokens + 7) / 8;
    const int max_blocks = num_sms * 4;
    if (blocks > max_blocks) blocks = max_blocks;
    if (blocks < 1) blocks = 1;
    dispatch_stage_kernel<<<blocks, 256, 0, stream>>>(a);
}

// =================================================================================================
// notify: lists + send_head + count exchange + receive layout. One CTA of 1024 threads.
// =================================================================================================
__device__ __forceinline__ uint32_t token_rank_mask(const NotifyArgs& a, int t) {
    uint32_t m = 0;
    if (a.is_token_in_rank != nullptr) {
        for (int r = 0; r < a.num_ranks; ++r) m |= (a.is_token_in_rank[(int64_t)t * a.num_ranks + r] ? 1u : 0u) << r;
    } else if (a.topk_idx != nullptr) {
        for (int k = 0; k < a.num_topk; ++k) {
            const int64_t e = a.topk_idx[(int64_t)t * a.num_topk + k];
            if (e >= 0 && e < a.num_experts) m |= 1u << (int)(e / a.num_local_experts);
        }
    }
    return m;
}

__global__ void __launch_bounds__(1024) dispatch_notify_kernel(NotifyArgs a) {
    extern __shared__ int s_ecnt[];  // [num_experts]
    __shared__ int s_ws[33];
    __shared__ int s_total[kMaxRanks];
    __shared__ int s_tc[kMaxRanks][kMaxRanks];
    const int tid = threadIdx.x, nt = blockDim.x;
    const int R = a.num_ranks;
    NormalCtrl* my_ctrl = ctrl_of(a.peers, a.layout, a.rank);

    if (!a.cached) {
        for (int i = tid; i < a.num_experts; i += nt) s_ecnt[i] = 0;
        __syncthreads();
        const int chunk = (a.num_tokens + nt - 1) / nt;
        const int t0 = min(a.num_tokens, tid * chunk), t1 = min(a.num_tokens, t0 + chunk);
        int cnt[kMaxRanks];
#pragma unroll
        for (int r = 0; r < kMaxRanks; ++r) cnt[r] = 0;
        for (int t = t0; t < t1; ++t) {
            const uint32_t m = token_rank_mask(a, t);
#pragma unroll
            for (int r = 0; r < kMaxRanks; ++r) cnt[r] += (m >> r) & 1u;
            if (a.topk_idx != nullptr) {
                for (int k = 0; k < a.num_topk; ++k) {
                    const int64_t e = a.topk_idx[(int64_t)t * a.num_topk + k];
                    if (e >= 0 && e < a.num_experts) atomicAdd(&s_ecnt[e], 1);
                }
            }
        }
        int base[kMaxRanks];
#pragma unroll
        for (int r = 0; r < kMaxRanks; ++r) {
            if (r < R) {
                int total;
                base[r] = block_exclusive_scan(cnt[r], &total, s_ws);
                if (tid == 0) s_total[r] = total;
            }
        }
        int* list = reinterpret_cast<int*>(static_cast<uint8_t*>(a.peers.base[a.rank]) + a.layout.list_off);
        const int cap = a.layout.capacity;
        for (int t = t0; t < t1; ++t) {
            const uint32_t m = token_rank_mask(a, t);
            for (int r = 0; r < R; ++r) {
                int pos = -1;
                if ((m >> r) & 1u) {
                    pos = base[r]++;
                    list[(int64_t)r * cap + pos] = t;
                }
                a.send_head[(int64_t)t * R + r] = pos;
            }
        }
        __syncthreads();
        // Push my count row and my per-expert counts into every destination's control block.
        for (int i = tid; i < R * R; i += nt) {
            const int dst = i / R, col = i % R;
            ctrl_of(a.peers, a.layout, dst)->token_counts[a.parity][a.rank][col] = s_total[col];
        }
        for (int i = tid; i < R * a.num_local_experts; i += nt) {
            const int dst = i / a.num_local_experts, le = i % a.num_local_experts;
            ctrl_of(a.peers, a.layout, dst)->expert_counts[a.parity][a.rank][le] =
                a.topk_idx != nullptr ? s_ecnt[dst * a.num_local_experts + le] : 0;
        }
    }
    __syncthreads();
    if (tid < R) {
        fence_sys();
        st_release_sys(&ctrl_of(a.peers, a.layout, tid)->notify_flag[a.rank], a.epoch);
        wait_ge(&my_ctrl->notify_flag[tid], a.epoch, a.st, kErrTimeoutNotify, tid);
    }
    __syncthreads();
    if (aborted(a.st) || a.cached) return;

    for (int i = tid; i < R * R; i += nt)
        s_tc[i / R][i % R] = ld_volatile(&my_ctrl->token_counts[a.parity][i / R][i % R]);
    __syncthreads();
    if (tid == 0) {
        for (int r = 0; r < R; ++r) {
            int acc = 0;
            for (int s = 0; s < R; ++s) {
                acc += s_tc[s][r];
                a.rank_prefix_matrix[s * R + r] = acc;
            }
        }
        for (int s = 0; s < R; ++s) {
            int acc = 0;
            for (int r = 0; r < R; ++r) {
                a.send_prefix_matrix[s * R + r] = acc;
                acc += s_tc[s][r];
            }
        }
        int acc = 0;
        a.recv_rank_prefix[0] = 0;
        for (int s = 0; s < R; ++s) {
            acc += s_tc[s][a.rank];
            a.recv_rank_prefix[s + 1] = acc;
        }
        *a.dev_num_recv = acc;
        if (a.host != nullptr) a.host->num_recv_tokens = acc;
    }
    for (int le = tid; le < a.num_local_experts; le += nt) {
        int c = 0;
        for (int s = 0; s < R; ++s) c += ld_volatile(&my_ctrl->expert_counts[a.parity][s][le]);
        if (a.cumulative_stats != nullptr) a.cumulative_stats[le] += c;
        const int al = a.expert_alignment > 1 ? (c + a.expert_alignment - 1) / a.expert_alignment * a.expert_alignment : c;
        a.num_recv_per_expert[le] = al;
        if (a.host != nullptr) a.host->num_recv_tokens_per_expert[le] = al;
    }
    __syncthreads();
    if (tid == 0 && a.host != nullptr) {
        __threadfence_system();
        *reinterpret_cast<volatile int*>(&a.host->ready_epoch) = a.epoch;
        __threadfence_system();
    }
}

void launch_dispatch_notify(const NotifyArgs& a, cudaStream_t stream) {
    const size_t smem = sizeof(int) * (a.num_experts > 0 ? a.num_experts : 1);
    dispatch_notify_kernel<<<1, 1024, smem, stream>>>(a);
}

// =================================================================================================
// pull: receivers TMA-load records from the sources' staging (peer memory) and TMA-store rows into
// their own outputs. Each warp runs an independent S-stage pipeline over chunks of 32 rows.
// =================================================================================================
__device__ __forceinline__ int find_source(const int* prefix, int R, int j) {
    int s = 0;
    while (s + 1 < R && j >= prefix[s + 1]) ++s;
    return s;
}

__global__ void __launch_bounds__(128) dispatch_pull_kernel(PullArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_prefix[kMaxRanks + 1];
    const int lane = lane_id(), warp = warp_id(), W = blockDim.x / 32;
    const int R = a.num_ranks, S = a.stages;
    const int stage_bytes = (a.rec.bytes + 127) / 128 * 128;
    uint8_t* wbuf = smem + (size_t)warp * S * stage_bytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)W * S * stage_bytes) + warp * S;

    if (lane == 0) {
        for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    if (threadIdx.x == 0) {
        s_prefix[0] = 0;
        for (int s = 0; s < R; ++s)
            s_prefix[s + 1] = a.rank_prefix_matrix[s * R + a.rank];  // inclusive prefix over sources
    }
    __syncthreads();

    const int num_recv = a.dev_num_recv != nullptr ? ld_volatile(a.dev_num_recv) : a.num_recv_host;
    const int K = a.num_topk;
    // Padding rows of a worst-case allocation: mark as empty.
    for (int j = num_recv + blockIdx.x * blockDim.x + threadIdx.x; j < a.num_out_rows; j += gridDim.x * blockDim.x) {
        if (a.recv_topk_idx != nullptr)
            for (int k = 0; k < K; ++k) a.recv_topk_idx[(int64_t)j * K + k] = -1;
        if (a.recv_topk_weights != nullptr)
            for (int k = 0; k < K; ++k) a.recv_topk_weights[(int64_t)j * K + k] = 0.f;
        if (a.recv_src_idx != nullptr) a.recv_src_idx[j] = -1;
    }
    if (num_recv > a.num_out_rows) {
        if (threadIdx.x == 0 && blockIdx.x == 0) report_error(a.st, kErrCapacity, -1, num_recv);
        return;
    }

    const int x_bytes = a.rec.x_bytes;
    const int nb = a.rec.scale_bytes > 0 ? a.layout.hidden / 128 : 0;
    const bool scales_bulk = a.recv_scales != nullptr && !a.scales_col_major && (nb * 4) % 16 == 0;
    const int E_l = a.num_local_experts;
    const int lo_e = a.rank * E_l;
    uint32_t phase = 0;  // per-stage parity bits (lane 0)
    const int num_chunks = (num_recv + 31) / 32;
    const int gw = blockIdx.x * W + warp, total_warps = gridDim.x * W;
    bool ok = true;

    for (int c = gw; c < num_chunks && ok; c += total_warps) {
        const int j = c * 32 + lane;
        const bool valid = j < num_recv;
        int src = 0, t = 0;
        if (valid) {
            src = find_source(s_prefix, R, j);
            const int pos = j - s_prefix[src];
            if (a.cached_src_idx != nullptr) {
                t = a.cached_src_idx[j];
            } else {
                const int* list = reinterpret_cast<const int*>(static_cast<const uint8_t*>(a.peers.base[src]) + a.layout.list_off) +
                                  (int64_t)a.rank * a.layout.capacity;
                t = ld_relaxed_sys(list + pos);
            }
        }
        const int n_rows = min(32, num_recv - c * 32);
        // Stages may still be read by stores of the previous chunk.
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
        // Prefetch the first S-1 rows.
        for (int i = 0; i < S - 1 && i < n_rows; ++i) {
            const int ps = __shfl_sync(0xffffffffu, src, i), pt = __shfl_sync(0xffffffffu, t, i);
            if (lane == 0) {
                const uint8_t* g = static_cast<const uint8_t*>(a.peers.base[ps]) + a.layout.staging_off +
                                   (int64_t)pt * a.layout.record_bytes;
                mbar_arrive_expect_tx(&bars[i], a.rec.bytes);
                tma_load_1d(wbuf + (size_t)i * stage_bytes, g, a.rec.bytes, &bars[i]);
            }
        }
        for (int i = 0; i < n_rows; ++i) {
            const int stage = i % S;
            const int jj = c * 32 + i;
            const int st_t = __shfl_sync(0xffffffffu, t, i);
            // rows i + S - 1 for the next load
            const int nxt = i + S - 1;
            const int ns = __shfl_sync(0xffffffffu, src, nxt & 31), ntk = __shfl_sync(0xffffffffu, t, nxt & 31);
            int good = 1;
            if (lane == 0) {
                good = mbar_wait(&bars[stage], (phase >> stage) & 1u, a.st, kErrTimeoutTma) ? 1 : 0;
                phase ^= 1u << stage;
            }
            good = __shfl_sync(0xffffffffu, good, 0);
            if (!good) {
                ok = false;
                break;
            }
            const uint8_t* buf = wbuf + (size_t)stage * stage_bytes;
            if (lane == 0) {
                tma_store_1d(static_cast<uint8_t*>(a.recv_x) + (int64_t)jj * x_bytes, buf, x_bytes);
                if (scales_bulk) tma_store_1d(a.recv_scales + (int64_t)jj * nb, buf + a.rec.scale_off, nb * 4);
                bulk_commit();
            }
            if (a.recv_scales != nullptr && !scales_bulk) {
                const float* sc = reinterpret_cast<const float*>(buf + a.rec.scale_off);
                for (int b = lane; b < nb; b += 32) {
                    if (a.scales_col_major) a.recv_scales[(int64_t)b * a.scales_ld + jj] = sc[b];
                    else a.recv_scales[(int64_t)jj * nb + b] = sc[b];
                }
            }
            if (lane < K) {
                const int e = reinterpret_cast<const int*>(buf + a.rec.idx_off)[lane];
                const float w = reinterpret_cast<const float*>(buf + a.rec.w_off)[lane];
                const bool mine = e >= lo_e && e < lo_e + E_l;
                if (a.recv_topk_idx != nullptr) a.recv_topk_idx[(int64_t)jj * K + lane] = mine ? (e - lo_e) : -1;
                if (a.recv_topk_weights != nullptr) a.recv_topk_weights[(int64_t)jj * K + lane] = mine ? w : 0.f;
            }
            if (lane == 0 && a.recv_src_idx != nullptr) a.recv_src_idx[jj] = st_t;
            __syncwarp();
            if (nxt < n_rows && lane == 0) {
                bulk_wait_read<1>();  // the store of row i-1 is done reading stage nxt % S
                const int nstage = nxt % S;
                const uint8_t* g = static_cast<const uint8_t*>(a.peers.base[ns]) + a.layout.staging_off +
                                   (int64_t)ntk * a.layout.record_bytes;
                mbar_arrive_expect_tx(&bars[nstage], a.rec.bytes);
                tma_load_1d(wbuf + (size_t)nstage * stage_bytes, g, a.rec.bytes, &bars[nstage]);
            }
            __syncwarp();
        }
    }
    if (lane == 0) bulk_wait<0>();
    __syncthreads();
    // The last block tells every source that its staging may be reused.
    if (threadIdx.x == 0) {
        NormalCtrl* my_ctrl = ctrl_of(a.peers, a.layout, a.rank);
        fence_sys();
        const int old = atom_add_acq_rel_gpu(&my_ctrl->pull_finished_blocks, 1);
        if (old == (int)gridDim.x - 1) {
            my_ctrl->pull_finished_blocks = 0;
            fence_sys();
            for (int s = 0; s < R; ++s) st_release_sys(&ctrl_of(a.peers, a.layout, s)->pull_done[a.rank], a.epoch);
        }
    }
}

static int smem_stages(int record_bytes, int warps, int max_stages) {
    const int stage_bytes = (record_bytes + 127) / 128 * 128;
    const int budget = 200 * 1024;
    int s = budget / (warps * (stage_bytes + 8));
    if (s > max_stages) s = max_stages;
    return s;
}

void launch_dispatch_pull(const PullArgs& a_in, int num_sms, cudaStream_t stream) {
    PullArgs a = a_in;
    const int warps = 4;
    if (a.stages <= 0) a.stages = smem_stages(a.rec.bytes, warps, 6);
    if (a.stages < 2) a.stages = 2;
    const int stage_bytes = (a.rec.bytes + 127) / 128 * 128;
    const size_t smem = (size_t)warps * a.stages * stage_bytes + (size_t)warps * a.stages * sizeof(uint64_t);
    cudaFuncSetAttribute(dispatch_pull_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    dispatch_pull_kernel<<<num_sms, warps * 32, smem, stream>>>(a);
}

// =================================================================================================
// combine push: expert-output rows -> the source rank's combine slots (peer memory).
// =================================================================================================
__global__ void __launch_bounds__(128) combine_push_kernel(CombinePushArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_prefix[kMaxRanks + 1];
    __shared__ int s_dst_base[kMaxRanks];
    const int lane = lane_id(), warp = warp_id(), W = blockDim.x / 32;
    const int R = a.num_ranks, S = a.stages, K = a.num_topk;
    const int H = a.layout.hidden;
    const int row_bytes = H * 2;
    const int stage_bytes = (row_bytes + 127) / 128 * 128;
    uint8_t* wbuf = smem + (size_t)warp * S * stage_bytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)W * S * stage_bytes) + warp * S;
    NormalCtrl* my_ctrl = ctrl_of(a.peers, a.layout, a.rank);

    // Destination `tid` must have finished reducing the previous combine before its slots are reused.
    if ((int)threadIdx.x < R) wait_ge(&my_ctrl->combine_ready[threadIdx.x], a.seq - 1, a.st, kErrTimeoutCombineReady, threadIdx.x);
    if (lane == 0) {
        for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    if (threadIdx.x == 0) {
        s_prefix[0] = 0;
        for (int s = 0; s < R; ++s) {
            s_prefix[s + 1] = a.rank_prefix_matrix[s * R + a.rank];
            s_dst_base[s] = a.send_prefix_matrix[s * R + a.rank];
        }
    }
    __syncthreads();
    if (aborted(a.st)) return;

    const int num_recv = min(s_prefix[R], a.num_recv_max);
    const int num_chunks = (num_recv + 31) / 32;
    const int gw = blockIdx.x * W + warp, total_warps = gridDim.x * W;
    const int64_t combine_rows_cap = (int64_t)a.layout.capacity * a.layout.num_ranks;
    uint32_t phase = 0;
    bool ok = true;
    for (int c = gw; c < num_chunks && ok; c += total_warps) {
        const int j = c * 32 + lane;
        const bool valid = j < num_recv;
        int dst = 0, drow = 0;
        if (valid) {
            dst = find_source(s_prefix, R, j);
            drow = s_dst_base[dst] + (j - s_prefix[dst]);
            if (drow < 0 || drow >= combine_rows_cap) {
                report_error(a.st, kErrBounds, dst, drow);
                dst = -1;
            }
        }
        const int n_rows = min(32, num_recv - c * 32);
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
        for (int i = 0; i < S - 1 && i < n_rows; ++i) {
            if (lane == 0) {
                mbar_arrive_expect_tx(&bars[i], row_bytes);
                tma_load_1d(wbuf + (size_t)i * stage_bytes, static_cast<const uint8_t*>(a.x) + (int64_t)(c * 32 + i) * row_bytes,
                            row_bytes, &bars[i]);
            }
        }
        for (int i = 0; i < n_rows; ++i) {
            const int stage = i % S;
            const int jj = c * 32 + i;
            const int d = __shfl_sync(0xffffffffu, dst, i), dr = __shfl_sync(0xffffffffu, drow, i);
            int good = 1;
            if (lane == 0) {
                good = mbar_wait(&bars[stage], (phase >> stage) & 1u, a.st, kErrTimeoutTma) ? 1 : 0;
                phase ^= 1u << stage;
            }
            good = __shfl_sync(0xffffffffu, good, 0);
            if (!good) {
                ok = false;
                break;
            }
            if (d >= 0) {
                uint8_t* peer = static_cast<uint8_t*>(a.peers.base[d]);
                if (lane == 0) {
                    tma_store_1d(peer + a.layout.combine_off + (int64_t)dr * row_bytes, wbuf + (size_t)stage * stage_bytes, row_bytes);
                }
                if (a.topk_weights != nullptr && lane < a.layout.topk_pad) {
                    float* wdst = reinterpret_cast<float*>(peer + a.layout.combine_w_off) + (int64_t)dr * a.layout.topk_pad;
                    wdst[lane] = lane < K ? a.topk_weights[(int64_t)jj * K + lane] : 0.f;
                }
            }
            if (lane == 0) bulk_commit();
            __syncwarp();
            const int nxt = i + S - 1;
            if (nxt < n_rows && lane == 0) {
                bulk_wait_read<1>();
                const int nstage = nxt % S;
                mbar_arrive_expect_tx(&bars[nstage], row_bytes);
                tma_load_1d(wbuf + (size_t)nstage * stage_bytes, static_cast<const uint8_t*>(a.x) + (int64_t)(c * 32 + nxt) * row_bytes,
                            row_bytes, &bars[nstage]);
            }
            __syncwarp();
        }
        // Rows of this chunk are complete in the destinations' memory: publish the counts.
        if (lane == 0) {
            bulk_wait<0>();
            fence_proxy_async_global();
        }
        __syncwarp();
        for (int d = 0; d < R; ++d) {
            const int cnt = __popc(__ballot_sync(0xffffffffu, valid && dst == d));
            if (cnt > 0 && lane == 0) {
                fence_sys();
                red_add_release_sys(&ctrl_of(a.peers, a.layout, d)->combine_arrived, cnt);
            }
        }
    }
}

void launch_combine_push(const CombinePushArgs& a_in, int num_sms, cudaStream_t stream) {
    CombinePushArgs a = a_in;
    const int warps = 4;
    if (a.stages <= 0) a.stages = smem_stages(a.layout.hidden * 2, warps, 4);
    if (a.stages < 2) a.stages = 2;
    const int stage_bytes = (a.layout.hidden * 2 + 127) / 128 * 128;
    const size_t smem = (size_t)warps * a.stages * stage_bytes + (size_t)warps * a.stages * sizeof(uint64_t);
    cudaFuncSetAttribute(combine_push_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    combine_push_kernel<<<num_sms, warps * 32, smem, stream>>>(a);
}

// =================================================================================================
// combine reduce: fp32 sum of the <= R contributions per token (+ bias) -> bf16; top-k weight sum.
// =================================================================================================
__global__ void __launch_bounds__(256) combine_reduce_kernel(CombineReduceArgs a) {
    __shared__ int s_base[kMaxRanks];
    const int R = a.num_ranks, K = a.num_topk, H = a.hidden;
    NormalCtrl* my_ctrl = ctrl_of(a.peers, a.layout, a.rank);
    if (threadIdx.x == 0) {
        int expected = 0;
        for (int r = 0; r < R; ++r) {
            const int prev = a.rank > 0 ? a.rank_prefix_matrix[(a.rank - 1) * R + r] : 0;
            expected += a.rank_prefix_matrix[a.rank * R + r] - prev;
            s_base[r] = a.send_prefix_matrix[a.rank * R + r];
        }
        wait_eq(&my_ctrl->combine_arrived, expected, a.st, kErrTimeoutCombineArrive, -1);
    }
    __syncthreads();
    if (!aborted(a.st)) {
        const int lane = lane_id();
        const int warps = blockDim.x / 32;
        const __nv_bfloat16* rows = reinterpret_cast<const __nv_bfloat16*>(static_cast<const uint8_t*>(a.peers.base[a.rank]) + a.layout.combine_off);
        const float* wrows = reinterpret_cast<const float*>(static_cast<const uint8_t*>(a.peers.base[a.rank]) + a.layout.combine_w_off);
        for (int t = blockIdx.x * warps + warp_id(); t < a.num_tokens; t += gridDim.x * warps) {
            int my_row = -1;
            if (lane < R) {
                const int p = a.send_head[(int64_t)t * R + lane];
                my_row = p >= 0 ? s_base[lane] + p : -1;
            }
            int src_rows[kMaxRanks];
            int n = 0;
#pragma unroll
            for (int r = 0; r < kMaxRanks; ++r) {
                const int v = __shfl_sync(0xffffffffu, my_row, r);
                if (r < R && v >= 0) src_rows[n++] = v;
            }
            for (int e0 = lane * 8; e0 < H; e0 += 256) {
                float acc[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) acc[i] = 0.f;
                for (int q = 0; q < n; ++q) {
                    const int4 v = *reinterpret_cast<const int4*>(rows + (int64_t)src_rows[q] * H + e0);
                    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float2 f = __bfloat1622float2(h2[i]);
                        acc[2 * i] += f.x;
                        acc[2 * i + 1] += f.y;
                    }
                }
                for (int b = 0; b < 2; ++b) {
                    const void* bias = b == 0 ? a.bias0 : a.bias1;
                    if (bias != nullptr) {
                        const int4 v = *reinterpret_cast<const int4*>(static_cast<const __nv_bfloat16*>(bias) + (int64_t)t * H + e0);
                        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const float2 f = __bfloat1622float2(h2[i]);
                            acc[2 * i] += f.x;
                            acc[2 * i + 1] += f.y;
                        }
                    }
                }
                int4 o;
                __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
                for (int i = 0; i < 4; ++i) o2[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
                *reinterpret_cast<int4*>(static_cast<__nv_bfloat16*>(a.out) + (int64_t)t * H + e0) = o;
            }
            if (a.out_topk_weights != nullptr && lane < K) {
                float w = 0.f;
                if (a.has_weights)
                    for (int q = 0; q < n; ++q) w += wrows[(int64_t)src_rows[q] * a.layout.topk_pad + lane];
                a.out_topk_weights[(int64_t)t * K + lane] = w;
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const int old = atom_add_acq_rel_gpu(&my_ctrl->combine_reduced_blocks, 1);
        if (old == (int)gridDim.x - 1) {
            my_ctrl->combine_reduced_blocks = 0;
            my_ctrl->combine_arrived = 0;
            fence_sys();
            for (int r = 0; r < R; ++r) st_release_sys(&ctrl_of(a.peers, a.layout, r)->combine_ready[a.rank], a.seq);
        }
    }
}

void launch_combine_reduce(const CombineReduceArgs& a, int num_sms, cudaStream_t stream) {
    int blocks = (a.num_tokens + 7) / 8;
    const int max_blocks = num_sms * 2;
    if (blocks > max_blocks) blocks = max_blocks;
    if (blocks < 1) blocks = 1;
    combine_reduce_kernel<<<blocks, 256, 0, stream>>>(a);
}

// =================================================================================================
// barrier across the NVLink domain (bounded).
// =================================================================================================
__global__ void barrier_kernel(PeerTable peers, int64_t ctrl_off, int rank, int num_ranks, int epoch, KernelStatus st) {
    const int r = threadIdx.x;
    if (r < num_ranks) {
        NormalCtrl* peer = reinterpret_cast<NormalCtrl*>(static_cast<uint8_t*>(peers.base[r]) + ctrl_off);
        NormalCtrl* mine = reinterpret_cast<NormalCtrl*>(static_cast<uint8_t*>(peers.base[rank]) + ctrl_off);
        fence_sys();
        st_release_sys(&peer->barrier_flag[rank], epoch);
        wait_ge(&mine->barrier_flag[r], epoch, st, kErrTimeoutBarrier, r);
    }
}

void launch_barrier(PeerTable peers, int64_t ctrl_off, int rank, int num_ranks, int epoch, KernelStatus st,
                    cudaStream_t stream) {
    barrier_kernel<<<1, 32, 0, stream>>>(peers, ctrl_off, rank, num_ranks, epoch, st);
}

}  // namespace ep
