// Normal-mode (throughput) expert-parallel kernels for one NVLink 5 / NVSwitch domain, sm_100a.
//
// Capability parity with the reference's intranode path ([DE]csrc/kernels/legacy/layout.cu:10-150,
// [DE]csrc/kernels/legacy/intranode.cu:25-1117, v2 [DE]deep_ep/include/deep_ep/impls/dispatch.cuh,
// combine.cuh, combine_reduce_epilogue.cuh), re-designed for B200:
//
//  dispatch = (count || stage) -> pull: the count step on a second stream concurrent with the
//  stage launch (default), or count -> pull with stage warps inside the pull launch
//  (DEEPEP_B200_DISPATCH_STAGE=warps); a cached handle with the concurrent stage runs no count step
//    * count  (up to 128 CTAs): waits until every receiver finished pulling the previous dispatch,
//               then builds the ordered per-destination token lists and `send_head` from the routing
//               alone (each CTA adds the per-destination counts its predecessors published) and the
//               per-expert counts; its last CTA pushes the count row and the per-expert counts into
//               every peer's control block, releases a flag, waits for every peer's flag and
//               computes the receive layout (prefix matrices, aligned per-expert counts).
//    * stage  (its own launch, or stage warps of the pull launch): each source writes one
//               16-byte-aligned RECORD per token into its own staging area (the row: bf16, or FP8
//               e4m3 with the 1x128 quantization fused here; its fp32 block scales; its top-k
//               ids/weights), in token order, and releases a staged flag per chunk of tokens in
//               every receiver's control block. The quantization is thereby off the count step's
//               critical path, and the pulls start on the first staged chunks.
//    * pull   (pull pairs): every receiver pulls the records it needs straight
//               out of the sources' staging with TMA bulk loads over NVLink (no multicast) into a
//               shared-memory ring, in the wavefront order (at step k pair g takes the next row of
//               source (k + g) % R, so all pairs walk every source's tokens in the order they are
//               staged), after a bounded wait on the (source, chunk) staged flag, and
//               TMA-stores them into its own output tensors. There is no receive ring and no copy
//               epilogue: the output tensors are written once. The last block publishes the
//               received counts to host-mapped memory (the CPU sync) and releases the sources' staging.
//  combine = one kernel, push and reduce overlapped
//    * push warps TMA-store this rank's expert-output rows into the source ranks' combine slots
//               (slot = send_prefix + position, known from the dispatch layout), walking the
//               destinations in a wavefront so each token's contributions arrive close together, and
//               announce arrivals per token in batches (one drain + system fence per batch);
//    * reducer warps (and push warps once done) take tokens from a shared cursor, wait until all
//               of a token's contributions arrived, sum them in fp32 (+ bias), cast to bf16, sum the
//               top-k weights; the last block releases `combine_ready` so peers may reuse the slots.
// Every wait is bounded and reports an error code instead of trapping.
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include "../include/ep/device.cuh"
#include "../include/ep/quant.cuh"
#include "../include/ep/schedule.cuh"
#include "api.h"

namespace ep {

namespace {

__device__ __forceinline__ NormalCtrl* ctrl_of(const PeerTable& p, const NormalLayout& l, int r) {
    return reinterpret_cast<NormalCtrl*>(static_cast<uint8_t*>(p.base[r]) + l.ctrl_off);
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
// Top-k ids and weights of token t into its record (lanes < topk_pad).
__device__ __forceinline__ void stage_record_meta(const StageArgs& a, int t, uint8_t* rec) {
    const int lane = lane_id();
    int idx = -1;
    float w = 0.f;
    if (lane < a.num_topk) {
        if (a.topk_idx != nullptr) idx = (int)a.topk_idx[(int64_t)t * a.num_topk + lane];
        if (a.topk_weights != nullptr) w = a.topk_weights[(int64_t)t * a.num_topk + lane];
    }
    if (lane < a.topk_pad) {
        reinterpret_cast<int*>(rec + a.rec.idx_off)[lane] = idx;
        reinterpret_cast<float*>(rec + a.rec.w_off)[lane] = w;
    }
}

// Whole record of token t through registers (one warp): quantized, copied bf16 or pre-quantized FP8
// row, its scales and the top-k metadata. Six 256-column groups in flight per lane (a 7168-wide
// row in five rounds).
__device__ __forceinline__ void stage_token_regs(const StageArgs& a, int t) {
    const int lane = lane_id();
    uint8_t* rec = a.staging + (int64_t)t * a.record_stride;
    if (a.quantize) {
        quantize_row_to_fp8<false, 6>(static_cast<const __nv_bfloat16*>(a.x) + (int64_t)t * a.hidden, rec,
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
    stage_record_meta(a, t, rec);
}

// After a warp staged token t (its stores ordered before lane 0 by __syncwarp): count the token in
// its chunk; the add that completes the chunk has acquired every earlier add of the chunk, so its
// releases of staged[rank][chunk] = epoch into every receiver's control block cover the whole chunk.
__device__ __forceinline__ void stage_signal_chunk(const StageArgs& a, int* chunk_done, int t) {
    const int c = t / a.chunk;
    const int target = min(a.chunk, a.num_tokens - c * a.chunk);
    if (a.writer_proxy_fence) fence_proxy_async_global();  // receivers read the staging with TMA (async proxy)
    const int before = a.signal_gpu_scope ? atom_add_acq_rel_gpu(&chunk_done[c], 1) : atom_add_acq_rel_sys(&chunk_done[c], 1);
    if (before == target - 1) {
        for (int r = 0; r < a.num_ranks; ++r)
            st_release_sys(&reinterpret_cast<NormalCtrl*>(static_cast<uint8_t*>(a.peers.base[r]) + a.layout.ctrl_off)->staged[a.rank][c],
                           a.epoch);
    }
}

// Standalone stage kernel: either before the count exchange (whose barrier then orders every peer's
// pull after this rank's staging), or concurrently with the count step with per-chunk signalling.
__global__ void __launch_bounds__(256, 2) dispatch_stage_kernel(StageArgs a) {
    // With tma_rows each warp owns one row buffer of dynamic shared memory: a single bulk copy brings
    // the whole bf16 row in (no registers held for loads in flight), the warp quantizes from there.
    extern __shared__ __align__(128) uint8_t s_rows[];
    __shared__ __align__(8) uint64_t s_bar[8];
    const uint64_t t_start = trace_begin(a.st);
    if (a.tma_rows && lane_id() == 0) {
        mbar_init(&s_bar[warp_id()], 1);
        fence_mbar_init();
    }
    if ((int)threadIdx.x < a.num_ranks && a.pull_done != nullptr) {
        // Receivers must have finished pulling the previous dispatch before the staging is rewritten.
        const int prev_epoch = a.epoch > 0 ? a.epoch - 1 : ld_volatile(a.dispatch_epoch);
        if (prev_epoch > 0) wait_ge(&a.pull_done[threadIdx.x], prev_epoch, a.st, kErrTimeoutPullDone, threadIdx.x);
    }
    int* chunk_done = a.signal_chunks ? reinterpret_cast<NormalCtrl*>(static_cast<uint8_t*>(a.peers.base[a.rank]) + a.layout.ctrl_off)->stage_chunk_done
                                      : nullptr;
    __syncthreads();
    if (threadIdx.x == 0) trace_end(a.st, kTraceWaitReceivers, t_start, a.num_tokens);
    if (aborted(a.st)) return;

    const int lane = lane_id();
    const int warps = blockDim.x / 32;
    const int total_warps = gridDim.x * warps;
    uint32_t phase = 0;
    for (int t = blockIdx.x * warps + warp_id(); t < a.num_tokens; t += total_warps) {
        if (!(a.quantize && a.tma_rows)) {
            stage_token_regs(a, t);
            if (chunk_done != nullptr) {
                __syncwarp();
                if (lane == 0) stage_signal_chunk(a, chunk_done, t);
            }
            continue;
        }
        uint8_t* rec = a.staging + (int64_t)t * a.record_stride;
        const uint32_t row_bytes = (uint32_t)a.hidden * 2;
        uint8_t* buf = s_rows + (size_t)warp_id() * row_bytes;
        if (lane == 0) {
            fence_proxy_async_smem();  // the previous row's generic reads precede this async write
            mbar_arrive_expect_tx(&s_bar[warp_id()], row_bytes);
            tma_load_1d(buf, static_cast<const uint8_t*>(a.x) + (int64_t)t * row_bytes, row_bytes, &s_bar[warp_id()]);
        }
        if (!__all_sync(0xffffffffu, mbar_wait(&s_bar[warp_id()], phase, a.st, kErrTimeoutTma) ? 1 : 0)) {
            if (lane == 0) mbar_wait(&s_bar[warp_id()], phase, a.st, kErrTimeoutTma);  // the row lands before exit
            break;
        }
        phase ^= 1u;
        quantize_row_to_fp8<true>(reinterpret_cast<const __nv_bfloat16*>(buf), rec,
                                  reinterpret_cast<float*>(rec + a.rec.scale_off), a.hidden, a.round_scale != 0);
        __syncwarp();
        stage_record_meta(a, t, rec);
        if (chunk_done != nullptr) {
            __syncwarp();
            if (lane == 0) stage_signal_chunk(a, chunk_done, t);
        }
    }
    if (a.st.trace != nullptr) {
        __syncthreads();
        if (threadIdx.x == 0) trace_end(a.st, kTraceStage, t_start, a.num_tokens);
    }
}

void launch_dispatch_stage(const StageArgs& a_in, int max_sms, cudaStream_t stream) {
    StageArgs a = a_in;
    int blocks = (a.num_tokens + 7) / 8;
    if (blocks < 1) blocks = 1;
    size_t smem = 0;
    const size_t row_bytes = (size_t)a.hidden * 2;
    // TMA row loads: 8 row buffers per block (two blocks per SM up to hidden 7168), 16-byte aligned rows.
    a.tma_rows = !a.regs_rows && a.quantize && row_bytes % 16 == 0 && 8 * row_bytes <= 112 * 1024 &&
                 reinterpret_cast<uintptr_t>(a.x) % 16 == 0;
    if (a.tma_rows) {
        smem = 8 * row_bytes;
        int sm_count = 148, dev = 0;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, dev);
        if (max_sms > 0 && max_sms < sm_count) sm_count = max_sms;
        if (blocks > 2 * sm_count) blocks = 2 * sm_count;  // grid-stride: every block resident
        cudaFuncSetAttribute(dispatch_stage_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    }
    dispatch_stage_kernel<<<blocks, 256, smem, stream>>>(a);
}

// =================================================================================================
// count: ordered per-destination lists + send_head + per-expert counts (all CTAs), then the count
// exchange and the receive layout (last CTA). Only the routing is read, so this step does not wait
// for the quantization; the staging runs concurrently (its own launch) or overlaps the pulls.
// =================================================================================================
__device__ __forceinline__ uint32_t token_rank_mask(const CountArgs& a, int t) {
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

// Block-wide exclusive scan of per-destination counts, two 32-bit counters per 64-bit word
// (destination 2w in the low half of word w, 2w + 1 in the high half): one scan for all
// destinations; each CTA counts at most tokens_per_cta < 2^31 tokens.
constexpr int kCountWords = kMaxRanks / 2;
__device__ void block_exclusive_scan_counts(uint64_t (&v)[kCountWords], uint64_t (&total)[kCountWords],
                                            uint64_t* ws /* kCountWords * 33 */) {
    const int lane = lane_id(), warp = warp_id(), nwarps = (blockDim.x + 31) / 32;
    uint64_t incl[kCountWords];
#pragma unroll
    for (int w = 0; w < kCountWords; ++w) incl[w] = v[w];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
#pragma unroll
        for (int w = 0; w < kCountWords; ++w) {
            const uint64_t n = __shfl_up_sync(0xffffffffu, incl[w], o);
            if (lane >= o) incl[w] += n;
        }
    }
    if (lane == 31)
#pragma unroll
        for (int w = 0; w < kCountWords; ++w) ws[w * 33 + warp] = incl[w];
    __syncthreads();
    if (warp == 0) {
#pragma unroll
        for (int w = 0; w < kCountWords; ++w) {
            const uint64_t own = lane < nwarps ? ws[w * 33 + lane] : 0;
            uint64_t sc = own;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint64_t n = __shfl_up_sync(0xffffffffu, sc, o);
                if (lane >= o) sc += n;
            }
            if (lane < nwarps) ws[w * 33 + lane] = sc - own;
            if (lane == nwarps - 1) ws[w * 33 + 32] = sc;
        }
    }
    __syncthreads();
#pragma unroll
    for (int w = 0; w < kCountWords; ++w) {
        v[w] = ws[w * 33 + warp] + incl[w] - v[w];
        total[w] = ws[w * 33 + 32];
    }
    __syncthreads();
}

__device__ __forceinline__ int count_of(const uint64_t (&v)[kCountWords], int r) {
    return (int)((v[r >> 1] >> (32 * (r & 1))) & 0xffffffffu);
}

constexpr int kCountThreads = 256;

__global__ void __launch_bounds__(kCountThreads) dispatch_count_kernel(CountArgs a) {
    extern __shared__ __align__(16) int s_ecnt[];  // [num_experts] per-CTA expert counts (fresh mode)
    __shared__ uint64_t s_ws[kCountWords * 33];
    __shared__ int s_base[kMaxRanks];
    __shared__ int s_total[kMaxRanks];
    __shared__ int s_tc[kMaxRanks][kMaxRanks];
    __shared__ int s_epoch, s_last;
    const int tid = threadIdx.x, nt = blockDim.x;
    const int R = a.num_ranks;
    NormalCtrl* my_ctrl = ctrl_of(a.peers, a.layout, a.rank);
    const uint64_t t_start = trace_begin(a.st);
    if (tid == 0) s_epoch = ld_volatile(&my_ctrl->dispatch_epoch) + 1;
    if (tid < kMaxRanks) s_base[tid] = 0;
    __syncthreads();
    const int epoch = s_epoch, parity = epoch & 1;
    // Every receiver must have finished pulling the previous dispatch (it reads my lists and my
    // staging) before this dispatch rewrites them.
    if (tid < R && epoch > 1) wait_ge(&my_ctrl->pull_done[tid], epoch - 1, a.st, kErrTimeoutPullDone, tid);
    __syncthreads();
    if (blockIdx.x == 0 && tid == 0) trace_end(a.st, kTraceWaitReceivers, t_start, a.num_tokens);
    if (aborted(a.st)) return;

    if (!a.cached) {
        const int per_thread = a.tokens_per_cta / nt;
        const int t0 = blockIdx.x * a.tokens_per_cta + tid * per_thread;
        const int t1 = min(a.num_tokens, t0 + per_thread);
        for (int i = tid; i < a.num_experts; i += nt) s_ecnt[i] = 0;
        __syncthreads();
        uint64_t cnt[kCountWords] = {};
        for (int t = t0; t < t1; ++t) {
            const uint32_t m = token_rank_mask(a, t);
#pragma unroll
            for (int r = 0; r < kMaxRanks; ++r) cnt[r >> 1] += (uint64_t)((m >> r) & 1u) << (32 * (r & 1));
            if (a.topk_idx != nullptr)
                for (int k = 0; k < a.num_topk; ++k) {
                    const int64_t e = a.topk_idx[(int64_t)t * a.num_topk + k];
                    if (e >= 0 && e < a.num_experts) atomicAdd(&s_ecnt[e], 1);
                }
        }
        uint64_t tot[kCountWords];
        block_exclusive_scan_counts(cnt, tot, s_ws);
        // Publish this CTA's counts, then add up those of the CTAs before it (all CTAs are resident:
        // the grid is at most kMaxCountCtas small CTAs).
        if (tid < R) {
            int mine = 0;  // count_of(tot, tid) with static indices (no local-memory copy of tot)
#pragma unroll
            for (int r = 0; r < kMaxRanks; ++r)
                if (r == tid) mine = count_of(tot, r);
            my_ctrl->count_cta_counts[blockIdx.x][tid] = mine;
        }
        __syncthreads();
        if (tid == 0) {
            __threadfence();
            st_release_sys(&my_ctrl->count_cta_flag[blockIdx.x], epoch);
        }
        if (tid < (int)blockIdx.x) {
            if (wait_ge(&my_ctrl->count_cta_flag[tid], epoch, a.st, kErrTimeoutNotify, -1))
                for (int r = 0; r < R; ++r) atomicAdd(&s_base[r], ld_volatile(&my_ctrl->count_cta_counts[tid][r]));
        }
        __syncthreads();
        if (aborted(a.st)) return;
        int pos[kMaxRanks];
#pragma unroll
        for (int r = 0; r < kMaxRanks; ++r) pos[r] = r < R ? s_base[r] + count_of(cnt, r) : 0;
        int* list = reinterpret_cast<int*>(static_cast<uint8_t*>(a.peers.base[a.rank]) + a.layout.list_off);
        const int cap = a.layout.capacity;
        for (int t = t0; t < t1; ++t) {
            const uint32_t m = token_rank_mask(a, t);
#pragma unroll
            for (int r = 0; r < kMaxRanks; ++r) {
                if (r >= R) break;
                int p = -1;
                if ((m >> r) & 1u) {
                    p = pos[r]++;
                    list[(int64_t)r * cap + p] = t;
                }
                a.send_head[(int64_t)t * R + r] = p;
            }
        }
        for (int i = tid; i < a.num_experts; i += nt)
            if (s_ecnt[i] != 0) atomicAdd(&a.expert_counts[i], s_ecnt[i]);
    }
    // The last CTA to finish runs the exchange.
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        s_last = atomicAdd(&my_ctrl->count_done_ctas, 1) == (int)gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (!a.cached) {
        if (tid < R) {
            int total = 0;
            for (int b = 0; b < (int)gridDim.x; ++b) total += ld_volatile(&my_ctrl->count_cta_counts[b][tid]);
            s_total[tid] = total;
        }
        __syncthreads();
        // Push my count row and my per-expert counts into every destination's control block.
        for (int i = tid; i < R * R; i += nt) {
            const int dst = i / R, col = i % R;
            ctrl_of(a.peers, a.layout, dst)->token_counts[parity][a.rank][col] = s_total[col];
        }
        for (int i = tid; i < R * a.num_local_experts; i += nt) {
            const int dst = i / a.num_local_experts, le = i % a.num_local_experts;
            int* c = &a.expert_counts[dst * a.num_local_experts + le];
            ctrl_of(a.peers, a.layout, dst)->expert_counts[parity][a.rank][le] = a.topk_idx != nullptr ? ld_volatile(c) : 0;
            *c = 0;  // ready for the next dispatch
        }
    }
    if (tid == 0) my_ctrl->count_done_ctas = 0;
    __syncthreads();
    const uint64_t t_wait = trace_begin(a.st);
    if (tid < R) {
        fence_sys();
        st_release_sys(&ctrl_of(a.peers, a.layout, tid)->notify_flag[a.rank], epoch);
        wait_ge(&my_ctrl->notify_flag[tid], epoch, a.st, kErrTimeoutNotify, tid);
    }
    __syncthreads();
    if (tid == 0) trace_end(a.st, kTraceCountExchange, t_wait, epoch);
    if (aborted(a.st)) return;
    if (a.cached) {
        if (tid == 0) {
            my_ctrl->dispatch_epoch = epoch;
            trace_end(a.st, kTraceCount, t_start, 1);
        }
        return;
    }

    for (int i = tid; i < R * R; i += nt)
        s_tc[i / R][i % R] = ld_volatile(&my_ctrl->token_counts[parity][i / R][i % R]);
    __syncthreads();
    if (tid < R) {
        // column `tid` of the inclusive prefix over sources, row `tid` of the exclusive prefix over destinations
        int acc = 0;
        for (int s = 0; s < R; ++s) {
            acc += s_tc[s][tid];
            a.rank_prefix_matrix[s * R + tid] = acc;
        }
        acc = 0;
        for (int r = 0; r < R; ++r) {
            a.send_prefix_matrix[tid * R + r] = acc;
            acc += s_tc[tid][r];
        }
    }
    if (tid == 0) {
        int acc = 0;
        a.recv_rank_prefix[0] = 0;
        for (int s = 0; s < R; ++s) {
            acc += s_tc[s][a.rank];
            a.recv_rank_prefix[s + 1] = acc;
        }
        *a.dev_num_recv = acc;
    }
    for (int le = tid; le < a.num_local_experts; le += nt) {
        int c = 0;
        for (int s = 0; s < R; ++s) c += ld_volatile(&my_ctrl->expert_counts[parity][s][le]);
        if (a.cumulative_stats != nullptr) a.cumulative_stats[le] += c;
        const int al = a.expert_alignment > 1 ? (c + a.expert_alignment - 1) / a.expert_alignment * a.expert_alignment : c;
        a.num_recv_per_expert[le] = al;
        if (a.host != nullptr) a.host->num_recv_tokens_per_expert[le] = al;
    }
    __syncthreads();
    if (tid == 0) {
        my_ctrl->dispatch_epoch = epoch;
        if (a.host != nullptr) {
            a.host->num_recv_tokens = *a.dev_num_recv;  // written by this thread above
            __threadfence_system();  // the counts (every thread's, ordered by the barrier) before the ticket
            *reinterpret_cast<volatile int*>(&a.host->ready_ticket) = a.host_ticket;
        }
        trace_end(a.st, kTraceCount, t_start, 0);
    }
}

void launch_dispatch_count(const CountArgs& a, cudaStream_t stream) {
    const int grid = a.cached ? 1 : std::max(1, (a.num_tokens + a.tokens_per_cta - 1) / a.tokens_per_cta);
    const size_t smem = sizeof(int) * (size_t)std::max(a.cached ? 1 : a.num_experts, 1);
    if (smem > 48 * 1024) cudaFuncSetAttribute(dispatch_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    dispatch_count_kernel<<<grid, kCountThreads, smem, stream>>>(a);
}

// =================================================================================================
// Row pipeline shared by pull (dispatch) and push (combine): each CTA runs kPairs independent
// (producer warp, consumer warp) pairs over an S-slot shared-memory ring. The producer's lane 0
// TMA-loads rows (from a peer's staging, or from local expert outputs) as soon as a slot is free;
// the consumer's lane 0 TMA-stores each landed row to its destination (local output, or a peer's
// combine slots) and returns the slot once the store has read it, keeping up to S/2 stores in
// flight (a store's read of shared memory completes only as its writes drain, ~2 us over NVLink, so
// a shallow store window starves the pipeline). Measured on B200: 32-64 CTAs of this pipeline pull
// ~745 GB/s from one peer.
// =================================================================================================
constexpr int kPairs = 2;
constexpr int kCombineThreads = 256;  // combine blocks: 2 push pairs (4 warps) + 4 reducer warps

struct PipeSmem;
__device__ __forceinline__ void release_slots(const PipeSmem& p, int k, int lag);

struct PipeSmem {
    uint8_t* slots;
    uint64_t* full;
    uint64_t* empty;
    int* side;  // two ints per slot of side information (source token / destination rank, token)
    int S, slot_bytes;
};

// Bytes of one pair's region, rounded to 128 so every pair's slots (TMA targets, 16-byte rule) and
// mbarriers (8-byte rule) stay aligned whatever the stage count.
__host__ __device__ __forceinline__ size_t pipe_pair_bytes(int S, int slot_bytes) {
    return ((size_t)S * slot_bytes + (size_t)S * 24 + 16 + 127) / 128 * 128;
}

__device__ __forceinline__ PipeSmem pipe_smem(uint8_t* smem, int pair, int S, int slot_bytes) {
    uint8_t* base = smem + (size_t)pair * pipe_pair_bytes(S, slot_bytes);
    PipeSmem p;
    p.slots = base;
    p.full = reinterpret_cast<uint64_t*>(base + (size_t)S * slot_bytes);
    p.empty = p.full + S;
    p.side = reinterpret_cast<int*>(p.empty + S);
    p.S = S;
    p.slot_bytes = slot_bytes;
    return p;
}

static size_t pipe_smem_bytes(int S, int slot_bytes) { return (size_t)kPairs * pipe_pair_bytes(S, slot_bytes); }

// Consumer lane 0, after committing the TMA store of pipeline row k: keep at most `lag` stores
// reading shared memory and hand the slot of row k - lag back to the producer.
__device__ __forceinline__ void release_slots(const PipeSmem& p, int k, int lag) {
    switch (lag) {
        case 1: bulk_wait_read<1>(); break;
        case 2: bulk_wait_read<2>(); break;
        case 3: bulk_wait_read<3>(); break;
        case 4: bulk_wait_read<4>(); break;
        case 5: bulk_wait_read<5>(); break;
        case 6: bulk_wait_read<6>(); break;
        case 7: bulk_wait_read<7>(); break;
        default: bulk_wait_read<8>(); lag = 8; break;
    }
    if (k >= lag) mbar_arrive(&p.empty[(k - lag) % p.S]);
}

__device__ __forceinline__ void pipe_init(const PipeSmem& p) {
    if (lane_id() == 0) {
        for (int s = 0; s < p.S; ++s) {
            mbar_init(&p.full[s], 1);
            mbar_init(&p.empty[s], 1);
        }
        fence_mbar_init();
    }
}

// =================================================================================================
// pull (dispatch receive): rows of my receive block are pulled from the sources' staging.
// =================================================================================================

constexpr int kStageWarps = 8;  // stage warps per pull block when the stage overlaps the pulls

// Stage warps of the pull launch: stage this rank's tokens in token order (grid-stride over warps,
// so low chunks complete first) and, once the last token of a chunk is in the staging, release
// staged[rank][chunk] = epoch in every receiver's control block. A warp's stores are ordered
// before lane 0's acq_rel add by __syncwarp; the add that completes a chunk has acquired every
// earlier add of that chunk, so its releases cover the whole chunk.
__device__ __forceinline__ void stage_warps_run(const PullArgs& a, NormalCtrl* my_ctrl) {
    const StageArgs& sa = a.stage;
    const int lane = lane_id();
    const int gw = blockIdx.x * kStageWarps + (warp_id() - 2 * kPairs), GW = gridDim.x * kStageWarps;
    for (int t = gw; t < sa.num_tokens; t += GW) {
        stage_token_regs(sa, t);
        __syncwarp();
        if (lane == 0) stage_signal_chunk(sa, my_ctrl->stage_chunk_done, t);
        if ((t & 63) == 0 && aborted(a.st)) break;
    }
}

__global__ void __launch_bounds__(64 * kPairs + 32 * kStageWarps) dispatch_pull_kernel(PullArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_prefix[kMaxRanks + 1];
    const int lane = lane_id(), warp = warp_id();
    const bool pull_warp = warp < 2 * kPairs;
    const int pair = warp >> 1;
    const bool producer = (warp & 1) == 0;
    const int R = a.num_ranks;
    const int slot_bytes = (a.rec.bytes + 127) / 128 * 128;
    NormalCtrl* my_ctrl = ctrl_of(a.peers, a.layout, a.rank);
    const int epoch = a.epoch > 0 ? a.epoch : ld_volatile(&my_ctrl->dispatch_epoch);
    const PipeSmem p = pipe_smem(smem, pull_warp ? pair : 0, a.stages, slot_bytes);
    if (pull_warp) pipe_init(p);
    if (threadIdx.x == 0) {
        s_prefix[0] = 0;
        for (int s = 0; s < R; ++s) s_prefix[s + 1] = a.rank_prefix_matrix[s * R + a.rank];
    }
    __syncthreads();

    const int num_recv = a.dev_num_recv != nullptr ? ld_volatile(a.dev_num_recv) : a.num_recv_host;
    const int K = a.num_topk;
    // Trace start of the pull (thread 0 reports it); read after the set-up barrier, so no 64-bit
    // value stays live through the pipeline loops.
    uint64_t t_pull = threadIdx.x == 0 ? trace_begin(a.st) : 0;
    if (!pull_warp) {
        // Stage warps: they never wait for the pulls, so every rank's pulls make progress.
        const uint64_t t_stage = trace_begin(a.st);
        if (a.stage_warps > 0 && !aborted(a.st)) stage_warps_run(a, my_ctrl);
        if (warp == 2 * kPairs && lane == 0 && a.stage_warps > 0) trace_end(a.st, kTraceStage, t_stage, a.stage.num_tokens);
    } else if (num_recv > a.num_out_rows) {
        if (threadIdx.x == 0 && blockIdx.x == 0) report_error(a.st, kErrCapacity, -1, num_recv);
    } else {
        const int pull_threads = 64 * kPairs;
        for (int j = num_recv + blockIdx.x * pull_threads + threadIdx.x; a.fill_padding && j < a.num_out_rows;
             j += gridDim.x * pull_threads) {
            if (a.recv_topk_idx != nullptr)
                for (int k = 0; k < K; ++k) a.recv_topk_idx[(int64_t)j * K + k] = -1;
            if (a.recv_topk_weights != nullptr)
                for (int k = 0; k < K; ++k) a.recv_topk_weights[(int64_t)j * K + k] = 0.f;
            if (a.recv_src_idx != nullptr) a.recv_src_idx[j] = -1;
        }
        // Host-mapped counts for the CPU (written here rather than by the count kernel, so PCIe
        // writes and their fence stay off the path to the first pull).
        if (blockIdx.x == gridDim.x - 1 && warp == 1 && a.host != nullptr) {
            for (int le = lane; le < a.num_local_experts; le += 32)
                a.host->num_recv_tokens_per_expert[le] = a.num_recv_per_expert[le];
            if (lane == 0) a.host->num_recv_tokens = num_recv;
            __syncwarp();
            if (lane == 0) {
                __threadfence_system();
                *reinterpret_cast<volatile int*>(&a.host->ready_ticket) = a.host_ticket;
            }
        }
        const int g = blockIdx.x * kPairs + pair, P = gridDim.x * kPairs;
        // With the stage overlapped, rows follow the wavefront order: at step k pair g takes the next
        // row of source (k + g) % R, so every pair walks every source's tokens in increasing order, at
        // the pace its stage warps release them, with the loads spread over all sources. Otherwise
        // rows are dealt in blocks (or chunks) of the receive order.
        const bool staged_flags = (a.stage_warps > 0 || a.wait_staged) && a.stage.chunk > 0;
        const bool wave = staged_flags;
        const int my_rows = wave ? wave_num_rows(g, P, s_prefix, R, num_recv) : pair_num_rows(g, P, num_recv, a.chunk);
        auto row_at = [&](int k) { return wave ? wave_row(g, P, k, s_prefix, R, num_recv) : pair_row(g, P, k, a.chunk, num_recv); };
        const int S = p.S;
        const int chunk = staged_flags ? a.stage.chunk : 0;

        if (producer) {
            // After an expired wait lane 0 issues nothing more (the consumer stops at the first row that
            // does not arrive) instead of waiting out every later row; then it drains what it issued.
            // Lanes look up 32 schedule steps at a time (a step past a source's rows is skipped).
            int failed = 0, issued = 0;
            for (int base = 0; issued < my_rows && !failed; base += 32) {
                const int kk = base + lane;
                int src = 0, t = 0;
                const int j = row_at(kk);
                if (j >= 0) {
                    src = find_source(s_prefix, R, j);
                    if (a.cached_src_idx != nullptr) {
                        t = a.cached_src_idx[j];
                    } else {
                        const int* list = reinterpret_cast<const int*>(static_cast<const uint8_t*>(a.peers.base[src]) + a.layout.list_off) +
                                          (int64_t)a.rank * a.layout.capacity;
                        t = ld_relaxed_sys(list + (j - s_prefix[src]));
                    }
                }
                // The sources stage concurrently: every lane checks its row's (source, chunk) staged flag
                // (local memory) at once; lane 0 later waits (bounded) only for rows whose chunk was not
                // staged yet, and a proxy fence orders its TMA reads after the flags it observed.
                int ready = 1;
                if (j >= 0 && chunk > 0) ready = (ld_acquire_sys(&my_ctrl->staged[src][t / chunk]) - epoch) >= 0;
                const uint32_t live = __ballot_sync(0xffffffffu, j >= 0);
                const uint32_t pending = __ballot_sync(0xffffffffu, !ready);
                if (lane == 0 && chunk > 0) fence_proxy_async_global();
                for (int i = 0; i < 32; ++i) {
                    if (!((live >> i) & 1u)) continue;
                    const int ps = __shfl_sync(0xffffffffu, src, i), pt = __shfl_sync(0xffffffffu, t, i);
                    if (lane == 0 && !failed) {
                        const int k = issued, slot = k % S;
                        if ((pending >> i) & 1u) {
                            if (!wait_ge(&my_ctrl->staged[ps][pt / chunk], epoch, a.st, kErrTimeoutStaged, ps)) {
                                failed = 1;
                                continue;
                            }
                            fence_proxy_async_global();
                        }
                        if (k >= S && !mbar_wait(&p.empty[slot], ((k / S) - 1) & 1, a.st, kErrTimeoutTma)) {
                            failed = 1;
                        } else {
                            p.side[2 * slot] = pt;
                            const uint8_t* gsrc = static_cast<const uint8_t*>(a.peers.base[ps]) + a.layout.staging_off +
                                                  (int64_t)pt * a.layout.record_bytes;
                            mbar_arrive_expect_tx(&p.full[slot], a.rec.bytes);
                            tma_load_1d(p.slots + (size_t)slot * slot_bytes, gsrc, a.rec.bytes, &p.full[slot]);
                            ++issued;
                        }
                    }
                }
                failed = __shfl_sync(0xffffffffu, failed, 0);
                issued = __shfl_sync(0xffffffffu, issued, 0);
            }
            if (lane == 0) ring_drain(p.full, S, issued, a.st, kErrTimeoutTma);
        } else {
            const int x_bytes = a.rec.x_bytes;
            const int nb = a.rec.scale_bytes > 0 ? a.layout.hidden / 128 : 0;
            const bool scales_bulk = a.recv_scales != nullptr && !a.scales_col_major && (nb * 4) % 16 == 0;
            const int E_l = a.num_local_experts, lo_e = a.rank * E_l;
            const int lag = S / 2 < 4 ? S / 2 : 4;  // peer loads are the slow leg: favour loads in flight
            for (int kk = 0, k = 0; k < my_rows; ++kk) {
                const int j = row_at(kk);
                if (j < 0) continue;
                const int slot = k % S;
                int good = 1;
                if (lane == 0) good = mbar_wait(&p.full[slot], (k / S) & 1, a.st, kErrTimeoutTma) ? 1 : 0;
                if (!__shfl_sync(0xffffffffu, good, 0)) break;
                const uint8_t* buf = p.slots + (size_t)slot * slot_bytes;
                if (lane == 0) {
                    tma_store_1d(static_cast<uint8_t*>(a.recv_x) + (int64_t)j * x_bytes, buf, x_bytes);
                    if (scales_bulk) tma_store_1d(a.recv_scales + (int64_t)j * nb, buf + a.rec.scale_off, nb * 4);
                    bulk_commit();
                }
                if (a.recv_scales != nullptr && !scales_bulk) {
                    const float* sc = reinterpret_cast<const float*>(buf + a.rec.scale_off);
                    for (int b = lane; b < nb; b += 32) {
                        if (a.scales_col_major) a.recv_scales[(int64_t)b * a.scales_ld + j] = sc[b];
                        else a.recv_scales[(int64_t)j * nb + b] = sc[b];
                    }
                }
                if (lane < K) {
                    const int e = reinterpret_cast<const int*>(buf + a.rec.idx_off)[lane];
                    const float w = reinterpret_cast<const float*>(buf + a.rec.w_off)[lane];
                    const bool mine = e >= lo_e && e < lo_e + E_l;
                    if (a.recv_topk_idx != nullptr) a.recv_topk_idx[(int64_t)j * K + lane] = mine ? (e - lo_e) : -1;
                    if (a.recv_topk_weights != nullptr) a.recv_topk_weights[(int64_t)j * K + lane] = mine ? w : 0.f;
                }
                if (lane == 0 && a.recv_src_idx != nullptr) a.recv_src_idx[j] = p.side[2 * slot];
                __syncwarp();
                if (lane == 0) release_slots(p, k, lag);
                ++k;
            }
            if (lane == 0) bulk_wait<0>();
        }
    }
    __syncthreads();
    // The last block tells every source that its staging may be reused.
    if (threadIdx.x == 0) {
        trace_end(a.st, kTracePull, t_pull, num_recv);
        fence_sys();
        const int old = atom_add_acq_rel_gpu(&my_ctrl->pull_finished_blocks, 1);
        if (old == (int)gridDim.x - 1) {
            my_ctrl->pull_finished_blocks = 0;
            // every stage of this dispatch is done (stage warps of this launch, or the stage launch
            // before it): its chunk counters start from zero for the next dispatch
            if ((a.stage_warps > 0 || a.wait_staged) && a.stage.chunk > 0)
                for (int c = 0; c * a.stage.chunk < a.stage.num_tokens; ++c) my_ctrl->stage_chunk_done[c] = 0;
            if (a.epoch > 0) my_ctrl->dispatch_epoch = a.epoch;  // no count step ran for this dispatch
            fence_sys();
            for (int s = 0; s < R; ++s) st_release_sys(&ctrl_of(a.peers, a.layout, s)->pull_done[a.rank], epoch);
        }
    }
}

static int pipe_stages(int slot_bytes, int max_stages) {
    const int budget = 200 * 1024;
    int s = (int)(budget / ((size_t)kPairs * (slot_bytes + 24) + 256));
    if (s > max_stages) s = max_stages;
    return s;
}

void launch_dispatch_pull(const PullArgs& a_in, int num_sms, cudaStream_t stream) {
    PullArgs a = a_in;
    const int slot_bytes = (a.rec.bytes + 127) / 128 * 128;
    if (a.stages <= 0) a.stages = pipe_stages(slot_bytes, 16);
    if (a.stages < 4) a.stages = 4;
    const size_t smem = pipe_smem_bytes(a.stages, slot_bytes);
    a.stage_warps = a.stage_warps > 0 ? kStageWarps : 0;
    cudaFuncSetAttribute(dispatch_pull_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    dispatch_pull_kernel<<<num_sms, 64 * kPairs + 32 * a.stage_warps, smem, stream>>>(a);
}

// =================================================================================================
// combine: one launch, two roles.
//  * push blocks (first `push_blocks`): producer/consumer pairs move each expert-output row to its
//    source rank's combine slot with TMA (load local, store to the peer). Once a row's store has
//    completed (bulk wait_group, not .read) the consumer adds 1 to the destination's arrival counter
//    of that token with a sys-scope release.
//  * reduce blocks (the rest): one warp per token of this rank, in token order; it waits until the
//    token's arrival counter equals its number of contributing ranks, sums the rows in fp32 (+ bias),
//    writes bf16, sums the top-k weights and resets the counter. Reduction overlaps the transfer.
// All blocks are co-resident (grid <= SM count, one block per SM by shared memory).
// =================================================================================================
template <int kU, int kN>
__device__ __forceinline__ void reduce_rows(const __nv_bfloat16* rows, const int* src_rows, int n, int H, int t,
                                            const void* bias0, const void* bias1, void* out, int e_start) {
    const int lane = lane_id();
    int4 v[kU][kN];
    for (int e0 = e_start + lane * 8; e0 - lane * 8 < H; e0 += 256 * kU) {
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int e = e0 + u * 256;
#pragma unroll
            for (int q = 0; q < kN; ++q)
                if (q < n && e < H) v[u][q] = *reinterpret_cast<const int4*>(rows + (int64_t)src_rows[q] * H + e);
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int e = e0 + u * 256;
            if (e >= H) break;
            float acc[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll
            for (int q = 0; q < kN; ++q) {
                if (q >= n) break;
                const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&v[u][q]);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float2 f = __bfloat1622float2(h2[i]);
                    acc[2 * i] += f.x;
                    acc[2 * i + 1] += f.y;
                }
            }
#pragma unroll
            for (int b = 0; b < 2; ++b) {
                const void* bias = b == 0 ? bias0 : bias1;
                if (bias != nullptr) {
                    const int4 bv = *reinterpret_cast<const int4*>(static_cast<const __nv_bfloat16*>(bias) + (int64_t)t * H + e);
                    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&bv);
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
            *reinterpret_cast<int4*>(static_cast<__nv_bfloat16*>(out) + (int64_t)t * H + e) = o;
        }
    }
}

// Reduce one token t (all its contributions must have arrived): fp32 sum (+ bias) -> bf16, weight sum.
__device__ __forceinline__ bool combine_reduce_token(const CombineArgs& a, int t, const int* s_base, const __nv_bfloat16* rows,
                                                     const float* wrows, int* arrival) {
    const int lane = lane_id();
    const int R = a.num_ranks, K = a.num_topk, H = a.layout.hidden;
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
    if (n > 0) {
        int good = 1;
        if (lane == 0) good = wait_eq(arrival + t, n, a.st, kErrTimeoutCombineArrive, t) ? 1 : 0;
        if (!__shfl_sync(0xffffffffu, good, 0)) return false;
    }
    if (n <= 1) reduce_rows<8, 1>(rows, src_rows, n, H, t, a.bias0, a.bias1, a.out, 0);
    else if (n == 2) reduce_rows<4, 2>(rows, src_rows, n, H, t, a.bias0, a.bias1, a.out, 0);
    else if (n <= 4) reduce_rows<2, 4>(rows, src_rows, n, H, t, a.bias0, a.bias1, a.out, 0);
    else reduce_rows<1, kMaxRanks>(rows, src_rows, n, H, t, a.bias0, a.bias1, a.out, 0);
    if (a.out_topk_weights != nullptr && lane < K) {
        float w = 0.f;
        if (a.has_weights)
            for (int q = 0; q < n; ++q) w += wrows[(int64_t)src_rows[q] * a.layout.topk_pad + lane];
        a.out_topk_weights[(int64_t)t * K + lane] = w;
    }
    __syncwarp();
    if (lane == 0 && n > 0) arrival[t] = 0;
    return true;
}

// Reducer loop: grab tokens from the shared cursor until none are left.
__device__ __forceinline__ void combine_reduce_loop(const CombineArgs& a, NormalCtrl* my_ctrl, const int* s_base) {
    const int lane = lane_id();
    const __nv_bfloat16* rows =
        reinterpret_cast<const __nv_bfloat16*>(static_cast<const uint8_t*>(a.peers.base[a.rank]) + a.layout.combine_off);
    const float* wrows = reinterpret_cast<const float*>(static_cast<const uint8_t*>(a.peers.base[a.rank]) + a.layout.combine_w_off);
    int* arrival = reinterpret_cast<int*>(static_cast<uint8_t*>(a.peers.base[a.rank]) + a.layout.arrival_off);
    while (true) {
        int t = 0;
        if (lane == 0) t = atomicAdd(&my_ctrl->combine_token_cursor, 1);
        t = __shfl_sync(0xffffffffu, t, 0);
        if (t >= a.num_tokens) break;
        if (!combine_reduce_token(a, t, s_base, rows, wrows, arrival)) break;
    }
}

// Expanded mode, sender side: bf16(sum_q w[q] * x[rows[q]]) of one token into a ring slot (shared
// memory), fp32 accumulation in q order. Each lane owns 8 columns per 256-column step and keeps
// kU x kN independent 16-byte loads in flight.
template <int kU, int kN>
__device__ __forceinline__ void expanded_rows_to_slot(const __nv_bfloat16* __restrict__ x, const int* rows, const float* ws,
                                                      int n, int H, uint8_t* slot) {
    const int lane = lane_id();
    int4 v[kU][kN];
    for (int e0 = lane * 8; e0 - lane * 8 < H; e0 += 256 * kU) {
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int e = e0 + u * 256;
#pragma unroll
            for (int q = 0; q < kN; ++q)
                if (q < n && e < H) v[u][q] = ld_nc_v4(reinterpret_cast<const int4*>(x + (int64_t)rows[q] * H + e));
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int e = e0 + u * 256;
            if (e >= H) break;
            float acc[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll
            for (int q = 0; q < kN; ++q) {
                if (q >= n) break;
                const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&v[u][q]);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float2 f = __bfloat1622float2(h2[i]);
                    acc[2 * i] = fmaf(ws[q], f.x, acc[2 * i]);
                    acc[2 * i + 1] = fmaf(ws[q], f.y, acc[2 * i + 1]);
                }
            }
            int4 o;
            __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
            for (int i = 0; i < 4; ++i) o2[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
            *reinterpret_cast<int4*>(slot + (size_t)e * 2) = o;
        }
    }
}

// More than 8 local rows of one token (top-k above 8): the q-th row and factor come from the lane
// that holds them (q-th set bit of `valid`) inside the column loop; off the common path.
__device__ __forceinline__ void expanded_rows_to_slot_many(const __nv_bfloat16* __restrict__ x, int r, float w,
                                                           uint32_t valid, int n, int H, uint8_t* slot) {
    const int lane = lane_id();
    for (int e0 = 0; e0 < H; e0 += 256) {
        const int e = e0 + lane * 8;
        float acc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = 0.f;
        for (int q = 0; q < n; ++q) {
            const int src = (int)__fns(valid, 0, q + 1);
            const int row = __shfl_sync(0xffffffffu, r, src);
            const float wq = __shfl_sync(0xffffffffu, w, src);
            if (e < H) {
                const int4 v = ld_nc_v4(reinterpret_cast<const int4*>(x + (int64_t)row * H + e));
                const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float2 f = __bfloat1622float2(h2[i]);
                    acc[2 * i] = fmaf(wq, f.x, acc[2 * i]);
                    acc[2 * i + 1] = fmaf(wq, f.y, acc[2 * i + 1]);
                }
            }
        }
        if (e < H) {
            int4 o;
            __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
            for (int i = 0; i < 4; ++i) o2[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
            *reinterpret_cast<int4*>(slot + (size_t)e * 2) = o;
        }
    }
}

// One token of the expanded mode into `slot`: gather its local rows and factors (row_map order),
// report and skip an out-of-range row (the call then fails on the host), reduce.
__device__ __forceinline__ void expanded_token_to_slot(const CombineArgs& a, int j, uint8_t* slot) {
    const int lane = lane_id(), K = a.row_map_k, H = a.layout.hidden;
    int r = -1;
    float w = 1.f;
    if (lane < K) {
        r = a.row_map[(int64_t)j * K + lane];
        if (a.row_weights != nullptr) w = a.row_weights[(int64_t)j * K + lane];
        if (r >= 0 && !in_window(r, 1, a.x_rows)) {
            report_error(a.st, kErrBounds, j, r);
            r = -1;
        }
    }
    const uint32_t valid = __ballot_sync(0xffffffffu, r >= 0);
    const int n = __popc(valid);
    const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(a.x);
    if (n > 8) {
        expanded_rows_to_slot_many(x, r, w, valid, n, H, slot);
        return;
    }
    int rows[8];
    float ws[8];
    uint32_t m = valid;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        const int src = m ? __ffs(m) - 1 : 0;
        rows[q] = __shfl_sync(0xffffffffu, r, src);
        ws[q] = __shfl_sync(0xffffffffu, w, src);
        if (m) m &= m - 1;
    }
    if (n <= 1) expanded_rows_to_slot<8, 1>(x, rows, ws, n, H, slot);
    else if (n == 2) expanded_rows_to_slot<4, 2>(x, rows, ws, n, H, slot);
    else if (n <= 4) expanded_rows_to_slot<2, 4>(x, rows, ws, n, H, slot);
    else expanded_rows_to_slot<1, 8>(x, rows, ws, n, H, slot);
}

template <bool kExpanded>
__global__ void __launch_bounds__(kCombineThreads) combine_kernel(CombineArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_prefix[kMaxRanks + 1];
    __shared__ int s_base[kMaxRanks];      // where my rows start in each destination's combine region
    __shared__ int s_red_base[kMaxRanks];  // where each rank's rows start in MY combine region
    const int lane = lane_id(), warp = warp_id();
    const int R = a.num_ranks, K = a.num_topk, H = a.layout.hidden;
    NormalCtrl* my_ctrl = ctrl_of(a.peers, a.layout, a.rank);
    const bool pusher = (int)blockIdx.x < a.push_blocks;
    const int row_bytes = H * 2;
    const int slot_bytes = (row_bytes + 127) / 128 * 128;
    const uint64_t t_start = trace_begin(a.st);

    if (pusher && (int)threadIdx.x < R)
        // Destination `tid` must have finished reducing the previous combine before its slots are reused.
        wait_ge(&my_ctrl->combine_ready[threadIdx.x], ld_volatile(&my_ctrl->combine_seq), a.st, kErrTimeoutCombineReady,
                threadIdx.x);
    if (threadIdx.x == 0) {
        s_prefix[0] = 0;
        for (int s = 0; s < R; ++s) {
            s_prefix[s + 1] = a.rank_prefix_matrix[s * R + a.rank];
            s_base[s] = a.send_prefix_matrix[s * R + a.rank];
            s_red_base[s] = a.send_prefix_matrix[a.rank * R + s];
        }
    }
    // Warps 0..2*kPairs-1 form the (producer, consumer) pairs. In the expanded mode the other warps of
    // a push block are extra producers (two per pair), since each row is computed, not copied.
    const bool pair_warp = warp < 2 * kPairs;
    const int pair = pair_warp ? warp >> 1 : (warp - 2 * kPairs) >> 1;
    constexpr int kProducers = kExpanded ? 1 + (kCombineThreads / 32 - 2 * kPairs) / kPairs : 1;
    const int prod_idx = pair_warp ? 0 : 1 + ((warp - 2 * kPairs) % (kProducers - 1 > 0 ? kProducers - 1 : 1));
    const PipeSmem p = pipe_smem(smem, pair, a.stages, slot_bytes);
    if (pusher && pair_warp) pipe_init(p);
    __syncthreads();

    if (pusher && (pair_warp || kExpanded) && !aborted(a.st)) {
        const bool producer = !pair_warp || (warp & 1) == 0;
        const int num_recv = min(s_prefix[R], a.num_recv_max);
        const int g = blockIdx.x * kPairs + pair, P = a.push_blocks * kPairs;
        const bool wave = a.chunk < 0;
        const int my_rows = wave ? wave_num_rows(g, P, s_prefix, R, num_recv) : pair_num_rows(g, P, num_recv, a.chunk);
        // k walks the schedule, c counts this pair's rows (pipeline slot / phase / announce index)
        auto row_at = [&](int k) { return wave ? wave_row(g, P, k, s_prefix, R, num_recv) : pair_row(g, P, k, a.chunk, num_recv); };
        const int S = p.S;
        const int64_t rows_cap = (int64_t)a.layout.capacity * a.layout.num_ranks;
        if (producer && kExpanded) {
            // Producer prod_idx computes the pair's rows c with c % kProducers == prod_idx straight into
            // their slots (generic stores, then a proxy fence so the consumer's TMA store sees them).
            int c = 0;
            for (int k = 0; c < my_rows; ++k) {
                const int j = row_at(k);
                if (j < 0) continue;
                if (c % kProducers == prod_idx) {
                    const int slot = c % S;
                    int good = 1;
                    if (lane == 0 && c >= S) good = mbar_wait(&p.empty[slot], ((c / S) - 1) & 1, a.st, kErrTimeoutTma) ? 1 : 0;
                    if (!__shfl_sync(0xffffffffu, good, 0)) break;
                    expanded_token_to_slot(a, j, p.slots + (size_t)slot * slot_bytes);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&p.full[slot]);
                }
                ++c;
            }
        } else if (producer) {
            // Only lane 0 works in this loop (no warp-wide step), so it alone stops at an expired
            // wait (the consumer stops at the first row that does not arrive) and drains what it issued.
            int c = 0;
            for (int k = 0; c < my_rows; ++k) {
                const int j = row_at(k);
                if (j < 0) continue;
                if (lane == 0) {
                    const int slot = c % S;
                    if (c >= S && !mbar_wait(&p.empty[slot], ((c / S) - 1) & 1, a.st, kErrTimeoutTma)) break;
                    mbar_arrive_expect_tx(&p.full[slot], row_bytes);
                    tma_load_1d(p.slots + (size_t)slot * slot_bytes, static_cast<const uint8_t*>(a.x) + (int64_t)j * row_bytes,
                                row_bytes, &p.full[slot]);
                }
                ++c;
            }
            if (lane == 0) ring_drain(p.full, S, c, a.st, kErrTimeoutTma);
        } else {
            // Slots recycle on read-completion (as in the pull). Arrivals are announced per batch of
            // kAnnounce rows: one drain of this thread's bulk stores, one sys-scope fence, then relaxed
            // reds (a release per row would wait for an NVLink round trip every row). With
            // `announce_lagged` the batch is announced when the NEXT batch is complete issued:
            // `wait_group kAnnounce` then only waits for the older batch, so the stores of the newer
            // one stay in flight instead of draining the pipe every kAnnounce rows.
            constexpr int kAnnounce = 16;
            const int lag = S / 2 < 4 ? S / 2 : 4;
            const bool lagged = a.announce_lagged != 0;
            int* arrivals[kMaxRanks];
#pragma unroll
            for (int r = 0; r < kMaxRanks; ++r)
                arrivals[r] = r < R ? reinterpret_cast<int*>(static_cast<uint8_t*>(a.peers.base[r]) + a.layout.arrival_off) : nullptr;
            int pend_t = -1, pend_d = 0;  // lane i holds the i-th row of the current announce batch
            int prev_t = -1, prev_d = 0, prev_cnt = 0;  // lagged mode: the batch waiting for announcement
            for (int kk = 0, k = 0; k < my_rows; ++kk) {
                const int j = row_at(kk);
                if (j < 0) continue;
                const int slot = k % S;
                const int d = find_source(s_prefix, R, j);
                const int64_t drow = s_base[d] + (j - s_prefix[d]);
                int good = 1;
                if (lane == 0) good = mbar_wait(&p.full[slot], (k / S) & 1, a.st, kErrTimeoutTma) ? 1 : 0;
                if (!__shfl_sync(0xffffffffu, good, 0)) break;
                if (!in_window(drow, 1, rows_cap)) {
                    if (lane == 0) report_error(a.st, kErrBounds, d, (int)drow);
                    break;
                }
                uint8_t* peer = static_cast<uint8_t*>(a.peers.base[d]);
                if (a.topk_weights != nullptr && lane < a.layout.topk_pad) {
                    float* wdst = reinterpret_cast<float*>(peer + a.layout.combine_w_off) + drow * a.layout.topk_pad;
                    wdst[lane] = lane < K ? a.topk_weights[(int64_t)j * K + lane] : 0.f;
                }
                if (lane == k % kAnnounce) {
                    pend_t = a.recv_src_idx[j];
                    pend_d = d;
                }
                __syncwarp();
                if (lane == 0) {
                    tma_store_1d(peer + a.layout.combine_off + drow * row_bytes, p.slots + (size_t)slot * slot_bytes, row_bytes);
                    bulk_commit();
                    release_slots(p, k, lag);
                }
                const bool flush = (k % kAnnounce) == kAnnounce - 1 || k + 1 == my_rows;
                if (flush && !lagged) {
                    const int cnt = (k % kAnnounce) + 1;
                    if (lane == 0) {
                        bulk_wait<0>();
                        fence_proxy_async_global();
                        fence_sys();  // weight stores of every lane precede the __syncwarp above
                    }
                    for (int i = 0; i < cnt; ++i) {
                        const int tt = __shfl_sync(0xffffffffu, pend_t, i), dd = __shfl_sync(0xffffffffu, pend_d, i);
                        if (lane == 0) atomicAdd_system(arrivals[dd] + tt, 1);
                    }
                } else if (flush) {
                    // The previous batch's groups are all older than the kAnnounce (or fewer) groups
                    // just committed for the current batch: waiting until at most kAnnounce remain
                    // completes exactly them. The last batch drains everything and announces both.
                    const int cnt = (k % kAnnounce) + 1;
                    const bool last = k + 1 == my_rows;
                    if (lane == 0) {
                        if (last || cnt < kAnnounce) bulk_wait<0>();
                        else bulk_wait<kAnnounce>();
                        fence_proxy_async_global();
                        fence_sys();
                    }
                    for (int i = 0; i < prev_cnt; ++i) {
                        const int tt = __shfl_sync(0xffffffffu, prev_t, i), dd = __shfl_sync(0xffffffffu, prev_d, i);
                        if (lane == 0) atomicAdd_system(arrivals[dd] + tt, 1);
                    }
                    if (last) {
                        for (int i = 0; i < cnt; ++i) {
                            const int tt = __shfl_sync(0xffffffffu, pend_t, i), dd = __shfl_sync(0xffffffffu, pend_d, i);
                            if (lane == 0) atomicAdd_system(arrivals[dd] + tt, 1);
                        }
                        prev_cnt = 0;
                    } else {
                        prev_t = pend_t;
                        prev_d = pend_d;
                        prev_cnt = cnt;
                    }
                }
                __syncwarp();
                ++k;
            }
            // After an early exit (an expired wait or a bounds error) stores of the unannounced batch
            // may still read the ring: complete them before this warp moves on.
            if (lane == 0) bulk_wait<0>();
            if (lagged && prev_cnt > 0) {
                // The loop left early (an expired wait or a bounds error): announce what completed.
                if (lane == 0) {
                    bulk_wait<0>();
                    fence_proxy_async_global();
                    fence_sys();
                }
                for (int i = 0; i < prev_cnt; ++i) {
                    const int tt = __shfl_sync(0xffffffffu, prev_t, i), dd = __shfl_sync(0xffffffffu, prev_d, i);
                    if (lane == 0) atomicAdd_system(arrivals[dd] + tt, 1);
                }
            }
        }
    }
    if (pusher && lane == 0 && pair_warp) trace_end(a.st, kTraceCombinePush, t_start, warp);
    // Every warp (push warps once their rows are sent) reduces tokens of this rank.
    if (!aborted(a.st)) combine_reduce_loop(a, my_ctrl, s_red_base);
    __syncthreads();
    if (threadIdx.x == 0) {
        trace_end(a.st, kTraceCombine, t_start, pusher ? 1 : 0);
        const int old = atom_add_acq_rel_gpu(&my_ctrl->combine_reduced_blocks, 1);
        if (old == (int)gridDim.x - 1) {
            my_ctrl->combine_reduced_blocks = 0;
            my_ctrl->combine_token_cursor = 0;
            const int seq = ld_volatile(&my_ctrl->combine_seq) + 1;
            my_ctrl->combine_seq = seq;
            fence_sys();
            for (int r = 0; r < R; ++r) st_release_sys(&ctrl_of(a.peers, a.layout, r)->combine_ready[a.rank], seq);
        }
    }
}

void launch_combine(const CombineArgs& a_in, int num_sms, cudaStream_t stream) {
    CombineArgs a = a_in;
    int sm_count = 148, dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, dev);
    const int slot_bytes = (a.layout.hidden * 2 + 127) / 128 * 128;
    if (a.stages <= 0) a.stages = pipe_stages(slot_bytes, 16);
    if (a.stages < 4) a.stages = 4;
    // All blocks co-resident (one per SM): push blocks carry 2 push pairs + 4 reducer warps, the
    // remaining SMs reduce only; push warps join the reduction when their rows are out.
    a.push_blocks = num_sms < sm_count ? num_sms : sm_count;
    if (a.push_blocks < 1) a.push_blocks = 1;
    const int reduce_blocks = sm_count - a.push_blocks;
    const size_t smem = pipe_smem_bytes(a.stages, slot_bytes);
    if (a.row_map != nullptr) {
        cudaFuncSetAttribute(combine_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        combine_kernel<true><<<a.push_blocks + reduce_blocks, kCombineThreads, smem, stream>>>(a);
    } else {
        cudaFuncSetAttribute(combine_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        combine_kernel<false><<<a.push_blocks + reduce_blocks, kCombineThreads, smem, stream>>>(a);
    }
}

// =================================================================================================
// barrier across the NVLink domain (bounded).
// =================================================================================================
__global__ void barrier_kernel(PeerTable peers, int64_t ctrl_off, int rank, int num_ranks, KernelStatus st) {
    const int r = threadIdx.x;
    const uint64_t t_start = trace_begin(st);
    NormalCtrl* mine = reinterpret_cast<NormalCtrl*>(static_cast<uint8_t*>(peers.base[rank]) + ctrl_off);
    const int epoch = ld_volatile(&mine->barrier_epoch) + 1;
    if (r < num_ranks) {
        NormalCtrl* peer = reinterpret_cast<NormalCtrl*>(static_cast<uint8_t*>(peers.base[r]) + ctrl_off);
        fence_sys();
        st_release_sys(&peer->barrier_flag[rank], epoch);
        wait_ge(&mine->barrier_flag[r], epoch, st, kErrTimeoutBarrier, r);
    }
    __syncwarp();
    if (r == 0) {
        mine->barrier_epoch = epoch;
        trace_end(st, kTraceBarrier, t_start, epoch);
    }
}

void launch_barrier(PeerTable peers, int64_t ctrl_off, int rank, int num_ranks, KernelStatus st, cudaStream_t stream) {
    barrier_kernel<<<1, 32, 0, stream>>>(peers, ctrl_off, rank, num_ranks, st);
}

__global__ void read_globaltimer_kernel(unsigned long long* out) { *out = globaltimer_ns(); }

void launch_read_globaltimer(unsigned long long* out, cudaStream_t stream) {
    read_globaltimer_kernel<<<1, 1, 0, stream>>>(out);
}

}  // namespace ep
