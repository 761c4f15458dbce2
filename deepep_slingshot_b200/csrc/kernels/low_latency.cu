// Low-latency (decode) expert-parallel kernels over NVLink 5 / NVSwitch, sm_100a.
//
// Capability parity with the reference's LL path ([DE]csrc/kernels/legacy/internode_ll.cu:129-555
// dispatch, :715-1230 combine, :1241-1256 clean, :1258-1289 mask ops; Python surface
// [DE]deep_ep/buffers/legacy.py:538-713), re-designed for one NVLink domain:
//
//  * dispatch send phase: one block per token; its 8 warps quantize the bf16 row to FP8 e4m3 with
//    1x128 scales (optional power-of-two / UE8M0 scales) into shared memory together, then warp k
//    claims a slot for top-k choice k in the destination's per-expert receive block with ONE remote
//    atomic (so rows land already compacted: valid rows of expert e are [0, recv_count[e]) with no
//    receive-side packing copy) and TMA-stores the row straight into `recv_x[e][slot]`; scales go into
//    the column-major scale block and (token, src rank, k) into the src-info arrays. The last block
//    sets a per-source `dispatch_done` flag in every destination.
//  * dispatch recv phase (the hook): bounded wait on the R flags (the last block resets them, so no
//    sequence numbers are needed and captured graphs replay), then per local expert read/reset the
//    slot counter and produce recv_count / layout_range / statistics.
//  * combine send phase: every received row (expert output) is TMA-copied back into the source
//    rank's [token][k] slot (with `use_logfmt` encoded in place to LogFMT-10 first); the last block
//    sets `combine_done`.
//  * combine recv phase (the hook): bounded wait, then the top-k WEIGHTED fp32 reduction + bf16 cast,
//    eight warps per token (decoding LogFMT groups on the fly).
// Two halves alternate (double buffering), as in the reference. In shrink mode an expired wait
// masks the silent rank instead of failing.
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include "../include/ep/device.cuh"
#include "../include/ep/logfmt.cuh"
#include "../include/ep/quant.cuh"
#include "api.h"

namespace ep {

namespace {

struct LLHalf {
    uint8_t* base;
    const LLLayout* l;
    __device__ LLCtrl* ctrl() const { return reinterpret_cast<LLCtrl*>(base + l->ctrl_off); }
    __device__ uint8_t* recv_x() const { return base + l->recv_x_off; }
    __device__ float* recv_scales() const { return reinterpret_cast<float*>(base + l->recv_scales_off); }
    __device__ int* src_info() const { return reinterpret_cast<int*>(base + l->recv_src_info_off); }
    __device__ int* src_meta() const { return reinterpret_cast<int*>(base + l->recv_src_meta_off); }
    __device__ __nv_bfloat16* combine_recv() const { return reinterpret_cast<__nv_bfloat16*>(base + l->combine_recv_off); }
    __device__ uint32_t* combine_meta() const { return reinterpret_cast<uint32_t*>(base + l->combine_meta_off); }
};

__device__ __forceinline__ LLHalf half_of(const PeerTable& p, const LLLayout& l, int rank, int half) {
    return LLHalf{static_cast<uint8_t*>(p.base[rank]) + (int64_t)half * l.half_bytes, &l};
}

// Shrink-mode mask, snapshotted into shared memory once per block (a volatile global load per
// (token, k) would put a round trip to L2 on every message).
__device__ __forceinline__ uint32_t load_mask_bits(const int* mask, int R) {
    uint32_t m = 0;
    if (mask != nullptr)
        for (int r = 0; r < R; ++r) m |= (ld_volatile(mask + r) != 0 ? 1u : 0u) << r;
    return m;
}

// Bounded wait used by LL receivers. In shrink mode an expired wait masks `peer` and succeeds.
__device__ bool ll_wait(const int* flag, int target, const KernelStatus& st, int code, int peer, int* mask, bool shrink,
                        int64_t* wait_stats) {
    const uint64_t t0 = globaltimer_ns();
    bool ok;
    if (shrink) {
        KernelStatus quiet = st;
        quiet.host_error = nullptr;
        quiet.abort_flag = nullptr;
        ok = wait_ge(flag, target, quiet, code, peer);
        if (!ok && mask != nullptr) atomicExch(mask + peer, 1);
        ok = true;
    } else {
        ok = wait_ge(flag, target, st, code, peer);
    }
    if (wait_stats != nullptr) atomicAdd(reinterpret_cast<unsigned long long*>(wait_stats + peer),
                                         (unsigned long long)(globaltimer_ns() - t0));
    return ok;
}

}  // namespace

// =================================================================================================
// LL dispatch
// =================================================================================================
__global__ void __launch_bounds__(256) ll_dispatch_kernel(LLDispatchArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_src_count[kMaxRanks];
    const LLLayout& L = a.layout;
    const int lane = lane_id(), warp = warp_id(), W = blockDim.x / 32;
    const int H = L.hidden, K = L.num_topk, R = L.num_ranks, E_l = L.num_local_experts;
    const int slots = R * L.max_tokens;
    const int nb = H / 128;
    const int row_bytes = a.use_fp8 ? H : 2 * H;
    const uint64_t t_start = trace_begin(a.st);
    __shared__ uint32_t s_masked;
    if (threadIdx.x == 0) s_masked = load_mask_bits(a.mask, R);
    __syncthreads();
    uint32_t masked = s_masked;

    if (a.phases & 1) {
        // One block per token: the 8 warps quantize the row cooperatively into shared memory, then
        // warp k claims a slot for top-k choice k (one remote atomic) and TMA-stores the row there.
        uint8_t* buf = smem;
        float* sbuf = reinterpret_cast<float*>(buf + row_bytes);
        for (int t = blockIdx.x; t < a.num_tokens; t += gridDim.x) {
            const __nv_bfloat16* xr = static_cast<const __nv_bfloat16*>(a.x) + (int64_t)t * H;
            for (int base = warp * 256; base < H; base += W * 256) {
                const int e = base + lane * 8;
                const bool valid = e < H;
                const int4 v = valid ? ld_nc_v4(reinterpret_cast<const int4*>(xr + e)) : make_int4(0, 0, 0, 0);
                if (a.use_fp8) {
                    float scale;
                    const uint2 q = quantize_8(v, a.round_scale != 0, &scale);
                    if (valid) {
                        *reinterpret_cast<uint2*>(buf + e) = q;
                        if ((lane & 15) == 0) sbuf[e / 128] = scale;
                    }
                } else if (valid) {
                    *reinterpret_cast<int4*>(buf + 2 * e) = v;
                }
            }
            fence_proxy_async_smem();  // generic smem writes -> visible to the TMA (async proxy)
            __syncthreads();
            if (warp < K) {
                const int k = warp;
                int dst_rank = -1, le = -1, slot = -1;
                if (lane == 0) {
                    const int64_t e = a.topk_idx[(int64_t)t * K + k];
                    if (e >= 0 && e < L.num_experts) {
                        dst_rank = (int)(e / E_l);
                        le = (int)(e % E_l);
                        if ((masked >> dst_rank) & 1u) {
                            dst_rank = -1;
                        } else {
                            LLHalf h = half_of(a.peers, L, dst_rank, a.half);
                            slot = atom_add_relaxed_sys(&h.ctrl()->slot_counter[le], 1);
                            if (slot >= slots) {
                                report_error(a.st, kErrCapacity, dst_rank, slot);
                                dst_rank = -1;
                            }
                        }
                    }
                }
                dst_rank = __shfl_sync(0xffffffffu, dst_rank, 0);
                le = __shfl_sync(0xffffffffu, le, 0);
                slot = __shfl_sync(0xffffffffu, slot, 0);
                if (dst_rank >= 0) {
                    LLHalf h = half_of(a.peers, L, dst_rank, a.half);
                    const int64_t row = (int64_t)le * slots + slot;
                    if (lane == 0) {
                        tma_store_1d(h.recv_x() + row * row_bytes, buf, row_bytes);
                        bulk_commit();
                        h.src_info()[row] = t;
                        h.src_meta()[row] = a.rank * K + k;
                    }
                    if (a.use_fp8) {
                        float* sc = h.recv_scales() + (int64_t)le * nb * slots;
                        for (int b = lane; b < nb; b += 32) sc[(int64_t)b * slots + slot] = sbuf[b];
                    }
                }
                if (lane == 0) bulk_wait_read<0>();  // the row buffer is rewritten for the next token
            }
            __syncthreads();
        }
        if (warp < K && lane == 0) {
            bulk_wait<0>();
            fence_proxy_async_global();
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            trace_end(a.st, kTraceLLDispatchSend, t_start, a.num_tokens);
            LLHalf mine = half_of(a.peers, L, a.rank, a.half);
            fence_sys();
            const int old = atom_add_acq_rel_gpu(&mine.ctrl()->send_finished_blocks, 1);
            if (old == (int)gridDim.x - 1) {
                mine.ctrl()->send_finished_blocks = 0;
                fence_sys();
                for (int d = 0; d < R; ++d) {
                    if ((masked >> d) & 1u) continue;
                    st_release_sys(&half_of(a.peers, L, d, a.half).ctrl()->dispatch_done[a.rank], 1);
                }
            }
        }
    }

    if (a.phases & 2) {
        const uint64_t t_recv = trace_begin(a.st);
        LLHalf mine = half_of(a.peers, L, a.rank, a.half);
        if ((int)threadIdx.x < R && !((masked >> threadIdx.x) & 1u))
            ll_wait(&mine.ctrl()->dispatch_done[threadIdx.x], 1, a.st, kErrTimeoutLLDispatch, threadIdx.x, a.mask,
                    a.shrink != 0, blockIdx.x == 0 ? a.wait_stats : nullptr);
        __syncthreads();
        // The last block that has seen every flag resets them for the next use of this half.
        if (threadIdx.x == 0) {
            const int old = atom_add_acq_rel_gpu(&mine.ctrl()->recv_finished_blocks, 1);
            if (old == (int)gridDim.x - 1) {
                mine.ctrl()->recv_finished_blocks = 0;
                for (int s = 0; s < R; ++s) mine.ctrl()->dispatch_done[s] = 0;
            }
        }
        for (int le = blockIdx.x; le < E_l; le += gridDim.x) {
            if (threadIdx.x < kMaxRanks) s_src_count[threadIdx.x] = 0;
            __syncthreads();
            const int count = min(ld_volatile(&mine.ctrl()->slot_counter[le]), slots);
            for (int j = threadIdx.x; j < count; j += blockDim.x) {
                const int src = ld_volatile(&mine.src_meta()[(int64_t)le * slots + j]) / K;
                if (src >= 0 && src < R) atomicAdd(&s_src_count[src], 1);
            }
            __syncthreads();
            if (threadIdx.x == 0) {
                a.recv_count[le] = count;
                mine.ctrl()->slot_counter[le] = 0;
                if (a.cumulative_stats != nullptr) a.cumulative_stats[le] += count;
            }
            if ((int)threadIdx.x < R && a.layout_range != nullptr)
                a.layout_range[(int64_t)le * R + threadIdx.x] = (int64_t)s_src_count[threadIdx.x];
            __syncthreads();
        }
        if (threadIdx.x == 0) trace_end(a.st, kTraceLLDispatchRecv, t_recv);
    }
}

void launch_ll_dispatch(const LLDispatchArgs& a, cudaStream_t stream) {
    const LLLayout& L = a.layout;
    const int W = 8;
    const int nb = L.hidden / 128;
    const int row_bytes = a.use_fp8 ? L.hidden : 2 * L.hidden;
    const size_t smem = (a.phases & 1) ? (size_t)((row_bytes + nb * 4 + 127) / 128 * 128) : 0;
    int num_sms = 148;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);
    int blocks = 1;
    if (a.phases & 1) blocks = a.num_tokens;  // one block per token
    if (a.phases & 2) blocks = blocks > L.num_local_experts ? blocks : L.num_local_experts;
    if (blocks > num_sms) blocks = num_sms;  // all blocks co-resident: the recv phase may wait on the send phase
    if (blocks < 1) blocks = 1;
    if (smem > 48 * 1024) cudaFuncSetAttribute(ll_dispatch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    ll_dispatch_kernel<<<blocks, W * 32, smem, stream>>>(a);
}

// =================================================================================================
// LL combine
// =================================================================================================
template <bool kLogFMT>
__global__ void __launch_bounds__(256) ll_combine_kernel(LLCombineArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t s_bar[8];
    const LLLayout& L = a.layout;
    const int lane = lane_id(), warp = warp_id(), W = blockDim.x / 32;
    const int H = L.hidden, K = L.num_topk, R = L.num_ranks, E_l = L.num_local_experts;
    const int slots = R * L.max_tokens;
    const int row_bytes = 2 * H;
    const uint64_t t_start = trace_begin(a.st);
    __shared__ uint32_t s_masked;
    if (threadIdx.x == 0) s_masked = load_mask_bits(a.mask, R);
    __syncthreads();
    uint32_t masked = s_masked;

    if (a.phases & 1) {
        uint8_t* buf = smem + (size_t)warp * ((row_bytes + 127) / 128 * 128);
        if (lane == 0) {
            mbar_init(&s_bar[warp], 1);
            fence_mbar_init();
        }
        __syncwarp();
        uint32_t phase = 0;
        LLHalf dsp = half_of(a.peers, L, a.rank, a.dispatch_half);
        bool ok = true;
        for (int64_t g = (int64_t)blockIdx.x * W + warp; g < (int64_t)E_l * slots && ok; g += (int64_t)gridDim.x * W) {
            const int le = (int)(g / slots), j = (int)(g % slots);
            if (j >= a.recv_count[le]) continue;
            const int meta = dsp.src_meta()[(int64_t)le * slots + j];
            const int t = dsp.src_info()[(int64_t)le * slots + j];
            const int src = meta / K, k = meta % K;
            if (!in_window(src, 1, R) || !in_window(t, 1, L.max_tokens)) {
                if (lane == 0) report_error(a.st, kErrBounds, src, t);
                continue;
            }
            if (((masked >> (src))) & 1u) continue;
            if constexpr (kLogFMT) {
                // Every lane waits for the row (the whole warp reads it), encodes it in place, then
                // lane 0 stores the compacted bytes; group metadata goes out with plain stores.
                if (lane == 0) {
                    bulk_wait_read<0>();
                    mbar_arrive_expect_tx(&s_bar[warp], row_bytes);
                    tma_load_1d(buf, static_cast<const uint8_t*>(a.x) + ((int64_t)le * slots + j) * row_bytes, row_bytes,
                                &s_bar[warp]);
                }
                __syncwarp();
                ok = __all_sync(0xffffffffu, mbar_wait(&s_bar[warp], phase, a.st, kErrTimeoutTma) ? 1 : 0) != 0;
                if (!ok && lane == 0) mbar_wait(&s_bar[warp], phase, a.st, kErrTimeoutTma);  // the row lands before exit
                phase ^= 1u;
                if (ok) {
                    LLHalf dh = half_of(a.peers, L, src, a.half);
                    uint32_t* meta = dh.combine_meta() + ((int64_t)t * K + k) * (H / 128);
                    const int n = logfmt_encode_row(buf, H, meta);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_1d(dh.combine_recv() + ((int64_t)t * K + k) * H, buf, n);
                        bulk_commit();
                    }
                }
            } else {
                if (lane == 0) {
                    bulk_wait_read<0>();
                    mbar_arrive_expect_tx(&s_bar[warp], row_bytes);
                    tma_load_1d(buf, static_cast<const uint8_t*>(a.x) + ((int64_t)le * slots + j) * row_bytes, row_bytes,
                                &s_bar[warp]);
                    ok = mbar_wait(&s_bar[warp], phase, a.st, kErrTimeoutTma);
                    if (!ok) mbar_wait(&s_bar[warp], phase, a.st, kErrTimeoutTma);  // the row lands before exit
                    phase ^= 1u;
                    if (ok) {
                        LLHalf dh = half_of(a.peers, L, src, a.half);
                        tma_store_1d(dh.combine_recv() + ((int64_t)t * K + k) * H, buf, row_bytes);
                        bulk_commit();
                    }
                }
                ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            }
        }
        if (lane == 0) {
            bulk_wait<0>();
            fence_proxy_async_global();
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            trace_end(a.st, kTraceLLCombineSend, t_start);
            LLHalf mine = half_of(a.peers, L, a.rank, a.half);
            fence_sys();
            const int old = atom_add_acq_rel_gpu(&mine.ctrl()->csend_finished_blocks, 1);
            if (old == (int)gridDim.x - 1) {
                mine.ctrl()->csend_finished_blocks = 0;
                fence_sys();
                for (int d = 0; d < R; ++d) {
                    if (((masked >> (d))) & 1u) continue;
                    st_release_sys(&half_of(a.peers, L, d, a.half).ctrl()->combine_done[a.rank], 1);
                }
            }
        }
    }

    if (a.phases & 2) {
        const uint64_t t_recv = trace_begin(a.st);
        LLHalf mine = half_of(a.peers, L, a.rank, a.half);
        if ((int)threadIdx.x < R && !((masked >> threadIdx.x) & 1u))
            ll_wait(&mine.ctrl()->combine_done[threadIdx.x], 1, a.st, kErrTimeoutLLCombine, threadIdx.x, a.mask,
                    a.shrink != 0, blockIdx.x == 0 ? a.wait_stats : nullptr);
        __syncthreads();
        if (threadIdx.x == 0) {
            const int old = atom_add_acq_rel_gpu(&mine.ctrl()->crecv_finished_blocks, 1);
            if (old == (int)gridDim.x - 1) {
                mine.ctrl()->crecv_finished_blocks = 0;
                for (int s = 0; s < R; ++s) mine.ctrl()->combine_done[s] = 0;
            }
        }
        if (aborted(a.st) && !a.shrink) return;
        masked = load_mask_bits(a.mask, R);  // ranks masked by an expired wait above
        const __nv_bfloat16* recv = mine.combine_recv();
        // Eight warps per token, each summing one eighth of the hidden dimension.
        const int span = (H / W + 7) / 8 * 8;
        for (int t = blockIdx.x; t < a.num_tokens; t += gridDim.x) {
            float wk = 0.f;
            int use = 0;
            if (lane < K) {
                const int64_t e = a.topk_idx[(int64_t)t * K + lane];
                if (e >= 0 && e < L.num_experts && !((masked >> (int)(e / E_l)) & 1u)) {
                    use = 1;
                    wk = a.topk_weights[(int64_t)t * K + lane];
                }
            }
            const uint32_t use_mask = __ballot_sync(0xffffffffu, use);
            int ks[kMaxTopk];
            float ws[kMaxTopk];
            int n = 0;
            for (int k = 0; k < K; ++k) {
                const float wv = __shfl_sync(0xffffffffu, wk, k);
                if ((use_mask >> k) & 1u) {
                    ks[n] = k;
                    ws[n] = wv;
                    ++n;
                }
            }
            const __nv_bfloat16* trow = recv + (int64_t)t * K * H;
            const int h0 = warp * span, h1 = min(H, h0 + span);
            if constexpr (kLogFMT) {
                // Encoded groups before each group of slot ks[q]: one ballot per 32 groups.
                const uint32_t* meta_t = mine.combine_meta() + (int64_t)t * K * (H / 128);
                const int groups = H / 128;
                uint32_t cmask[kMaxTopk][kLogFmtMaxGroupsPerLane];
                for (int q = 0; q < n; ++q)
#pragma unroll
                    for (int i = 0; i < kLogFmtMaxGroupsPerLane; ++i) {
                        const int gg = i * 32 + lane;
                        const uint32_t m = gg < groups ? ld_volatile_u32(meta_t + (int64_t)ks[q] * groups + gg) : 0u;
                        cmask[q][i] = __ballot_sync(0xffffffffu, (m & 0x8000u) != 0);
                    }
                for (int e0 = h0 + lane * 8; e0 < h1; e0 += 256) {
                    const int g = e0 >> 7, p = e0 & 127;
                    float acc[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
                    for (int q = 0; q < n; ++q) {
                        int before = 0;
#pragma unroll
                        for (int i = 0; i < kLogFmtMaxGroupsPerLane; ++i) {
                            const int lo = i * 32;
                            if (g > lo) before += __popc(g - lo >= 32 ? cmask[q][i] : (cmask[q][i] & ((1u << (g - lo)) - 1u)));
                        }
                        const uint32_t m = ld_volatile_u32(meta_t + (int64_t)ks[q] * groups + g);
                        logfmt_accumulate8(reinterpret_cast<const uint8_t*>(trow + (int64_t)ks[q] * H), g, p, before, m,
                                           ws[q], acc);
                    }
                    int4 o;
                    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
                    for (int i = 0; i < 4; ++i) o2[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
                    *reinterpret_cast<int4*>(static_cast<__nv_bfloat16*>(a.out) + (int64_t)t * H + e0) = o;
                }
                continue;
            }
            for (int e0 = h0 + lane * 8; e0 < h1; e0 += 256) {
                int4 v[kMaxTopk];
#pragma unroll
                for (int q = 0; q < kMaxTopk; ++q)
                    if (q < n) v[q] = *reinterpret_cast<const int4*>(trow + (int64_t)ks[q] * H + e0);
                float acc[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll
                for (int q = 0; q < kMaxTopk; ++q) {
                    if (q >= n) break;
                    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&v[q]);
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
                *reinterpret_cast<int4*>(static_cast<__nv_bfloat16*>(a.out) + (int64_t)t * H + e0) = o;
            }
        }
        if (threadIdx.x == 0) trace_end(a.st, kTraceLLCombineRecv, t_recv, a.num_tokens);
    }
}

void launch_ll_combine(const LLCombineArgs& a, cudaStream_t stream) {
    const LLLayout& L = a.layout;
    const int W = 8;
    const size_t smem = (a.phases & 1) ? (size_t)W * ((2 * L.hidden + 127) / 128 * 128) : 0;
    int num_sms = 148;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);
    int blocks = num_sms;
    if (!(a.phases & 1)) {
        blocks = a.num_tokens;  // receive: one block (8 warps) per token
        if (blocks > num_sms) blocks = num_sms;
    }
    if (blocks < 1) blocks = 1;
    if (a.use_logfmt) {
        if (smem > 48 * 1024) cudaFuncSetAttribute(ll_combine_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        ll_combine_kernel<true><<<blocks, W * 32, smem, stream>>>(a);
    } else {
        if (smem > 48 * 1024) cudaFuncSetAttribute(ll_combine_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        ll_combine_kernel<false><<<blocks, W * 32, smem, stream>>>(a);
    }
}

// =================================================================================================
// LL clean: zero the slot counters of both halves (flags are epoch-valued and need no reset).
// =================================================================================================
__global__ void ll_clean_kernel(PeerTable peers, LLLayout layout, int rank) {
    for (int h = 0; h < 2; ++h) {
        LLHalf mine = half_of(peers, layout, rank, h);
        for (int i = threadIdx.x; i < kMaxLocalExperts; i += blockDim.x) mine.ctrl()->slot_counter[i] = 0;
        if (threadIdx.x == 0) {
            mine.ctrl()->send_finished_blocks = 0;
            mine.ctrl()->csend_finished_blocks = 0;
            mine.ctrl()->recv_finished_blocks = 0;
            mine.ctrl()->crecv_finished_blocks = 0;
        }
        if (threadIdx.x < kMaxRanks) {
            mine.ctrl()->dispatch_done[threadIdx.x] = 0;
            mine.ctrl()->combine_done[threadIdx.x] = 0;
        }
    }
}

void launch_ll_clean(PeerTable peers, LLLayout layout, int rank, KernelStatus st, cudaStream_t stream) {
    (void)st;
    ll_clean_kernel<<<1, 256, 0, stream>>>(peers, layout, rank);
}

}  // namespace ep
