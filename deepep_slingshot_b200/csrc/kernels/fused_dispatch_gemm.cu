// Normal-mode dispatch receive fused with the gate/up grouped FP8 GEMM (tcgen05 + TMEM), sm_100a.
//
// One persistent launch (one CTA per SM) after the dispatch's stage and notify steps:
//  * pull role (the first `pull_ctas` CTAs, four producer/consumer warp pairs each): every received
//    row's record is TMA-loaded from its source's staging over NVLink (no multicast) into a
//    shared-memory ring, as in the plain pull. The consumer claims, for every local expert the token
//    selected, the next slot of that expert (one atomic), TMA-stores the FP8 row and its 1x128 scales
//    straight into the expert-grouped, 128-aligned GEMM operand (`a`, `sa`), and writes the row map
//    (received token, k) -> operand row and the local top-k weights. Once a row's stores are complete
//    (`cp.async.bulk.wait_group`, a proxy fence) the consumer adds the row to its 128-row tile's landed
//    counter with a release.
//  * GEMM role (every other CTA at once; the pull CTAs when their rows are done): tiles are taken
//    from a global counter in level order (schedule.cuh `fused_gemm_tile`: every expert's first
//    m-tile, then every second m-tile, ... the order in which tiles fill). The producer waits
//    (bounded, acquire) until the tile's landed counter equals its row count, fences the async
//    proxy and TMA-loads A / B; warp 1 issues `tcgen05.mma.kind::f8f6f4` into one of two TMEM
//    accumulators; warps 2..9 promote each 128-K block with sa * sb in fp32 and write the tile's
//    valid bf16 rows. Tile ids go from the producer to the MMA and epilogue warps through a small
//    shared-memory queue.
// The transfer and the expert math overlap tile by tile, and no permute pass is needed. Waits on
// rows landed by other CTAs of this launch are safe because every CTA is resident (grid <= SMs,
// one CTA per SM) and the pull role never waits on the GEMM role. Every wait is bounded: an expired
// wait reports and the CTA winds down (sentinel tile ids release the consumers).
#include <cuda.h>
#include <cuda_bf16.h>

#include "../include/ep/device.cuh"
#include "../include/ep/schedule.cuh"
#include "gemm.h"
#include "tcgen05_common.cuh"

namespace ep {

namespace {

constexpr int kBM = 128, kBN = 128, kBK = 128;
constexpr int kStageBytes = (kBM + kBN) * kBK;  // 32 KiB
constexpr int kGemmStages = 6;
constexpr int kEpiWarps = 8;
constexpr int kThreads = (2 + kEpiWarps) * 32;
constexpr uint32_t kTmemCols = 2 * kBN;
constexpr int kPullPairs = 4;   // pull role: warps 0..7 form producer / consumer pairs
constexpr int kLag = 4;         // rows per consumer whose stores may still be in flight
constexpr int kTileQ = 4;       // tile-id queue depth
constexpr int kMaxLevels = 512; // m-tiles per expert

__host__ __device__ constexpr uint32_t idesc_e4m3_f32(int m, int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_f8(uint32_t tmem_d, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mbar_inval(uint64_t* bar) {
    asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void red_add_release_gpu(int* p, int v) {
    asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait for a landed-row counter written by other CTAs of this launch.
__device__ __forceinline__ bool wait_landed(const int* p, int target, const KernelStatus& st, int detail) {
    if (ld_acquire_gpu(p) >= target) return true;
    const uint64_t start = globaltimer_ns();
    uint32_t iter = 0;
    while (true) {
        if (ld_acquire_gpu(p) >= target) return true;
        if ((++iter & 255u) == 0) {
            if (globaltimer_ns() - start > st.timeout_ns) {
                report_error(st, kErrTimeoutTma, -1, detail);
                return false;
            }
            if (aborted(st)) return false;
        }
    }
}

// Per-pair pull ring: [S slots][slot_bytes] | full[S] | empty[S] | side[S] | pend[kLag + 1][kMaxTopk].
struct PullRing {
    uint8_t* slots;
    uint64_t* full;
    uint64_t* empty;
    int* side;
    int* pend;
    int S, slot_bytes;
};

__host__ __device__ __forceinline__ size_t pull_pair_bytes(int S, int slot_bytes) {
    return ((size_t)S * slot_bytes + (size_t)S * 20 + (size_t)(kLag + 1) * kMaxTopk * 4 + 127) / 128 * 128;
}

__device__ __forceinline__ PullRing pull_ring(uint8_t* smem, int pair, int S, int slot_bytes) {
    uint8_t* base = smem + (size_t)pair * pull_pair_bytes(S, slot_bytes);
    PullRing r;
    r.slots = base;
    r.full = reinterpret_cast<uint64_t*>(base + (size_t)S * slot_bytes);
    r.empty = r.full + S;
    r.side = reinterpret_cast<int*>(r.empty + S);
    r.pend = r.side + S;
    r.S = S;
    r.slot_bytes = slot_bytes;
    return r;
}

struct FusedShared {
    int off[kMaxLocalExperts + 1];  // 128-aligned first operand row of every expert
    int cnt[kMaxLocalExperts];      // received rows per expert
    int order[kMaxLocalExperts];    // experts by decreasing m-tile count
    int level[kMaxLevels + 1];      // tile-row prefix per level
    int prefix[kMaxRanks + 1];      // receive rows per source rank (prefix)
    int levels;
    int tq[kTileQ];
    uint32_t tmem_base;
};

// Landed rows a tile waits for.
__device__ __forceinline__ int tile_rows(const FusedShared& sh, int e, int mt) { return min(kBM, sh.cnt[e] - mt * kBM); }

// ------------------------------------------------------------------------------------------------ pull role
__device__ void pull_role(const FusedDispatchGemmArgs& a, FusedShared& sh, uint8_t* smem, int S) {
    const int lane = lane_id(), warp = warp_id();
    const int R = a.num_ranks, K = a.num_topk, E_l = a.num_local_experts, lo_e = a.rank * E_l;
    const int slot_bytes = (a.rec.bytes + 127) / 128 * 128;
    const int nb = a.layout.hidden / 128;
    const uint64_t t_start = trace_begin(a.st);
    const int num_recv = ld_volatile(a.dev_num_recv);
    const bool active = warp < 2 * kPullPairs;
    const int pair = warp >> 1;
    const bool producer = (warp & 1) == 0;
    // Checked before the ring's mbarriers exist, so that an early return leaves none behind.
    if (num_recv > a.num_out_rows) {
        if (threadIdx.x == 0 && blockIdx.x == 0) report_error(a.st, kErrCapacity, -1, num_recv);
        return;
    }
    PullRing p{};
    if (active) {
        p = pull_ring(smem, pair, S, slot_bytes);
        if (producer && lane == 0) {
            for (int s = 0; s < S; ++s) {
                mbar_init(&p.full[s], 1);
                mbar_init(&p.empty[s], 1);
            }
            fence_mbar_init();
        }
    }
    // Host-mapped counts for the CPU (one idle warp of the first pull CTA).
    if (blockIdx.x == 0 && warp == 2 * kPullPairs && a.host != nullptr) {
        for (int le = lane; le < E_l; le += 32) a.host->num_recv_tokens_per_expert[le] = a.num_recv_per_expert[le];
        if (lane == 0) a.host->num_recv_tokens = num_recv;
        __syncwarp();
        if (lane == 0) {
            __threadfence_system();
            *reinterpret_cast<volatile int*>(&a.host->ready_ticket) = a.host_ticket;
        }
    }
    __syncthreads();
    if (active) {
        const int g = blockIdx.x * kPullPairs + pair, P = a.pull_ctas * kPullPairs;
        const int my_rows = pair_num_rows(g, P, num_recv, a.chunk);
        if (producer) {
            // Lane 0 issues the loads; after an expired wait it issues no more (the consumer stops
            // at the first row that does not arrive) instead of waiting out every later row.
            int failed = 0, issued = 0;
            for (int base = 0; base < my_rows; base += 32) {
                const int kk = base + lane;
                int src = 0, t = 0;
                if (kk < my_rows) {
                    const int j = pair_row(g, P, kk, a.chunk, num_recv);
                    src = find_source(sh.prefix, R, j);
                    const int* list = reinterpret_cast<const int*>(static_cast<const uint8_t*>(a.peers.base[src]) + a.layout.list_off) +
                                      (int64_t)a.rank * a.layout.capacity;
                    t = ld_relaxed_sys(list + (j - sh.prefix[src]));
                }
                const int n = min(32, my_rows - base);
                for (int i = 0; i < n; ++i) {
                    const int ps = __shfl_sync(0xffffffffu, src, i), pt = __shfl_sync(0xffffffffu, t, i);
                    if (lane == 0 && !failed) {
                        const int k = base + i, slot = k % S;
                        if (k >= S && !mbar_wait(&p.empty[slot], ((k / S) - 1) & 1, a.st, kErrTimeoutTma)) {
                            failed = 1;
                        } else {
                            p.side[slot] = pt;
                            const uint8_t* gsrc = static_cast<const uint8_t*>(a.peers.base[ps]) + a.layout.staging_off +
                                                  (int64_t)pt * a.layout.record_bytes;
                            mbar_arrive_expect_tx(&p.full[slot], a.rec.bytes);
                            tma_load_1d(p.slots + (size_t)slot * slot_bytes, gsrc, a.rec.bytes, &p.full[slot]);
                            ++issued;
                        }
                    }
                }
                if (__shfl_sync(0xffffffffu, failed, 0)) break;
            }
            // Every issued load lands before the ring's shared memory is reused (after a failure the
            // consumer may have stopped short of them).
            if (lane == 0) ring_drain(p.full, S, issued, a.st, kErrTimeoutTma);
        } else {
            // Lane 0 issues the stores and, kLag rows later, publishes their completion: it alone
            // observed the completion, fenced the async proxy and releases the counters.
            auto publish = [&](int kk) {
                const int* pend = p.pend + (kk % (kLag + 1)) * kMaxTopk;
                for (int q = 0; q < K; ++q)
                    if (pend[q] >= 0) red_add_release_gpu(a.landed + pend[q], 1);
            };
            int k = 0;
            for (; k < my_rows; ++k) {
                const int j = pair_row(g, P, k, a.chunk, num_recv), slot = k % S;
                int good = 1;
                if (lane == 0) good = mbar_wait(&p.full[slot], (k / S) & 1, a.st, kErrTimeoutTma) ? 1 : 0;
                if (!__shfl_sync(0xffffffffu, good, 0)) break;
                const uint8_t* buf = p.slots + (size_t)slot * slot_bytes;
                int row = -1, tile = -1;
                if (lane < K) {
                    const int e = reinterpret_cast<const int*>(buf + a.rec.idx_off)[lane];
                    const float w = reinterpret_cast<const float*>(buf + a.rec.w_off)[lane];
                    const bool mine = e >= lo_e && e < lo_e + E_l;
                    if (mine) {
                        const int le = e - lo_e;
                        const int s = atomicAdd(a.claim + le, 1);
                        if (s < sh.cnt[le]) {
                            row = sh.off[le] + s;
                            tile = le * a.max_mtiles + s / kBM;
                        } else {
                            report_error(a.st, kErrBounds, le, s);
                        }
                    }
                    a.row_map[(int64_t)j * K + lane] = row;
                    a.recv_topk_weights[(int64_t)j * K + lane] = row >= 0 ? w : 0.f;
                    p.pend[(k % (kLag + 1)) * kMaxTopk + lane] = tile;
                }
                for (int q = 0; q < K; ++q) {
                    const int r = __shfl_sync(0xffffffffu, row, q);
                    if (lane == 0 && r >= 0) {
                        tma_store_1d(a.a + (int64_t)r * a.layout.hidden, buf, a.rec.x_bytes);
                        tma_store_1d(a.sa + (int64_t)r * nb, buf + a.rec.scale_off, nb * 4);
                    }
                }
                __syncwarp();
                if (lane == 0) {
                    bulk_commit();
                    a.recv_src_idx[j] = p.side[slot];
                    bulk_wait<kLag>();  // rows <= k - kLag: stores complete, slot read
                    if (k >= kLag) {
                        fence_proxy_async_global();
                        publish(k - kLag);
                        mbar_arrive(&p.empty[(k - kLag) % S]);
                    }
                }
                __syncwarp();
            }
            if (lane == 0) {
                bulk_wait<0>();
                fence_proxy_async_global();
                for (int kk = max(0, k - kLag); kk < k; ++kk) publish(kk);
            }
        }
    }
    __syncthreads();
    // The ring's shared memory becomes GEMM stages: retire its mbarriers first.
    if (active && !producer && lane == 0)
        for (int s = 0; s < S; ++s) {
            mbar_inval(&p.full[s]);
            mbar_inval(&p.empty[s]);
        }
    // The last pull CTA tells every source that its staging may be reused.
    if (threadIdx.x == 0) {
        trace_end(a.st, kTracePull, t_start, num_recv);
        NormalCtrl* my_ctrl = reinterpret_cast<NormalCtrl*>(static_cast<uint8_t*>(a.peers.base[a.rank]) + a.layout.ctrl_off);
        fence_sys();
        const int old = atom_add_acq_rel_gpu(&my_ctrl->pull_finished_blocks, 1);
        if (old == a.pull_ctas - 1) {
            my_ctrl->pull_finished_blocks = 0;
            const int epoch = ld_volatile(&my_ctrl->dispatch_epoch);
            fence_sys();
            for (int s = 0; s < R; ++s) {
                NormalCtrl* c = reinterpret_cast<NormalCtrl*>(static_cast<uint8_t*>(a.peers.base[s]) + a.layout.ctrl_off);
                st_release_sys(&c->pull_done[a.rank], epoch);
            }
        }
    }
}

// ------------------------------------------------------------------------------------------------ GEMM role
__device__ void gemm_role(const CUtensorMap* map_a, const CUtensorMap* map_b, const FusedDispatchGemmArgs& a,
                          FusedShared& sh, uint8_t* smem) {
    __shared__ __align__(8) uint64_t s_full[kGemmStages], s_empty[kGemmStages];
    __shared__ __align__(8) uint64_t s_tfull[2], s_tempty[2];
    __shared__ __align__(8) uint64_t s_qfull[kTileQ], s_qempty[kTileQ];
    const int warp = warp_id(), lane = lane_id();
    const int KB = a.layout.hidden / kBK;
    const int n_tiles = a.n / kBN;
    const int levels = sh.levels;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kGemmStages; ++s) {
            mbar_init(&s_full[s], 1);
            mbar_init(&s_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&s_tfull[b], 1);
            mbar_init(&s_tempty[b], kEpiWarps);
        }
        for (int q = 0; q < kTileQ; ++q) {
            mbar_init(&s_qfull[q], 1);
            mbar_init(&s_qempty[q], 1 + kEpiWarps);
        }
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sh.tmem_base)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem_base = sh.tmem_base;
    // Consumers of the tile queue wait as long as a producer may wait for rows to land, and more.
    KernelStatus st_q = a.st;
    st_q.timeout_ns = 2 * a.st.timeout_ns + 1000000000ull;

    if (warp == 0) {
        // ---------------------------------------------------------------- tile fetch + TMA producer
        if (lane == 0) {
            uint32_t g = 0;
            bool ok = levels >= 0;
            for (int q = 0;; ++q) {
                const int t = ok ? atomicAdd(a.tile_counter, 1) : -1;
                int mt = 0, e = 0, nt = 0;
                const bool valid = ok && fused_gemm_tile(t, n_tiles, sh.level, levels, sh.order, mt, e, nt);
                const int slot = q % kTileQ;
                if (!mbar_wait(&s_qempty[slot], ((q / kTileQ) & 1) ^ 1, st_q, kErrTimeoutTma)) break;
                sh.tq[slot] = valid ? t : -1;  // -1: no more tiles (or a failure): the consumers stop
                mbar_arrive(&s_qfull[slot]);
                if (!valid) break;
                // After an expired wait the tile is still loaded (whatever the rows hold) so its MMA
                // and epilogue complete; the error is reported and the next fetch ends the loop.
                if (!wait_landed(a.landed + e * a.max_mtiles + mt, tile_rows(sh, e, mt), a.st, t)) ok = false;
                fence_proxy_async_global();  // rows landed by other CTAs' bulk stores -> this thread's TMA reads
                const int a_row = sh.off[e] + mt * kBM, b_row = e * a.n + nt * kBN;
                bool loaded = true;
                for (int kb = 0; kb < KB; ++kb, ++g) {
                    const int s = g % kGemmStages;
                    if (!mbar_wait(&s_empty[s], ((g / kGemmStages) & 1) ^ 1, a.st, kErrTimeoutTma)) {
                        loaded = false;  // the MMA warp has stopped: its own waits expired
                        break;
                    }
                    uint8_t* sa_tile = smem + (size_t)s * kStageBytes;
                    mbar_arrive_expect_tx(&s_full[s], kStageBytes);
                    tc::tma_load_2d(sa_tile, map_a, kb * kBK, a_row, &s_full[s]);
                    tc::tma_load_2d(sa_tile + kBM * kBK, map_b, kb * kBK, b_row, &s_full[s]);
                }
                if (!loaded) {
                    ring_drain(s_full, kGemmStages, (int)g, a.st, kErrTimeoutTma);  // issued loads land first
                    break;
                }
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_e4m3_f32(kBM, kBN);
            uint32_t g = 0;
            bool ok = true;
            for (int q = 0; ok; ++q) {
                const int slot = q % kTileQ;
                if (!mbar_wait(&s_qfull[slot], (q / kTileQ) & 1, st_q, kErrTimeoutTma)) break;
                const int t = sh.tq[slot];
                mbar_arrive(&s_qempty[slot]);
                if (t < 0) break;
                for (int kb = 0; kb < KB && ok; ++kb, ++g) {
                    const int s = g % kGemmStages, b = g & 1;
                    ok = mbar_wait(&s_tempty[b], ((g >> 1) & 1) ^ 1, a.st, kErrTimeoutTma) &&
                         mbar_wait(&s_full[s], (g / kGemmStages) & 1, a.st, kErrTimeoutTma);
                    if (!ok) break;
                    tc::fence_after();
                    const uint32_t sa_addr = smem_u32(smem + (size_t)s * kStageBytes);
                    const uint64_t da = tc::smem_desc_sw128(sa_addr), db = tc::smem_desc_sw128(sa_addr + kBM * kBK);
                    const uint32_t d_tmem = tmem_base + (uint32_t)(b * kBN);
#pragma unroll
                    for (int k = 0; k < kBK / 32; ++k)
                        mma_f8(d_tmem, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc, k > 0 ? 1u : 0u);
                    tc::mma_commit(&s_empty[s]);
                    tc::mma_commit(&s_tfull[b]);
                }
            }
            // After an expired wait: issued MMAs complete before the TMEM is freed.
            if (!ok && g > 0)
                mbar_wait(&s_empty[(g - 1) % kGemmStages], ((g - 1) / kGemmStages) & 1, a.st, kErrTimeoutTma);
        }
    } else {
        // ---------------------------------------------------------------- epilogue / scale promotion
        const int ew = warp - 2;
        const int qd = warp & 3;  // TMEM lane quarter
        const int h = ew >> 2;    // column half
        const int r_in = 32 * qd + lane;
        const int nb = a.layout.hidden / 128;
        uint32_t g = 0;
        bool ok = true;
        for (int q = 0; ok; ++q) {
            const int slot = q % kTileQ;
            int t = -1;
            if (lane == 0) t = mbar_wait(&s_qfull[slot], (q / kTileQ) & 1, st_q, kErrTimeoutTma) ? sh.tq[slot] : -2;
            t = __shfl_sync(0xffffffffu, t, 0);
            if (t == -2) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_qempty[slot]);
            int mt, e, nt;
            if (t < 0 || !fused_gemm_tile(t, n_tiles, sh.level, levels, sh.order, mt, e, nt)) break;
            const int rows = tile_rows(sh, e, mt);
            // The tile's rows and scales were stored by pull CTAs, and the producer may not have
            // seen them land yet: acquire the landed counter before reading the scales. After an
            // expired wait the tile still completes, as in the producer.
            if (lane == 0) wait_landed(a.landed + e * a.max_mtiles + mt, rows, a.st, t);
            __syncwarp();
            const int m = sh.off[e] + mt * kBM + r_in;
            const float* sa_row = a.sa + (int64_t)m * nb;
            const float* sb_blk = a.sb + ((int64_t)e * (a.n / 128) + nt) * KB;
            float acc[64];
#pragma unroll
            for (int i = 0; i < 64; ++i) acc[i] = 0.f;
            // the scales of K block kb + 1 load while block kb is waited for and promoted
            float pa = r_in < rows ? sa_row[0] : 0.f, pb = sb_blk[0];
            for (int kb = 0; kb < KB; ++kb, ++g) {
                const int b = g & 1;
                const float scale = pa * pb;
                if (kb + 1 < KB) {
                    pa = r_in < rows ? sa_row[kb + 1] : 0.f;
                    pb = sb_blk[kb + 1];
                }
                int good = 1;
                if (lane == 0) good = mbar_wait(&s_tfull[b], (g >> 1) & 1, a.st, kErrTimeoutTma) ? 1 : 0;
                if (!__shfl_sync(0xffffffffu, good, 0)) {
                    ok = false;
                    break;
                }
                tc::fence_after();
                float v[64];
                const uint32_t taddr = tmem_base + ((uint32_t)(32 * qd) << 16) + (uint32_t)(b * kBN + 64 * h);
                tc::tmem_ld_32(taddr, v);
                tc::tmem_ld_32(taddr + 32, v + 32);
                tc::tmem_wait_ld();
                tc::fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&s_tempty[b]);
#pragma unroll
                for (int i = 0; i < 64; ++i) acc[i] = fmaf(scale, v[i], acc[i]);
            }
            if (!ok) break;
            if (r_in < rows) {
                __nv_bfloat16* d = static_cast<__nv_bfloat16*>(a.d) + (int64_t)m * a.n + nt * kBN + 64 * h;
#pragma unroll
                for (int c = 0; c < 64; c += 8) {
                    int4 o;
                    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
                    for (int i = 0; i < 4; ++i) o2[i] = __floats2bfloat162_rn(acc[c + 2 * i], acc[c + 2 * i + 1]);
                    *reinterpret_cast<int4*>(d + c) = o;
                }
            }
        }
    }
    tc::fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols) : "memory");
    }
}

}  // namespace

__global__ void __launch_bounds__(kThreads, 1) fused_dispatch_gemm_kernel(const __grid_constant__ CUtensorMap map_a,
                                                                        const __grid_constant__ CUtensorMap map_b,
                                                                        FusedDispatchGemmArgs a, int pull_stages) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ FusedShared sh;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const int E_l = a.num_local_experts;
    if (threadIdx.x == 0) {
        int acc = 0;
        int* m_tiles = reinterpret_cast<int*>(smem);  // scratch until the rings start
        int* hist = m_tiles + kMaxLocalExperts;
        for (int e = 0; e < E_l; ++e) {
            sh.off[e] = acc;
            acc += a.num_recv_per_expert[e];  // 128-aligned counts from the notify step
            sh.cnt[e] = a.raw_counts[e];
            m_tiles[e] = (sh.cnt[e] + kBM - 1) / kBM;
        }
        sh.off[E_l] = acc;
        sh.levels = fused_gemm_levels(m_tiles, E_l, sh.order, sh.level, min(a.max_mtiles, kMaxLevels), hist);
        if (sh.levels < 0 || acc > a.rows_cap) {
            report_error(a.st, kErrCapacity, -1, acc);
            sh.levels = -1;
        }
        sh.prefix[0] = 0;
        for (int s = 0; s < a.num_ranks; ++s) sh.prefix[s + 1] = a.rank_prefix_matrix[s * a.num_ranks + a.rank];
    }
    __syncthreads();
    if ((int)blockIdx.x < a.pull_ctas) {
        if (sh.levels >= 0) pull_role(a, sh, smem, pull_stages);
        __syncthreads();  // the ring's shared memory becomes GEMM stages
    }
    gemm_role(&map_a, &map_b, a, sh, smem);
}

int launch_fused_dispatch_gemm(const FusedDispatchGemmArgs& a, int num_sms, cudaStream_t stream) {
    const int H = a.layout.hidden;
    if (H % kBK != 0 || a.n % kBN != 0 || a.num_local_experts <= 0 || a.num_local_experts > kMaxLocalExperts ||
        a.max_mtiles <= 0 || a.max_mtiles > kMaxLevels || a.pull_ctas <= 0 || a.pull_ctas > num_sms ||
        a.num_topk > kMaxTopk || a.rec.x_bytes != H || (H / 128 * 4) % 16 != 0 || a.rows_cap <= 0)
        return 1;
    CUtensorMap map_a, map_b;
    if (!tc::make_map_2d(&map_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.a, (uint64_t)a.rows_cap, (uint64_t)H, 128)) return 2;
    if (!tc::make_map_2d(&map_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.b, (uint64_t)a.num_local_experts * a.n, (uint64_t)H, 128))
        return 2;
    const int slot_bytes = (a.rec.bytes + 127) / 128 * 128;
    const size_t gemm_bytes = (size_t)kGemmStages * kStageBytes;
    int pull_stages = 8;
    while (pull_stages > kLag + 1 && (size_t)kPullPairs * pull_pair_bytes(pull_stages, slot_bytes) > gemm_bytes) --pull_stages;
    const size_t pull_bytes = (size_t)kPullPairs * pull_pair_bytes(pull_stages, slot_bytes);
    if (pull_stages <= kLag || pull_bytes > gemm_bytes) return 1;
    // The setup scratch (m-tile counts and a histogram) also lives in the dynamic region.
    const size_t smem = gemm_bytes + 1024;
    cudaFuncSetAttribute(fused_dispatch_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    fused_dispatch_gemm_kernel<<<num_sms, kThreads, smem, stream>>>(map_a, map_b, a, pull_stages);
    return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

}  // namespace ep
