// Host models of device-side logic (no GPU needed; compiled by nvcc for the host).
//
// The scheduling and LogFMT helpers below are the same __host__ __device__ functions the kernels
// call (csrc/include/ep/schedule.cuh, logfmt.cuh), so these checks exercise the production code:
//   1. row dealing of the pull / push pipelines covers every row exactly once and every loop ends;
//   2. the pipeline-ring credit protocol (counters, slots, ring directions) delivers every message in
//      order, never overwrites an unconsumed slot and never deadlocks, under random interleavings;
//   3. LogFMT-10 packing round-trips and the code -> value mapping stays within its error bound;
//   4. the masked grouped GEMM's tile order covers every tile once and balances decode batches;
//   5. the fused dispatch -> GEMM tile order covers every live tile once, level by level;
//   6. the down projection -> combine index rules (csrc/include/ep/gemm_combine.cuh): over random
//      routings of 1..8 ranks, every expert row lands in exactly one slot of its token's source rank,
//      and the source's reduction over its own routing equals the direct top-k weighted sum.
// Prints "ALL OK" and exits 0 on success.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <deque>
#include <random>
#include <vector>

#include "../../deepep_slingshot_b200/csrc/include/ep/gemm_combine.cuh"
#include "../../deepep_slingshot_b200/csrc/include/ep/logfmt.cuh"
#include "../../deepep_slingshot_b200/csrc/include/ep/schedule.cuh"

#define CHECK(cond, ...)                                   \
    do {                                                   \
        if (!(cond)) {                                     \
            std::printf("FAILED %s:%d: ", __FILE__, __LINE__); \
            std::printf(__VA_ARGS__);                      \
            std::printf("\n");                             \
            std::exit(1);                                  \
        }                                                  \
    } while (0)

static void check_dealing(std::mt19937& rng) {
    for (int trial = 0; trial < 4000; ++trial) {
        const int R = 1 + rng() % 8;
        const int P = std::vector<int>{1, 2, 4, 16, 128, 296}[rng() % 6];
        std::vector<int> prefix(R + 1, 0);
        for (int s = 0; s < R; ++s) {
            const int kind = rng() % 4;
            const int len = kind == 0 ? 0 : kind == 1 ? 1 + rng() % 5 : rng() % 3000;
            prefix[s + 1] = prefix[s] + len;
        }
        const int n = (rng() % 4 == 0) ? (int)(rng() % (prefix[R] + 1)) : prefix[R];
        // wavefront (combine push)
        std::vector<int> owner(n, -1);
        for (int g = 0; g < P; ++g) {
            const int rows = ep::wave_num_rows(g, P, prefix.data(), R, n);
            int c = 0;
            for (int k = 0; c < rows; ++k) {
                CHECK(k < 100000000, "wave loop does not end (g=%d)", g);
                const int j = ep::wave_row(g, P, k, prefix.data(), R, n);
                if (j < 0) continue;
                CHECK(j < n && owner[j] == -1, "wave row %d dealt twice", j);
                owner[j] = g;
                ++c;
            }
        }
        for (int j = 0; j < n; ++j) CHECK(owner[j] >= 0, "wave row %d never dealt (R=%d P=%d)", j, R, P);
        // chunked / contiguous (pull, combine with chunk >= 0)
        for (int chunk : {0, 1, 8, 33}) {
            std::vector<int> seen(n, 0);
            for (int g = 0; g < P; ++g) {
                const int rows = ep::pair_num_rows(g, P, n, chunk);
                for (int k = 0; k < rows; ++k) {
                    const int j = ep::pair_row(g, P, k, chunk, n);
                    CHECK(j >= 0 && j < n, "pair_row out of range (chunk %d)", chunk);
                    seen[j]++;
                }
            }
            for (int j = 0; j < n; ++j) CHECK(seen[j] == 1, "chunk %d: row %d dealt %d times", chunk, j, seen[j]);
        }
        for (int j = 0; j < prefix[R]; ++j) {
            const int s = ep::find_source(prefix.data(), R, j);
            CHECK(prefix[s] <= j && j < prefix[s + 1], "find_source(%d) = %d", j, s);
        }
    }
    std::printf("dealing ok\n");
}

// Pipeline ring: the counters and credit rule of pp_copy_kernel, the slot sets chosen with
// ring_dir as in SymmetricRegion::pp_send / pp_recv.
struct RankState {
    int send_count[2] = {0, 0}, recv_count[2] = {0, 0};
    int arrival[2] = {0, 0}, release[2] = {0, 0};
    std::vector<long> slots[2];  // message id per slot, -1 = free
};

static void check_pp_ring(std::mt19937& rng) {
    for (int trial = 0; trial < 3000; ++trial) {
        const int R = 1 + rng() % 8, msgs = 1 + rng() % 12;
        // With one or two ranks both neighbours are the same rank and share one slot ring, so the two
        // sends of an iteration need two slots (fewer would block the stream, as on the GPU).
        const int inflight = (R <= 2 ? 2 : 1) + rng() % 3;
        std::vector<RankState> st(R);
        for (auto& s : st)
            for (int d = 0; d < 2; ++d) s.slots[d].assign(inflight, -1);
        // program per rank: per message: send next, send prev, recv prev, recv next (stream order)
        struct Op { int kind, peer; };  // kind 0 send, 1 recv
        std::vector<std::vector<Op>> prog(R);
        for (int r = 0; r < R; ++r) {
            const int prev = (r + R - 1) % R, next = (r + 1) % R;
            for (int m = 0; m < msgs; ++m) {
                prog[r].push_back({0, next});
                prog[r].push_back({0, prev});
                prog[r].push_back({1, prev});
                prog[r].push_back({1, next});
            }
        }
        // sent[src][dst] = FIFO of message ids in flight from src to dst (per slot set)
        std::vector<std::vector<std::deque<long>>> fifo(R, std::vector<std::deque<long>>(R));
        std::vector<size_t> pc(R, 0);
        long next_id = 0;
        int idle = 0;
        while (true) {
            bool all_done = true;
            for (int r = 0; r < R; ++r) all_done &= pc[r] == prog[r].size();
            if (all_done) break;
            const int r = rng() % R;
            if (pc[r] == prog[r].size()) continue;
            const Op op = prog[r][pc[r]];
            bool progressed = false;
            if (op.kind == 0) {
                const int dst = op.peer, ds = ep::ring_dir(r, dst, R), dr = ep::ring_dir(dst, r, R);
                const int c = st[r].send_count[ds];
                if (st[r].release[ds] - (c + 1 - inflight) >= 0) {  // credit rule of the kernel
                    long& slot = st[dst].slots[dr][(unsigned)c % (unsigned)inflight];
                    CHECK(slot == -1, "send %d->%d overwrites an unconsumed slot", r, dst);
                    slot = next_id;
                    fifo[r][dst].push_back(next_id++);
                    st[dst].arrival[dr] += 1;
                    st[r].send_count[ds] = c + 1;
                    progressed = true;
                }
            } else {
                const int src = op.peer, dr = ep::ring_dir(r, src, R), ds = ep::ring_dir(src, r, R);
                const int c = st[r].recv_count[dr];
                if (st[r].arrival[dr] - (c + 1) >= 0) {
                    long& slot = st[r].slots[dr][(unsigned)c % (unsigned)inflight];
                    CHECK(slot != -1, "recv %d<-%d reads an empty slot", r, src);
                    // with two ranks both neighbours are one rank: the slot set is shared, FIFO per pair
                    CHECK(!fifo[src][r].empty() && fifo[src][r].front() == slot, "recv %d<-%d out of order", r, src);
                    fifo[src][r].pop_front();
                    slot = -1;
                    st[src].release[ds] += 1;
                    st[r].recv_count[dr] = c + 1;
                    progressed = true;
                }
            }
            if (progressed) {
                ++pc[r];
                idle = 0;
            } else {
                CHECK(++idle < 100000, "pipeline ring deadlock (R=%d inflight=%d)", R, inflight);
            }
        }
        for (int a = 0; a < R; ++a)
            for (int b = 0; b < R; ++b) CHECK(fifo[a][b].empty(), "undelivered messages %d->%d", a, b);
    }
    std::printf("pipeline ring ok\n");
}

static void check_logfmt(std::mt19937& rng) {
    // packing round trip
    for (int trial = 0; trial < 20000; ++trial) {
        uint32_t c[8], out[8];
        uint8_t bytes[10];
        for (int i = 0; i < 8; ++i) c[i] = rng() & 0x3ffu;
        ep::logfmt_pack4(c, bytes);
        ep::logfmt_pack4(c + 4, bytes + 5);
        uint16_t words[5];
        for (int i = 0; i < 5; ++i) words[i] = (uint16_t)(bytes[2 * i] | (bytes[2 * i + 1] << 8));
        ep::logfmt_unpack8(words, out);
        for (int i = 0; i < 8; ++i) CHECK(out[i] == c[i], "pack/unpack code %d: %u != %u", i, out[i], c[i]);
    }
    // code -> value: nearest level in linear space, within one step of relative error
    std::uniform_real_distribution<float> u(0.f, 1.f);
    for (int trial = 0; trial < 2000; ++trial) {
        const float amax = std::ldexp(0.5f + 0.5f * u(rng), -(int)(rng() % 20));  // below 1
        const float amin = amax * std::ldexp(u(rng) + 1e-3f, -(int)(rng() % 40));
        const ep::LogFmtGroup p = ep::logfmt_params(amax, amin);
        if (!p.cast) continue;
        const float inv = 1.0f / p.step;
        const float up = log2f((1.0f + exp2f(p.step)) * 0.5f) * inv;
        uint32_t last = 0;
        for (int i = 0; i <= 200; ++i) {
            const float v = amin + (amax - amin) * (float)i / 200.f;
            const uint32_t code = ep::logfmt_code(v, p, inv, up);
            CHECK((code >> 9) == 0, "positive value got a sign bit");
            CHECK((code & 511u) >= (last & 511u), "codes not monotonic");
            last = code;
            const float back = ep::logfmt_value(code, p);
            if (v >= exp2f(p.log_amin)) {  // values below the clamped range flush towards zero by design
                const float rel = std::fabs(back - v) / v;
                CHECK(rel <= exp2f(p.step) - 1.f + 1e-5f, "relative error %g above the level spacing", rel);
            }
            const uint32_t neg = ep::logfmt_code(-v, p, inv, up);
            CHECK(neg == (code | (v != 0.f ? 512u : 0u)) || (v == 0.f && neg == 512u), "sign handling");
        }
        CHECK(ep::logfmt_code(0.f, p, inv, up) == 0 && ep::logfmt_value(0, p) == 0.f, "zero encodes to code 0");
    }
    std::printf("logfmt ok\n");
}

// Masked grouped GEMM tile order: every potential tile is visited exactly once over the grid, the
// live tiles (m0 < count) are exactly those the roles compute, and a decode batch (count <= 128 per
// expert) gives every CTA floor or ceil of its share of live tiles.
static void check_masked_tiles(std::mt19937& rng) {
    for (int trial = 0; trial < 3000; ++trial) {
        const int E = 1 + rng() % 64, n_tiles = 1 + rng() % 64, slots = 1 + rng() % 2048;
        const int m_tiles = (slots + 127) / 128;
        const int G = std::vector<int>{1, 7, 148, 296}[rng() % 4];
        const bool decode = rng() % 2 == 0;
        std::vector<int> count(E);
        for (int e = 0; e < E; ++e) count[e] = decode ? rng() % 129 : rng() % (slots + 1);
        std::vector<int> seen((size_t)E * n_tiles * m_tiles, 0);
        int live_min = 1 << 30, live_max = 0;
        for (int c = 0; c < G; ++c) {
            int live = 0;
            int mt, e, nt;
            for (int t = c; ep::masked_gemm_tile(t, E, n_tiles, m_tiles, mt, e, nt); t += G) {
                CHECK(mt >= 0 && mt < m_tiles && e >= 0 && e < E && nt >= 0 && nt < n_tiles, "tile %d out of range", t);
                ++seen[((size_t)mt * E + e) * n_tiles + nt];
                if (mt * 128 < count[e]) ++live;
            }
            live_min = std::min(live_min, live);
            live_max = std::max(live_max, live);
        }
        for (size_t i = 0; i < seen.size(); ++i) CHECK(seen[i] == 1, "tile %zu visited %d times", i, seen[i]);
        int mt, e, nt;
        CHECK(!ep::masked_gemm_tile(E * n_tiles * m_tiles, E, n_tiles, m_tiles, mt, e, nt), "tile past the end accepted");
        if (decode) {
            bool all_nonempty = true;
            for (int x = 0; x < E; ++x) all_nonempty &= count[x] > 0;
            if (all_nonempty) CHECK(live_max - live_min <= 1, "decode imbalance %d..%d (E=%d NT=%d G=%d)", live_min, live_max, E, n_tiles, G);
        }
    }
}

// Fused dispatch -> GEMM tile order: every (expert, m-tile, n-tile) with m-tile < the expert's count
// appears exactly once, levels come in order, and each level lists experts with that many tiles.
static void check_fused_tiles(std::mt19937& rng) {
    for (int trial = 0; trial < 3000; ++trial) {
        const int E = 1 + rng() % 300, n_tiles = 1 + rng() % 40, max_levels = 1 + rng() % 64;
        std::vector<int> mt(E), order(E, -1), prefix(max_levels + 1, 0), hist(max_levels + 1);
        for (int e = 0; e < E; ++e) mt[e] = rng() % 3 == 0 ? 0 : (int)(rng() % (max_levels + 1));
        const int levels = ep::fused_gemm_levels(mt.data(), E, order.data(), prefix.data(), max_levels, hist.data());
        int want = 0;
        for (int e = 0; e < E; ++e) want = std::max(want, mt[e]);
        CHECK(levels == want, "levels %d != %d", levels, want);
        std::vector<int> pos(E, 0);
        for (int i = 0; i < E; ++i) {
            CHECK(order[i] >= 0 && order[i] < E && ++pos[order[i]] == 1, "order is not a permutation");
            if (i) CHECK(mt[order[i - 1]] >= mt[order[i]], "order not descending");
        }
        std::vector<int> seen((size_t)E * (max_levels + 1) * n_tiles, 0);
        int total = 0, last_level = 0;
        int l, e, nt;
        for (int t = 0; ep::fused_gemm_tile(t, n_tiles, prefix.data(), levels, order.data(), l, e, nt); ++t) {
            CHECK(l < mt[e] && nt >= 0 && nt < n_tiles, "invalid tile %d (l=%d e=%d mt=%d)", t, l, e, mt[e]);
            CHECK(l >= last_level, "levels out of order");
            last_level = l;
            CHECK(++seen[((size_t)e * (max_levels + 1) + l) * n_tiles + nt] == 1, "tile visited twice");
            ++total;
        }
        int expect = 0;
        for (int x = 0; x < E; ++x) expect += mt[x] * n_tiles;
        CHECK(total == expect, "%d tiles visited, expected %d", total, expect);
    }
    int hist[4], order[2], prefix[4];
    const int too_many[2] = {5, 1};
    CHECK(ep::fused_gemm_levels(too_many, 2, order, prefix, 3, hist) == -1, "overflow not reported");
}

// Down projection -> combine. Dispatch semantics as the library's: receiver r gets, in source-rank
// order and token order, every token with at least one expert on r; its routing row keeps the k
// positions (local expert id, -1 elsewhere); the permute gives each (received token, k) with a local
// expert one operand row of that expert's 128-aligned block. The receiver's GEMM output for a row is
// modelled by a value that names (source, token, global expert); the row goes to the slot that the
// same destination-word rule as the row-destination kernel gives.
static double expert_value(int s, int t, int e) { return 1000.0 * s + t + 0.001 * e; }

static void check_gemm_combine(std::mt19937& rng) {
    for (int trial = 0; trial < 1500; ++trial) {
        const int R = 1 + rng() % 8, E_l = 1 + rng() % 6, E = R * E_l, K = 1 + rng() % std::min(8, E);
        std::vector<int> N(R);
        std::vector<std::vector<int>> topk(R);      // [t * K + k] global expert or -1
        std::vector<std::vector<double>> w(R);
        for (int s = 0; s < R; ++s) {
            N[s] = rng() % 4 == 0 ? 0 : (int)(rng() % 40);
            topk[s].assign((size_t)N[s] * K, -1);
            w[s].resize((size_t)N[s] * K);
            for (int t = 0; t < N[s]; ++t) {
                std::vector<int> perm(E);
                for (int e = 0; e < E; ++e) perm[e] = e;
                std::shuffle(perm.begin(), perm.end(), rng);
                for (int k = 0; k < K; ++k) {
                    topk[s][(size_t)t * K + k] = rng() % 5 == 0 ? -1 : perm[k];
                    w[s][(size_t)t * K + k] = (double)(rng() % 1000) / 997.0;
                }
            }
        }
        // send[s][r] = tokens s sends to r; rank_prefix_matrix[s][r] = sum over s' <= s
        std::vector<int> rpm((size_t)R * R, 0);
        for (int r = 0; r < R; ++r) {
            int acc = 0;
            for (int s = 0; s < R; ++s) {
                for (int t = 0; t < N[s]; ++t) {
                    bool to_r = false;
                    for (int k = 0; k < K; ++k) to_r |= topk[s][(size_t)t * K + k] >= 0 && topk[s][(size_t)t * K + k] / E_l == r;
                    acc += to_r;
                }
                rpm[(size_t)s * R + r] = acc;
            }
        }
        std::vector<std::vector<double>> slots(R);
        std::vector<std::vector<int>> written(R);
        for (int s = 0; s < R; ++s) {
            slots[s].assign((size_t)N[s] * K, 0.0);
            written[s].assign((size_t)N[s] * K, 0);
        }
        for (int r = 0; r < R; ++r) {
            std::vector<int> src_idx, recv_topk;  // received tokens
            for (int s = 0; s < R; ++s)
                for (int t = 0; t < N[s]; ++t) {
                    bool to_r = false;
                    for (int k = 0; k < K; ++k) to_r |= topk[s][(size_t)t * K + k] >= 0 && topk[s][(size_t)t * K + k] / E_l == r;
                    if (!to_r) continue;
                    src_idx.push_back(t);
                    for (int k = 0; k < K; ++k) {
                        const int e = topk[s][(size_t)t * K + k];
                        recv_topk.push_back(e >= 0 && e / E_l == r ? e % E_l : -1);
                    }
                }
            const int num_recv = (int)src_idx.size();
            CHECK(num_recv == rpm[(size_t)(R - 1) * R + r], "receive count");
            // permute: 128-aligned blocks per local expert, rows in (token, k) order
            std::vector<int> count(E_l, 0), offset(E_l + 1, 0);
            for (int x : recv_topk)
                if (x >= 0) ++count[x];
            for (int e = 0; e < E_l; ++e) offset[e + 1] = offset[e] + (count[e] + 127) / 128 * 128;
            const int rows = std::max(offset[E_l], 1);
            std::vector<int> row_map((size_t)num_recv * K, -1), fill(E_l, 0);
            for (int j = 0; j < num_recv; ++j)
                for (int k = 0; k < K; ++k) {
                    const int e = recv_topk[(size_t)j * K + k];
                    if (e >= 0) row_map[(size_t)j * K + k] = offset[e] + fill[e]++;
                }
            // destination words (the row-destination kernel's rule) and the GEMM's rows
            std::vector<int> prefix(R + 1, 0);
            for (int s = 0; s < R; ++s) prefix[s + 1] = rpm[(size_t)s * R + r];
            std::vector<int> dest(rows, -1);
            std::vector<double> y(rows, 0.0);
            for (int j = 0; j < num_recv; ++j)
                for (int k = 0; k < K; ++k) {
                    const int row = row_map[(size_t)j * K + k];
                    if (row < 0) continue;
                    const int s = ep::gc_source_of(prefix.data(), R, j);
                    const int t = src_idx[j];
                    dest[row] = ep::gc_encode(s, t, k, K);
                    y[row] = expert_value(s, t, r * E_l + recv_topk[(size_t)j * K + k]);
                }
            // the epilogue: rows with a destination go to that slot, padding rows nowhere
            for (int row = 0; row < rows; ++row) {
                if (dest[row] < 0) continue;
                const int s = ep::gc_rank_of(dest[row]), slot = ep::gc_slot_of(dest[row]);
                CHECK(s >= 0 && s < R && slot >= 0 && slot < N[s] * K, "destination out of range");
                CHECK(++written[s][slot] == 1, "slot written twice");
                slots[s][slot] = y[row];
            }
        }
        // source reduction over its own routing == direct top-k weighted sum
        for (int s = 0; s < R; ++s)
            for (int t = 0; t < N[s]; ++t) {
                double got = 0.0, want = 0.0;
                for (int k = 0; k < K; ++k) {
                    const int e = topk[s][(size_t)t * K + k];
                    const bool valid = e >= 0;
                    CHECK(written[s][(size_t)t * K + k] == (valid ? 1 : 0), "slot (%d, %d) of rank %d written %d times",
                          t, k, s, written[s][(size_t)t * K + k]);
                    if (!valid) continue;
                    got += w[s][(size_t)t * K + k] * slots[s][(size_t)t * K + k];
                    want += w[s][(size_t)t * K + k] * expert_value(s, t, e);
                }
                CHECK(std::fabs(got - want) <= 1e-9 * (1.0 + std::fabs(want)), "reduction mismatch");
            }
    }
    CHECK(ep::gc_rank_of(ep::gc_encode(7, (1 << 21) - 1, 7, 8)) == 7 && ep::gc_slot_of(ep::gc_encode(7, (1 << 21) - 1, 7, 8)) == (1 << 24) - 1,
          "largest destination word");
}

int main() {
    std::mt19937 rng(12345);
    check_dealing(rng);
    check_masked_tiles(rng);
    check_fused_tiles(rng);
    check_gemm_combine(rng);
    check_pp_ring(rng);
    check_logfmt(rng);
    std::printf("ALL OK\n");
    return 0;
}
