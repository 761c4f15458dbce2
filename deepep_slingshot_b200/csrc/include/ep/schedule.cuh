// Row schedules of the pipelined dispatch-pull and combine-push kernels (host + device, so the host
// model tests exercise the exact functions the kernels run).
#pragma once

#include <cuda_runtime.h>

namespace ep {

__host__ __device__ __forceinline__ int sched_min(int a, int b) { return a < b ? a : b; }

// Rows are dealt to pairs in chunks of `chunk`: pair g owns chunks g, g + P, g + 2P, ... so every
// pair sees rows of every source/destination rank (receive rows are sorted by rank).
// chunk == 0 deals contiguous ranges instead (pair g owns rows [g*per, (g+1)*per)).
__host__ __device__ __forceinline__ int pair_row(int g, int P, int k, int chunk, int n) {
    if (chunk == 0) return g * ((n + P - 1) / P) + k;
    return ((k / chunk) * P + g) * chunk + (k % chunk);
}

// Combine push order with chunk == -1 ("wavefront"): at step k pair g serves destination
// s = (k + g) % R, row (k / R) * P + g of that destination's segment (-1 past its end). Every pair
// spreads its stores over all destinations (no incast), and all ranks walk each destination's tokens
// in increasing order at the same pace, so a token's contributions from every source land close
// together and the reducers (which take tokens in increasing order) follow the pushes instead of
// waiting for the end of the push phase.
__host__ __device__ __forceinline__ int wave_row(int g, int P, int k, const int* prefix, int R, int n) {
    const int s = (k + g) % R;
    const int i = (k / R) * P + g;
    const int lo = sched_min(prefix[s], n), hi = sched_min(prefix[s + 1], n);
    return i < hi - lo ? lo + i : -1;
}
__host__ __device__ __forceinline__ int wave_num_rows(int g, int P, const int* prefix, int R, int n) {
    int rows = 0;
    for (int s = 0; s < R; ++s) {
        const int len = sched_min(prefix[s + 1], n) - sched_min(prefix[s], n);
        if (len > g) rows += (len - g + P - 1) / P;
    }
    return rows;
}
__host__ __device__ __forceinline__ int pair_num_rows(int g, int P, int n, int chunk) {
    if (chunk == 0) {
        const int per = (n + P - 1) / P;
        const int r0 = sched_min(n, g * per);
        return sched_min(n, r0 + per) - r0;
    }
    const int full_chunks = n / chunk, rem = n % chunk;
    int c = full_chunks > g ? (full_chunks - g + P - 1) / P : 0;
    int rows = c * chunk;
    if (rem > 0 && full_chunks % P == g) rows += rem;  // the trailing partial chunk
    return rows;
}

// Contiguous row range of pair `g` out of `total_pairs` for `n` rows.
__host__ __device__ __forceinline__ void pair_range(int n, int g, int total_pairs, int& r0, int& r1) {
    const int per = (n + total_pairs - 1) / total_pairs;
    r0 = sched_min(n, g * per);
    r1 = sched_min(n, r0 + per);
}

// Source rank of receive row j (rows sorted by source; prefix[s] = first row of source s).
__host__ __device__ __forceinline__ int find_source(const int* prefix, int R, int j) {
    int s = 0;
    while (s + 1 < R && j >= prefix[s + 1]) ++s;
    return s;
}

// Pipeline ring direction of `other` seen from `me`: 0 when `other` is my previous rank, else 1.
// With two ranks (or one) the neighbour is both and the index is 0 on both sides.
__host__ __device__ __forceinline__ int ring_dir(int me, int other, int num_ranks) {
    return other == (me + num_ranks - 1) % num_ranks ? 0 : 1;
}

// Tile order of the masked grouped GEMM: (m-tile, expert, n-tile), n-tile innermost. A grid of G
// persistent CTAs takes tiles c, c + G, ...; the first E * n_tiles tiles are every expert's first
// m-tile, so a decode batch (at most one m-tile per expert) spreads evenly over the CTAs.
// Returns false past the last potential tile.
__host__ __device__ __forceinline__ bool masked_gemm_tile(int t, int E, int n_tiles, int m_tiles, int& mt, int& e, int& nt) {
    const int per_mt = E * n_tiles;
    if (t < 0 || t >= per_mt * m_tiles) return false;
    mt = t / per_mt;
    const int r = t - mt * per_mt;
    e = r / n_tiles;
    nt = r - e * n_tiles;
    return true;
}

// Tile order of the fused dispatch -> grouped GEMM: level-major, where level l holds the l-th m-tile
// of every expert that has more than l m-tiles, n-tile innermost. The receive side fills each
// expert's rows in claim order, so an expert's tile l completes before its tile l + 1 and the
// level-0 tiles of all experts complete first; taking tiles in level order follows the arrivals.
// `fused_gemm_levels` sorts experts by decreasing m-tile count (counting sort) so each level's
// experts are a prefix of `order`, and writes level_prefix[l] = tiles (in units of n-tile rows)
// before level l, for l = 0..levels. `hist` needs max_levels + 1 ints. Returns the number of
// levels (the largest m-tile count), or -1 if it exceeds max_levels.
__host__ __device__ __forceinline__ int fused_gemm_levels(const int* m_tiles, int E, int* order, int* level_prefix,
                                                          int max_levels, int* hist) {
    int levels = 0;
    for (int v = 0; v <= max_levels; ++v) hist[v] = 0;
    for (int e = 0; e < E; ++e) {
        const int v = m_tiles[e];
        if (v > max_levels) return -1;
        ++hist[v];
        if (v > levels) levels = v;
    }
    // Descending order: experts with value v start after all experts with a larger value.
    int above = 0;  // experts with m_tiles > v
    for (int v = max_levels; v >= 0; --v) {
        const int c = hist[v];
        hist[v] = above;  // first position of value v
        above += c;
    }
    for (int e = 0; e < E; ++e) order[hist[m_tiles[e]]++] = e;
    // After the placement hist[v] = first position of value v + its count = experts with m_tiles >= v.
    level_prefix[0] = 0;
    for (int l = 0; l < levels; ++l) level_prefix[l + 1] = level_prefix[l] + hist[l + 1];
    return levels;
}

// Tile t of the fused order: (level mt, expert e, n-tile nt); false past the last tile.
__host__ __device__ __forceinline__ bool fused_gemm_tile(int t, int n_tiles, const int* level_prefix, int levels,
                                                         const int* order, int& mt, int& e, int& nt) {
    if (t < 0 || levels <= 0) return false;
    const int r = t / n_tiles;
    if (r >= level_prefix[levels]) return false;
    int lo = 0, hi = levels - 1;  // largest level with level_prefix[level] <= r
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (level_prefix[mid] <= r) lo = mid;
        else hi = mid - 1;
    }
    mt = lo;
    e = order[r - level_prefix[lo]];
    nt = t - r * n_tiles;
    return true;
}

}  // namespace ep
