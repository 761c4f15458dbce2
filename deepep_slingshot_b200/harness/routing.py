"""Routing tables for the EP benchmark with exactly controlled traffic.

`skew_routes` (the reference's receiver-skew calibration, backend/tests/routing.py:12-42, written
anew): every token goes to exactly two distinct destination ranks with `topk / 2` experts on each,
so the rows a rank receives are fixed by construction. Rank 0 receives `skew` times the mean; the
others share the remainder evenly. Total assignments and transmitted rows do not change with the
skew, unlike top-k of random logits. Two-destination pairs come from splitting the sorted multiset
of destinations in half (no destination fills more than half of it, so the halves never agree at
the same position).

Other routings: `uniform` (top-k of uniform logits), `hot_rank` (every token on rank 0's first
experts: the other ranks receive nothing), `self` (every token stays on its own rank: no NVLink
traffic), `remote` (two destinations, never the source rank).

Count-driven routings (the reference replays per-expert counts of real traces,
backend/tests/bank_routing.py:25-61; the trace data itself is not part of this library):
`routes_from_counts` realises exact per-expert counts as a top-k table with distinct experts per
token, `greedy_placement` / `random_placement` map logical experts to physical ids. Names:
`zipf<s>[_greedy|_random]` (Zipf(s) expert popularity per rank), `counts:<file.npy>[:greedy|:random]`
(a [ranks, experts] array of per-rank counts, e.g. from a router trace) and `bank:<scenario>[:greedy|:random]`
(the built-in scenario tables of `BANK`).
"""
from typing import Tuple

import numpy as np
import torch

ROUTINGS = ['uniform', 'mixed', 'skew1.5', 'skew2', 'skew4', 'hot_rank', 'self', 'remote', 'zipf1.1', 'zipf1.1_greedy']


def skew_routes(num_tokens: int, num_ranks: int, num_experts: int, num_topk: int, skew: float, seed: int,
                exclude_self: bool = False) -> Tuple[np.ndarray, np.ndarray]:
    """Global routing table `[num_ranks * num_tokens, num_topk]` (rank r owns rows r*N .. r*N+N-1) and
    the `[src, dst]` row-count matrix."""
    R, N, K = num_ranks, num_tokens, num_topk
    assert K % 2 == 0 and num_experts % R == 0 and R >= 2
    if not 1.0 <= skew <= R / 2:
        raise ValueError('two distinct destinations per token need 1 <= skew <= num_ranks / 2')
    total = R * N
    counts = np.empty(R, dtype=np.int64)
    counts[0] = int(round(2 * N * skew))
    rest = 2 * total - counts[0]
    counts[1:] = rest // (R - 1)
    counts[1:1 + rest - counts[1:].sum()] += 1
    assert counts.sum() == 2 * total and counts.max() <= total
    deck = np.sort(np.repeat(np.arange(R), counts))
    pairs = np.stack([deck[:total], deck[total:]], axis=1)
    rng = np.random.default_rng(seed)
    pairs = pairs[rng.permutation(total)]
    if exclude_self:
        # Balanced remote-only traffic: source s deals its tokens round-robin over the other ranks.
        assert skew == 1.0, 'remote routing is defined for balanced traffic'
        assert R >= 3, 'two distinct remote destinations need at least three ranks'
        src = np.arange(total) // N
        i = np.arange(total) % N
        pairs = np.stack([(src + 1 + i % (R - 1)) % R, (src + 1 + (i + 1) % (R - 1)) % R], axis=1)
        assert np.all(pairs != src[:, None])
    assert np.all(pairs[:, 0] != pairs[:, 1])
    le = num_experts // R
    half = K // 2
    assert half <= le
    start = rng.integers(0, le, size=(total, 1))
    local = (start + np.arange(half)[None, :]) % le
    idx = np.concatenate([pairs[:, :1] * le + local, pairs[:, 1:] * le + local], axis=1)
    matrix = np.zeros((R, R), dtype=np.int64)
    for s in range(R):
        matrix[s] = np.bincount(pairs[s * N:(s + 1) * N].ravel(), minlength=R)
    return idx.astype(np.int64), matrix


def routes_from_counts(counts, num_tokens: int, num_topk: int, seed: int) -> np.ndarray:
    """`[num_tokens, num_topk]` expert ids whose histogram is exactly `counts` (sum <= tokens*topk, each
    count <= tokens), distinct experts per token; missing assignments are -1. A cursor walks the token
    positions cyclically and each expert (random order) takes its count of consecutive positions, so
    every position is visited exactly `num_topk` times and no expert meets a token twice; tokens are
    then shuffled."""
    counts = np.asarray(counts, dtype=np.int64)
    n, k = num_tokens, num_topk
    deficit = n * k - int(counts.sum())
    if deficit < 0 or (counts.size and counts.max() > n) or deficit > n * k:
        raise ValueError('counts must sum to at most tokens * topk with no count above tokens')
    rng = np.random.default_rng(seed)
    full = np.append(counts, deficit)  # last entry: the "no expert" filler
    table = np.full((n, k), -1, dtype=np.int64)
    fill = np.zeros(n, dtype=np.int64)
    cursor = 0
    for e in rng.permutation(full.size):
        left = int(full[e])
        while left > 0:  # only the filler can exceed n; it may repeat a token (several -1 entries)
            c = min(left, n)
            pos = (cursor + np.arange(c)) % n
            table[pos, fill[pos]] = e if e < counts.size else -1
            fill[pos] += 1
            cursor = (cursor + c) % n
            left -= c
    assert (fill == k).all()
    return table[rng.permutation(n)]


def greedy_placement(load, experts_per_rank: int) -> np.ndarray:
    """perm[logical expert] = physical expert id: experts by decreasing load, each onto the
    least-loaded rank with a free slot (balanced partition, no replicas)."""
    load = np.asarray(load, dtype=np.float64)
    ranks = load.size // experts_per_rank
    rank_load = np.zeros(ranks)
    fill = np.zeros(ranks, dtype=np.int64)
    perm = np.empty(load.size, dtype=np.int64)
    for e in np.argsort(-load, kind='stable'):
        free = np.nonzero(fill < experts_per_rank)[0]
        r = free[np.argmin(rank_load[free])]
        perm[e] = r * experts_per_rank + fill[r]
        fill[r] += 1
        rank_load[r] += load[e]
    return perm


def random_placement(num_experts: int, seed: int) -> np.ndarray:
    """A seeded random permutation of the experts (a placement that ignores load)."""
    return np.random.default_rng(seed).permutation(num_experts)


def zipf_counts(num_experts: int, num_tokens: int, num_topk: int, s: float, seed: int) -> np.ndarray:
    """Per-expert counts summing to tokens * topk with Zipf(s) popularity over a random expert order,
    capped at `num_tokens` per expert (overflow redistributed)."""
    rng = np.random.default_rng(seed)
    w = 1.0 / np.arange(1, num_experts + 1) ** s
    w = w[rng.permutation(num_experts)]
    total = num_tokens * num_topk
    counts = np.floor(w / w.sum() * total).astype(np.int64)
    counts[np.argsort(-w)[: total - counts.sum()]] += 1
    while counts.max() > num_tokens:
        over = counts - num_tokens
        spill = int(over[over > 0].sum())
        counts = np.minimum(counts, num_tokens)
        room = num_tokens - counts
        order = np.argsort(room)[::-1]
        for e in order:
            take = min(int(room[e]), spill)
            counts[e] += take
            spill -= take
            if spill == 0:
                break
    return counts


def _spread(total: int, weights: np.ndarray, cap: int) -> np.ndarray:
    """Integer counts proportional to `weights`, summing to `total`, none above `cap` (the overflow of
    a capped entry goes to the others in proportion)."""
    w = np.asarray(weights, dtype=np.float64)
    counts = np.zeros(w.size, dtype=np.int64)
    free = w > 0
    left = total
    while left > 0 and free.any():
        share = np.where(free, w, 0.0)
        raw = share / share.sum() * left
        add = np.minimum(np.floor(raw).astype(np.int64), cap - counts)
        if add.sum() == 0:  # hand out the remainder one by one, largest weights first
            for e in np.argsort(-share):
                if left == 0 or not free[e]:
                    break
                if counts[e] < cap:
                    counts[e] += 1
                    left -= 1
        else:
            counts += add
            left -= int(add.sum())
        free &= counts < cap
    if left > 0:
        raise ValueError('the capped counts cannot hold the total')
    return counts


# Built-in bank of per-expert count tables: named routing scenarios, deterministic per (rank, seed),
# that stress the count-driven paths the way recorded router traces do (the reference replays per-
# layer count tables of real traces, backend/tests/bank_routing.py:25-105; no trace is shipped
# here, so the scenarios below are synthetic and named for the shape they produce).
#   hot8        8 experts, the same on every rank, take half of all assignments; the rest is uniform
#   drift       Zipf(1.2) popularity whose expert order differs per rank (rank-local hot experts)
#   dead        a quarter of the experts (a random set shared by all ranks) receive nothing
#   saturated   the top-k-1 most popular experts are chosen by every token (count = tokens, the cap);
#               the last choice is uniform over the others
BANK = ('hot8', 'drift', 'dead', 'saturated')


def bank_counts(name: str, rank: int, num_ranks: int, N: int, E: int, K: int, seed: int) -> np.ndarray:
    """This rank's per-expert counts (sum N * K, each <= N) for bank scenario `name`."""
    total = N * K
    shared = np.random.default_rng(seed)           # the same on every rank
    local = np.random.default_rng(seed * 977 + rank)  # this rank's own
    if name == 'hot8':
        hot = shared.permutation(E)[:min(8, E)]
        w = np.full(E, 0.5 / max(E - hot.size, 1))
        w[hot] = 0.5 / hot.size
        return _spread(total, w, N)
    if name == 'drift':
        w = 1.0 / np.arange(1, E + 1) ** 1.2
        return _spread(total, w[local.permutation(E)], N)
    if name == 'dead':
        w = np.ones(E)
        w[shared.permutation(E)[:E // 4]] = 0.0
        return _spread(total, w, N)
    if name == 'saturated':
        if K < 2 or E <= K:
            raise ValueError('bank scenario saturated needs 2 <= topk < experts')
        top = shared.permutation(E)[:K - 1]
        counts = np.zeros(E, dtype=np.int64)
        counts[top] = N
        rest = np.setdiff1d(np.arange(E), top)
        counts[rest] = _spread(N, np.ones(rest.size), N)
        return counts
    raise ValueError(f'unknown bank scenario {name} (known: {", ".join(BANK)})')


def _count_routing(name: str, rank: int, num_ranks: int, N: int, E: int, K: int, seed: int) -> torch.Tensor:
    placement = None
    if name.startswith('bank:'):
        parts = name.split(':')
        counts = bank_counts(parts[1], rank, num_ranks, N, E, K, seed)
        placement = parts[2] if len(parts) > 2 else None
        load = sum(bank_counts(parts[1], r, num_ranks, N, E, K, seed) for r in range(num_ranks)).astype(np.float64)
    elif name.startswith('counts:'):
        parts = name.split(':')
        all_counts = np.load(parts[1])
        counts = np.asarray(all_counts[rank % all_counts.shape[0]], dtype=np.int64)
        placement = parts[2] if len(parts) > 2 else None
        load = np.asarray(all_counts, dtype=np.float64).sum(0)
    else:
        base, _, placement = name.partition('_')
        s = float(base[4:])
        counts = zipf_counts(E, N, K, s, seed * 100 + rank)
        load = sum(zipf_counts(E, N, K, s, seed * 100 + r) for r in range(num_ranks)).astype(np.float64)
    if counts.size != E:
        raise ValueError(f'counts have {counts.size} experts, the model has {E}')
    idx = routes_from_counts(counts, N, K, seed * 1000 + rank)
    if placement in ('greedy', 'random'):
        perm = greedy_placement(load, E // num_ranks) if placement == 'greedy' else random_placement(E, seed)
        idx = np.where(idx >= 0, np.append(perm, -1)[idx], -1)
    return torch.from_numpy(idx.astype(np.int64))


def make_routing(name: str, rank: int, num_ranks: int, num_tokens: int, num_experts: int, num_topk: int,
                 seed: int) -> torch.Tensor:
    """This rank's `[num_tokens, num_topk]` int64 expert ids for routing `name` (CPU tensor)."""
    N, E, K, R = num_tokens, num_experts, num_topk, num_ranks
    if name == 'uniform':
        g = torch.Generator().manual_seed(seed * 100 + rank)
        return torch.rand((N, E), generator=g).topk(K, dim=1).indices.to(torch.int64)
    if name == 'hot_rank':
        if K > E // R:
            raise ValueError(f'routing hot_rank puts all top-{K} choices on rank 0, which owns only {E // R} experts')
        return torch.arange(K, dtype=torch.int64)[None, :].expand(N, K).contiguous()
    if name == 'self':
        le = E // R
        if K > le:
            raise ValueError(f'routing self keeps all top-{K} choices on the source rank, which owns only {le} experts')
        g = torch.Generator().manual_seed(seed * 100 + rank)
        return (torch.rand((N, le), generator=g).topk(K, dim=1).indices + rank * le).to(torch.int64)
    if name.startswith('zipf') or name.startswith('counts:') or name.startswith('bank:'):
        return _count_routing(name, rank, R, N, E, K, seed)
    if R == 1:
        raise ValueError(f'routing {name} needs at least two ranks')
    if name == 'mixed':
        skew, excl = 1.0, False
    elif name == 'remote':
        skew, excl = 1.0, True
    elif name.startswith('skew'):
        skew, excl = float(name[4:]), False
    else:
        raise ValueError(f'unknown routing {name}')
    idx, _ = skew_routes(N, R, E, K, skew, seed, exclude_self=excl)
    return torch.from_numpy(idx[rank * N:(rank + 1) * N].copy())


def route_matrix(idx: np.ndarray, num_ranks: int, num_experts: int) -> np.ndarray:
    """Rows this rank sends to each destination (a token counts once per destination rank)."""
    le = num_experts // num_ranks
    out = np.zeros(num_ranks, dtype=np.int64)
    dst = np.where(idx >= 0, idx // le, -1)
    for r in range(num_ranks):
        out[r] = int((dst == r).any(axis=1).sum())
    return out
