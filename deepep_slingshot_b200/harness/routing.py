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
"""
from typing import Tuple

import numpy as np
import torch

ROUTINGS = ['uniform', 'mixed', 'skew1.5', 'skew2', 'skew4', 'hot_rank', 'self', 'remote']


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


def make_routing(name: str, rank: int, num_ranks: int, num_tokens: int, num_experts: int, num_topk: int,
                 seed: int) -> torch.Tensor:
    """This rank's `[num_tokens, num_topk]` int64 expert ids for routing `name` (CPU tensor)."""
    N, E, K, R = num_tokens, num_experts, num_topk, num_ranks
    if name == 'uniform':
        g = torch.Generator().manual_seed(seed * 100 + rank)
        return torch.rand((N, E), generator=g).topk(K, dim=1).indices.to(torch.int64)
    if name == 'hot_rank':
        assert K <= E // R
        return torch.arange(K, dtype=torch.int64)[None, :].expand(N, K).contiguous()
    if name == 'self':
        le = E // R
        assert K <= le
        g = torch.Generator().manual_seed(seed * 100 + rank)
        return (torch.rand((N, le), generator=g).topk(K, dim=1).indices + rank * le).to(torch.int64)
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
