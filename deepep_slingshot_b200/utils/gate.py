"""Routing (gate) generators for tests and benchmarks.

Parity with the reference's `deep_ep/utils/gate.py:4-180` (balanced / unbalanced score generators)
and `backend/tests/routing.py:12-78` (receiver-skew, local / remote routings), plus the popularity
skews named in the benchmark configs: N(0,1) logits, uniform logits, Zipf(s) expert popularity.
Every generator returns (topk_idx int64 [N, K], topk_weights fp32 [N, K]) with softmax weights over
the selected K logits.
"""
from typing import Optional, Tuple

import torch


def _select(scores: torch.Tensor, num_topk: int) -> Tuple[torch.Tensor, torch.Tensor]:
    vals, idx = torch.topk(scores, num_topk, dim=-1, largest=True, sorted=False)
    weights = torch.softmax(vals.float(), dim=-1)
    return idx.to(torch.int64), weights.to(torch.float32)


def normal_routing(num_tokens: int, num_experts: int, num_topk: int, generator: Optional[torch.Generator] = None,
                   device='cpu') -> Tuple[torch.Tensor, torch.Tensor]:
    """Top-k of N(0,1) router logits (DeepSeek-V3 config)."""
    scores = torch.randn((num_tokens, num_experts), generator=generator, dtype=torch.float32).to(device)
    return _select(scores, num_topk)


def uniform_routing(num_tokens: int, num_experts: int, num_topk: int, generator: Optional[torch.Generator] = None,
                    device='cpu') -> Tuple[torch.Tensor, torch.Tensor]:
    """Top-k of U(0,1) router logits (uniform expert choice)."""
    scores = torch.rand((num_tokens, num_experts), generator=generator, dtype=torch.float32).to(device)
    return _select(scores, num_topk)


def zipf_routing(num_tokens: int, num_experts: int, num_topk: int, s: float = 1.1,
                 generator: Optional[torch.Generator] = None, device='cpu') -> Tuple[torch.Tensor, torch.Tensor]:
    """Expert popularity ~ Zipf(s): logits = log(p_e) + Gumbel noise, so top-k samples without
    replacement proportionally to p_e. Expert ids are permuted so hot experts spread over ranks."""
    ranks = torch.arange(1, num_experts + 1, dtype=torch.float64)
    p = ranks.pow(-s)
    p = p / p.sum()
    perm = torch.randperm(num_experts, generator=generator)
    logp = torch.empty(num_experts, dtype=torch.float64)
    logp[perm] = p.log()
    u = torch.rand((num_tokens, num_experts), generator=generator, dtype=torch.float64).clamp_(1e-12, 1 - 1e-12)
    gumbel = -torch.log(-torch.log(u))
    scores = (logp.unsqueeze(0) + gumbel).float().to(device)
    return _select(scores, num_topk)


def get_scores_by_factor(num_tokens: int, num_experts: int, num_ranks: int, factor: float,
                         generator: Optional[torch.Generator] = None) -> torch.Tensor:
    """Router scores where rank 0's experts draw from U(0, factor) and all others from U(0, 1): a
    factor above 1 makes rank 0 hot."""
    epr = num_experts // num_ranks
    scores = torch.rand((num_tokens, num_experts), generator=generator)
    scores[:, :epr] *= factor
    return scores


def _rank0_ratio(scores: torch.Tensor, num_ranks: int, num_topk: int) -> float:
    epr = scores.shape[1] // num_ranks
    ranks = torch.topk(scores, num_topk, dim=-1).indices // epr
    hit = torch.zeros((scores.shape[0], num_ranks), dtype=torch.bool)
    hit.scatter_(1, ranks, True)
    per_rank = hit.float().sum(0)
    return float(per_rank[0] / per_rank[1:].mean().clamp_min(1e-9))


def map_unbalanced_ratio_to_factor(num_tokens: int, num_experts: int, num_ranks: int, num_topk: int, ratio: float,
                                   generator: Optional[torch.Generator] = None, iterations: int = 20) -> float:
    """Bisection for the score factor whose top-k routing sends rank 0 about `ratio` times the tokens
    of an average other rank."""
    lo, hi = 1.0, 100.0
    for _ in range(iterations):
        mid = (lo + hi) / 2
        r = _rank0_ratio(get_scores_by_factor(num_tokens, num_experts, num_ranks, mid, generator), num_ranks, num_topk)
        if r > ratio:
            hi = mid
        else:
            lo = mid
    return lo


def get_random_unbalanced_scores(num_tokens: int, num_experts: int, num_ranks: int, num_topk: int, ratio: float,
                                 generator: Optional[torch.Generator] = None) -> torch.Tensor:
    """Random scores whose top-k makes rank 0 receive about `ratio` times the average traffic."""
    factor = 1.0 if ratio == 1.0 else map_unbalanced_ratio_to_factor(num_tokens, num_experts, num_ranks, num_topk,
                                                                     ratio, generator)
    return get_scores_by_factor(num_tokens, num_experts, num_ranks, factor, generator)


def generate_rank_count(num_tokens: int, num_experts: int, num_ranks: int, num_topk: int, ratio: float,
                        generator: Optional[torch.Generator] = None) -> torch.Tensor:
    """`[num_tokens, num_ranks]` int32: how many of token t's top-k experts live on rank r, with every
    row summing to `num_topk`, and rank 0 (the special rank) holding experts of `ratio` times as many
    tokens as an average other rank (exact up to rounding). Each token spreads over as many distinct
    ranks as uniform top-k routing would give it (capped so the special rank's share stays reachable);
    the special rank is put on the chosen number of tokens, the other rank slots are dealt round-robin
    over a random order of the other ranks."""
    assert ratio >= 1.0 and num_ranks >= 1
    R, N, K = num_ranks, num_tokens, num_topk
    epr = num_experts // R
    if R == 1:
        return torch.full((N, 1), K, dtype=torch.int32)
    # distinct ranks per token under uniform top-k, capped so the special rank's share is reachable
    ranks = torch.topk(torch.rand((N, num_experts), generator=generator), K, dim=-1).indices // epr
    hit = torch.zeros((N, R), dtype=torch.bool)
    hit.scatter_(1, ranks, True)
    cap = min(R, int((R - 1) / ratio) + 1)
    spread = hit.sum(1).clamp(min=max(1, -(-K // epr)), max=cap)
    total = int(spread.sum())
    must = spread == R  # a token on every rank includes the special rank
    special = round(total * ratio / (R - 1 + ratio))
    special = min(N, max(int(must.sum()), special))
    rest = torch.nonzero(~must).flatten()
    rest = rest[torch.randperm(rest.numel(), generator=generator)]
    with_special = must.clone()
    with_special[rest[:special - int(must.sum())]] = True
    counts = torch.zeros((N, R), dtype=torch.int32)
    normal = (torch.randperm(R - 1, generator=generator) + 1).tolist()
    cursor = 0
    spread_l, special_l = spread.tolist(), with_special.tolist()
    for t in range(N):
        a = spread_l[t]
        picks = [0] if special_l[t] else []
        seen = set(picks)
        while len(picks) < a:  # a - len(picks) <= R - 1 distinct normal ranks always exist
            r = normal[cursor % (R - 1)]
            cursor += 1
            if r not in seen:
                seen.add(r)
                picks.append(r)
        for i in range(K):  # the k experts over the picked ranks, at most epr per rank
            counts[t, picks[i % a]] += 1
    return counts


def generate_topk_idx(rank_count: torch.Tensor, num_tokens: int, num_experts: int, num_ranks: int, num_topk: int,
                      generator: Optional[torch.Generator] = None) -> torch.Tensor:
    """Expert ids realising `rank_count`: `rank_count[t, r]` distinct random experts of rank r per token."""
    assert tuple(rank_count.shape) == (num_tokens, num_ranks)
    assert bool((rank_count.sum(1) == num_topk).all())
    epr = num_experts // num_ranks
    perm = torch.argsort(torch.rand((num_tokens, num_ranks, epr), generator=generator), dim=-1)
    experts = perm + torch.arange(num_ranks).view(1, num_ranks, 1) * epr
    take = torch.arange(epr).view(1, 1, epr) < rank_count.cpu().view(num_tokens, num_ranks, 1)
    return experts[take].view(num_tokens, num_topk).to(torch.int64)


def get_precise_unbalanced_scores(num_tokens: int, num_experts: int, num_ranks: int, num_topk: int, ratio: float,
                                  generator: Optional[torch.Generator] = None) -> torch.Tensor:
    """Scores whose top-k follows `generate_rank_count` exactly: chosen experts score in (0.9, 1],
    the rest in [0, 0.9)."""
    counts = generate_rank_count(num_tokens, num_experts, num_ranks, num_topk, ratio, generator)
    idx = generate_topk_idx(counts, num_tokens, num_experts, num_ranks, num_topk, generator)
    scores = torch.rand((num_tokens, num_experts), generator=generator) * 0.9
    top = 0.9 + 1e-6 + torch.rand((num_tokens, num_topk), generator=generator) * (0.1 - 1e-6)
    scores.scatter_(1, idx, top)
    return scores


def get_unbalanced_scores(num_tokens: int, num_experts: int, num_ranks: int, num_topk: int, ratio: float = 1.0,
                          precise: bool = False, generator: Optional[torch.Generator] = None) -> torch.Tensor:
    """Router scores with rank 0 receiving about (`precise`: exactly) `ratio` times the average traffic."""
    if precise:
        return get_precise_unbalanced_scores(num_tokens, num_experts, num_ranks, num_topk, ratio, generator)
    return get_random_unbalanced_scores(num_tokens, num_experts, num_ranks, num_topk, ratio, generator)


def hot_rank_routing(num_tokens: int, num_experts: int, num_ranks: int, num_topk: int, hot_rank: int = 0,
                     generator: Optional[torch.Generator] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Every token picks experts of one rank only (every other rank receives nothing)."""
    epr = num_experts // num_ranks
    assert num_topk <= epr
    scores = torch.full((num_tokens, num_experts), -1e9)
    scores[:, hot_rank * epr:(hot_rank + 1) * epr] = torch.randn((num_tokens, epr), generator=generator)
    return _select(scores, num_topk)


def local_routing(num_tokens: int, num_experts: int, num_ranks: int, num_topk: int, rank: int,
                  generator: Optional[torch.Generator] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Tokens stay on their own rank (no NVLink traffic)."""
    return hot_rank_routing(num_tokens, num_experts, num_ranks, num_topk, hot_rank=rank, generator=generator)


def drop_tokens(topk_idx: torch.Tensor, topk_weights: torch.Tensor, ratio: float,
                generator: Optional[torch.Generator] = None) -> None:
    """Mask a random fraction of (token, k) selections with -1 (the reference's dropped-token cases)."""
    if ratio <= 0:
        return
    m = torch.rand(topk_idx.shape, generator=generator) < ratio
    topk_idx.masked_fill_(m.to(topk_idx.device), -1)
    topk_weights.masked_fill_(m.to(topk_weights.device), 0)
