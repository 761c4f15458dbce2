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


def get_unbalanced_scores(num_tokens: int, num_experts: int, num_ranks: int, num_topk: int, ratio: float = 1.0,
                          generator: Optional[torch.Generator] = None) -> torch.Tensor:
    """Scores whose rank-level load is skewed by `ratio` (1.0 = balanced): the first rank's experts get
    their logits lifted so it receives about `ratio` times the average traffic."""
    scores = torch.randn((num_tokens, num_experts), generator=generator).abs() + 1
    if ratio > 1.0:
        epr = num_experts // num_ranks
        scores[:, :epr] *= ratio
    return scores


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
