"""Functional reference of dispatch / combine (the reference's `deep_ep/utils/refs.py` API shape),
built on the `ReferenceBuffer` oracle. Works on any process group backend (gloo on CPU, NCCL).

`dispatch` returns received rows sorted by (source rank, source token) with their global source
index `src_rank * num_max_tokens_per_rank + src_token`; `combine` reduces `[tokens, topk, hidden]`
contributions either in top-k order or as per-rank partials (bf16-rounded, as they travel) summed in
rank order; `generate_pre_combine_data` makes deterministic per-(token, k) test rows.
"""
import math
from typing import Optional, Tuple, Union

import torch
import torch.distributed as dist


def dispatch(x: Union[torch.Tensor, Tuple[torch.Tensor, torch.Tensor]], topk_idx: torch.Tensor,
             topk_weights: Optional[torch.Tensor], num_max_tokens_per_rank: int, num_experts: int,
             group: Optional[dist.ProcessGroup] = None):
    """(recv_x, recv_topk_idx (local ids, -1 elsewhere), recv_topk_weights, recv_src_token_global_idx,
    num_recv_tokens_per_rank)."""
    from ..parallel.reference import ReferenceBuffer
    group = group or dist.group.WORLD
    ref = ReferenceBuffer(group)
    weights = topk_weights if topk_weights is not None else torch.ones(topk_idx.shape, dtype=torch.float32,
                                                                       device=topk_idx.device)
    rx, ri, rw, _, handle, _ = ref.dispatch(x, topk_idx=topk_idx, topk_weights=weights, num_experts=num_experts)
    rank_prefix, src_idx = handle[0], handle[3].to(torch.int64)
    R, me = group.size(), group.rank()
    starts = torch.cat([torch.zeros(1, dtype=torch.int64), rank_prefix[:, me].to(torch.int64).cpu()])
    per_rank = (starts[1:] - starts[:-1]).to(torch.int)
    src_rank = torch.repeat_interleave(torch.arange(R), per_rank.long()).to(src_idx.device)
    global_idx = src_rank * num_max_tokens_per_rank + src_idx
    return rx, ri, (rw if topk_weights is not None else None), global_idx, per_rank


def generate_pre_combine_data(src_token_global_idx: torch.Tensor, num_max_tokens_per_rank: int, num_topk: int,
                              hidden: int, seed: int = 0) -> torch.Tensor:
    """Deterministic bf16 rows `[tokens, num_topk, hidden]` that depend only on (global token, k),
    so every rank regenerates the contribution it expects back."""
    key = (src_token_global_idx.to(torch.int64).unsqueeze(1) * num_topk +
           torch.arange(num_topk, device=src_token_global_idx.device).unsqueeze(0))
    phase = ((key * 2654435761 + seed * 97) % 1000003).float() / 1000003.0
    cols = torch.arange(1, hidden + 1, device=src_token_global_idx.device, dtype=torch.float32)
    return torch.cos(phase.unsqueeze(-1) * cols * 0.37 + math.pi * phase.unsqueeze(-1)).to(torch.bfloat16)


def ordered_accumulate(data: torch.Tensor, initial_value: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Sum `data [tokens, k, hidden]` over k in order, in fp32, starting from `initial_value`."""
    acc = initial_value.float().clone() if initial_value is not None else \
        torch.zeros((data.shape[0], data.shape[2]), dtype=torch.float32, device=data.device)
    for k in range(data.shape[1]):
        acc += data[:, k].float()
    return acc.to(data.dtype)


def combine(y: torch.Tensor, topk_idx: torch.Tensor, num_scaleout_ranks: int, num_scaleup_ranks: int,
            num_experts: int, bias: Union[None, torch.Tensor, Tuple[torch.Tensor, torch.Tensor]] = None,
            reduce_in_local: bool = True, reduce_in_scaleup: bool = False) -> torch.Tensor:
    """Combine `y [tokens, k, hidden]` (the contribution of each top-k choice) into `[tokens, hidden]`.

    reduce_in_local=False: every copy is added in top-k order. reduce_in_local=True: copies of experts
    on one rank are summed first (fp32) and rounded to bf16 (the partial that travels), then partials
    are added in rank order. With a single scale-out group `reduce_in_scaleup` adds nothing."""
    assert not (reduce_in_scaleup and not reduce_in_local), 'invalid reduction configuration'
    n, k, h = y.shape
    num_ranks = num_scaleout_ranks * num_scaleup_ranks
    epr = num_experts // num_ranks
    b0, b1 = (bias if isinstance(bias, tuple) else (bias, None))
    acc = torch.zeros((n, h), dtype=torch.float32, device=y.device)
    for b in (b0, b1):
        if b is not None:
            acc += b.float()
    valid = topk_idx >= 0
    if not reduce_in_local:
        for j in range(k):
            acc += torch.where(valid[:, j:j + 1], y[:, j].float(), torch.zeros((), device=y.device))
        return acc.to(torch.bfloat16)
    dest = torch.where(valid, topk_idx // epr, torch.full_like(topk_idx, -1))
    for r in range(num_ranks):
        part = torch.zeros((n, h), dtype=torch.float32, device=y.device)
        for j in range(k):
            part += torch.where((dest[:, j] == r).unsqueeze(1), y[:, j].float(), torch.zeros((), device=y.device))
        has = (dest == r).any(1, keepdim=True)
        acc += torch.where(has, part.to(torch.bfloat16).float(), torch.zeros((), device=y.device))
    return acc.to(torch.bfloat16)
