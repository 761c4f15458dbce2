"""Permute dispatched tokens into the expert-grouped layout of the grouped GEMMs, and back.

`permute` groups the rows of every (token, k) selection by local expert (deterministic order),
padding each expert's block to `alignment` rows, and returns the map needed by `unpermute`.
`unpermute` is the top-k weighted fp32 gather-sum back to one row per token (bf16).
The torch functions `permute_reference` / `unpermute_reference` are the numerics oracle.
"""
from typing import NamedTuple, Optional

import torch

from .._ext import require_ext


class Permuted(NamedTuple):
    """Result of `permute`: expert-grouped rows (and scales / probs), the (token, k) -> row map and the
    per-expert offsets and counts."""
    x: torch.Tensor                 # [rows, H] grouped by expert (rows past offsets[E] unused)
    scales: Optional[torch.Tensor]  # [rows, H/128] FP8 block scales
    probs: Optional[torch.Tensor]   # [rows] top-k weight of each grouped row
    row_map: torch.Tensor           # [N, K] int32 grouped row of (t, k), -1 if none
    expert_offsets: torch.Tensor    # [E+1] int32, aligned exclusive prefix
    expert_counts: torch.Tensor     # [E] int32, unpadded counts


def permute(x: torch.Tensor, topk_idx: torch.Tensor, num_experts: int, alignment: int = 1,
            probs: Optional[torch.Tensor] = None, x_scales: Optional[torch.Tensor] = None,
            num_out_rows: int = 0, zero_padding: bool = False) -> Permuted:
    """`zero_padding` zeroes each expert's alignment rows (and their scales), so grouped GEMMs may run
    over whole aligned groups."""
    out = require_ext().permute(x, x_scales, topk_idx, probs, num_experts, alignment, num_out_rows, zero_padding)
    return Permuted(*out)


def unpermute(y: torch.Tensor, row_map: torch.Tensor, weights: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Sum each token's rows back from the expert-grouped layout (`row_map [N, K]`, -1 = none),
    weighted by `probs [N, K]` when given (sm_100a kernel)."""
    return require_ext().unpermute(y, row_map, weights)


def permute_reference(topk_idx: torch.Tensor, num_experts: int, alignment: int = 1):
    """(counts, aligned offsets) of the grouped layout, computed with torch."""
    valid = topk_idx[topk_idx >= 0]
    counts = torch.bincount(valid, minlength=num_experts)[:num_experts].to(torch.int32)
    aligned = (counts + alignment - 1) // alignment * alignment
    offsets = torch.zeros(num_experts + 1, dtype=torch.int32, device=topk_idx.device)
    offsets[1:] = aligned.cumsum(0)
    return counts, offsets


def unpermute_reference(y: torch.Tensor, row_map: torch.Tensor, weights: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Torch oracle of `unpermute` (fp32 accumulation, bf16 result)."""
    N, K = row_map.shape
    w = weights if weights is not None else torch.ones((N, K), device=y.device)
    valid = row_map >= 0
    g = y[row_map.clamp(min=0).long()].float() * (w * valid).unsqueeze(-1)
    return g.sum(1).to(torch.bfloat16)


def unpermute_backward(g_tok: torch.Tensor, row_map: torch.Tensor, weights: torch.Tensor, y: torch.Tensor,
                       g_y: torch.Tensor) -> torch.Tensor:
    """Backward of the weighted unpermute (sm_100a kernel): writes `g_y[row_map[j, k]] =
    bf16(g_tok[j] * weights[j, k])` into the caller's zeroed `g_y` and returns the weight gradient
    `[N, K]` fp32, `<g_tok[j], y[row_map[j, k]]>` (0 where row_map is -1)."""
    return require_ext().unpermute_backward(g_tok, row_map, weights, y, g_y)


def unpermute_backward_reference(g_tok: torch.Tensor, row_map: torch.Tensor, weights: torch.Tensor, y: torch.Tensor):
    """Torch oracle of `unpermute_backward` (fp32 math): returns (g_y, g_w)."""
    valid = row_map >= 0
    rows = row_map[valid].long()
    t_of = torch.arange(row_map.shape[0], device=g_tok.device).unsqueeze(1).expand_as(row_map)[valid]
    g_y = torch.zeros_like(y)
    g_y[rows] = (g_tok[t_of].float() * weights[valid].unsqueeze(1)).to(torch.bfloat16)
    g_w = torch.zeros_like(weights)
    g_w[valid] = (g_tok[t_of].float() * y[rows].float()).sum(-1)
    return g_y, g_w


def zero_group_padding(tensors, offsets: torch.Tensor, counts: torch.Tensor) -> None:
    """Zero the alignment padding rows `[offsets[e] + counts[e], offsets[e + 1])` of up to three
    expert-grouped 2D tensors in place (sm_100a kernel)."""
    require_ext().zero_group_padding(list(tensors), offsets, counts)
