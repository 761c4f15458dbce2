"""Normal-mode down projection with the combine as its epilogue.

In the MoE layer the down projection's output rows only exist to be sent back to their tokens'
source ranks and summed there with the top-k weights. `GemmCombine` fuses that send into the grouped
FP8 GEMM: its epilogue stores every finished bf16 row over NVLink into slot (t, k) of token t's
source rank, so the transfer overlaps the remaining GEMM tiles and the unfused path's separate
combine launch (and its read of the GEMM output) goes away; the source rank then sums its own slots
with its own top-k weights in fp32.

    gc = GemmCombine(group, num_max_tokens, num_topk, hidden)      # collective, once per layer
    y = gc.send(a, a_scales, w2, w2_scales, offsets, counts, row_map, handle, keep_local=True)
    out = gc.reduce(topk_idx, topk_weights)                       # [num_tokens, hidden] bf16

`a`/`a_scales` are the expert-grouped FP8 rows (`permute(..., alignment=128)` layout) and `row_map`
the permute's (received token, k) -> row map; `handle` is `Buffer.dispatch`'s. Every rank calls
`send` and then `reduce`, in the same order; the epochs that order the slot reuse are host counters,
so the pair is not CUDA-graph replayable. The unfused composition is
`Buffer.combine(y, handle, row_map=row_map, row_weights=recv_topk_weights)`; this one sends up to
top-k rows per (token, rank) instead of one sender-reduced row and hides them behind the GEMM.

Capability reference: DeepEP's combine after a separate expert GEMM
([DE]csrc/kernels/legacy/intranode.cu:705) and its low-latency weighted receive
([DE]csrc/kernels/legacy/internode_ll.cu:715-1230); the reference has no GEMM of its own.
The functions `row_destinations`, `exchange_reference` and `reduce_reference` restate the kernels'
index rules in torch (CPU and gloo tests check them against `ReferenceBuffer.combine`).
"""
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

from .symmetric import SymmetricRegion

SLOT_BITS = 24
MAX_SLOTS = 1 << SLOT_BITS


def row_destinations(row_map: torch.Tensor, recv_src_idx: torch.Tensor, rank_prefix_matrix: torch.Tensor,
                     rank: int, rows: int) -> torch.Tensor:
    """Destination word of every operand row: (source rank << 24) | (t * K + k), -1 for none.
    Same rule as the row-destination kernel: received token j comes from the source s with
    prefix[s] <= j < prefix[s + 1], prefix[s + 1] = rank_prefix_matrix[s][rank]."""
    num_recv, K = row_map.shape
    dest = torch.full((rows,), -1, dtype=torch.int64)
    rm = row_map.long().cpu()
    prefix = torch.cat([torch.zeros(1, dtype=torch.int64), rank_prefix_matrix[:, rank].long().cpu()])
    j = torch.arange(num_recv)
    src = (torch.searchsorted(prefix[1:], j, right=True)).clamp(max=prefix.numel() - 2)
    t = recv_src_idx.long().cpu()
    for k in range(K):
        ok = rm[:, k] >= 0
        dest[rm[ok, k]] = (src[ok] << SLOT_BITS) | (t[ok] * K + k)
    return dest.to(torch.int32)


def exchange_reference(group: dist.ProcessGroup, y: torch.Tensor, row_dest: torch.Tensor,
                       num_tokens: int, num_topk: int) -> torch.Tensor:
    """Every rank's slots [num_tokens * K, H] after the sends (rows gathered over `group`).
    Slots no rank writes stay zero."""
    R, me = group.size(), group.rank()
    H = y.shape[1]
    d = row_dest.long()
    keep = d >= 0
    packed = torch.cat([d[keep].unsqueeze(1).to(torch.float64), y[keep].double()], dim=1)
    sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(R)]
    dist.all_gather(sizes, torch.tensor([packed.shape[0]], dtype=torch.int64), group=group)
    mx = int(max(s.item() for s in sizes))
    pad = torch.zeros((mx, H + 1), dtype=torch.float64)
    pad[:packed.shape[0]] = packed
    parts = [torch.zeros_like(pad) for _ in range(R)]
    dist.all_gather(parts, pad, group=group)
    slots = torch.zeros((num_tokens * num_topk, H), dtype=torch.float64)
    for r in range(R):
        rows = parts[r][:int(sizes[r].item())]
        words = rows[:, 0].long()
        mine = (words >> SLOT_BITS) == me
        slots[words[mine] & (MAX_SLOTS - 1)] = rows[mine, 1:]
    return slots.to(y.dtype)


def reduce_reference(slots: torch.Tensor, topk_idx: torch.Tensor, topk_weights: Optional[torch.Tensor]) -> torch.Tensor:
    """out[t] = bf16(sum over k with topk_idx[t][k] >= 0 of w[t][k] * slot (t, k)), fp32 in k order."""
    N, K = topk_idx.shape
    H = slots.shape[1]
    s = slots.float().view(N, K, H)
    w = topk_weights.float() if topk_weights is not None else torch.ones((N, K))
    acc = torch.zeros((N, H), dtype=torch.float32)
    for k in range(K):
        acc += torch.where((topk_idx[:, k] >= 0).unsqueeze(1), w[:, k:k + 1] * s[:, k], torch.zeros_like(acc))
    return acc.to(torch.bfloat16)


class GemmCombine:
    """One GEMM-combine region per rank of `group`: slots for `num_max_tokens x num_topk` bf16 rows
    of `hidden` (the same on every rank). Construction is collective."""

    def __init__(self, group: dist.ProcessGroup, num_max_tokens: int, num_topk: int, hidden: int,
                 timeout_secs: Optional[float] = None):
        if num_max_tokens * num_topk > MAX_SLOTS:
            raise ValueError(f'num_max_tokens * num_topk must not exceed {MAX_SLOTS}')
        if hidden % 128:
            raise ValueError('hidden must be a multiple of 128')
        self.group = group
        self.num_max_tokens, self.num_topk, self.hidden = int(num_max_tokens), int(num_topk), int(hidden)
        self.region = SymmetricRegion(group, self.size_hint(num_max_tokens, num_topk, hidden), timeout_secs)

    @staticmethod
    def size_hint(num_max_tokens: int, num_topk: int, hidden: int) -> int:
        """Bytes of slot storage per rank."""
        return int(num_max_tokens) * int(num_topk) * int(hidden) * 2

    def send(self, a: torch.Tensor, a_scales: torch.Tensor, w: torch.Tensor, w_scales: torch.Tensor,
             expert_offsets: torch.Tensor, expert_counts: Optional[torch.Tensor], row_map: torch.Tensor,
             handle: Tuple, keep_local: bool = True, num_sms: int = 0) -> Optional[torch.Tensor]:
        """Grouped FP8 GEMM `a @ w[e]^T` (fp32 1x128 / 128x128 scales) whose rows go to their tokens'
        source ranks; returns the rows (`[rows, hidden]` bf16) when `keep_local` (the backward of
        the routing weights needs them), else None."""
        rank_prefix_matrix, _, _, recv_src_idx = handle[:4]
        if w.shape[1] != self.hidden:
            raise ValueError(f'the weights produce {w.shape[1]} columns, the region holds rows of {self.hidden}')
        if row_map.shape[1] != self.num_topk:
            raise ValueError(f'row_map has top-k {row_map.shape[1]}, the region {self.num_topk}')
        y = self.region.runtime.gemm_combine_send(a, a_scales, w, w_scales, expert_offsets.to(torch.int32).contiguous(),
                                                  None if expert_counts is None else expert_counts.to(torch.int32).contiguous(),
                                                  row_map.contiguous(), recv_src_idx.contiguous(),
                                                  rank_prefix_matrix.contiguous(), bool(keep_local), int(num_sms))
        return y if keep_local else None

    def reduce(self, topk_idx: torch.Tensor, topk_weights: Optional[torch.Tensor] = None,
               num_sms: int = 0) -> torch.Tensor:
        """This rank's tokens: the top-k weighted fp32 sum of their slots, bf16 `[num_tokens, hidden]`."""
        if topk_idx.shape[0] > self.num_max_tokens:
            raise ValueError(f'{topk_idx.shape[0]} tokens exceed the region ({self.num_max_tokens})')
        w = None if topk_weights is None else topk_weights.float().contiguous()
        return self.region.runtime.gemm_combine_reduce(topk_idx.to(torch.int64).contiguous(), w, int(num_sms))

    def __call__(self, a, a_scales, w, w_scales, expert_offsets, expert_counts, row_map, handle, topk_idx,
                 topk_weights=None, keep_local: bool = True) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
        y = self.send(a, a_scales, w, w_scales, expert_offsets, expert_counts, row_map, handle, keep_local)
        return self.reduce(topk_idx, topk_weights), y

    def check_error(self) -> None:
        self.region.check_error()

    def destroy(self) -> None:
        """Collective: every rank's kernels finish and the ranks meet before any region is unmapped."""
        if self.region is not None:
            torch.cuda.synchronize()
            dist.barrier(self.group)
            self.region.destroy()
            self.region = None


def max_tokens_over_group(group: dist.ProcessGroup, num_tokens: int, device) -> int:
    """The largest token count of any rank (the region size every rank must agree on)."""
    t = torch.tensor([int(num_tokens)], dtype=torch.int64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return int(t.item())


__all__: List[str] = ['GemmCombine', 'row_destinations', 'exchange_reference', 'reduce_reference',
                      'max_tokens_over_group']
