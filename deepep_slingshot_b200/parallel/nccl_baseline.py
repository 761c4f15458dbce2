"""The NCCL all-to-all baseline: expert-parallel dispatch / combine as a PyTorch user would write them
with `torch.distributed.all_to_all_single` over NCCL, with no custom kernel.

It is what the fused NVLink kernels are measured against (the "path that only calls NCCL
all-to-all"), not the product. Same `Buffer` API and the same receive order as the NVLink kernels
(rows grouped by source rank, then by source token index), so the EP benchmark checks it exactly
against the oracle before timing it. Written for speed rather than as an oracle:
  * routing is vectorized (one destination mask, one `nonzero` for the send order);
  * each dispatch moves one packed row per (token, destination): FP8 row (quantized with torch ops)
    or bf16 row, fp32 scales, int64 top-k ids, fp32 top-k weights and the int64 source index, in a
    single `all_to_all_single`; the counts travel in a first, tiny one (the host needs them to size
    the payload: one sync), and the per-expert counts list needs a second sync;
  * combine sends the bf16 rows (+ fp32 weights) back in one `all_to_all_single` and sums them per
    token with `index_add_` in fp32; no host sync.
The cached dispatch (handle reuse) skips the routing and the count exchange.
"""
from typing import Optional, Tuple, Union

import torch
import torch.distributed as dist

from ..utils.math import align, per_token_cast_to_fp8


class _Done:
    """Event stand-in: NCCL calls are stream-ordered, nothing to wait for."""

    def current_stream_wait(self) -> None:
        pass


def _byte_cols(t: torch.Tensor) -> torch.Tensor:
    return t.contiguous().view(torch.uint8).reshape(t.shape[0], -1)


class NcclAllToAllEP:
    """Dispatch / combine over `all_to_all_single` (NCCL on GPUs): the baseline arm of the benchmark."""

    def __init__(self, group: dist.ProcessGroup, **_unused) -> None:
        self.group = group
        self.rank = group.rank()
        self.group_size = group.size()

    def _dest_mask(self, topk_idx: torch.Tensor, num_experts: int) -> torch.Tensor:
        R = self.group_size
        valid = topk_idx >= 0
        dst = torch.where(valid, topk_idx // (num_experts // R), torch.full_like(topk_idx, R))
        mask = torch.zeros((topk_idx.shape[0], R + 1), dtype=torch.bool, device=topk_idx.device)
        mask.scatter_(1, dst, True)
        return mask[:, :R]

    def get_dispatch_layout(self, topk_idx: torch.Tensor, num_experts: int, previous_event=None, async_finish=False,
                            allocate_on_comm_stream=False):
        valid = topk_idx >= 0
        per_expert = torch.bincount(topk_idx[valid], minlength=num_experts).to(torch.int32)
        mask = self._dest_mask(topk_idx, num_experts)
        return mask.sum(0).to(torch.int32), None, per_expert, mask, _Done()

    def dispatch(self, x: Union[torch.Tensor, Tuple[torch.Tensor, torch.Tensor]], handle: Optional[tuple] = None,
                 num_tokens_per_rank=None, num_tokens_per_rdma_rank=None, is_token_in_rank=None,
                 num_tokens_per_expert=None, topk_idx=None, topk_weights=None, expert_alignment: int = 1,
                 num_worst_tokens: int = 0, config=None, previous_event=None, async_finish=False,
                 allocate_on_comm_stream=False, num_experts: Optional[int] = None, quantize_fp8: bool = False,
                 round_scale: bool = False):
        R, me = self.group_size, self.rank
        x, x_scales = x if isinstance(x, tuple) else (x, None)
        if quantize_fp8:
            x, x_scales = per_token_cast_to_fp8(x, round_scale=round_scale)
        N, H = x.shape
        dev = x.device
        if handle is not None:
            order, send_counts, recv_counts, recv_src_idx, itir, send_head = handle
            topk_idx = topk_weights = None
        else:
            if num_experts is None:
                num_experts = num_tokens_per_expert.numel()
            itir = is_token_in_rank if is_token_in_rank is not None else self._dest_mask(topk_idx, num_experts)
            pairs = itir.t().nonzero()                      # (destination, token), destination-major
            order = pairs[:, 1]
            counts = itir.sum(0).to(torch.int64)
            rc = torch.empty(R, dtype=torch.int64, device=dev)
            dist.all_to_all_single(rc, counts, group=self.group)
            send_counts, recv_counts = counts.tolist(), rc.tolist()
            starts = torch.cumsum(counts, 0) - counts
            send_head = torch.full((N, R), -1, dtype=torch.int32, device=dev)
            send_head[order, pairs[:, 0]] = (torch.arange(order.numel(), device=dev) - starts[pairs[:, 0]]).to(torch.int32)
        cols = [_byte_cols(x)]
        if x_scales is not None:
            cols.append(_byte_cols(x_scales.float()))
        K = topk_idx.shape[1] if topk_idx is not None else 0
        if K:
            cols.append(_byte_cols(topk_idx.to(torch.int64)))
            w = topk_weights if topk_weights is not None else torch.zeros((N, K), device=dev)
            cols.append(_byte_cols(w.float()))
        if handle is None:
            cols.append(_byte_cols(torch.arange(N, device=dev, dtype=torch.int64).unsqueeze(1)))
        packed = torch.cat(cols, dim=1).index_select(0, order)
        row_bytes = packed.shape[1]
        recv = torch.empty((sum(recv_counts), row_bytes), dtype=torch.uint8, device=dev)
        dist.all_to_all_single(recv.view(-1), packed.view(-1), [c * row_bytes for c in recv_counts],
                               [c * row_bytes for c in send_counts], group=self.group)
        off = H * x.element_size()
        recv_x = recv[:, :off].contiguous().view(x.dtype)
        recv_scales = None
        if x_scales is not None:
            nb = x_scales.shape[1]
            recv_scales = recv[:, off:off + 4 * nb].contiguous().view(torch.float32)
            off += 4 * nb
        recv_topk_idx = recv_topk_weights = None
        per_expert_list = []
        if K:
            g = recv[:, off:off + 8 * K].contiguous().view(torch.int64)
            w = recv[:, off + 8 * K:off + 12 * K].contiguous().view(torch.float32)
            off += 12 * K
            epr = num_experts // R
            mine = (g >= me * epr) & (g < (me + 1) * epr)
            recv_topk_idx = torch.where(mine, g - me * epr, torch.full_like(g, -1))
            recv_topk_weights = torch.where(mine, w, torch.zeros_like(w))
            counts_e = torch.bincount(recv_topk_idx[mine], minlength=epr)
            per_expert_list = [align(c, expert_alignment) for c in counts_e.tolist()]
        if handle is None:
            recv_src_idx = recv[:, off:off + 8].contiguous().view(torch.int64).flatten().to(torch.int32)
            # fields 3..5 as in `Buffer`'s handle: source index, destination mask, send_head
            new_handle = (order, send_counts, recv_counts, recv_src_idx, itir, send_head)
        else:
            new_handle = handle
        if num_worst_tokens > 0:
            pad = num_worst_tokens - recv_x.shape[0]
            assert pad >= 0, 'num_worst_tokens is smaller than the received rows'
            recv_x = torch.cat([recv_x, recv_x.new_zeros((pad, H))])
            if recv_scales is not None:
                recv_scales = torch.cat([recv_scales, recv_scales.new_zeros((pad, recv_scales.shape[1]))])
            if recv_topk_idx is not None:
                recv_topk_idx = torch.cat([recv_topk_idx, recv_topk_idx.new_full((pad, K), -1)])
                recv_topk_weights = torch.cat([recv_topk_weights, recv_topk_weights.new_zeros((pad, K))])
            per_expert_list = []
        out_x = (recv_x, recv_scales) if recv_scales is not None else recv_x
        return out_x, recv_topk_idx, recv_topk_weights, per_expert_list, new_handle, _Done()

    def combine(self, x: torch.Tensor, handle: tuple, topk_weights: Optional[torch.Tensor] = None,
                bias: Union[torch.Tensor, Tuple[torch.Tensor, torch.Tensor], None] = None, config=None,
                previous_event=None, async_finish=False, allocate_on_comm_stream=False):
        order, send_counts, recv_counts, _, _, send_head = handle
        N, H = send_head.shape[0], x.shape[1]
        n_recv = sum(recv_counts)
        cols = [_byte_cols(x[:n_recv].to(torch.bfloat16))]
        K = topk_weights.shape[1] if topk_weights is not None else 0
        if K:
            cols.append(_byte_cols(topk_weights[:n_recv].float()))
        rows = torch.cat(cols, dim=1) if len(cols) > 1 else cols[0]
        row_bytes = rows.shape[1]
        back = torch.empty((order.numel(), row_bytes), dtype=torch.uint8, device=x.device)
        dist.all_to_all_single(back.view(-1), rows.contiguous().view(-1), [c * row_bytes for c in send_counts],
                               [c * row_bytes for c in recv_counts], group=self.group)
        acc = torch.zeros((N, H), dtype=torch.float32, device=x.device)
        acc.index_add_(0, order, back[:, :2 * H].contiguous().view(torch.bfloat16).float())
        out_w = None
        if K:
            out_w = torch.zeros((N, K), dtype=torch.float32, device=x.device)
            out_w.index_add_(0, order, back[:, 2 * H:].contiguous().view(torch.float32))
        if bias is not None:
            for b in (bias if isinstance(bias, tuple) else (bias,)):
                acc += b.float()
        return acc.to(torch.bfloat16), out_w, _Done()
