"""Pure-PyTorch reference backend: the correctness oracle of every GPU kernel, and the CPU/gloo path.

`ReferenceBuffer` has the same methods and return values as `Buffer` (`get_dispatch_layout`,
`dispatch`, `combine`, `low_latency_dispatch`, `low_latency_combine`) but moves bytes with
`torch.distributed.all_to_all_single` over any backend (gloo on CPU ranks, NCCL on GPUs). It follows
the reference's independent-oracle design: a variable-size all-to-all byte transport of payload,
scales, ids, weights and source ids (`backend/tests/common.py:36-65`) and the single-process
reference dispatch/combine of DeepEP ([DE]deep_ep/utils/refs.py:10-243).

Receive order is the one the NVLink kernels produce: grouped by source rank, then by source token
index, so normal-mode results compare exactly. Low-latency rows are compacted per local expert and
sorted by (source rank, token) here; the GPU order inside an expert is arrival order, so tests
compare per-expert row sets.
"""
from typing import List, Optional, Tuple, Union

import torch
import torch.distributed as dist

from ..utils.math import align, per_token_cast_to_fp8


class _Evt:
    """Stand-in event for the synchronous reference (nothing to wait for)."""

    def current_stream_wait(self) -> None:
        pass


def _as_bytes(t: torch.Tensor) -> torch.Tensor:
    cols = t.element_size()
    for d in t.shape[1:]:
        cols *= d
    return t.contiguous().view(torch.uint8).reshape(t.shape[0], cols)


def _from_bytes(b: torch.Tensor, dtype: torch.dtype, cols: int) -> torch.Tensor:
    # a fresh copy: a one-row slice counts as contiguous but keeps the parent's row stride and offset
    return torch.empty(b.shape, dtype=b.dtype, device=b.device).copy_(b).view(dtype).reshape(b.shape[0], cols)


class ReferenceBuffer:
    """Synchronous pure-torch EP buffer with the `Buffer` API (see module docstring)."""

    def __init__(self, group: dist.ProcessGroup, num_nvl_bytes: int = 0, num_rdma_bytes: int = 0,
                 low_latency_mode: bool = False, **_unused) -> None:
        self.group = group
        self.rank = group.rank()
        self.group_size = group.size()
        self.num_nvl_bytes = num_nvl_bytes
        self.num_rdma_bytes = num_rdma_bytes
        self.low_latency_mode = low_latency_mode

    # ------------------------------------------------------------------ transport
    def _exchange(self, rows: torch.Tensor, send_counts: List[int]) -> Tuple[torch.Tensor, List[int]]:
        """Variable all-to-all of uint8 rows [n, row_bytes]; returns (received rows, recv counts)."""
        R = self.group_size
        dev = rows.device
        sc = torch.tensor(send_counts, dtype=torch.int64, device=dev)
        rc = torch.empty(R, dtype=torch.int64, device=dev)
        dist.all_to_all_single(rc, sc, group=self.group)
        recv_counts = rc.tolist()
        row_bytes = rows.shape[1]
        out = torch.empty((sum(recv_counts), row_bytes), dtype=torch.uint8, device=dev)
        dist.all_to_all_single(out.view(-1), rows.reshape(-1), [c * row_bytes for c in recv_counts],
                               [c * row_bytes for c in send_counts], group=self.group)
        return out, recv_counts

    # ------------------------------------------------------------------ layout
    def get_dispatch_layout(self, topk_idx: torch.Tensor, num_experts: int, previous_event=None, async_finish=False,
                            allocate_on_comm_stream=False):
        R = self.group_size
        epr = num_experts // R
        valid = topk_idx >= 0
        num_tokens_per_expert = torch.zeros(num_experts, dtype=torch.int32, device=topk_idx.device)
        ids = topk_idx[valid]
        num_tokens_per_expert.scatter_add_(0, ids, torch.ones_like(ids, dtype=torch.int32))
        dst = torch.where(valid, topk_idx // epr, torch.full_like(topk_idx, -1))
        is_token_in_rank = torch.zeros((topk_idx.shape[0], R), dtype=torch.bool, device=topk_idx.device)
        for r in range(R):
            is_token_in_rank[:, r] = (dst == r).any(dim=1)
        num_tokens_per_rank = is_token_in_rank.sum(dim=0).to(torch.int32)
        return num_tokens_per_rank, None, num_tokens_per_expert, is_token_in_rank, _Evt()

    # ------------------------------------------------------------------ normal mode
    def dispatch(self, x: Union[torch.Tensor, Tuple[torch.Tensor, torch.Tensor]], handle: Optional[tuple] = None,
                 num_tokens_per_rank=None, num_tokens_per_rdma_rank=None, is_token_in_rank=None,
                 num_tokens_per_expert=None, topk_idx=None, topk_weights=None, expert_alignment: int = 1,
                 num_worst_tokens: int = 0, config=None, previous_event=None, async_finish=False,
                 allocate_on_comm_stream=False, num_experts: Optional[int] = None, quantize_fp8: bool = False,
                 round_scale: bool = False):
        R, me = self.group_size, self.rank
        x, x_scales = x if isinstance(x, tuple) else (x, None)
        if quantize_fp8:
            assert x_scales is None
            x, x_scales = per_token_cast_to_fp8(x, round_scale=round_scale)
        N, H = x.shape
        cached = handle is not None
        if cached:
            is_token_in_rank = handle[4]
            topk_idx = topk_weights = None
        if num_experts is None and num_tokens_per_expert is not None:
            num_experts = num_tokens_per_expert.numel()
        if is_token_in_rank is None:
            _, _, _, is_token_in_rank, _ = self.get_dispatch_layout(topk_idx, num_experts)
        K = topk_idx.shape[1] if topk_idx is not None else 0
        parts, send_counts, send_head = [], [], torch.full((N, R), -1, dtype=torch.int32, device=x.device)
        for r in range(R):
            idx = torch.nonzero(is_token_in_rank[:, r]).flatten()
            send_head[idx, r] = torch.arange(idx.numel(), dtype=torch.int32, device=x.device)
            cols = [_as_bytes(x[idx])]
            if x_scales is not None:
                cols.append(_as_bytes(x_scales[idx].float()))
            if topk_idx is not None:
                cols.append(_as_bytes(topk_idx[idx].to(torch.int64)))
                w = topk_weights[idx] if topk_weights is not None else torch.zeros((idx.numel(), K), device=x.device)
                cols.append(_as_bytes(w.float()))
            cols.append(_as_bytes(idx.to(torch.int64).unsqueeze(1)))
            parts.append(torch.cat(cols, dim=1))
            send_counts.append(idx.numel())
        rows, recv_counts = self._exchange(torch.cat(parts, dim=0), send_counts)
        off = 0
        xb = H * x.element_size()
        recv_x = _from_bytes(rows[:, off:off + xb], x.dtype, H)
        off += xb
        recv_scales = None
        if x_scales is not None:
            nb = x_scales.shape[1]
            recv_scales = _from_bytes(rows[:, off:off + 4 * nb], torch.float32, nb)
            off += 4 * nb
        recv_topk_idx = recv_topk_weights = None
        num_recv_tokens_per_expert_list = []
        if topk_idx is not None:
            g = _from_bytes(rows[:, off:off + 8 * K], torch.int64, K)
            off += 8 * K
            w = _from_bytes(rows[:, off:off + 4 * K], torch.float32, K)
            off += 4 * K
            epr = num_experts // R
            mine = (g >= me * epr) & (g < (me + 1) * epr)
            recv_topk_idx = torch.where(mine, g - me * epr, torch.full_like(g, -1))
            recv_topk_weights = torch.where(mine, w, torch.zeros_like(w))
            for e in range(epr):
                num_recv_tokens_per_expert_list.append(align(int((recv_topk_idx == e).sum().item()), expert_alignment))
        recv_src_idx = _from_bytes(rows[:, off:off + 8], torch.int64, 1).flatten().to(torch.int32)
        rc = torch.tensor(recv_counts, dtype=torch.int64)
        # rank_prefix_matrix[s][r] = tokens from sources <= s to r: gather every rank's send counts
        all_counts = [torch.zeros(R, dtype=torch.int64, device=x.device) for _ in range(R)]
        dist.all_gather(all_counts, torch.tensor(send_counts, dtype=torch.int64, device=x.device), group=self.group)
        matrix = torch.stack(all_counts).to(torch.int32)  # [src][dst]
        rank_prefix_matrix = matrix.cumsum(dim=0).to(torch.int32)
        send_prefix_matrix = (matrix.cumsum(dim=1) - matrix).to(torch.int32)
        recv_rank_prefix = torch.cat([torch.zeros(1, dtype=torch.int64), rc.cumsum(0)]).to(torch.int32).to(x.device)
        handle = (rank_prefix_matrix, send_prefix_matrix, recv_rank_prefix, recv_src_idx, is_token_in_rank, send_head)
        if num_worst_tokens > 0:
            pad = num_worst_tokens - recv_x.shape[0]
            assert pad >= 0
            recv_x = torch.cat([recv_x, torch.zeros((pad, H), dtype=recv_x.dtype, device=x.device)])
            if recv_scales is not None:
                recv_scales = torch.cat([recv_scales, torch.zeros((pad, recv_scales.shape[1]), device=x.device)])
            if recv_topk_idx is not None:
                recv_topk_idx = torch.cat([recv_topk_idx, torch.full((pad, K), -1, dtype=torch.int64, device=x.device)])
                recv_topk_weights = torch.cat([recv_topk_weights, torch.zeros((pad, K), device=x.device)])
            num_recv_tokens_per_expert_list = []
        out_x = (recv_x, recv_scales) if recv_scales is not None else recv_x
        if cached:
            recv_topk_idx = recv_topk_weights = None
        return out_x, recv_topk_idx, recv_topk_weights, num_recv_tokens_per_expert_list, handle, _Evt()

    def combine(self, x: torch.Tensor, handle: tuple, topk_weights: Optional[torch.Tensor] = None,
                bias: Union[torch.Tensor, Tuple[torch.Tensor, torch.Tensor], None] = None, config=None,
                previous_event=None, async_finish=False, allocate_on_comm_stream=False,
                row_map: Optional[torch.Tensor] = None, row_weights: Optional[torch.Tensor] = None):
        R, me = self.group_size, self.rank
        rank_prefix_matrix, _, recv_rank_prefix, recv_src_idx, is_token_in_rank, send_head = handle
        N = send_head.shape[0]
        H = x.shape[1]
        num_recv = int(recv_rank_prefix[-1].item())
        if row_map is not None:
            # Expanded mode: fp32 sum of each received token's local rows, weighted by row_weights,
            # rounded to bf16 before the exchange (the row that crosses the link).
            rm = row_map[:num_recv].long()
            wts = row_weights[:num_recv].float() if row_weights is not None else torch.ones(rm.shape, device=x.device)
            valid = rm >= 0
            rows_f = x.float()[rm.clamp(min=0)] * (wts * valid).unsqueeze(-1)
            x = torch.zeros((num_recv, H), dtype=torch.float32, device=x.device)
            for k in range(rm.shape[1]):  # k order, as the kernel accumulates
                x += rows_f[:, k]
            x = x.to(torch.bfloat16)
        x = x[:num_recv]
        K = topk_weights.shape[1] if topk_weights is not None else 0
        counts = (recv_rank_prefix[1:] - recv_rank_prefix[:-1]).tolist()
        cols = [_as_bytes(x.to(torch.bfloat16))]
        if topk_weights is not None:
            cols.append(_as_bytes(topk_weights[:num_recv].float()))
        rows, back_counts = self._exchange(torch.cat(cols, dim=1), counts)
        back_x = _from_bytes(rows[:, :2 * H], torch.bfloat16, H).float()
        acc = torch.zeros((N, H), dtype=torch.float32, device=x.device)
        acc_w = torch.zeros((N, K), dtype=torch.float32, device=x.device) if K else None
        off = 0
        for r in range(R):
            idx = torch.nonzero(is_token_in_rank[:, r]).flatten()
            n = back_counts[r]
            assert n == idx.numel()
            acc.index_add_(0, idx, back_x[off:off + n])
            if K:
                acc_w.index_add_(0, idx, _from_bytes(rows[off:off + n, 2 * H:2 * H + 4 * K], torch.float32, K))
            off += n
        if bias is not None:
            for b in (bias if isinstance(bias, tuple) else (bias,)):
                acc += b.float()
        return acc.to(torch.bfloat16), acc_w, _Evt()

    # ------------------------------------------------------------------ low-latency mode
    def low_latency_dispatch(self, x: torch.Tensor, topk_idx: torch.Tensor, num_max_dispatch_tokens_per_rank: int,
                             num_experts: int, cumulative_local_expert_recv_stats=None,
                             dispatch_wait_recv_cost_stats=None, use_fp8: bool = True, round_scale: bool = False,
                             use_ue8m0: bool = False, async_finish: bool = False, return_recv_hook: bool = False):
        R, me = self.group_size, self.rank
        N, H = x.shape
        K = topk_idx.shape[1]
        epr = num_experts // R
        maxT = num_max_dispatch_tokens_per_rank
        if use_fp8:
            q, s = per_token_cast_to_fp8(x, round_scale=round_scale)
        parts, counts = [], []
        for r in range(R):
            t_idx, k_idx = torch.nonzero((topk_idx >= r * epr) & (topk_idx < (r + 1) * epr), as_tuple=True)
            e_local = topk_idx[t_idx, k_idx] - r * epr
            cols = [_as_bytes(q[t_idx]), _as_bytes(s[t_idx])] if use_fp8 else [_as_bytes(x[t_idx].to(torch.bfloat16))]
            meta = torch.stack([e_local, t_idx.to(torch.int64), torch.full_like(t_idx, me), k_idx.to(torch.int64)], dim=1)
            cols.append(_as_bytes(meta))
            parts.append(torch.cat(cols, dim=1))
            counts.append(t_idx.numel())
        rows, _ = self._exchange(torch.cat(parts, dim=0), counts)
        xb = H if use_fp8 else 2 * H
        nb = H // 128
        off = xb + (4 * nb if use_fp8 else 0)
        meta = _from_bytes(rows[:, off:off + 32], torch.int64, 4)
        slots = R * maxT
        dt = torch.float8_e4m3fn if use_fp8 else torch.bfloat16
        packed_x = torch.zeros((epr, slots, H), dtype=dt, device=x.device)
        packed_s = torch.zeros((epr, slots, nb), dtype=torch.float32, device=x.device) if use_fp8 else None
        src_info = torch.full((epr, slots), -1, dtype=torch.int32, device=x.device)
        src_meta = torch.full((epr, slots), -1, dtype=torch.int32, device=x.device)
        recv_count = torch.zeros(epr, dtype=torch.int32, device=x.device)
        layout_range = torch.zeros((epr, R), dtype=torch.int64, device=x.device)
        for e in range(epr):
            sel = torch.nonzero(meta[:, 0] == e).flatten()
            key = meta[sel, 2] * (maxT + 1) + meta[sel, 1]
            sel = sel[torch.argsort(key)]
            n = sel.numel()
            recv_count[e] = n
            packed_x[e, :n] = _from_bytes(rows[sel, :xb], dt, H)
            if use_fp8:
                packed_s[e, :n] = _from_bytes(rows[sel, xb:xb + 4 * nb], torch.float32, nb)
            src_info[e, :n] = meta[sel, 1].to(torch.int32)
            src_meta[e, :n] = (meta[sel, 2] * K + meta[sel, 3]).to(torch.int32)
            for r in range(R):
                layout_range[e, r] = int((meta[sel, 2] == r).sum().item())
        if cumulative_local_expert_recv_stats is not None:
            cumulative_local_expert_recv_stats += recv_count
        recv = (packed_x, packed_s) if use_fp8 else packed_x
        handle = (src_info, layout_range, maxT, H, num_experts, recv_count, 0, src_meta)
        hook = (lambda: None) if return_recv_hook else None
        return recv, recv_count, handle, _Evt(), hook

    def low_latency_combine(self, x: torch.Tensor, topk_idx: torch.Tensor, topk_weights: torch.Tensor, handle: tuple,
                            use_logfmt: bool = False, zero_copy: bool = False, async_finish: bool = False,
                            return_recv_hook: bool = False, out: Optional[torch.Tensor] = None,
                            combine_wait_recv_cost_stats=None):
        R, me = self.group_size, self.rank
        src_info, layout_range, maxT, H, num_experts, recv_count, _, src_meta = handle
        K = topk_idx.shape[1]
        epr = num_experts // R
        if use_logfmt:
            from ..utils.math import logfmt10_roundtrip
            x = logfmt10_roundtrip(x)
        parts, counts = [], []
        for r in range(R):
            rows_r = []
            for e in range(epr):
                n = int(recv_count[e].item())
                sel = torch.nonzero(src_meta[e, :n] // K == r).flatten()
                t = src_info[e, sel].to(torch.int64)
                k = (src_meta[e, sel] % K).to(torch.int64)
                meta = torch.stack([t, k], dim=1)
                rows_r.append(torch.cat([_as_bytes(x[e, sel].float()), _as_bytes(meta)], dim=1))
            part = torch.cat(rows_r, dim=0) if rows_r else torch.empty((0, 4 * H + 16), dtype=torch.uint8, device=x.device)
            parts.append(part)
            counts.append(part.shape[0])
        rows, _ = self._exchange(torch.cat(parts, dim=0), counts)
        vals = _from_bytes(rows[:, :4 * H], torch.float32, H)
        meta = _from_bytes(rows[:, 4 * H:4 * H + 16], torch.int64, 2)
        N = topk_idx.shape[0]
        w = topk_weights[meta[:, 0], meta[:, 1]].float().unsqueeze(1)
        acc = torch.zeros((N, H), dtype=torch.float32, device=x.device)
        acc.index_add_(0, meta[:, 0], vals * w)
        res = acc.to(torch.bfloat16)
        if out is not None:
            out.copy_(res)
            res = out
        hook = (lambda: None) if return_recv_hook else None
        return res, _Evt(), hook
