"""Expert-parallel SwiGLU MoE FFN layer (forward + backward) on the B200 kernels.

Forward per rank (every step on hand-written sm_100a kernels):
  dispatch (FP8 1x128 quantization fused) -> permute (expert-grouped, 128-aligned) ->
  grouped FP8 GEMM gate/up (tcgen05, 1x128 x 128x128 block scales) -> fused SwiGLU + FP8 requant ->
  grouped FP8 GEMM down -> combine with the top-k weighted reduction of each token's grouped rows
  fused into its sender side (one kernel: weighted fp32 sum, bf16 cast, NVLink push, sum over ranks).
Backward: combine^T = cached dispatch of the output gradient; unpermute^T (the gradient scattered to
the grouped rows, scaled by the routing weights, and the routing weights' gradient in one kernel);
the expert GEMM gradients in bf16 (straight-through through the FP8 quantization) as this library's
tcgen05 grouped GEMMs with MN-major operands (no transposes) and the fused SwiGLU backward kernel;
permute^T + dispatch^T = the weighted-expanded combine. Every alignment padding row stays zero, so
the grouped GEMMs run over whole 128-row groups without masks.

The reference library has no model layer (its expert compute is SGLang + DeepGEMM,
backend/tests/sglang_dispatcher_smoke.py:107-124); this is the flagship workload of the benchmark
config "full MoE layer forward+backward".
"""
import os
from types import SimpleNamespace
from typing import Optional

import torch

from ..ops.gemm import grouped_gemm_fp8, quantize_weights_fp8
from ..ops.permute import permute, unpermute_backward, zero_group_padding
from ..ops.quant import per_token_cast_back, swiglu_backward
from .._ext import require_ext


# Backward expert GEMMs: `tcgen05_mn` (default: this library's tcgen05 grouped bf16 GEMMs reading the
# weights and activations as they lie through MN-major operand descriptors, no transposes), `tcgen05`
# (the same kernels with K-major operands: the weights are transposed every step), `grouped`
# (torch's grouped bf16 GEMM, a library stand-in kept for A/B), `loop` (per-expert matmuls).
# DEEPEP_B200_MOE_FUSED_DISPATCH=1: the forward's dispatch receive and gate/up GEMM run as one kernel
# (Buffer.dispatch_gemm) instead of dispatch -> permute -> grouped GEMM.
_FUSED_DISPATCH = {'enabled': os.environ.get('DEEPEP_B200_MOE_FUSED_DISPATCH', '0') == '1'}
_BWD = {'mode': os.environ.get('DEEPEP_B200_MOE_BWD', 'tcgen05_mn')}
# DEEPEP_B200_MOE_UE8M0=1: every FP8 scale of the forward (dispatched activations, weights, SwiGLU
# output) is a power of two, and the grouped GEMMs let the tensor core apply the scales
# (`grouped_gemm_fp8(..., ue8m0=True)`, kind::mxf8f6f4.block_scale) instead of promoting every K block.
_UE8M0 = {'enabled': os.environ.get('DEEPEP_B200_MOE_UE8M0', '0') == '1'}
# DEEPEP_B200_MOE_FUSED_COMBINE=1: the down projection's epilogue sends every row into its token's
# combine slot on the source rank and the source reduces its slots (parallel.gemm_combine) instead of
# grouped GEMM -> weighted expanded combine. fp32-scale GEMMs after the plain dispatch only (not with
# UE8M0 or the fused dispatch, whose handle rows past the received count are not row-mapped).
_FUSED_COMBINE = {'enabled': os.environ.get('DEEPEP_B200_MOE_FUSED_COMBINE', '0') == '1'}


def _aligned_rows(per_expert, alignment: int = 128) -> int:
    """Rows of the expert-grouped layout from the host's per-expert counts (no device read)."""
    return sum((c + alignment - 1) // alignment * alignment for c in per_expert)


def _expert_grads(g_y, a, h, xf, offsets, counts, w1, w2, inter):
    """(g_xp [R, H], g_w1, g_w2) of the expert FFNs over the grouped rows [0, R): padding rows of every
    operand are zero, so whole 128-aligned groups can be multiplied. The SwiGLU backward is the
    library's kernel in every mode."""
    offs32 = offsets.to(torch.int32).contiguous()
    mode = _BWD['mode']
    if mode in ('tcgen05_mn', 'tcgen05'):
        from ..ops.gemm import grouped_gemm_bf16, grouped_gemm_bf16_wgrad, grouped_gemm_bf16_wgrad_rows
        if mode == 'tcgen05_mn':
            g_a = grouped_gemm_bf16(g_y, w2, offs32, counts, b_mn_major=True)             # [R, I]
            g_w2 = grouped_gemm_bf16_wgrad_rows(g_y, a, offs32)                           # [E, H, I]
            g_h = swiglu_backward(h, g_a)                                                 # [R, 2I]
            g_xp = grouped_gemm_bf16(g_h, w1, offs32, counts, b_mn_major=True)            # [R, H]
            g_w1 = grouped_gemm_bf16_wgrad_rows(g_h, xf, offs32)                          # [E, 2I, H]
            return g_xp, g_w1, g_w2
        g_a = grouped_gemm_bf16(g_y, w2.transpose(1, 2).contiguous(), offs32, counts)
        g_w2 = grouped_gemm_bf16_wgrad(g_y.t().contiguous(), a.t().contiguous(), offs32)
        g_h = swiglu_backward(h, g_a)
        g_xp = grouped_gemm_bf16(g_h, w1.transpose(1, 2).contiguous(), offs32, counts)
        g_w1 = grouped_gemm_bf16_wgrad(g_h.t().contiguous(), xf.t().contiguous(), offs32)
        return g_xp, g_w1, g_w2
    if mode == 'grouped' and hasattr(torch, '_grouped_mm'):
        offs = offs32[1:]
        g_a = torch._grouped_mm(g_y, w2, offs=offs)
        g_w2 = torch._grouped_mm(g_y.t(), a, offs=offs)
        g_h = swiglu_backward(h, g_a.contiguous())
        g_xp = torch._grouped_mm(g_h, w1, offs=offs)
        g_w1 = torch._grouped_mm(g_h.t(), xf, offs=offs)
        empty = counts == 0
        g_w1[empty] = 0
        g_w2[empty] = 0
        return g_xp, g_w1.contiguous(), g_w2.contiguous()
    g_xp = torch.zeros_like(xf)
    g_w1, g_w2 = torch.zeros_like(w1), torch.zeros_like(w2)
    off, cnt = offsets.tolist(), counts.tolist()
    for e in range(w1.shape[0]):
        r0, r1 = off[e], off[e] + cnt[e]
        if r1 <= r0:
            continue
        g_a = g_y[r0:r1] @ w2[e]
        g_w2[e] = g_y[r0:r1].t() @ a[r0:r1]
        g_h = swiglu_backward(h[r0:r1].contiguous(), g_a.contiguous())
        g_xp[r0:r1] = g_h @ w1[e]
        g_w1[e] = g_h.t() @ xf[r0:r1]
    return g_xp, g_w1, g_w2


class _MoEFunction(torch.autograd.Function):

    @staticmethod
    def forward(ctx, x, topk_idx, topk_weights, w1, w2, buffer, num_experts, config, gemm_combine=None):
        E_l = w1.shape[0]
        inter = w1.shape[1] // 2
        ue8m0 = _UE8M0['enabled'] and not _FUSED_DISPATCH['enabled']
        if _FUSED_DISPATCH['enabled']:
            w1q, w1s = quantize_weights_fp8(w1.detach())
            # Dispatch receive and gate/up GEMM in one launch, tile by tile (Buffer.dispatch_gemm).
            h, grp, handle = buffer.dispatch_gemm(x, topk_idx, topk_weights.float().contiguous(), num_experts, w1q,
                                                  w1s.contiguous())
            p = SimpleNamespace(x=grp['x'], scales=grp['scales'], row_map=grp['row_map'],
                                expert_offsets=grp['expert_offsets'], expert_counts=grp['expert_counts'])
            rw = grp['topk_weights']
            rows = _aligned_rows(grp['num_recv_tokens_per_expert_list'], 1)
            # The fused receive leaves the alignment padding of its operand unwritten: zero it (and
            # the GEMM's rows computed from it) so the padding stays zero through the layer.
            zero_group_padding([p.x, p.scales, h], p.expert_offsets, p.expert_counts)
        else:
            (rxq, rxs), ridx, rw, per_expert, handle, _ = buffer.dispatch(
                x, topk_idx=topk_idx, topk_weights=topk_weights, num_experts=num_experts, quantize_fp8=True,
                round_scale=ue8m0, config=config)
            p = permute(rxq, ridx, E_l, alignment=128, probs=rw, x_scales=rxs, zero_padding=True)
            rows = _aligned_rows(per_expert)
            w1q, w1s = quantize_weights_fp8(w1.detach(), round_scale=ue8m0)
            h = grouped_gemm_fp8(p.x, p.scales, w1q, w1s.contiguous(), p.expert_offsets, p.expert_counts, ue8m0=ue8m0)
        a, aq, as_ = require_ext().swiglu_quant(h, ue8m0)
        w2q, w2s = quantize_weights_fp8(w2.detach(), round_scale=ue8m0)
        if gemm_combine is not None and not ue8m0 and not _FUSED_DISPATCH['enabled']:
            # The down projection's epilogue sends each row to its token's slot on the source rank;
            # the source sums its slots with its own top-k weights. y stays local for the backward.
            y = gemm_combine.send(aq, as_, w2q, w2s.contiguous(), p.expert_offsets, p.expert_counts, p.row_map, handle,
                                  keep_local=True)
            out = gemm_combine.reduce(topk_idx, topk_weights)
        else:
            y = grouped_gemm_fp8(aq, as_, w2q, w2s.contiguous(), p.expert_offsets, p.expert_counts, ue8m0=ue8m0)
            # Top-k weighted reduction of the grouped rows, bf16 cast and exchange in one kernel.
            out, _, _ = buffer.combine(y, handle, config=config, row_map=p.row_map, row_weights=rw)
        ctx.buffer, ctx.config, ctx.inter, ctx.rows = buffer, config, inter, rows
        ctx.handle = handle
        ctx.save_for_backward(p.x, p.scales, p.row_map, p.expert_offsets, p.expert_counts, rw, h, a, y, w1, w2)
        return out

    @staticmethod
    def backward(ctx, g_out):
        xp, xs, row_map, offsets, counts, rw, h, a, y, w1, w2 = ctx.saved_tensors
        buffer, config, inter, R = ctx.buffer, ctx.config, ctx.inter, ctx.rows
        g_out = g_out.contiguous().to(torch.bfloat16)
        # combine^T: send the output gradient to the ranks that computed each token (cached layout)
        g_tok, *_ = buffer.dispatch(g_out, handle=ctx.handle, config=config)
        # unpermute^T: grouped output gradient (scaled by the routing weight) and the weight gradient
        g_y = torch.zeros((R, y.shape[1]), dtype=torch.bfloat16, device=y.device)
        g_rw = unpermute_backward(g_tok, row_map, rw, y[:R], g_y)
        xf = per_token_cast_back(xp[:R], xs[:R])  # zero padding rows dequantize to zero
        g_xp, g_w1, g_w2 = _expert_grads(g_y, a[:R], h[:R], xf, offsets, counts, w1, w2, inter)
        # permute^T (sum of each received token's rows) fused with dispatch^T = combine (sum over ranks)
        g_x, g_topk_w, _ = buffer.combine(g_xp, ctx.handle, topk_weights=g_rw, config=config, row_map=row_map)
        return g_x, None, g_topk_w, g_w1, g_w2, None, None, None, None


class MoEFFN(torch.nn.Module):
    """SwiGLU MoE FFN with `num_experts / group_size` local experts per rank.

    Weights: w1 [E_local, 2*inter, hidden] (gate rows then up rows), w2 [E_local, hidden, inter],
    bf16 master copies, quantized to FP8 with 128x128 block scales inside every forward.
    """

    def __init__(self, buffer, hidden: int, inter: int, num_experts: int, num_topk: int,
                 config=None, init_std: float = 0.02, generator: Optional[torch.Generator] = None):
        super().__init__()
        world = buffer.group_size
        assert num_experts % world == 0
        self.buffer, self.config = buffer, config
        self.hidden, self.inter, self.num_experts, self.num_topk = hidden, inter, num_experts, num_topk
        e_l = num_experts // world
        g = generator
        self.w1 = torch.nn.Parameter((torch.randn((e_l, 2 * inter, hidden), generator=g) * init_std)
                                     .to(torch.bfloat16).cuda())
        self.w2 = torch.nn.Parameter((torch.randn((e_l, hidden, inter), generator=g) * init_std)
                                     .to(torch.bfloat16).cuda())

    def forward(self, x: torch.Tensor, topk_idx: torch.Tensor, topk_weights: torch.Tensor) -> torch.Tensor:
        return _MoEFunction.apply(x, topk_idx, topk_weights, self.w1, self.w2, self.buffer, self.num_experts,
                                  self.config, self._gemm_combine(topk_idx))

    def _gemm_combine(self, topk_idx: torch.Tensor):
        """The layer's GEMM-combine region when DEEPEP_B200_MOE_FUSED_COMBINE=1 (created at the first
        forward, a collective call; its slots hold the buffer's token capacity on every rank)."""
        if not _FUSED_COMBINE['enabled'] or _UE8M0['enabled'] or _FUSED_DISPATCH['enabled']:
            return None
        gc = getattr(self, '_gc', None)
        if gc is None:
            from ..parallel.gemm_combine import GemmCombine
            gc = GemmCombine(self.buffer.group, self.buffer.get_capacity(self.hidden), topk_idx.shape[1], self.hidden)
            self._gc = gc
        return gc

    def release(self) -> None:
        """Free the layer's GEMM-combine region (collective: every rank calls it)."""
        gc = getattr(self, '_gc', None)
        if gc is not None:
            gc.destroy()
            self._gc = None

    def quantized_weights(self):
        """FP8 weights with 128x128 scales (w1q, w1s, w2q, w2s), re-quantized only after the bf16
        master weights change (inference reuses them across decode steps)."""
        key = (self.w1.data_ptr(), self.w1._version, self.w2.data_ptr(), self.w2._version)
        if getattr(self, '_wq_key', None) != key:
            w1q, w1s = quantize_weights_fp8(self.w1.detach())
            w2q, w2s = quantize_weights_fp8(self.w2.detach())
            self._wq = (w1q, w1s.contiguous(), w2q, w2s.contiguous())
            self._wq_key = key
        return self._wq

    @torch.no_grad()
    def forward_low_latency(self, ll_buffer, x: torch.Tensor, topk_idx: torch.Tensor, topk_weights: torch.Tensor,
                            num_max_dispatch_tokens_per_rank: int, fuse_combine: bool = True) -> torch.Tensor:
        """Decode forward (inference) on the low-latency path, every step a hand-written sm_100a kernel:
        FP8 dispatch with its receive fused into the masked gate/up GEMM
        (`Buffer.low_latency_dispatch_gemm`) -> masked SwiGLU + FP8 requant -> masked down GEMM ->
        top-k weighted `low_latency_combine`. `ll_buffer` is a `Buffer` with a low-latency region for
        (num_max_dispatch_tokens_per_rank, hidden, num_experts); no permute, no packing copy. With
        `fuse_combine` the down projection's epilogue stores its rows straight into the sources'
        combine slots (`Buffer.low_latency_gemm_combine`)."""
        from ..ops.gemm import masked_grouped_gemm_fp8
        from ..ops.quant import swiglu_quant
        w1q, w1s, w2q, w2s = self.quantized_weights()
        h, counts, handle, _ = ll_buffer.low_latency_dispatch_gemm(x, topk_idx, num_max_dispatch_tokens_per_rank,
                                                                   self.num_experts, w1q, w1s)
        _, aq, as_ = swiglu_quant(h, counts=counts)
        if fuse_combine:
            # down projection whose epilogue is the combine's send, then the weighted receive
            return ll_buffer.low_latency_gemm_combine(aq, as_, w2q, w2s, topk_idx, topk_weights.float().contiguous(), handle)
        y = masked_grouped_gemm_fp8(aq, as_, counts, w2q, w2s)
        out, _, _ = ll_buffer.low_latency_combine(y, topk_idx, topk_weights, handle)
        return out


def moe_reference(x, topk_idx, topk_weights, w1_all, w2_all, round_scale: bool = False):
    """Single-process fp32 oracle with the layer's quantization points (FP8 x, FP8 weights, bf16 h,
    FP8 a, bf16 y); w*_all hold every expert of the group: [E, 2I, H] and [E, H, I]. `round_scale`:
    power-of-two scales everywhere (the layer's UE8M0 mode)."""
    from ..ops.gemm import dequant_blocks, quantize_weights_fp8_reference
    from ..utils.math import per_token_cast_back, per_token_cast_to_fp8
    inter = w1_all.shape[1] // 2
    xq, xs = per_token_cast_to_fp8(x, round_scale=round_scale)
    xf = per_token_cast_back(xq, xs).float()
    w1q, w1s = quantize_weights_fp8_reference(w1_all, round_scale)
    w2q, w2s = quantize_weights_fp8_reference(w2_all, round_scale)
    w1f, w2f = dequant_blocks(w1q, w1s), dequant_blocks(w2q, w2s)
    out = torch.zeros_like(x, dtype=torch.float32)
    for k in range(topk_idx.shape[1]):
        for e in topk_idx[:, k].unique().tolist():
            if e < 0:
                continue
            sel = topk_idx[:, k] == e
            h = (xf[sel] @ w1f[e].t()).to(torch.bfloat16).float()
            a = (torch.nn.functional.silu(h[:, :inter]) * h[:, inter:]).to(torch.bfloat16)
            aq, as_ = per_token_cast_to_fp8(a, round_scale=round_scale)
            y = (per_token_cast_back(aq, as_).float() @ w2f[e].t()).to(torch.bfloat16).float()
            out[sel] += topk_weights[sel, k].unsqueeze(1) * y
    return out.to(torch.bfloat16)
