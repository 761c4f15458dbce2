"""Grouped GEMMs on the B200 tensor cores (tcgen05 + TMEM, hand-written sm_100a kernels).

`grouped_gemm_fp8`: rows of A grouped by expert (128-aligned blocks from `permute(..., alignment=128)`),
per-token 1x128 activation scales, 128x128 weight scales, fp32 promotion per 128-wide K block, bf16 out.
`masked_grouped_gemm_fp8`: the same math over the low-latency per-expert padded layout `[E, slots, k]`
with per-expert valid-row counts (the decode path; fused with the dispatch receive in
`Buffer.low_latency_dispatch_gemm`).
`grouped_gemm_bf16` / `grouped_gemm_bf16_wgrad`: bf16 x bf16 -> fp32 TMEM accumulation, the backward
(input- and weight-gradient) GEMMs of the expert FFN. `*_reference` are the fp32 torch oracles.
"""
from typing import Optional

import torch

from .._ext import require_ext


def grouped_gemm_fp8(a: torch.Tensor, sa: torch.Tensor, b: torch.Tensor, sb: torch.Tensor, offsets: torch.Tensor,
                     counts: Optional[torch.Tensor] = None, num_sms: int = 0, timeout_s: float = 10.0,
                     ue8m0: bool = False) -> torch.Tensor:
    """Grouped block-scaled FP8 GEMM on tcgen05: rows of `a [rows, k]` (1x128 scales `sa`) grouped by
    expert at 128-aligned `offsets`, times `b [E, n, k]` (128x128 scales `sb`) -> `[rows, n]` bf16; only the
    first `counts[e]` rows of each group are meaningful.

    With `ue8m0=True` every scale must be a power of two (`round_scale=True` quantization): the
    tensor core then applies the scales itself (`kind::mxf8f6f4.block_scale`) and accumulates over
    the whole K range in TMEM, with no per-K-block promotion."""
    return require_ext().grouped_gemm_fp8(a, sa, b, sb, offsets, counts, num_sms, timeout_s, ue8m0)


def grouped_gemm_bf16(a: torch.Tensor, b: torch.Tensor, offsets: torch.Tensor, counts: Optional[torch.Tensor] = None,
                      num_sms: int = 0, timeout_s: float = 10.0, b_mn_major: bool = False) -> torch.Tensor:
    """M-grouped bf16 GEMM on tcgen05: rows of `a [rows, k]` grouped by expert (`offsets [E+1]`,
    128-aligned) times `b [E, n, k]` (K-major weights) -> `[rows, n]` bf16 (fp32 accumulation).
    With `b_mn_major=True`, `b` is `[E, k, n]` and is read as it lies (no transpose copy): the forward
    weights of the layer serve the input-gradient GEMM directly."""
    return require_ext().grouped_gemm_bf16(a, b, offsets, counts, 0, num_sms, timeout_s, False, b_mn_major)


def grouped_gemm_bf16_wgrad(a_t: torch.Tensor, b_t: torch.Tensor, offsets: torch.Tensor, num_sms: int = 0,
                            timeout_s: float = 10.0) -> torch.Tensor:
    """K-grouped bf16 GEMM on tcgen05 (weight gradients): `a_t [m, Ktot]`, `b_t [n, Ktot]` with expert e
    owning K range [offsets[e], offsets[e+1]) -> `[E, m, n]` = per-expert a_t[:, K_e] @ b_t[:, K_e]^T."""
    return require_ext().grouped_gemm_bf16(a_t, b_t, offsets, None, 1, num_sms, timeout_s)


def grouped_gemm_bf16_wgrad_rows(a: torch.Tensor, b: torch.Tensor, offsets: torch.Tensor, num_sms: int = 0,
                                 timeout_s: float = 10.0) -> torch.Tensor:
    """K-grouped bf16 GEMM on tcgen05 over row-major activations, read as they lie (MN-major operands,
    no transposes): `a [Ktot, m]`, `b [Ktot, n]` with expert e owning rows [offsets[e], offsets[e+1])
    (64-aligned) -> `[E, m, n]` = per-expert a[K_e]^T @ b[K_e]."""
    return require_ext().grouped_gemm_bf16(a, b, offsets, None, 1, num_sms, timeout_s, True, True)


def grouped_gemm_bf16_reference(a, b, offsets, counts=None) -> torch.Tensor:
    """fp32 torch oracle of `grouped_gemm_bf16` (mode 0); rows past `counts[e]` stay zero."""
    out = torch.zeros((a.shape[0], b.shape[1]), dtype=torch.float32, device=a.device)
    off = offsets.tolist()
    for e in range(b.shape[0]):
        r1 = off[e] + (int(counts[e]) if counts is not None else off[e + 1] - off[e])
        if r1 > off[e]:
            out[off[e]:r1] = a[off[e]:r1].float() @ b[e].float().t()
    return out


def grouped_gemm_bf16_wgrad_reference(a_t, b_t, offsets) -> torch.Tensor:
    """fp32 torch oracle of `grouped_gemm_bf16_wgrad` (K-grouped)."""
    off = offsets.tolist()
    E = len(off) - 1
    out = torch.zeros((E, a_t.shape[0], b_t.shape[0]), dtype=torch.float32, device=a_t.device)
    for e in range(E):
        if off[e + 1] > off[e]:
            out[e] = a_t[:, off[e]:off[e + 1]].float() @ b_t[:, off[e]:off[e + 1]].float().t()
    return out


def op_error_state(clear: bool = False):
    """(code, peer, detail, rank) of the last bounded wait that expired in a standalone op."""
    return require_ext().op_error_state(clear)


def dequant_rows(x: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """fp8 [m, k] with 1x128 scales [m, k/128] -> fp32."""
    m, k = x.shape
    return (x.float().view(m, k // 128, 128) * s.view(m, k // 128, 1)).view(m, k)


def dequant_blocks(w: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """fp8 [E, n, k] with 128x128 scales [E, n/128, k/128] -> fp32."""
    E, n, k = w.shape
    return (w.float().view(E, n // 128, 128, k // 128, 128) * s.view(E, n // 128, 1, k // 128, 1)).view(E, n, k)


def quantize_weights_fp8(w: torch.Tensor, round_scale: bool = False):
    """bf16/fp32 [E, n, k] -> (fp8 [E, n, k], fp32 128x128 block scales [E, n/128, k/128]).
    With `round_scale` the scales are rounded up to powers of two (exact as UE8M0, what the
    block-scaled MMA path of `grouped_gemm_fp8(..., ue8m0=True)` needs).
    Contiguous bf16 CUDA weights go through the sm_100a block-quantization kernel (one HBM pass);
    other inputs use `quantize_weights_fp8_reference` (the same numerics in torch)."""
    if w.is_cuda and w.dtype == torch.bfloat16 and w.is_contiguous() and w.dim() == 3:
        return require_ext().quantize_weights_fp8(w, round_scale)
    return quantize_weights_fp8_reference(w, round_scale)


def quantize_weights_fp8_reference(w: torch.Tensor, round_scale: bool = False):
    """Torch definition of the 128x128 block weight quantization (oracle of the kernel)."""
    E, n, k = w.shape
    v = w.float().view(E, n // 128, 128, k // 128, 128)
    amax = v.abs().amax(dim=(2, 4)).clamp(min=1e-4)
    c448 = torch.full_like(amax, 448.0)
    scale = amax / c448
    if round_scale:
        scale = torch.pow(2.0, torch.ceil(torch.log2(scale)))
        mult = 1.0 / scale
    else:
        mult = c448 / amax  # one factor per block, as the kernel applies it
    q = (v * mult.view(E, n // 128, 1, k // 128, 1)).clamp(-448, 448).to(torch.float8_e4m3fn)
    return q.view(E, n, k), scale


def grouped_gemm_fp8_reference(a, sa, b, sb, offsets, counts=None) -> torch.Tensor:
    """fp32 torch oracle of `grouped_gemm_fp8` with the same dequantisation; rows past
    `counts[e]` stay zero."""
    af = dequant_rows(a, sa)
    bf = dequant_blocks(b, sb)
    out = torch.zeros((a.shape[0], b.shape[1]), dtype=torch.float32, device=a.device)
    E = b.shape[0]
    off = offsets.tolist()
    cnt = counts.tolist() if counts is not None else [off[e + 1] - off[e] for e in range(E)]
    for e in range(E):
        r0, r1 = off[e], off[e] + cnt[e]
        if r1 > r0:
            out[r0:r1] = af[r0:r1] @ bf[e].t()
    return out


def masked_grouped_gemm_fp8(a: torch.Tensor, sa: torch.Tensor, counts: torch.Tensor, b: torch.Tensor, sb: torch.Tensor,
                            num_sms: int = 0, timeout_s: float = 10.0) -> torch.Tensor:
    """Masked grouped FP8 GEMM on tcgen05 over the low-latency per-expert padded layout:
    `a [E, slots, k]` e4m3 with 1x128 scales `sa [E, slots, k/128]` (any strides, e.g. the dispatch's
    column-major scales), `counts [E]` int32 valid rows per expert, `b [E, n, k]` e4m3 with 128x128
    scales `sb [E, n/128, k/128]` -> `[E, slots, n]` bf16. Rows at or beyond `counts[e]` are left
    unwritten. `Buffer.low_latency_dispatch_gemm` runs the same kernel fused with the dispatch receive."""
    return require_ext().masked_grouped_gemm_fp8(a, sa, counts, b, sb, num_sms, timeout_s)


def masked_grouped_gemm_fp8_reference(a, sa, counts, b, sb) -> torch.Tensor:
    """fp32 torch oracle of `masked_grouped_gemm_fp8` (rows at or beyond `counts[e]` are zero)."""
    E, slots, k = a.shape
    bf = dequant_blocks(b, sb)
    out = torch.zeros((E, slots, b.shape[1]), dtype=torch.float32, device=a.device)
    for e, c in enumerate(counts.tolist()):
        c = max(0, min(int(c), slots))
        if c > 0:
            out[e, :c] = dequant_rows(a[e, :c], sa[e, :c].contiguous()) @ bf[e].t()
    return out
