"""Per-token 1x128 FP8 e4m3 cast kernels (sm_100a) with the numerics of `utils.math`'s torch oracle."""
from typing import Optional, Tuple

import torch

from .._ext import require_ext


def per_token_cast_to_fp8(x: torch.Tensor, round_scale: bool = False) -> Tuple[torch.Tensor, torch.Tensor]:
    """bf16 [N, H] -> (fp8 e4m3 [N, H], fp32 scales [N, H/128]); scale = amax/448 (power of two if
    `round_scale`)."""
    return require_ext().per_token_cast_to_fp8(x, round_scale)


def per_token_cast_back(x: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """FP8 e4m3 [N, H] with 1x128 fp32 scales [N, H/128] -> bf16 (sm_100a kernel)."""
    return require_ext().per_token_cast_back(x, scales)


def swiglu_quant(h: torch.Tensor, round_scale: bool = False, counts: Optional[torch.Tensor] = None):
    """SwiGLU + 1x128 FP8 requantization on sm_100a: `h [rows, 2I]` (gate | up) -> (a bf16 [rows, I],
    a_q fp8 [rows, I], a_s fp32 [rows, I/128]). With `counts` (int32 [E]) `h` is the masked per-expert
    layout `[E, slots, 2I]`, outputs keep that shape, and rows at or beyond `counts[e]` are skipped
    (left unwritten)."""
    return require_ext().swiglu_quant(h, round_scale, counts)


def swiglu_quant_reference(h: torch.Tensor, round_scale: bool = False):
    """Torch oracle of `swiglu_quant` (fp32 math, bf16 `a`, then the per-token cast)."""
    from ..utils.math import per_token_cast_to_fp8 as cast
    inter = h.shape[-1] // 2
    hf = h.float()
    a = (torch.nn.functional.silu(hf[..., :inter]) * hf[..., inter:]).to(torch.bfloat16)
    aq, as_ = cast(a.reshape(-1, inter), round_scale)
    return a, aq.view(a.shape), as_.view(*a.shape[:-1], inter // 128)


def swiglu_backward(h: torch.Tensor, g_a: torch.Tensor) -> torch.Tensor:
    """SwiGLU backward on sm_100a: `h [rows, 2I]` (gate | up) and the gradient of `a = silu(gate) * up`
    `g_a [rows, I]` (bf16) -> `g_h [rows, 2I]` bf16 (fp32 math)."""
    return require_ext().swiglu_backward(h, g_a)


def swiglu_backward_reference(h: torch.Tensor, g_a: torch.Tensor) -> torch.Tensor:
    """Torch oracle of `swiglu_backward` (fp32 math, bf16 result)."""
    inter = h.shape[1] // 2
    gate, up, ga = h[:, :inter].float(), h[:, inter:].float(), g_a.float()
    s = torch.sigmoid(gate)
    return torch.cat([ga * up * s * (1 + gate * (1 - s)), ga * gate * s], dim=1).to(torch.bfloat16)
