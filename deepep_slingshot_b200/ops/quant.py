"""Per-token 1x128 FP8 e4m3 cast kernels (sm_100a) with the numerics of `utils.math`'s torch oracle."""
from typing import Tuple

import torch

from .._ext import require_ext


def per_token_cast_to_fp8(x: torch.Tensor, round_scale: bool = False) -> Tuple[torch.Tensor, torch.Tensor]:
    """bf16 [N, H] -> (fp8 e4m3 [N, H], fp32 scales [N, H/128]); scale = amax/448 (power of two if
    `round_scale`)."""
    return require_ext().per_token_cast_to_fp8(x, round_scale)


def per_token_cast_back(x: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    return require_ext().per_token_cast_back(x, scales)
