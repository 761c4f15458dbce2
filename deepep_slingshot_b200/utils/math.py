"""Small numeric helpers and the pure-torch FP8 reference casts.

Parity with the reference's `deep_ep/utils/math.py` ([DE]deep_ep/utils/math.py:5-103): `calc_diff`,
`ceil_div`, `align`, `per_token_cast_to_fp8` (1x128 amax, scale = amax/448, amax clamped at 1e-4),
`per_token_cast_back` (also accepts packed UE8M0 scales), `inplace_unique`, `count_bytes`, hashes.
The torch versions here are the numerics oracle of the sm_100a cast kernels (`ops.quant`).
"""
from typing import Tuple

import torch


def calc_diff(x: torch.Tensor, y: torch.Tensor) -> float:
    """1 - 2<x+1, y+1> / (|x+1|^2 + |y+1|^2): 0 for identical tensors (the reference's comparison
    metric)."""
    x, y = x.double() + 1, y.double() + 1
    denominator = (x * x + y * y).sum()
    sim = 2 * (x * y).sum() / denominator
    return (1 - sim).item()


def safe_div(a, b) -> float:
    """a / b; 0 / 0 is 0 (any other division by zero raises)."""
    if b == 0:
        if a == 0:
            return 0
        raise ZeroDivisionError
    return a / b


def ceil_div(x: int, y: int) -> int:
    """Ceiling of a / b for positive integers."""
    return (x + y - 1) // y


def align(x: int, y: int) -> int:
    """`x` rounded up to a multiple of `y`."""
    return ceil_div(x, y) * y


def per_token_cast_to_fp8(x: torch.Tensor, round_scale: bool = False) -> Tuple[torch.Tensor, torch.Tensor]:
    """bf16/fp32 [m, n] -> (fp8 e4m3 [m, n], fp32 scales [m, ceil(n/128)])."""
    assert x.dim() == 2
    m, n = x.shape
    aligned_n = align(n, 128)
    if m == 0:
        return (torch.empty((0, n), dtype=torch.float8_e4m3fn, device=x.device),
                torch.empty((0, aligned_n // 128), dtype=torch.float32, device=x.device))
    x_padded = torch.nn.functional.pad(x, (0, aligned_n - n), mode='constant', value=0)
    x_view = x_padded.view(m, -1, 128)
    x_amax = x_view.abs().float().amax(dim=2).view(m, -1).clamp(1e-4)
    # Tensor/tensor divisions: one IEEE rounding, as in the kernels (a Python-scalar divisor would
    # make torch multiply by a rounded reciprocal instead).
    c448 = torch.full_like(x_amax, 448.0)
    scale = x_amax / c448
    if round_scale:
        scale = torch.pow(2.0, torch.ceil(torch.log2(scale)))
        mult = 1.0 / scale
    else:
        mult = c448 / x_amax
    q = x_view.float() * mult.unsqueeze(2)
    q = q.clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    return q.view(m, aligned_n)[:, :n].contiguous(), scale.view(m, -1)


def per_token_cast_back(x_fp8: torch.Tensor, x_scales: torch.Tensor) -> torch.Tensor:
    """Torch definition of the FP8 -> bf16 cast with 1x128 scales (oracle of the kernel)."""
    if x_fp8.numel() == 0:
        return x_fp8.to(torch.bfloat16)
    assert x_fp8.dim() == 2
    m, n = x_fp8.shape
    aligned_n = align(n, 128)
    x_padded = torch.nn.functional.pad(x_fp8.view(torch.uint8), (0, aligned_n - n), value=0).view(torch.float8_e4m3fn)
    if x_scales.dtype == torch.int:
        x_scales = x_scales.view(dtype=torch.uint8).to(torch.int) << 23
        x_scales = x_scales.view(dtype=torch.float)
    x_fp32 = x_padded.to(torch.float32).view(m, -1, 128)
    x_scales = x_scales.reshape(m, -1, 1)
    return (x_fp32 * x_scales).view(m, aligned_n).to(torch.bfloat16)[:, :n].contiguous()


def logfmt10_roundtrip(x: torch.Tensor) -> torch.Tensor:
    """What a LogFMT-10 receiver reconstructs from bf16 rows `x [..., hidden]` (fp32 result): per
    128-group, groups with max|x| < 1 and some spread are coded as sign + 9-bit log2 level between
    log2(min|x|) (clamped to log2(max|x|) - 32) and log2(max|x|), rounded to the nearer level in linear
    space; other groups pass through unchanged. Oracle of the sm_100a LL combine with `use_logfmt`."""
    shape = x.shape
    g = x.to(torch.bfloat16).float().reshape(-1, shape[-1] // 128, 128)
    a = g.abs()
    amax = a.amax(-1, keepdim=True)
    amin = a.amin(-1, keepdim=True)
    log_amax = torch.log2(amax)
    log_amin = torch.maximum(torch.log2(amin), log_amax - 32)
    cast = (log_amax < 0) & (log_amin < log_amax)
    step = (log_amax - log_amin) / 510
    safe_step = torch.where(cast, step, torch.ones_like(step))
    up = torch.log2((1 + torch.exp2(safe_step)) * 0.5) / safe_step
    t = (torch.log2(a) - log_amin) / safe_step
    code = torch.floor(t + 2 - up).clamp(0, 511)
    code = torch.where(a == 0, torch.zeros_like(code), code)
    dec = torch.where(code == 0, torch.zeros_like(a), torch.exp2((code - 1) * safe_step + log_amin)) * torch.sign(g)
    out = torch.where(cast, dec, g)
    return out.reshape(shape)


def pack_ue8m0(scales: torch.Tensor) -> torch.Tensor:
    """fp32 power-of-two scales [..., nb] -> packed UE8M0 int32 [..., nb/4] (exponent bytes, little endian)."""
    assert scales.shape[-1] % 4 == 0
    exp = ((scales.contiguous().view(torch.int32) >> 23) & 0xff).to(torch.uint8)
    return exp.view(*scales.shape[:-1], scales.shape[-1] // 4, 4).contiguous().view(torch.int32).view(*scales.shape[:-1], scales.shape[-1] // 4)


def inplace_unique(x: torch.Tensor, num_slots: int) -> None:
    """Replace each row of `x` (values in [0, num_slots) or negative) by its unique values in
    descending order, padded with -1 (in place)."""
    assert x.dim() == 2
    mask = x < 0
    x_padded = x.masked_fill(mask, num_slots)
    bin_count = torch.zeros((x.size(0), num_slots + 1), dtype=x.dtype, device=x.device)
    bin_count.scatter_add_(1, x_padded, torch.ones_like(x_padded))
    bin_count = bin_count[:, :num_slots]
    sorted_bin_count, sorted_bin_idx = torch.sort(bin_count, dim=-1, descending=True)
    sorted_bin_idx.masked_fill_(sorted_bin_count == 0, -1)
    sorted_bin_idx = torch.sort(sorted_bin_idx, descending=True, dim=-1).values
    x[:, :].fill_(-1)
    valid_len = min(num_slots, x.size(1))
    x[:, :valid_len] = sorted_bin_idx[:, :valid_len]


def hash_tensor(t: torch.Tensor) -> int:
    """Sum of the tensor's bytes viewed as int32: a cheap content checksum (insensitive to element
    order), for comparing runs."""
    return t.view(torch.int).sum().item()


def count_bytes(*tensors) -> int:
    """Total bytes of the given tensors (nested tuples / lists allowed, None entries count 0)."""
    total = 0
    for t in tensors:
        if isinstance(t, (tuple, list)):
            total += count_bytes(*t)
        elif t is not None:
            total += t.numel() * t.element_size()
    return total


def create_grouped_scores(scores: torch.Tensor, group_idx: torch.Tensor, num_groups: int) -> torch.Tensor:
    """Zero the scores of every expert group a token did not select (group-limited routing):
    `scores [N, E]` viewed as `[N, num_groups, E / num_groups]`, `group_idx [N, g]` the kept groups."""
    n, e = scores.shape
    keep = torch.zeros((n, num_groups), dtype=torch.bool, device=scores.device)
    keep.scatter_(1, group_idx, True)
    return (scores.view(n, num_groups, -1) * keep.unsqueeze(-1)).view(n, e)


def hash_tensors(*tensors) -> int:
    """XOR of `hash_tensor` over tensors (nested tuples / lists allowed, None skipped)."""
    value = 0
    for t in tensors:
        if isinstance(t, (tuple, list)):
            value ^= hash_tensors(*t)
        elif isinstance(t, torch.Tensor):
            value ^= hash_tensor(t)
    return value
