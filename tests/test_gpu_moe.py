"""GPU test of the expert-parallel MoE FFN layer (forward + backward) against torch oracles.

Forward is compared with a single-process fp32 oracle that applies the same quantization points;
backward with torch autograd on unquantized fp32 math (the layer's gradients are straight-through
the FP8 quantization), weight gradients all-reduced over ranks before comparison.
"""
import pytest
import torch
import torch.distributed as dist

from tests._dist import run_ranks
from tests.test_gpu_intranode import _worlds

pytestmark = pytest.mark.gpu


def _ref_autograd(x, idx, w, w1_all, w2_all):
    inter = w1_all.shape[1] // 2
    out = torch.zeros_like(x)
    for k in range(idx.shape[1]):
        for e in idx[:, k].unique().tolist():
            if e < 0:
                continue
            sel = idx[:, k] == e
            h = x[sel] @ w1_all[e].t()
            a = torch.nn.functional.silu(h[:, :inter]) * h[:, inter:]
            out = out.index_add(0, torch.nonzero(sel).flatten(), w[sel, k].unsqueeze(1) * (a @ w2_all[e].t()))
    return out


def _moe_body(rank, world, N, H, I, E, K, bwd='tcgen05_mn', ue8m0=False):
    from deepep_slingshot_b200 import Buffer
    from deepep_slingshot_b200.models import MoEFFN, moe_reference
    from deepep_slingshot_b200.models import moe as moe_mod
    moe_mod._BWD['mode'] = bwd
    moe_mod._UE8M0['enabled'] = ue8m0
    from deepep_slingshot_b200.utils import gate
    from deepep_slingshot_b200.utils.math import calc_diff
    group = dist.group.WORLD
    buf = Buffer(group, num_nvl_bytes=Buffer.get_nvl_buffer_size_hint(N, H, world), num_gpu_timeout_secs=20)
    gw = torch.Generator().manual_seed(1234)  # same weights on every rank
    w1_all = (torch.randn((E, 2 * I, H), generator=gw) * 0.05).to(torch.bfloat16).cuda()
    w2_all = (torch.randn((E, H, I), generator=gw) * 0.05).to(torch.bfloat16).cuda()
    e_l = E // world
    layer = MoEFFN(buf, H, I, E, K)
    with torch.no_grad():
        layer.w1.copy_(w1_all[rank * e_l:(rank + 1) * e_l])
        layer.w2.copy_(w2_all[rank * e_l:(rank + 1) * e_l])
    g = torch.Generator().manual_seed(rank + 7)
    x = torch.randn((N, H), generator=g).to(torch.bfloat16).cuda()
    idx, w = gate.normal_routing(N, E, K, generator=g)
    idx, w = idx.cuda(), w.cuda()
    x.requires_grad_(True)
    w.requires_grad_(True)
    out = layer(x, idx, w)
    ref = moe_reference(x.detach(), idx, w.detach(), w1_all, w2_all, round_scale=ue8m0)
    torch.cuda.synchronize()
    d = calc_diff(out.float(), ref.float())
    assert d < 2e-4, d
    # backward
    go = torch.randn((N, H), generator=g).to(torch.bfloat16).cuda()
    (out.float() * go.float()).sum().backward()
    xr = x.detach().float().requires_grad_(True)
    wr = w.detach().clone().requires_grad_(True)
    w1r = w1_all.float().requires_grad_(True)
    w2r = w2_all.float().requires_grad_(True)
    (_ref_autograd(xr, idx, wr, w1r, w2r) * go.float()).sum().backward()
    g_w1 = w1r.grad.clone()
    g_w2 = w2r.grad.clone()
    dist.all_reduce(g_w1)
    dist.all_reduce(g_w2)
    sl = slice(rank * e_l, (rank + 1) * e_l)
    # Routing-weight gradients are <g_out, y> with y from the FP8 forward: looser bound.
    for name, got, exp, tol in (('x', x.grad, xr.grad, 2e-3), ('w', w.grad, wr.grad, 6e-3),
                                ('w1', layer.w1.grad, g_w1[sl], 2e-3), ('w2', layer.w2.grad, g_w2[sl], 2e-3)):
        dd = calc_diff(got.float(), exp.float())
        assert dd < tol, (name, dd)
    buf.check_error()


@pytest.mark.parametrize('world', _worlds())
@pytest.mark.parametrize('bwd', ['tcgen05_mn', 'tcgen05', 'grouped', 'loop'])
def test_moe_layer_forward_backward(world, bwd):
    """Forward against the quantization-aware oracle; backward gradients (x, routing weights, w1, w2)
    against fp32 autograd, with the backward GEMMs on the tcgen05 kernels (MN-major operands, the
    default, or K-major), torch's grouped GEMM (A/B stand-in) or per-expert matmuls."""
    run_ranks(_moe_body, world, 'nccl', args=(256, 1024, 512, 16, 4, bwd))


@pytest.mark.parametrize('world', _worlds()[:2])
def test_moe_layer_ue8m0_forward_backward(world):
    """The layer with power-of-two scales and the block-scaled forward GEMMs, against the oracle with
    the same quantization points (and the same backward checks)."""
    run_ranks(_moe_body, world, 'nccl', args=(256, 1024, 512, 16, 4, 'tcgen05_mn', True))
