"""GPU tests of the normal-mode down projection with the combine as its epilogue
(`parallel/gemm_combine.py`, kernels in gemm_sm100.cu `kSend` and gemm_combine.cu).

Compared, at every world size the box offers and over three back-to-back epochs (slot reuse):
  * the rows the GEMM keeps locally against the plain grouped FP8 GEMM (same arithmetic: bit-exact);
  * the reduced tokens against the unfused composition (plain GEMM, then `Buffer.combine` in its
    expanded weighted mode), weighted and unweighted, tokens routed nowhere included;
  * the MoE layer forward and backward with `DEEPEP_B200_MOE_FUSED_COMBINE` against the unfused layer.
The host-side ordering rules (reduce without a send, two sends without a reduce) raise on the host.

All of them passed at world 1 on their first B200 run; the multi-rank parametrisations need a box
with more GPUs.
"""
import pytest
import torch
import torch.distributed as dist

from tests._dist import run_ranks

pytestmark = pytest.mark.gpu


def _worlds():
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    return [w for w in (1, 2, 4, 8) if w <= n] or [1]


def _body(rank, world, N, H, E, K):
    from deepep_slingshot_b200 import Buffer
    from deepep_slingshot_b200.ops.gemm import grouped_gemm_fp8, quantize_weights_fp8
    from deepep_slingshot_b200.ops.permute import permute
    from deepep_slingshot_b200.parallel.gemm_combine import GemmCombine
    from deepep_slingshot_b200.utils import gate
    group = dist.group.WORLD
    buf = Buffer(group, num_nvl_bytes=Buffer.get_nvl_buffer_size_hint(N, H, world), num_gpu_timeout_secs=20)
    gc = GemmCombine(group, N, K, H, timeout_secs=20)
    E_l = E // world
    gw = torch.Generator(device='cuda').manual_seed(99 + rank)
    wq, ws = quantize_weights_fp8((torch.randn((E_l, H, H), generator=gw, device='cuda') * 0.05).to(torch.bfloat16))
    ws = ws.contiguous()
    with pytest.raises(RuntimeError):
        gc.reduce(torch.zeros((4, K), dtype=torch.int64, device='cuda'))  # no send to reduce
    for it in range(3):
        g = torch.Generator().manual_seed(100 * it + rank)
        n = N - 7 * rank - it
        x = torch.randn((n, H), generator=g).to(torch.bfloat16).cuda()
        idx, w = gate.normal_routing(n, E, K, generator=g)
        idx[torch.rand(idx.shape, generator=g) < 0.1] = -1
        idx[:3] = -1  # routed nowhere
        idx, w = idx.cuda(), w.cuda()
        (rxq, rxs), ridx, rw, _, h, _ = buf.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E, quantize_fp8=True)
        p = permute(rxq, ridx, E_l, alignment=128, probs=rw, x_scales=rxs, zero_padding=True)
        rows = int(p.expert_offsets[-1].item())
        y_ref = grouped_gemm_fp8(p.x, p.scales, wq, ws, p.expert_offsets, p.expert_counts)
        out_ref, _, _ = buf.combine(y_ref, h, row_map=p.row_map, row_weights=rw)
        out_ref_u, _, _ = buf.combine(y_ref, h, row_map=p.row_map)
        y = gc.send(p.x, p.scales, wq, ws, p.expert_offsets, p.expert_counts, p.row_map, h, keep_local=True)
        if it == 0:
            with pytest.raises(RuntimeError):  # the previous send is not reduced yet
                gc.send(p.x, p.scales, wq, ws, p.expert_offsets, p.expert_counts, p.row_map, h)
        out = gc.reduce(idx, w)
        y2 = gc.send(p.x, p.scales, wq, ws, p.expert_offsets, p.expert_counts, p.row_map, h, keep_local=False)
        out_u = gc.reduce(idx, None)
        torch.cuda.synchronize()
        gc.check_error()
        buf.check_error()
        assert y2 is None
        assert torch.equal(y[:rows], y_ref[:rows])
        assert out.shape == (n, H) and out.dtype == torch.bfloat16
        tol = dict(atol=2e-2, rtol=2e-2)
        assert torch.allclose(out.float(), out_ref.float(), **tol), (it, (out.float() - out_ref.float()).abs().max())
        assert torch.allclose(out_u.float(), out_ref_u.float(), **tol), (it, (out_u.float() - out_ref_u.float()).abs().max())
        assert torch.count_nonzero(out[:3]) == 0
    gc.destroy()


@pytest.mark.parametrize('world', _worlds())
def test_gemm_combine_matches_the_unfused_path(world):
    run_ranks(_body, world, backend='nccl', args=(256, 1024, 16, 4))


@pytest.mark.parametrize('world', _worlds())
def test_gemm_combine_deepseek_shape(world):
    """hidden 7168, top-8 (32 experts keep the square [experts, hidden, hidden] test weights small)."""
    run_ranks(_body, world, backend='nccl', args=(512, 7168, 32, 8))


def _moe_body(rank, world, N, H, I, E, K):
    from deepep_slingshot_b200 import Buffer
    from deepep_slingshot_b200.models import MoEFFN
    from deepep_slingshot_b200.models import moe as moe_mod
    from deepep_slingshot_b200.utils import gate
    from deepep_slingshot_b200.utils.math import calc_diff
    group = dist.group.WORLD
    buf = Buffer(group, num_nvl_bytes=Buffer.get_nvl_buffer_size_hint(N, H, world), num_gpu_timeout_secs=20)
    layer = MoEFFN(buf, H, I, E, K, generator=torch.Generator().manual_seed(5 + rank))
    g = torch.Generator().manual_seed(rank + 7)
    x = torch.randn((N, H), generator=g).to(torch.bfloat16).cuda()
    idx, w = gate.normal_routing(N, E, K, generator=g)
    idx, w = idx.cuda(), w.cuda()
    go = torch.randn((N, H), generator=g).to(torch.bfloat16).cuda()
    res = {}
    for fused in (False, True):
        moe_mod._FUSED_COMBINE['enabled'] = fused
        layer.zero_grad(set_to_none=True)
        xi = x.clone().requires_grad_(True)
        wi = w.clone().requires_grad_(True)
        out = layer(xi, idx, wi)
        (out.float() * go.float()).sum().backward()
        torch.cuda.synchronize()
        res[fused] = (out.detach(), xi.grad, wi.grad, layer.w1.grad.clone(), layer.w2.grad.clone())
    moe_mod._FUSED_COMBINE['enabled'] = False
    assert getattr(layer, '_gc', None) is not None  # the fused run went through the region
    for name, a, b in zip(('out', 'x', 'w', 'w1', 'w2'), res[False], res[True]):
        d = calc_diff(a.float(), b.float())
        assert d < 1e-4, (name, d)
    layer.release()
    buf.check_error()


@pytest.mark.parametrize('world', _worlds())
def test_moe_layer_with_fused_down_projection_combine(world):
    run_ranks(_moe_body, world, backend='nccl', args=(256, 1024, 512, 16, 4))
