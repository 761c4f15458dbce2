"""GPU tests of the normal-mode combine in its weighted expanded mode.

The expanded mode takes one row per (received token, local expert) in the expert-grouped layout that
`permute` produces, and reduces each token's rows with its top-k weights on the sender before the
exchange; the source rank then sums the ranks' rows. It is checked, at every world size the box
offers, against
  * a plain fp32 torch oracle of the whole operation (`ReferenceBuffer.combine` with `row_map`:
    fp32 weighted sum, bf16 rounding of each rank's row, fp32 sum over ranks, bf16), and
  * the unfused composition it replaces (weighted `unpermute`, then the plain combine),
for bf16 and FP8 dispatch, alignment 1 and 128, with and without a bias, and unweighted.
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
    from deepep_slingshot_b200 import Buffer, ReferenceBuffer
    from deepep_slingshot_b200.ops.permute import permute, unpermute
    from deepep_slingshot_b200.utils import gate
    group = dist.group.WORLD
    buf = Buffer(group, num_nvl_bytes=Buffer.get_nvl_buffer_size_hint(N, H, world), num_gpu_timeout_secs=20)
    ref = ReferenceBuffer(group)
    E_l = E // world
    cases = [(False, 1, False, True), (True, 128, True, True), (False, 128, False, False), (True, 1, False, True)]
    for it, (fp8, align, with_bias, weighted) in enumerate(cases):
        g = torch.Generator().manual_seed(1000 * it + rank)
        n = N - 5 * rank
        x = torch.randn((n, H), generator=g).to(torch.bfloat16).cuda()
        idx, w = gate.normal_routing(n, E, K, generator=g)
        idx, w = idx.cuda(), w.cuda()
        if fp8:
            (rx, rs), ridx, rw, _, h, _ = buf.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E, quantize_fp8=True)
        else:
            rx, ridx, rw, _, h, _ = buf.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E)
            rs = None
        eh = ref.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E)[4]  # the oracle's own handle
        p = permute(rx, ridx, E_l, alignment=align, probs=rw, x_scales=rs)
        # expanded expert outputs: a different random row per (token, local expert)
        y = torch.randn((p.x.shape[0], H), generator=g).to(torch.bfloat16).cuda()
        row_w = rw if weighted else None
        bias = torch.randn((n, H), generator=g).to(torch.bfloat16).cuda() if with_bias else None
        out, out_w, _ = buf.combine(y, h, topk_weights=rw, bias=bias, row_map=p.row_map, row_weights=row_w)
        # fp32 oracle of the whole operation, over the oracle's own exchange
        eo, eow, _ = ref.combine(y, eh, topk_weights=rw, bias=bias, row_map=p.row_map, row_weights=row_w)
        # unfused composition: weighted unpermute kernel, then the plain combine
        uo, uow, _ = buf.combine(unpermute(y, p.row_map, row_w), h, topk_weights=rw, bias=bias)
        torch.cuda.synchronize()
        tol = dict(atol=2e-2, rtol=2e-2)
        assert out.shape == (n, H) and out.dtype == torch.bfloat16
        assert torch.allclose(out.float(), eo.float(), **tol), (it, (out.float() - eo.float()).abs().max())
        assert torch.allclose(out.float(), uo.float(), **tol), (it, (out.float() - uo.float()).abs().max())
        assert torch.allclose(out_w, eow, atol=1e-6) and torch.allclose(out_w, uow, atol=1e-6)
        # tokens routed nowhere come back as zero (+ bias)
        dead = (idx < 0).all(dim=1)
        if bool(dead.any()):
            expect = bias[dead].float() if bias is not None else torch.zeros_like(out[dead].float())
            assert torch.allclose(out[dead].float(), expect, atol=1e-2)


@pytest.mark.parametrize('world', _worlds())
def test_weighted_expanded_combine(world):
    run_ranks(_body, world, backend='nccl', args=(512, 2048, 32, 8))


@pytest.mark.parametrize('world', _worlds())
def test_weighted_expanded_combine_deepseek_shape(world):
    """hidden 7168, 256 experts, top-8: at one GPU every token has 8 local rows."""
    run_ranks(_body, world, backend='nccl', args=(1024, 7168, 256, 8))


def _roundtrip_body(rank, world):
    """combine(dispatch(x)) in the expanded mode with the received rows as expert outputs gives
    x times the sum of its top-k weights (the library's plumbing invariant)."""
    from deepep_slingshot_b200 import Buffer
    from deepep_slingshot_b200.ops.permute import permute
    from deepep_slingshot_b200.utils import gate
    N, H, E, K = 300, 1024, 16, 4
    buf = Buffer(dist.group.WORLD, num_nvl_bytes=Buffer.get_nvl_buffer_size_hint(N, H, world), num_gpu_timeout_secs=20)
    g = torch.Generator().manual_seed(7 + rank)
    x = torch.randn((N, H), generator=g).to(torch.bfloat16).cuda()
    idx, w = gate.normal_routing(N, E, K, generator=g)
    idx, w = idx.cuda(), w.cuda()
    rx, ridx, rw, _, h, _ = buf.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E)
    p = permute(rx, ridx, E // world, alignment=1, probs=rw)
    out, _, _ = buf.combine(p.x, h, row_map=p.row_map, row_weights=rw)
    torch.cuda.synchronize()
    expect = x.float() * torch.where(idx >= 0, w, torch.zeros_like(w)).sum(1, keepdim=True)
    assert torch.allclose(out.float(), expect, atol=3e-2, rtol=3e-2), (out.float() - expect).abs().max()


@pytest.mark.parametrize('world', _worlds())
def test_weighted_combine_roundtrip(world):
    run_ranks(_roundtrip_body, world, backend='nccl')
