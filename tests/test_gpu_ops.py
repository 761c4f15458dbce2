"""GPU tests of the standalone sm_100a ops against torch oracles: permute / unpermute."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize('N,H,E,K,align,fp8', [(1000, 1024, 32, 8, 128, True), (4096, 7168, 32, 8, 128, True),
                                                (77, 256, 8, 2, 1, False), (513, 2048, 256, 8, 64, False)])
def test_permute_unpermute(N, H, E, K, align, fp8):
    from deepep_slingshot_b200.ops.permute import permute, permute_reference, unpermute, unpermute_reference
    from deepep_slingshot_b200.utils.math import per_token_cast_to_fp8
    g = torch.Generator().manual_seed(N)
    x = torch.randn((N, H), generator=g).to(torch.bfloat16).cuda()
    idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(N)]).cuda()
    idx[torch.rand((N, K), generator=g).cuda() < 0.1] = -1
    w = torch.rand((N, K), generator=g).cuda()
    xs = None
    if fp8:
        x, xs = per_token_cast_to_fp8(x)
    p = permute(x, idx, E, alignment=align, probs=w, x_scales=xs)
    p2 = permute(x, idx, E, alignment=align, probs=w, x_scales=xs)
    torch.cuda.synchronize()
    counts, offsets = permute_reference(idx, E, align)
    assert torch.equal(p.expert_counts, counts) and torch.equal(p.expert_offsets, offsets)
    assert torch.equal(p.row_map, p2.row_map)  # deterministic order
    rm = p.row_map
    valid = rm >= 0
    assert torch.equal(valid, idx >= 0)
    rows = rm[valid].long()
    assert rows.unique().numel() == rows.numel()
    t_of = torch.arange(N, device='cuda').unsqueeze(1).expand(N, K)[valid]
    e_of = idx[valid]
    assert ((rows >= offsets[e_of].long()) & (rows < (offsets[e_of] + counts[e_of]).long())).all()
    assert torch.equal(p.x[rows].view(torch.uint8), x[t_of].view(torch.uint8))
    assert torch.equal(p.probs[rows], w[valid])
    if fp8:
        assert torch.equal(p.scales[rows], xs[t_of])
    # unpermute (bf16 expert outputs)
    y = torch.randn((p.x.shape[0], H), generator=g).to(torch.bfloat16).cuda()
    out = unpermute(y, rm, w)
    ref = unpermute_reference(y, rm, w)
    assert torch.allclose(out.float(), ref.float(), atol=2e-2, rtol=1e-2)


def test_permute_zero_padding():
    from deepep_slingshot_b200.ops.permute import permute
    from deepep_slingshot_b200.utils.math import per_token_cast_to_fp8
    g = torch.Generator().manual_seed(5)
    N, H, E, K = 300, 512, 8, 2
    x, xs = per_token_cast_to_fp8(torch.randn((N, H), generator=g).to(torch.bfloat16).cuda())
    idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(N)]).cuda()
    p = permute(x, idx, E, alignment=128, x_scales=xs, zero_padding=True)
    torch.cuda.synchronize()
    off, cnt = p.expert_offsets.tolist(), p.expert_counts.tolist()
    for e in range(E):
        pad = slice(off[e] + cnt[e], off[e + 1])
        assert (p.x[pad].view(torch.uint8) == 0).all() and (p.scales[pad] == 0).all()


@pytest.mark.parametrize('K', [8, 12])
def test_unpermute_backward_matches_torch(K):
    """g_y scatter (bf16(g * w)) exactly, routing-weight gradient (fp32 dots) within fp32 tolerance."""
    from deepep_slingshot_b200.ops.permute import permute, unpermute_backward, unpermute_backward_reference
    g = torch.Generator().manual_seed(K)
    N, H, E = 700, 7168, 16
    idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(N)]).cuda()
    idx[torch.rand((N, K), generator=g).cuda() < 0.3] = -1
    w = torch.rand((N, K), generator=g).cuda()
    x = torch.randn((N, H), generator=g).to(torch.bfloat16).cuda()
    p = permute(x, idx, E, alignment=128, probs=w, zero_padding=True)
    R = int(p.expert_offsets[-1])
    y = torch.randn((R, H), generator=g).to(torch.bfloat16).cuda()
    g_tok = torch.randn((N, H), generator=g).to(torch.bfloat16).cuda()
    g_y = torch.zeros_like(y)
    g_w = unpermute_backward(g_tok, p.row_map, w, y, g_y)
    ref_gy, ref_gw = unpermute_backward_reference(g_tok, p.row_map, w, y)
    torch.cuda.synchronize()
    assert torch.equal(g_y, ref_gy)
    assert torch.allclose(g_w, ref_gw, rtol=1e-4, atol=1e-2), (g_w - ref_gw).abs().max()
    assert bool((g_w[p.row_map < 0] == 0).all())


def test_swiglu_backward_matches_torch():
    from deepep_slingshot_b200.ops.quant import swiglu_backward, swiglu_backward_reference
    g = torch.Generator().manual_seed(5)
    h = (torch.randn((1000, 4096), generator=g) * 3).to(torch.bfloat16).cuda()
    g_a = torch.randn((1000, 2048), generator=g).to(torch.bfloat16).cuda()
    got = swiglu_backward(h, g_a)
    exp = swiglu_backward_reference(h, g_a)
    torch.cuda.synchronize()
    # fp32 math on both sides; the kernel's exp and division round differently from torch's: one bf16 ulp
    assert torch.allclose(got.float(), exp.float(), rtol=1e-2, atol=1e-3), (got.float() - exp.float()).abs().max()


def test_zero_group_padding():
    from deepep_slingshot_b200.ops.permute import zero_group_padding
    offsets = torch.tensor([0, 128, 128, 384], dtype=torch.int32, device='cuda')
    counts = torch.tensor([100, 0, 129], dtype=torch.int32, device='cuda')
    a = torch.full((384, 64), 7.0, dtype=torch.bfloat16, device='cuda')
    b = torch.full((384, 4), 3.0, dtype=torch.float32, device='cuda')
    zero_group_padding([a, b], offsets, counts)
    torch.cuda.synchronize()
    live = torch.zeros(384, dtype=torch.bool, device='cuda')
    live[0:100] = True
    live[128:257] = True
    assert bool((a[live] == 7).all()) and bool((a[~live] == 0).all())
    assert bool((b[live] == 3).all()) and bool((b[~live] == 0).all())
