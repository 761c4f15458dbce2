"""CPU/gloo plumbing check (world size 2, no GPU): the reference backend's dispatch/combine semantics.

Config: per rank 64 tokens, hidden 256, fp32 ~N(0,1) from seed 0; 8 experts (4 per rank), top-2 of
N(0,1) router logits, softmax weights over the chosen 2. combine(dispatch(x)) with identity experts
weighted by the received top-k weights equals x * sum(top-k weights); per-expert receive counts
from get_dispatch_layout are exact.
"""
import torch
import torch.distributed as dist

from tests._dist import run_ranks


def _body(rank, world):
    from deepep_slingshot_b200 import ReferenceBuffer
    from deepep_slingshot_b200.utils.gate import normal_routing
    g = torch.Generator().manual_seed(rank)
    torch.manual_seed(0)
    N, H, E, K = 64, 256, 8, 2
    x = torch.randn((N, H), generator=torch.Generator().manual_seed(rank * 7 + 0))
    topk_idx, topk_w = normal_routing(N, E, K, generator=g)
    buf = ReferenceBuffer(dist.group.WORLD)
    ntpr, _, ntpe, itir, _ = buf.get_dispatch_layout(topk_idx, E)
    # exact per-expert counts: all-reduce of the local counts must equal the global histogram
    all_idx = [torch.zeros_like(topk_idx) for _ in range(world)]
    dist.all_gather(all_idx, topk_idx)
    hist = torch.bincount(torch.cat(all_idx).flatten(), minlength=E).to(torch.int32)
    tot = ntpe.clone()
    dist.all_reduce(tot)
    assert torch.equal(tot, hist)
    x_bf = x.to(torch.bfloat16)
    (recv_x, recv_idx, recv_w, per_expert, handle, _) = buf.dispatch(
        x_bf, num_tokens_per_rank=ntpr, is_token_in_rank=itir, num_tokens_per_expert=ntpe, topk_idx=topk_idx,
        topk_weights=topk_w)
    # receive counts per local expert match the global histogram slice
    epr = E // world
    assert per_expert == hist[rank * epr:(rank + 1) * epr].tolist()
    # identity experts: each received row scaled by the sum of its local weights
    y = (recv_x.float() * recv_w.sum(dim=1, keepdim=True)).to(torch.bfloat16)
    out, out_w, _ = buf.combine(y, handle, topk_weights=recv_w)
    expect = x_bf.float() * topk_w.sum(dim=1, keepdim=True)
    assert torch.allclose(out.float(), expect, atol=3e-2, rtol=2e-2), (out.float() - expect).abs().max()
    assert torch.allclose(out_w, topk_w, atol=1e-6)
    # weighted expanded combine: one row per (received token, local expert), reduced with the
    # received top-k weights on the sender, gives the same result
    valid = recv_idx >= 0
    row_map = torch.full(recv_idx.shape, -1, dtype=torch.int32)
    row_map[valid] = torch.arange(int(valid.sum()), dtype=torch.int32)
    y_exp = recv_x[torch.nonzero(valid)[:, 0]]
    out3, out3_w, _ = buf.combine(y_exp, handle, topk_weights=recv_w, row_map=row_map, row_weights=recv_w)
    assert torch.allclose(out3.float(), expect, atol=3e-2, rtol=2e-2), (out3.float() - expect).abs().max()
    assert torch.allclose(out3_w, topk_w, atol=1e-6)
    # low-latency reference: weighted combine of identity experts gives x * sum(w) as well
    recv, cnt, h, _, hook = buf.low_latency_dispatch(x_bf, topk_idx, 64, E, use_fp8=False, return_recv_hook=True)
    hook()
    out2, _, _ = buf.low_latency_combine(recv, topk_idx, topk_w, h)
    assert torch.allclose(out2.float(), expect, atol=3e-2, rtol=2e-2)


def test_gloo_world2_plumbing():
    run_ranks(_body, 2, 'gloo')


def _edge_oracle_body(rank, world):
    """Oracle with ranks holding 0..3 tokens and a hot rank (CPU, gloo)."""
    import torch.distributed as dist
    from deepep_slingshot_b200 import ReferenceBuffer
    ref = ReferenceBuffer(dist.group.WORLD)
    H, E, K = 256, 8, 2
    g = torch.Generator().manual_seed(rank)
    for case in range(3):
        N = [0, 1, 3, 2][(rank + case) % 4]
        x = torch.randn((N, H), generator=g).to(torch.bfloat16)
        if case == 2:
            idx = torch.arange(K, dtype=torch.int64).expand(N, K).contiguous()
        else:
            idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(N)]) if N else \
                torch.empty((0, K), dtype=torch.int64)
        w = torch.rand((N, K), generator=g)
        for fp8 in (False, True):
            rx, ri, rw, lst, h, _ = ref.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E, quantize_fp8=fp8)
            n = (rx[0] if fp8 else rx).shape[0]
            out, ow, _ = ref.combine(torch.ones((n, H), dtype=torch.bfloat16), h, topk_weights=rw)
            # every token comes back once per destination rank holding one of its experts
            dst = (idx // (E // world)).tolist()
            expect = torch.tensor([len(set(d)) for d in dst], dtype=torch.float32)
            assert out.shape == (N, H) and torch.equal(out[:, 0].float(), expect)


def test_reference_edge_cases_gloo():
    from tests._dist import run_ranks
    run_ranks(_edge_oracle_body, 2)


def _refs_body(rank, world):
    """Functional reference API (dispatch / generate_pre_combine_data / combine / ordered_accumulate)."""
    import torch.distributed as dist
    from deepep_slingshot_b200.utils import refs
    from deepep_slingshot_b200.utils.gate import normal_routing
    N, H, E, K, maxT = 32, 128, 8, 2, 64
    g = torch.Generator().manual_seed(rank)
    x = torch.randn((N, H), generator=g).to(torch.bfloat16)
    idx, w = normal_routing(N, E, K, generator=g)
    rx, ri, rw, gidx, per_rank = refs.dispatch(x, idx, w, maxT, E)
    assert int(per_rank.sum()) == rx.shape[0] and torch.equal(gidx, torch.sort(gidx).values)
    # every received row is the source token identified by its global index
    all_x = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(all_x, x)
    for i, gi in enumerate(gidx.tolist()):
        assert torch.equal(rx[i], all_x[gi // maxT][gi % maxT])
    # the same (token, k) data regenerates identically on every rank
    y = refs.generate_pre_combine_data(torch.arange(N) + rank * maxT, maxT, K, H)
    y2 = refs.generate_pre_combine_data(torch.arange(N) + rank * maxT, maxT, K, H)
    assert torch.equal(y, y2) and y.shape == (N, K, H)
    flat = refs.combine(y, idx, 1, world, E, reduce_in_local=False)
    assert torch.equal(flat, refs.ordered_accumulate(y))
    local = refs.combine(y, idx, 1, world, E, reduce_in_local=True)
    assert torch.allclose(local.float(), flat.float(), atol=3e-2, rtol=2e-2)


def test_functional_refs_gloo():
    from tests._dist import run_ranks
    run_ranks(_refs_body, 2)


def test_small_helpers():
    from deepep_slingshot_b200.utils.math import create_grouped_scores, hash_tensors
    from deepep_slingshot_b200.utils.testing import empty_suppress, suppress_stdout_stderr
    s = torch.arange(16, dtype=torch.float32).view(2, 8) + 1
    gs = create_grouped_scores(s, torch.tensor([[0], [3]]), 4)
    assert gs[0, :2].tolist() == [1.0, 2.0] and gs[0, 2:].abs().sum() == 0 and gs[1, 6:].tolist() == [15.0, 16.0]
    a, b = torch.arange(4, dtype=torch.int32), torch.ones(3, dtype=torch.int32)
    assert hash_tensors(a, [b, None]) == (int(a.sum()) ^ int(b.sum()))
    with suppress_stdout_stderr():
        print('hidden')
    with empty_suppress():
        pass


def _matrix_oracle_body(rank, world):
    """The oracle over the normal-mode matrix the GPU test enumerates (CPU, gloo): FP8 / bf16 x
    expert alignment 1 / 128 x 0 / 1 / 2 biases, and the cached dispatch through a copied handle."""
    import itertools
    from deepep_slingshot_b200 import ReferenceBuffer
    ref = ReferenceBuffer(dist.group.WORLD)
    N, H, E, K = 24 - rank, 256, 8, 2
    g = torch.Generator().manual_seed(50 + rank)
    for i, (fp8, align, nbias) in enumerate(itertools.product((True, False), (1, 128), (0, 1, 2))):
        x = torch.randn((N, H), generator=g).to(torch.bfloat16)
        idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(N)])
        w = torch.rand((N, K), generator=g)
        rx, ri, rw, counts, h, _ = ref.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E,
                                                expert_alignment=align, quantize_fp8=fp8)
        assert all(c % align == 0 for c in counts)
        hc = tuple(t.clone() if isinstance(t, torch.Tensor) else t for t in h)
        cx = ref.dispatch(x, handle=hc, quantize_fp8=fp8)[0]
        if fp8:
            assert torch.equal(cx[0].view(torch.uint8), rx[0].view(torch.uint8)) and torch.equal(cx[1], rx[1])
        else:
            assert torch.equal(cx, rx)
        n = (rx[0] if fp8 else rx).shape[0]
        biases = [torch.full((N, H), float(b + 1), dtype=torch.bfloat16) for b in range(nbias)]
        bias = None if nbias == 0 else (biases[0] if nbias == 1 else tuple(biases))
        out, ow, _ = ref.combine(torch.ones((n, H), dtype=torch.bfloat16), h, topk_weights=rw, bias=bias)
        dst = (idx // (E // world)).tolist()
        expect = torch.tensor([len(set(d)) for d in dst], dtype=torch.float32) + sum(b + 1 for b in range(nbias))
        assert torch.equal(out[:, 0].float(), expect), (i, out[:, 0], expect)
        assert torch.allclose(ow, w, atol=1e-6)


def test_reference_mode_matrix_gloo():
    run_ranks(_matrix_oracle_body, 2, 'gloo')
