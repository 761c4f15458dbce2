"""GPU tests of the v2 API (`ElasticBuffer` / `EPHandle`): normal and expanded layouts, cached
handles, combine (incl. expanded combine), and the shrink-mode mask APIs of `Buffer`."""
import pytest
import torch
import torch.distributed as dist

from tests._dist import run_ranks
from tests.test_gpu_intranode import _make_inputs, _worlds

pytestmark = pytest.mark.gpu


def _elastic_body(rank, world, N, H, E, K):
    from deepep_slingshot_b200 import ElasticBuffer, ReferenceBuffer
    from deepep_slingshot_b200.ops.permute import unpermute_reference
    group = dist.group.WORLD
    buf = ElasticBuffer(group, num_max_tokens_per_rank=N, hidden=H, num_topk=K, use_fp8_dispatch=True,
                        num_gpu_timeout_secs=20)
    ref = ReferenceBuffer(group)
    assert buf.get_logical_domain_size() == (1, world) and buf.get_physical_domain_size() == (1, world)
    E_l = E // world
    for it in range(2):
        x, idx, w = _make_inputs(rank, N - rank, H, E, K, seed=it)
        # normal layout, fused FP8
        (rx, rs), ri, rw, h, _ = buf.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E, quantize_fp8=True)
        (ex, es), ei, ew, _, eh, _ = ref.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E, quantize_fp8=True)
        torch.cuda.synchronize()
        assert torch.equal(rx.view(torch.uint8), ex.view(torch.uint8)) and torch.equal(rs, es)
        assert torch.equal(ri, ei) and torch.equal(rw, ew)
        assert int(h.psum_num_recv_tokens_per_scaleup_rank[-1]) == rx.shape[0]
        src_rank = h.recv_src_metadata[:, 1].long()
        assert torch.equal(h.recv_src_metadata[:, 0] - src_rank * N, eh[3].long().to(torch.int32))
        # cached
        (cx, cs), *_ = buf.dispatch(x, handle=h, quantize_fp8=True)
        torch.cuda.synchronize()
        assert torch.equal(cx.view(torch.uint8), rx.view(torch.uint8))
        # combine (unweighted sum over ranks) + weights sum
        y = torch.randn((rx.shape[0], H), device='cuda').to(torch.bfloat16)
        out, ow, _ = buf.combine(y, h, topk_weights=rw)
        eo, eow, _ = ref.combine(y, eh, topk_weights=ew)
        torch.cuda.synchronize()
        assert torch.allclose(out.float(), eo.float(), atol=1e-2, rtol=1e-2)
        assert torch.allclose(ow, eow, atol=1e-6)
        # expanded layout: one row per (token, local expert), grouped by expert, aligned to 128
        (xx, xs), xi, xw, xh, _ = buf.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E, quantize_fp8=True,
                                               expert_alignment=128, do_expand=True)
        torch.cuda.synchronize()
        rm = xh.row_map
        valid = rm >= 0
        assert torch.equal(valid, ri >= 0)
        rows = rm[valid].long()
        tok = torch.arange(ri.shape[0], device='cuda').unsqueeze(1).expand_as(ri)[valid]
        assert torch.equal(xx[rows].view(torch.uint8), rx[tok].view(torch.uint8))
        assert torch.equal(xs[rows], rs[tok])
        off = xh.expert_offsets
        e_of = ri[valid]
        assert ((rows >= off[e_of].long()) & (rows < xh.psum_num_recv_tokens_per_expert[e_of].long())).all()
        assert (off[:-1] % 128 == 0).all() and xx.shape[0] == int(off[-1])
        # expanded combine: rows of a token are summed, then combined across ranks
        ye = torch.randn((xx.shape[0], H), device='cuda').to(torch.bfloat16)
        xo, _, _ = buf.combine(ye, xh)
        yt = unpermute_reference(ye, rm)
        eo2, _, _ = ref.combine(yt, eh)
        torch.cuda.synchronize()
        assert torch.allclose(xo.float(), eo2.float(), atol=3e-2, rtol=2e-2)
    buf.barrier(with_cpu_sync=True)


@pytest.mark.parametrize('world', _worlds())
def test_elastic_buffer(world):
    run_ranks(_elastic_body, world, 'nccl', args=(200, 1024, 32, 6))


def _mask_body(rank, world):
    from deepep_slingshot_b200 import Buffer
    buf = Buffer(dist.group.WORLD, num_rdma_bytes=Buffer.get_low_latency_rdma_size_hint(16, 256, world, 8 * world),
                 low_latency_mode=True, enable_shrink=True)
    status = torch.zeros(world, dtype=torch.int32, device='cuda')
    buf.low_latency_query_mask_buffer(status)
    assert status.sum().item() == 0
    buf.low_latency_update_mask_buffer(world - 1, True)
    buf.low_latency_query_mask_buffer(status)
    torch.cuda.synchronize()
    assert status.tolist() == [0] * (world - 1) + [1]
    buf.low_latency_update_mask_buffer(world - 1, False)
    buf.low_latency_update_mask_buffer(0, True)
    buf.low_latency_clean_mask_buffer()
    buf.low_latency_query_mask_buffer(status)
    torch.cuda.synchronize()
    assert status.sum().item() == 0


def test_shrink_mask_apis():
    run_ranks(_mask_body, 1, 'nccl')
