"""GPU edge cases against the oracle: ranks with 0, 1, 2 or 3 tokens, a hot rank that receives every
token while the others receive none, and low-latency calls with empty ranks."""
import pytest
import torch
import torch.distributed as dist

from tests._dist import run_ranks
from tests.test_gpu_intranode import _worlds

pytestmark = pytest.mark.gpu


def _edge_body(rank, world):
    from deepep_slingshot_b200 import Buffer, ReferenceBuffer
    group = dist.group.WORLD
    H, E, K = 256, 8, 2
    buf = Buffer(group, num_nvl_bytes=Buffer.get_nvl_buffer_size_hint(64, H, world),
                 num_rdma_bytes=Buffer.get_low_latency_rdma_size_hint(8, H, world, E), low_latency_mode=True,
                 num_gpu_timeout_secs=20)
    ref = ReferenceBuffer(group)
    g = torch.Generator().manual_seed(rank)
    for case in range(3):
        N = [0, 1, 3, 2][(rank + case) % 4]
        x = torch.randn((N, H), generator=g).to(torch.bfloat16).cuda()
        if case == 2:  # hot rank: every token on rank 0's experts, other ranks receive nothing
            idx = torch.arange(K, dtype=torch.int64).expand(N, K).contiguous().cuda()
        else:
            idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(N)]).cuda() if N else \
                torch.empty((0, K), dtype=torch.int64, device='cuda')
        w = torch.rand((N, K), generator=g).cuda()
        for fp8 in (False, True):
            kw = dict(topk_idx=idx, topk_weights=w, num_experts=E, quantize_fp8=fp8)
            rx, ri, rw, lst, h, _ = buf.dispatch(x, **kw)
            ex, ei, ew, elst, eh, _ = ref.dispatch(x, **kw)
            torch.cuda.synchronize()
            if fp8:
                assert torch.equal(rx[0].view(torch.uint8), ex[0].view(torch.uint8)) and torch.equal(rx[1], ex[1])
                n = rx[0].shape[0]
            else:
                assert torch.equal(rx, ex)
                n = rx.shape[0]
            assert torch.equal(ri, ei) and torch.equal(rw, ew) and lst == elst
            y = torch.randn((n, H), generator=g).to(torch.bfloat16).cuda()
            out, ow, _ = buf.combine(y, h, topk_weights=rw)
            eo, eow, _ = ref.combine(y, eh, topk_weights=ew)
            torch.cuda.synchronize()
            assert out.shape == (N, H) and torch.allclose(out.float(), eo.float(), atol=1e-2, rtol=1e-2)
        # low latency with possibly empty ranks
        recv, cnt, lh, _, hook = buf.low_latency_dispatch(x, idx, 8, E, use_fp8=False, return_recv_hook=True)
        hook()
        erecv, ecnt, elh, _, _ = ref.low_latency_dispatch(x, idx, 8, E, use_fp8=False)
        torch.cuda.synchronize()
        assert torch.equal(cnt, ecnt)
        ly = torch.zeros((E // world, 8 * world, H), dtype=torch.bfloat16, device='cuda')
        lo, _, chook = buf.low_latency_combine(ly, idx, w, lh, return_recv_hook=True)
        chook()
        torch.cuda.synchronize()
        assert lo.shape == (N, H) and (lo == 0).all()
    buf.check_error()


@pytest.mark.parametrize('world', _worlds())
def test_edge_cases(world):
    run_ranks(_edge_body, world, backend='nccl')
