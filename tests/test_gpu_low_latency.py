"""GPU tests of the low-latency (decode) kernels against the pure-torch oracle.

Rows inside one local expert arrive in NVLink arrival order, so per-expert row sets are compared
after sorting by (source rank, source token).
"""
import pytest
import torch
import torch.distributed as dist

from tests._dist import run_ranks
from tests.test_gpu_intranode import _make_inputs, _worlds

pytestmark = pytest.mark.gpu


def _sorted_rows(n, src_info, src_meta, K, *tensors):
    key = (src_meta[:n] // K).to(torch.int64) * 1_000_000 + src_info[:n].to(torch.int64)
    order = torch.argsort(key)
    return [t[:n][order] for t in tensors]


def _ll_body(rank, world, N, H, E, K, use_fp8, hook):
    from deepep_slingshot_b200 import Buffer, ReferenceBuffer
    group = dist.group.WORLD
    maxT = N
    buf = Buffer(group, num_rdma_bytes=Buffer.get_low_latency_rdma_size_hint(maxT, H, world, E), low_latency_mode=True,
                 num_gpu_timeout_secs=20)
    ref = ReferenceBuffer(group)
    E_l = E // world
    for it in range(4):
        x, idx, w = _make_inputs(rank, N - rank, H, E, K, seed=it, kind='uniform' if it % 2 else 'drop')
        stats = torch.zeros(E_l, dtype=torch.int32, device='cuda')
        recv, cnt, h, ev, hk = buf.low_latency_dispatch(x, idx, maxT, E, cumulative_local_expert_recv_stats=stats,
                                                        use_fp8=use_fp8, return_recv_hook=hook)
        if hook:
            hk()
        erecv, ecnt, eh, _, _ = ref.low_latency_dispatch(x, idx, maxT, E, use_fp8=use_fp8)
        torch.cuda.synchronize()
        assert torch.equal(cnt, ecnt), (cnt, ecnt)
        assert torch.equal(stats, ecnt)
        assert torch.equal(h[1], eh[1])  # per-source counts
        for e in range(E_l):
            n = int(cnt[e])
            if use_fp8:
                gx, gs, gi, gm = _sorted_rows(n, h[0][e], h[7][e], K, recv[0][e].view(torch.uint8), recv[1][e], h[0][e], h[7][e])
                rx_, rs_, ri_, rm_ = _sorted_rows(n, eh[0][e], eh[7][e], K, erecv[0][e].view(torch.uint8), erecv[1][e], eh[0][e], eh[7][e])
                assert torch.equal(gx, rx_) and torch.equal(gs, rs_)
            else:
                gx, gi, gm = _sorted_rows(n, h[0][e], h[7][e], K, recv[e], h[0][e], h[7][e])
                rx_, ri_, rm_ = _sorted_rows(n, eh[0][e], eh[7][e], K, erecv[e], eh[0][e], eh[7][e])
                assert torch.equal(gx, rx_)
            assert torch.equal(gi, ri_) and torch.equal(gm, rm_)
        # expert outputs: dequantized rows scaled per expert; combine is top-k weighted
        if use_fp8:
            from deepep_slingshot_b200.utils.math import per_token_cast_back
            xs = torch.stack([per_token_cast_back(recv[0][e], recv[1][e]) for e in range(E_l)])
        else:
            xs = recv.clone()
        xs = (xs.float() * (1 + torch.arange(E_l, device='cuda').view(-1, 1, 1) * 0.25)).to(torch.bfloat16)
        out, _, chk = buf.low_latency_combine(xs, idx, w, h, return_recv_hook=hook)
        if hook:
            chk()
        # oracle combine uses the oracle's row order
        if use_fp8:
            exs = torch.stack([per_token_cast_back(erecv[0][e], erecv[1][e]) for e in range(E_l)])
        else:
            exs = erecv.clone()
        exs = (exs.float() * (1 + torch.arange(E_l, device='cuda').view(-1, 1, 1) * 0.25)).to(torch.bfloat16)
        eout, _, _ = ref.low_latency_combine(exs, idx, w, eh)
        torch.cuda.synchronize()
        assert torch.allclose(out.float(), eout.float(), atol=2e-2, rtol=2e-2), (out.float() - eout.float()).abs().max()
    buf.check_error()


@pytest.mark.parametrize('world', _worlds())
@pytest.mark.parametrize('use_fp8', [True, False])
@pytest.mark.parametrize('hook', [True, False])
def test_low_latency(world, use_fp8, hook):
    run_ranks(_ll_body, world, 'nccl', args=(64, 1024, 32, 8, use_fp8, hook))


@pytest.mark.parametrize('world', _worlds()[-1:])
def test_low_latency_deepseek_shape(world):
    run_ranks(_ll_body, world, 'nccl', args=(128, 7168, 256, 8, True, True))


def _ll_logfmt_body(rank, world, N, H, E, K, hook):
    """LL combine with `use_logfmt=True`: expert outputs below 1 travel LogFMT-10 encoded, larger
    ones as raw bf16 groups; compared with the oracle that applies the same number format."""
    from deepep_slingshot_b200 import Buffer, ReferenceBuffer
    from deepep_slingshot_b200.utils.math import calc_diff
    group = dist.group.WORLD
    buf = Buffer(group, num_rdma_bytes=Buffer.get_low_latency_rdma_size_hint(N, H, world, E), low_latency_mode=True,
                 num_gpu_timeout_secs=20)
    ref = ReferenceBuffer(group)
    E_l = E // world
    for it in range(3):
        x, idx, w = _make_inputs(rank, N - rank, H, E, K, seed=10 + it, kind='uniform')
        recv, cnt, h, _, hk = buf.low_latency_dispatch(x, idx, N, E, use_fp8=False, return_recv_hook=hook)
        if hook:
            hk()
        erecv, ecnt, eh, _, _ = ref.low_latency_dispatch(x, idx, N, E, use_fp8=False)
        # most experts produce small outputs (encoded); expert 0 produces large ones (raw groups);
        # the first 64 columns are zeroed on expert 1 (zeros inside encoded groups)
        scale = torch.full((E_l, 1, 1), 0.03, device='cuda')
        scale[0] = 2.0
        xs = (recv.float() * scale).to(torch.bfloat16)
        exs = (erecv.float() * scale).to(torch.bfloat16)
        if E_l > 1:
            xs[1, :, :64] = 0
            exs[1, :, :64] = 0
        out, _, chk = buf.low_latency_combine(xs, idx, w, h, use_logfmt=True, return_recv_hook=hook)
        if hook:
            chk()
        eout, _, _ = ref.low_latency_combine(exs, idx, w, eh, use_logfmt=True)
        plain, _, _ = ref.low_latency_combine(exs, idx, w, eh)
        torch.cuda.synchronize()
        assert calc_diff(out.float(), eout.float()) < 1e-5, calc_diff(out.float(), eout.float())
        assert torch.allclose(out.float(), eout.float(), atol=2e-3, rtol=3e-2)
        assert calc_diff(out.float(), plain.float()) < 1e-4  # the format itself stays close to bf16
    buf.check_error()


@pytest.mark.parametrize('world', _worlds())
@pytest.mark.parametrize('hook', [True, False])
def test_low_latency_logfmt(world, hook):
    run_ranks(_ll_logfmt_body, world, 'nccl', args=(64, 2048, 32, 8, hook))
