"""GPU tests of the normal-mode NVLink kernels against the pure-torch oracle (`ReferenceBuffer`).

Every check runs on 1 rank, and on 2/4/8 ranks when the box has that many GPUs. Each case compares
bytes exactly where the math is exact (rows, FP8 bytes, scales, ids, counts, source indices) and
within bf16 tolerance for the combine sums.
"""
import pytest
import torch
import torch.distributed as dist

from tests._dist import run_ranks

pytestmark = pytest.mark.gpu


def _gpus():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _worlds():
    n = _gpus()
    return [w for w in (1, 2, 4, 8) if w <= n] or [1]


def _make_inputs(rank, N, H, E, K, seed=0, kind='normal'):
    from deepep_slingshot_b200.utils import gate
    g = torch.Generator().manual_seed(seed * 1000 + rank)
    x = torch.randn((N, H), generator=g).to(torch.bfloat16).cuda()
    if kind == 'uniform':
        idx, w = gate.uniform_routing(N, E, K, generator=g)
    else:
        idx, w = gate.normal_routing(N, E, K, generator=g)
    if kind == 'drop':
        gate.drop_tokens(idx, w, 0.2, generator=g)
    return x, idx.cuda(), w.cuda()


def _intranode_body(rank, world, N, H, E, K, kind):
    from deepep_slingshot_b200 import Buffer, ReferenceBuffer
    group = dist.group.WORLD
    buf = Buffer(group, num_nvl_bytes=Buffer.get_nvl_buffer_size_hint(N, H, world), num_gpu_timeout_secs=20)
    ref = ReferenceBuffer(group)
    for it in range(3):
        x, idx, w = _make_inputs(rank, N - rank * 3, H, E, K, seed=it, kind=kind)
        # layout
        a = buf.get_dispatch_layout(idx, E)
        b = ref.get_dispatch_layout(idx, E)
        assert torch.equal(a[0], b[0]) and torch.equal(a[2], b[2]) and torch.equal(a[3], b[3])
        ntpr, _, ntpe, itir, _ = a
        # bf16 dispatch
        rx, ri, rw, lst, h, _ = buf.dispatch(x, num_tokens_per_rank=ntpr, is_token_in_rank=itir,
                                             num_tokens_per_expert=ntpe, topk_idx=idx, topk_weights=w,
                                             expert_alignment=4 if it == 1 else 1)
        ex, ei, ew, elst, eh, _ = ref.dispatch(x, num_tokens_per_rank=ntpr, is_token_in_rank=itir,
                                               num_tokens_per_expert=ntpe, topk_idx=idx, topk_weights=w,
                                               expert_alignment=4 if it == 1 else 1)
        torch.cuda.synchronize()
        assert rx.shape == ex.shape and torch.equal(rx, ex)
        assert torch.equal(ri, ei) and torch.equal(rw, ew)
        assert lst == elst
        assert torch.equal(h[3], eh[3])  # recv_src_idx
        assert torch.equal(h[0], eh[0].to(h[0].device))  # rank prefix matrix
        assert torch.equal(h[5], eh[5])  # send_head
        # combine (unweighted sum + weights sum), with bias on the second iteration
        y = (rx.float() * (rank + 1) * 0.5).to(torch.bfloat16)
        bias = torch.randn_like(x) if it == 2 else None
        out, out_w, _ = buf.combine(y, h, topk_weights=rw, bias=bias)
        eo, eow, _ = ref.combine(y, eh, topk_weights=ew, bias=bias)
        torch.cuda.synchronize()
        assert torch.allclose(out.float(), eo.float(), atol=1e-2, rtol=1e-2), (out.float() - eo.float()).abs().max()
        assert torch.allclose(out_w, eow, atol=1e-6)
        # fused FP8 quantization dispatch (bytes and scales exact)
        (qx, qs), qi, qw, qlst, qh, _ = buf.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E, quantize_fp8=True)
        (fx, fs), fi, fw, flst, fh, _ = ref.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E, quantize_fp8=True)
        torch.cuda.synchronize()
        assert torch.equal(qx.view(torch.uint8), fx.view(torch.uint8))
        assert torch.equal(qs, fs)
        assert torch.equal(qi, fi) and qlst == flst
        # pre-quantized FP8 input, column-major scales
        (px, ps), *_ = buf.dispatch((fx_in := ref_quant(x)), topk_idx=idx, topk_weights=w, num_experts=E,
                                     scales_col_major=True)
        torch.cuda.synchronize()
        assert torch.equal(px.view(torch.uint8), fx.view(torch.uint8)) and torch.equal(ps, fs)
        # cached dispatch reuses the handle
        cx, *_ = buf.dispatch(x, handle=h)
        torch.cuda.synchronize()
        assert torch.equal(cx, rx)
        # no-CPU-sync (worst case) dispatch
        worst = N * world
        wx, wi, ww, wl, wh, _ = buf.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E, num_worst_tokens=worst)
        torch.cuda.synchronize()
        n = rx.shape[0]
        assert wx.shape[0] == worst and wl == []
        assert torch.equal(wx[:n], rx) and torch.equal(wi[:n], ri) and (wi[n:] == -1).all()
        # async + previous_event on the comm stream
        ev = Buffer.capture()
        ax, ai, aw, al, ah, aev = buf.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E, previous_event=ev,
                                               async_finish=True, allocate_on_comm_stream=True)
        aev.current_stream_wait()
        assert torch.equal(ax, rx)
        ao, _, aev2 = buf.combine(y, ah, async_finish=True)
        aev2.current_stream_wait()
        eo2, _, _ = ref.combine(y, eh)
        assert torch.allclose(ao.float(), eo2.float(), atol=1e-2, rtol=1e-2)
    buf.check_error()


def ref_quant(x):
    from deepep_slingshot_b200.utils.math import per_token_cast_to_fp8
    return per_token_cast_to_fp8(x)


@pytest.mark.parametrize('world', _worlds())
@pytest.mark.parametrize('kind', ['normal', 'drop'])
def test_intranode_dispatch_combine(world, kind):
    run_ranks(_intranode_body, world, 'nccl', args=(256, 1024, 32, 8, kind))


@pytest.mark.parametrize('world', _worlds()[-1:])
def test_intranode_deepseek_shape(world):
    run_ranks(_intranode_body, world, 'nccl', args=(1024, 7168, 256, 8, 'normal'))


def _timeout_body(rank, world):
    """Delayed peer: rank 1 skips a dispatch; rank 0's bounded notify wait must expire, report
    TIMEOUT as a Python exception (no trap, GPU stays usable), and a new buffer must work."""
    from deepep_slingshot_b200 import Buffer
    group = dist.group.WORLD
    N, H, E, K = 64, 256, 16, 4
    buf = Buffer(group, num_nvl_bytes=Buffer.get_nvl_buffer_size_hint(N, H, world), num_gpu_timeout_secs=1.0,
                 explicitly_destroy=True)
    x, idx, w = _make_inputs(rank, N, H, E, K)
    if rank == 0:
        with pytest.raises(RuntimeError, match='timeout'):
            buf.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E)
        torch.cuda.synchronize()
        code = buf.get_error_state()[0]
        assert code == 1, code
    dist.barrier()
    torch.cuda.synchronize()
    buf.destroy()
    dist.barrier()
    buf2 = Buffer(group, num_nvl_bytes=Buffer.get_nvl_buffer_size_hint(N, H, world), num_gpu_timeout_secs=10)
    rx, *_ = buf2.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E)
    torch.cuda.synchronize()
    buf2.check_error()


@pytest.mark.skipif(_gpus() < 2, reason='needs 2 GPUs')
def test_delayed_peer_timeout_reports():
    run_ranks(_timeout_body, 2, 'nccl')


def test_fp8_cast_kernels_match_torch():
    from deepep_slingshot_b200.ops.quant import per_token_cast_back, per_token_cast_to_fp8
    from deepep_slingshot_b200.utils import math as m
    x = torch.randn((1000, 7168), dtype=torch.bfloat16, device='cuda') * 3
    for rs in (False, True):
        q, s = per_token_cast_to_fp8(x, round_scale=rs)
        rq, rsc = m.per_token_cast_to_fp8(x, round_scale=rs)
        assert torch.equal(q.view(torch.uint8), rq.view(torch.uint8))
        assert torch.equal(s, rsc)
        assert torch.equal(per_token_cast_back(q, s), m.per_token_cast_back(rq, rsc))
