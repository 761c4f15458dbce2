"""GPU test of the low-latency FP8 dispatch options DeepEP's low-latency test covers and the other
GPU tests do not: power-of-two scales (`round_scale`), packed UE8M0 scales (`use_ue8m0`), and the
asynchronous mode without a hook (`async_finish` + the returned event), against `ReferenceBuffer`.
"""
import pytest
import torch
import torch.distributed as dist

from tests._dist import run_ranks
from tests.test_gpu_intranode import _make_inputs, _worlds
from tests.test_gpu_low_latency import _sorted_rows

pytestmark = pytest.mark.gpu


def _unpack_ue8m0(packed: torch.Tensor) -> torch.Tensor:
    """int32 [slots, nb/4] (4 exponent bytes each) -> fp32 [slots, nb] powers of two."""
    b = packed.contiguous().view(torch.uint8).to(torch.int32)
    return (b << 23).view(torch.float32)


def _options_body(rank, world, N, H, E, K):
    from deepep_slingshot_b200 import Buffer, ReferenceBuffer
    group = dist.group.WORLD
    buf = Buffer(group, num_rdma_bytes=Buffer.get_low_latency_rdma_size_hint(N, H, world, E), low_latency_mode=True,
                 num_gpu_timeout_secs=20)
    ref = ReferenceBuffer(group)
    E_l = E // world
    for i, (ue8m0, hook) in enumerate([(False, True), (True, True), (False, False), (True, False)]):
        x, idx, w = _make_inputs(rank, N - rank, H, E, K, seed=i, kind='uniform')
        recv, cnt, h, ev, hk = buf.low_latency_dispatch(x, idx, N, E, use_fp8=True, round_scale=True, use_ue8m0=ue8m0,
                                                        async_finish=not hook, return_recv_hook=hook)
        if hook:
            hk()
        else:
            ev.current_stream_wait()
        erecv, ecnt, eh, _, _ = ref.low_latency_dispatch(x, idx, N, E, use_fp8=True, round_scale=True)
        torch.cuda.synchronize()
        tag = f'ue8m0={ue8m0} hook={hook}'
        assert torch.equal(cnt, ecnt), tag
        for e in range(E_l):
            n = int(cnt[e])
            scales = _unpack_ue8m0(recv[1][e]) if ue8m0 else recv[1][e]
            if ue8m0:
                assert recv[1].dtype == torch.int32 and recv[1].shape[-1] == H // 512, tag
            gx, gs = _sorted_rows(n, h[0][e], h[7][e], K, recv[0][e].view(torch.uint8), scales)
            rx, rs = _sorted_rows(n, eh[0][e], eh[7][e], K, erecv[0][e].view(torch.uint8), erecv[1][e])
            assert torch.equal(gx, rx), tag
            assert torch.equal(gs, rs), tag
            # power-of-two scales: the mantissa bits are zero
            assert bool(((gs.view(torch.int32) & 0x7fffff) == 0).all()), tag
        # the combine of the dispatched rows still works after every mode
        from deepep_slingshot_b200.utils.math import per_token_cast_back
        xs = torch.stack([per_token_cast_back(recv[0][e], (_unpack_ue8m0(recv[1][e]) if ue8m0 else recv[1][e]).contiguous())
                          for e in range(E_l)])
        out, _, _ = buf.low_latency_combine(xs, idx, w, h)
        exs = torch.stack([per_token_cast_back(erecv[0][e], erecv[1][e]) for e in range(E_l)])
        eout, _, _ = ref.low_latency_combine(exs, idx, w, eh)
        torch.cuda.synchronize()
        assert torch.allclose(out.float(), eout.float(), atol=2e-2, rtol=2e-2), tag
    buf.check_error()


@pytest.mark.parametrize('world', _worlds()[:2])
def test_low_latency_fp8_options(world):
    run_ranks(_options_body, world, 'nccl', args=(64, 2048, 8 * world, 4))
