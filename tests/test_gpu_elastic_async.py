"""GPU test of the v2 dispatch in asynchronous mode (`async_with_compute_stream=True`): the wrapper's
post-processing (source metadata, expert prefix sums, the expanded layout) runs on the comm stream
after the kernels, the returned event covers it, and every output equals the synchronous call's.
"""
import pytest
import torch
import torch.distributed as dist

from tests._dist import run_ranks
from tests.test_gpu_intranode import _make_inputs, _worlds

pytestmark = pytest.mark.gpu


def _async_body(rank, world, N, H, E, K):
    from deepep_slingshot_b200 import ElasticBuffer
    buf = ElasticBuffer(dist.group.WORLD, num_max_tokens_per_rank=N, hidden=H, num_topk=K, use_fp8_dispatch=True,
                        num_gpu_timeout_secs=20)
    for it, expand in enumerate((False, True)):
        x, idx, w = _make_inputs(rank, N - rank, H, E, K, seed=it)
        kw = dict(topk_idx=idx, topk_weights=w, num_experts=E, quantize_fp8=True, do_expand=expand,
                  expert_alignment=128 if expand else 1)
        (sx, ss), si, sw, sh, _ = buf.dispatch(x, **kw)
        torch.cuda.synchronize()
        (ax, as_), ai, aw, ah, ev = buf.dispatch(x, **kw, async_with_compute_stream=True)
        ev.current_stream_wait()
        assert torch.equal(ax.view(torch.uint8), sx.view(torch.uint8)), ('x', expand)
        assert torch.equal(as_, ss), ('scales', expand)
        assert torch.equal(ai, si) and torch.equal(aw, sw), ('ids/weights', expand)
        assert torch.equal(ah.recv_src_metadata, sh.recv_src_metadata)
        assert torch.equal(ah.psum_num_recv_tokens_per_expert, sh.psum_num_recv_tokens_per_expert)
        # cached dispatch through the async handle, asynchronously as well
        (cx, cs), *_, cev = buf.dispatch(x, handle=ah, quantize_fp8=True, async_with_compute_stream=True)
        cev.current_stream_wait()
        assert torch.equal(cx.view(torch.uint8), sx.view(torch.uint8)) and torch.equal(cs, ss)
        torch.cuda.synchronize()
    buf.barrier(with_cpu_sync=True)


@pytest.mark.parametrize('world', _worlds()[:2])
def test_elastic_dispatch_async(world):
    run_ranks(_async_body, world, 'nccl', args=(128, 512, 16, 4))
