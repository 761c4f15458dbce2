"""GPU test of the normal-mode API over the mode matrix DeepEP's elastic test enumerates
(tests/elastic/test_ep.py:22-558 of the DeepEP tree): dispatch dtype FP8 / bf16 x expert alignment
1 / 128 x bias none / one / two x (previous event + async + allocation on the comm stream) on / off
x a copied handle for the cached dispatch, every case against `ReferenceBuffer`.
"""
import copy
import itertools

import pytest
import torch
import torch.distributed as dist

from tests._dist import run_ranks
from tests.test_gpu_intranode import _make_inputs, _worlds

pytestmark = pytest.mark.gpu


def _matrix_body(rank, world, N, H, E, K):
    from deepep_slingshot_b200 import Buffer, ReferenceBuffer
    group = dist.group.WORLD
    buf = Buffer(group, num_nvl_bytes=Buffer.get_nvl_buffer_size_hint(N, H, world), num_gpu_timeout_secs=20)
    ref = ReferenceBuffer(group)
    cases = list(itertools.product((True, False), (1, 128), (0, 1, 2), (False, True)))
    for i, (fp8, align, nbias, overlap) in enumerate(cases):
        x, idx, w = _make_inputs(rank, N - rank, H, E, K, seed=i)
        kw = dict(topk_idx=idx, topk_weights=w, num_experts=E, expert_alignment=align, quantize_fp8=fp8)
        extra = {}
        if overlap:
            extra = dict(previous_event=Buffer.capture(), async_finish=True, allocate_on_comm_stream=True)
        rx, ri, rw, counts, h, ev = buf.dispatch(x, **kw, **extra)
        if overlap:
            ev.current_stream_wait()
        ex, ei, ew, ecounts, eh, _ = ref.dispatch(x, **kw)
        torch.cuda.synchronize()
        tag = f'case {i}: fp8={fp8} align={align} bias={nbias} overlap={overlap}'
        if fp8:
            assert torch.equal(rx[0].view(torch.uint8), ex[0].view(torch.uint8)), tag
            assert torch.equal(rx[1], ex[1]), tag
        else:
            assert torch.equal(rx, ex), tag
        assert torch.equal(ri, ei) and torch.equal(rw, ew), tag
        assert list(counts) == list(ecounts), tag
        # cached dispatch through a copy of the handle (fresh tensors: only the handle's contents count)
        hc = tuple(t.clone() if isinstance(t, torch.Tensor) else copy.copy(t) for t in h)
        cx = buf.dispatch(x, handle=hc, quantize_fp8=fp8, **extra_for_cached(overlap, Buffer))
        if overlap:
            cx[5].current_stream_wait()
        torch.cuda.synchronize()
        if fp8:
            assert torch.equal(cx[0][0].view(torch.uint8), rx[0].view(torch.uint8)), tag
        else:
            assert torch.equal(cx[0], rx), tag
        # combine with 0, 1 or 2 bias tensors
        n = (rx[0] if fp8 else rx).shape[0]
        y = torch.randn((n, H), device='cuda').to(torch.bfloat16)
        gb = torch.Generator(device='cuda').manual_seed(77 + i + rank)
        biases = [torch.randn((N - rank, H), device='cuda', generator=gb).to(torch.bfloat16) for _ in range(nbias)]
        bias = None if nbias == 0 else (biases[0] if nbias == 1 else tuple(biases))
        cextra = dict(async_finish=True, allocate_on_comm_stream=True,
                      previous_event=Buffer.capture()) if overlap else {}
        out, ow, cev = buf.combine(y, h, topk_weights=rw, bias=bias, **cextra)
        if overlap:
            cev.current_stream_wait()
        eo, eow, _ = ref.combine(y, eh, topk_weights=ew, bias=bias)
        torch.cuda.synchronize()
        assert torch.allclose(out.float(), eo.float(), atol=2e-2, rtol=2e-2), tag
        assert torch.allclose(ow, eow, atol=1e-6), tag
    buf.check_error()


def extra_for_cached(overlap, Buffer):
    return dict(previous_event=Buffer.capture(), async_finish=True, allocate_on_comm_stream=True) if overlap else {}


@pytest.mark.parametrize('world', _worlds()[:2])
def test_normal_mode_matrix(world):
    run_ranks(_matrix_body, world, 'nccl', args=(96, 512, 16, 4))
