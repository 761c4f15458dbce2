"""GPU tests of the SGLang-style normal-mode dispatcher adapter: two layers share one buffer,
dispatch/combine match the oracle, one live dispatch per buffer, reference-counted teardown."""
import pytest
import torch
import torch.distributed as dist

from tests._dist import run_ranks
from tests.test_gpu_intranode import _make_inputs, _worlds

pytestmark = pytest.mark.gpu


def _adapter_body(rank, world):
    from deepep_slingshot_b200 import ReferenceBuffer
    from deepep_slingshot_b200.integrations.sglang_dispatcher import DeepEPB200Normal
    group = dist.group.WORLD
    H, E, K, N = 1024, 32, 4, 300
    layers = [DeepEPB200Normal(group, H, E, expert_alignment=128) for _ in range(2)]
    ref = ReferenceBuffer(group)
    for it, layer in enumerate(layers * 2):
        x, idx, w = _make_inputs(rank, N - rank, H, E, K, seed=it)
        rx, ri, rw, counts, _ = layer._dispatch_core(x, idx, w)
        ex, ei, ew, ecounts, eh, _ = ref.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E, expert_alignment=128)
        torch.cuda.synchronize()
        assert torch.equal(rx, ex) and torch.equal(ri, ei) and torch.equal(rw, ew) and list(counts) == list(ecounts)
        other = layers[1 - layers.index(layer)]
        with pytest.raises(RuntimeError):
            other._dispatch_core(x, idx, w)  # the shared buffer has a live dispatch
        y = (rx.float() * 0.5).to(torch.bfloat16)
        out, _ = layer._combine_core(y)
        eo, _, _ = ref.combine(y, eh)
        torch.cuda.synchronize()
        assert torch.allclose(out.float(), eo.float(), atol=1e-2, rtol=1e-2)
    assert layers[0].buffer is layers[1].buffer
    layers[0].close()
    assert len(DeepEPB200Normal.pool) == 1
    layers[1].close()
    assert len(DeepEPB200Normal.pool) == 0


@pytest.mark.parametrize('world', _worlds())
def test_sglang_adapter(world):
    run_ranks(_adapter_body, world, backend='nccl')
