"""GPU tests of the bf16 tcgen05 grouped GEMMs with MN-major operands (weights and activations read
as they lie, no transposes), against fp32 torch references.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(got, ref):
    return float((got.float() - ref).norm() / ref.norm().clamp_min(1e-6))


def test_dgrad_mn_major_weights():
    from deepep_slingshot_b200.ops.gemm import grouped_gemm_bf16, grouped_gemm_bf16_reference
    torch.manual_seed(0)
    E, k, n = 3, 256, 384
    counts = torch.tensor([128, 5, 200], dtype=torch.int32, device='cuda')
    aligned = ((counts + 127) // 128) * 128
    offsets = torch.zeros(E + 1, dtype=torch.int32, device='cuda')
    offsets[1:] = torch.cumsum(aligned, 0)
    rows = int(offsets[-1])
    a = torch.randn((rows, k), device='cuda').to(torch.bfloat16)
    w = (torch.randn((E, k, n), device='cuda') * 0.1).to(torch.bfloat16)  # forward layout [E, k, n]
    d = grouped_gemm_bf16(a, w, offsets, counts, b_mn_major=True)
    ref = grouped_gemm_bf16_reference(a, w.transpose(1, 2).contiguous(), offsets, counts)
    torch.cuda.synchronize()
    off = offsets.tolist()
    for e, c in enumerate(counts.tolist()):
        assert _rel(d[off[e]:off[e] + c], ref[off[e]:off[e] + c]) < 1e-2
    # the K-major path on transposed weights agrees
    d_k = grouped_gemm_bf16(a, w.transpose(1, 2).contiguous(), offsets, counts)
    for e, c in enumerate(counts.tolist()):
        assert _rel(d[off[e]:off[e] + c], d_k[off[e]:off[e] + c].float()) < 1e-3


def test_wgrad_mn_major_rows():
    from deepep_slingshot_b200.ops.gemm import grouped_gemm_bf16_wgrad_reference, grouped_gemm_bf16_wgrad_rows
    torch.manual_seed(1)
    m, n = 256, 384
    offsets = torch.tensor([0, 128, 128, 384], dtype=torch.int32, device='cuda')  # expert 1 has no rows
    K = int(offsets[-1])
    a = torch.randn((K, m), device='cuda').to(torch.bfloat16)
    b = torch.randn((K, n), device='cuda').to(torch.bfloat16)
    d = grouped_gemm_bf16_wgrad_rows(a, b, offsets)
    ref = grouped_gemm_bf16_wgrad_reference(a.t().contiguous(), b.t().contiguous(), offsets)
    torch.cuda.synchronize()
    assert d.shape == (3, m, n)
    assert float(d[1].abs().max()) == 0.0
    for e in (0, 2):
        assert _rel(d[e], ref[e]) < 1e-2


def _moe_mn_body(rank, world, *args):
    from tests.test_gpu_moe import _moe_body
    _moe_body(rank, world, *args, bwd='tcgen05_mn')


@pytest.mark.parametrize('world', [1, 2])
def test_moe_layer_backward_mn_major(world):
    """The MoE layer's gradients with the MN-major tcgen05 backward GEMMs (no transposes) against
    fp32 autograd, as the K-major and torch paths are checked in tests/test_gpu_moe.py."""
    from tests._dist import run_ranks
    if torch.cuda.device_count() < world:
        pytest.skip(f'needs {world} GPUs')
    run_ranks(_moe_mn_body, world, 'nccl', args=(256, 1024, 512, 16, 4))
