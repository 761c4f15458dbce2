"""Host-side unit tests (no GPU): region layouts, record formats, FP8 reference math, routings."""
import pytest
import torch

from deepep_slingshot_b200.utils import gate
from deepep_slingshot_b200.utils.math import align, pack_ue8m0, per_token_cast_back, per_token_cast_to_fp8


def _ext():
    from deepep_slingshot_b200._ext import load_ext
    ext = load_ext()
    if ext is None:
        pytest.skip('extension not built')
    return ext


@pytest.mark.parametrize('hidden', [256, 2048, 4096, 7168])
@pytest.mark.parametrize('ranks', [1, 2, 4, 8])
def test_normal_region_capacity(hidden, ranks):
    ext = _ext()
    for tokens in (128, 4096, 8192):
        size = ext.normal_region_size_for(tokens, hidden, ranks)
        assert size % (2 << 20) == 0
        cap = ext.normal_layout_capacity(size, hidden, ranks)
        assert cap >= tokens, (tokens, cap)


def test_ll_region_size_monotonic():
    ext = _ext()
    a = ext.ll_region_size_for(128, 7168, 8, 256)
    b = ext.ll_region_size_for(256, 7168, 8, 256)
    assert 0 < a < b and a % (2 << 20) == 0


def test_fp8_reference_roundtrip():
    x = torch.randn(64, 7168, dtype=torch.bfloat16)
    q, s = per_token_cast_to_fp8(x)
    assert q.dtype == torch.float8_e4m3fn and s.shape == (64, 56)
    back = per_token_cast_back(q, s)
    rel = ((back.float() - x.float()).abs().max() / x.float().abs().max()).item()
    assert rel < 0.07
    q2, s2 = per_token_cast_to_fp8(x, round_scale=True)
    e = torch.log2(s2)
    assert torch.equal(e, torch.round(e))
    packed = pack_ue8m0(s2)
    assert packed.shape == (64, 14) and packed.dtype == torch.int32
    back2 = per_token_cast_back(q2, packed)
    assert torch.equal(back2, per_token_cast_back(q2, s2))


def test_routings_shapes_and_weights():
    g = torch.Generator().manual_seed(0)
    for fn in (gate.normal_routing, gate.uniform_routing, gate.zipf_routing):
        idx, w = fn(512, 256, 8, generator=g)
        assert idx.shape == (512, 8) and idx.dtype == torch.int64
        assert torch.allclose(w.sum(1), torch.ones(512))
        assert (idx.sort(1).values.diff(dim=1) > 0).all()  # distinct experts per token
    idx, _ = gate.zipf_routing(8192, 256, 8, s=1.1, generator=g)
    counts = torch.bincount(idx.flatten(), minlength=256).float()
    assert counts.max() > 4 * counts.mean()  # skewed popularity


def test_align():
    assert align(5, 4) == 8 and align(8, 4) == 8
