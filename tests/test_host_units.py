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


@pytest.mark.parametrize('tokens,hidden,ranks,experts', [(128, 7168, 8, 256), (64, 2048, 2, 32), (1, 256, 1, 8)])
def test_ll_layout_offsets(tokens, hidden, ranks, experts):
    """Low-latency half layout: ordered, 128-byte aligned, non-overlapping sections that fit the half
    (the LogFMT metadata section included)."""
    ext = _ext()
    l = ext.ll_layout(tokens, hidden, ranks, experts)
    order = ['ctrl_off', 'recv_x_off', 'recv_scales_off', 'recv_src_info_off', 'recv_src_meta_off',
             'combine_recv_off', 'combine_send_off', 'combine_meta_off']
    offs = [l[k] for k in order]
    assert all(o % 128 == 0 for o in offs)
    assert offs == sorted(offs) and len(set(offs)) == len(offs)
    e_l, slots = experts // ranks, ranks * tokens
    assert l['recv_scales_off'] - l['recv_x_off'] >= e_l * slots * hidden * 2
    assert l['combine_send_off'] - l['combine_recv_off'] >= tokens * 16 * hidden * 2
    assert l['half_bytes'] - l['combine_meta_off'] >= tokens * 16 * (hidden // 128) * 4
    assert 2 * l['half_bytes'] <= ext.ll_region_size_for(tokens, hidden, ranks, experts)


@pytest.mark.parametrize('hidden,ranks', [(7168, 8), (1024, 2)])
def test_normal_layout_offsets(hidden, ranks):
    ext = _ext()
    size = ext.normal_region_size_for(4096, hidden, ranks)
    l = ext.normal_layout(size, hidden, ranks)
    for k in ('list_off', 'staging_off', 'combine_off', 'combine_w_off', 'scratch_off', 'arrival_off'):
        assert l[k] % 128 == 0 and l[k] < l['total_bytes'] <= size, k
    assert l['record_bytes'] % 16 == 0 and l['record_bytes'] >= hidden  # FP8 row + metadata, TMA-sized
    assert l['capacity'] >= 4096


def test_symmetric_ctrl_fits():
    ext = _ext()
    assert ext.sym_ctrl_struct_bytes <= ext.sym_ctrl_bytes and ext.sym_ctrl_bytes % 4096 == 0


def test_logfmt_oracle_properties():
    from deepep_slingshot_b200.utils.math import logfmt10_roundtrip
    g = torch.Generator().manual_seed(0)
    small = (torch.randn((8, 1024), generator=g) * 0.05).to(torch.bfloat16)
    big = (torch.randn((8, 1024), generator=g) * 4).to(torch.bfloat16)
    rs = logfmt10_roundtrip(small)
    rel = (rs - small.float()).abs() / small.float().abs().clamp_min(1e-30)
    assert float(rel[small != 0].max()) < 0.05          # 9-bit log levels over <= 32 octaves
    assert torch.equal(torch.sign(rs), torch.sign(small.float()))
    assert torch.equal(logfmt10_roundtrip(big), big.float())  # groups with |x| >= 1 travel raw
    z = small.clone()
    z[:, :128] = 0
    assert (logfmt10_roundtrip(z)[:, :128] == 0).all()


def test_analyze_trace_synthetic():
    from deepep_slingshot_b200.harness.analyze_trace import analyze
    ev = []
    for r in range(2):
        off = 10.0 * r
        for name, s, d in (('dispatch.wait_receivers', 0, 1), ('dispatch.count', 0, 20), ('dispatch.stage', 25, 30),
                           ('dispatch.pull', 25, 100), ('combine.block', 160, 200)):
            ev.append({'name': name, 'pid': r, 'ts': s + off, 'dur': d})
    rep = analyze({'traceEvents': ev})
    assert len(rep) == 1
    p = rep[0]['phases']
    assert p['dispatch.stage']['start_spread_us'] == 10.0 and p['combine.block']['last_rank'] == 1
    assert [c['phase'] for c in rep[0]['critical_path']] == ['dispatch.count', 'dispatch.pull', 'combine.block']


def test_ep_benchmark_byte_counts():
    from deepep_slingshot_b200.harness.ep_benchmark import combine_bytes, dispatch_bytes
    assert dispatch_bytes(10, 7168, 8, True) == 10 * (7168 + 56 * 4 + 64 + 32)
    assert dispatch_bytes(10, 7168, 8, False) == 10 * (2 * 7168 + 64 + 32)
    assert combine_bytes(10, 7168, 8) == 10 * (2 * 7168 + 32)


@pytest.mark.parametrize('ratio', [1.0, 1.5, 3.0])
def test_precise_unbalanced_routing(ratio):
    g = torch.Generator().manual_seed(3)
    N, E, R, K = 2048, 256, 8, 8
    counts = gate.generate_rank_count(N, E, R, K, ratio, generator=g)
    assert (counts.sum(1) == K).all() and int(counts.max()) <= E // R
    tokens_per_rank = (counts > 0).sum(0).float()
    assert abs(float(tokens_per_rank[0] / tokens_per_rank[1:].mean()) - ratio) < 0.05 * ratio
    idx = gate.generate_topk_idx(counts, N, E, R, K, generator=g)
    assert idx.shape == (N, K)
    assert (torch.sort(idx, 1).values.diff(dim=1) != 0).all()
    back = torch.zeros((N, R), dtype=torch.int32)
    back.scatter_add_(1, idx // (E // R), torch.ones_like(idx, dtype=torch.int32))
    assert torch.equal(back, counts)
    scores = gate.get_unbalanced_scores(N, E, R, K, ratio, precise=True, generator=g)
    assert scores.shape == (N, E)


def test_random_unbalanced_scores_ratio():
    g = torch.Generator().manual_seed(4)
    scores = gate.get_unbalanced_scores(4096, 256, 8, 8, 2.0, generator=g)
    epr = 32
    hit = torch.zeros((4096, 8), dtype=torch.bool)
    hit.scatter_(1, torch.topk(scores, 8, dim=-1).indices // epr, True)
    per = hit.float().sum(0)
    assert 1.6 < float(per[0] / per[1:].mean()) < 2.4


def test_elastic_side_feature_size_hints():
    from deepep_slingshot_b200.parallel.elastic import ElasticBuffer

    class G:
        def size(self):
            return 8
    a = ElasticBuffer.get_elastic_buffer_alignment()
    gpu, cpu = ElasticBuffer.get_engram_storage_size_hint(1000, 4096, 128)
    assert gpu % a == 0 and cpu % a == 0 and cpu >= 1000 * 4096 * 2
    pp = ElasticBuffer.get_pp_buffer_size_hint(3 << 20, 2)
    assert pp % a == 0 and pp >= 2 * 2 * (3 << 20)
    nb = ElasticBuffer.get_agrs_num_max_session_bytes(G(), [(33, 64), (7,)], torch.bfloat16)
    assert nb == (8 * 33 * 64 * 2 + 31) // 32 * 32 + (8 * 7 * 2 + 31) // 32 * 32
    assert ElasticBuffer.get_agrs_buffer_size_hint(G(), nb) % a == 0


def test_nvlink_gbs_with_fake_nvml(monkeypatch):
    """NVLink bandwidth from the NVML link count (a fake NVML: reads only, nothing is changed)."""
    import sys
    import types
    from deepep_slingshot_b200.utils import envs

    def fake(links_up):
        m = types.ModuleType('pynvml')
        m.NVML_FEATURE_ENABLED = 1

        class NVMLError(Exception):
            pass
        m.NVMLError = NVMLError
        m.nvmlInit = lambda: None
        m.nvmlShutdown = lambda: None
        m.nvmlDeviceGetHandleByIndex = lambda i: 'h'

        def state(h, i):
            if i >= 18:
                raise NVMLError()
            return 1 if i < links_up else 0
        m.nvmlDeviceGetNvLinkState = state
        return m
    monkeypatch.setitem(sys.modules, 'pynvml', fake(18))
    assert abs(envs.get_nvlink_gbs() - envs.B200_NVLINK_GBS) < 1e-6
    monkeypatch.setitem(sys.modules, 'pynvml', fake(9))
    assert abs(envs.get_nvlink_gbs() - envs.B200_NVLINK_GBS / 2) < 1e-6
    monkeypatch.setitem(sys.modules, 'pynvml', fake(0))
    assert envs.get_nvlink_gbs() == envs.B200_NVLINK_GBS  # no links reported: measured fallback


def test_masked_gemm_oracle_matches_grouped_oracle():
    """The masked-layout oracle equals the packed grouped oracle on the same rows (CPU), and leaves
    rows at or beyond the counts zero."""
    from deepep_slingshot_b200.ops.gemm import (grouped_gemm_fp8_reference, masked_grouped_gemm_fp8_reference,
                                                quantize_weights_fp8_reference)
    from deepep_slingshot_b200.utils.math import per_token_cast_to_fp8
    torch.manual_seed(0)
    E, slots, K, N = 3, 256, 256, 128
    xq, xs = per_token_cast_to_fp8(torch.randn((E * slots, K)))
    a, sa = xq.view(E, slots, K), xs.view(E, slots, K // 128)
    wq, ws = quantize_weights_fp8_reference(torch.randn((E, N, K)) * 0.05)
    counts = torch.tensor([5, 0, 256], dtype=torch.int32)
    masked = masked_grouped_gemm_fp8_reference(a, sa.transpose(1, 2).contiguous().transpose(1, 2), counts, wq, ws)
    offsets = torch.arange(0, (E + 1) * slots, slots, dtype=torch.int32)
    packed = grouped_gemm_fp8_reference(xq, xs, wq, ws, offsets, counts).view(E, slots, N)
    assert torch.equal(masked, packed)
    assert masked[0, 5:].abs().sum() == 0 and masked[1].abs().sum() == 0


def test_bench_moe_roofline_bounds():
    """The MoE step's lower bound is the largest of compute, NVLink and the weight bytes through HBM."""
    import importlib.util
    import os
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), 'bench.py')
    spec = importlib.util.spec_from_file_location('_bench_under_test', path)
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    one = bench.moe_roofline_seconds(32768, 7168, 2048, 256, 1, 4096)
    assert one['nvlink'] == 0 and one['bound'] == one['hbm']          # all 256 experts on one GPU
    assert abs(one['hbm'] - 8 * 256 * 3 * 7168 * 2048 / 6558.4e9) < 1e-12
    eight = bench.moe_roofline_seconds(32768, 7168, 2048, 32, 8, 21900)
    assert eight['bound'] == eight['compute'] and eight['hbm'] == one['hbm'] / 8
    assert abs(eight['compute'] - (6 * 32768 * 7168 * 2048 / (2 * 1650.1e12) + 12 * 32768 * 7168 * 2048 / 1650.1e12)) < 1e-12


def test_bench_moe_roofline_uses_the_slowest_rank():
    """Under a skewed routing the step's bound is the rank that holds the popular experts: its own
    expert rows and its own remote traffic, not the average rank's."""
    import importlib.util
    import os
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), 'bench.py')
    spec = importlib.util.spec_from_file_location('_bench_under_test2', path)
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    E, world, N, K = 16, 4, 6, 2
    idx = torch.tensor([[0, 1], [0, 5], [2, -1], [9, 13], [3, 4], [-1, -1]])
    rows, toks = bench.moe_route_loads(idx, E, world)
    assert rows.tolist() == [5, 2, 1, 1] and toks.tolist() == [4, 2, 1, 1]
    # every rank sends the same routing: rank 0 computes 20 of the 36 rows
    rows_to = [4 * r for r in rows.tolist()]
    tokens_from = [toks.tolist() for _ in range(world)]
    worst = bench.moe_step_roofline(rows_to, tokens_from, 7168, 2048, E // world)
    assert worst['rank'] == 0 and worst['rows'] == 20
    assert worst['remote_in'] == 3 * 4 and worst['remote_out'] == 2 + 1 + 1
    alone = bench.moe_roofline_seconds(20, 7168, 2048, E // world, world, 0, remote_in=12, remote_out=4)
    assert abs(worst['bound'] - alone['bound']) < 1e-15
    mean = bench.moe_roofline_seconds(sum(rows_to) / world, 7168, 2048, E // world, world, 0, remote_in=12,
                                      remote_out=4)
    assert worst['compute'] > mean['compute']
    # per direction: a rank that only receives tokens takes in their FP8 rows and one bf16 gradient
    # row each, and sends back two bf16 rows each (forward combine, backward gradient combine)
    b = bench.moe_roofline_seconds(0, 7168, 2048, 1, 2, 0, remote_in=100, remote_out=0, nvlink_bytes_per_s=1.0)
    assert b['nvlink'] == max(100 * ((7168 + 56 * 4) + 2 * 7168), 100 * 2 * 2 * 7168)


def test_elastic_previous_event_unwrapping():
    """v2 calls accept the `EventOverlap` that dispatch / combine return as `previous_event` (the
    native call gets its event), a native event as is, or nothing."""
    from deepep_slingshot_b200.parallel.elastic import _native_event
    from deepep_slingshot_b200.utils.event import EventOverlap
    native = object()
    assert _native_event(EventOverlap(native)) is native
    assert _native_event(native) is native
    assert _native_event(None) is None
