"""Host unit tests (CPU): routing tables with exact traffic, benchmark summaries, trace decoding."""
import json
import os

import numpy as np
import pytest
import torch


@pytest.mark.parametrize('skew', [1.0, 1.5, 2.0, 4.0])
def test_skew_routes_exact(skew):
    from deepep_slingshot_b200.harness.routing import skew_routes
    idx, m = skew_routes(512, 8, 256, 8, skew, seed=3)
    received = m.sum(0)
    assert m.sum() == 2 * 512 * 8                      # two destinations per token
    assert abs(received.max() / received.mean() - skew) <= 1 / 512
    assert (np.diff(np.sort(idx, axis=1), axis=1) != 0).all()  # distinct experts per token
    le = 256 // 8
    dst = idx // le
    assert ((dst == dst[:, :1]).sum(1) == 4).all()     # half of the top-k on each destination


def test_named_routings():
    from deepep_slingshot_b200.harness.routing import make_routing, route_matrix
    remote = make_routing('remote', 2, 8, 64, 256, 8, 0).numpy()
    assert route_matrix(remote, 8, 256)[2] == 0
    selfr = make_routing('self', 5, 8, 64, 256, 8, 0).numpy()
    assert (route_matrix(selfr, 8, 256) == np.eye(8, dtype=np.int64)[5] * 64).all()
    hot = make_routing('hot_rank', 1, 8, 16, 256, 8, 0).numpy()
    assert (hot // 32 == 0).all()
    with pytest.raises(ValueError):
        make_routing('mixed', 0, 1, 16, 32, 4, 0)


def test_summarize(tmp_path):
    from deepep_slingshot_b200.harness.summarize import summarize_dir
    for rank in range(2):
        with open(tmp_path / f'timings-rank{rank}.jsonl', 'w') as f:
            for seed in range(2):
                rec = {'kind': 'timing', 'model': 'qwen3', 'tokens_per_rank': 4096, 'ranks': 2, 'dispatch_dtype': 'fp8',
                       'routing': 'mixed', 'seed': seed, 'op': 'dispatch', 'bytes': 1_000_000 * (rank + 1),
                       'rank_max_us': [10.0, 12.0, 11.0, 30.0], 'max_host_us_per_iteration': 50.0 + rank}
                f.write(json.dumps(rec) + '\n')
    rows = summarize_dir(str(tmp_path))
    assert len(rows) == 2
    r = rows[0]
    assert r['median_rank_max_us'] == 11.5 and r['max_host_us_per_iteration'] == 51.0
    assert r['gbps_bottleneck_rank'] == round(2e6 / 11.5e-6 / 1e9, 1)
    rep = json.load(open(tmp_path / 'repeatability.json'))
    assert list(rep.values())[0]['cv'] == 0.0
    assert os.path.exists(tmp_path / 'summary.csv')


def test_trace_decode_and_chrome():
    from deepep_slingshot_b200.utils.trace import TRACE_DTYPE, decode, summarize, to_chrome_trace
    rec = np.zeros(3, dtype=TRACE_DTYPE)
    rec['start_ns'] = [1000, 1500, 5000]
    rec['end_ns'] = [2000, 2500, 6000]
    rec['event'] = [104, 104, 110]
    rec['block'] = [0, 1, 0]
    raw = torch.from_numpy(np.frombuffer(rec.tobytes(), dtype=np.uint8).copy()).view(3, 40)
    out = decode(raw)
    assert (out['event'] == rec['event']).all()
    s = summarize(out)
    assert s['dispatch.pull']['count'] == 2 and s['dispatch.pull']['union_us'] == 1.5
    tr = to_chrome_trace({0: out}, {0: 0})
    assert len(tr['traceEvents']) == 3 and tr['traceEvents'][0]['ts'] == 0.0


def test_routes_from_counts_exact():
    from deepep_slingshot_b200.harness.routing import routes_from_counts, zipf_counts
    for seed in range(5):
        counts = zipf_counts(256, 4096, 6, 1.2, seed)
        assert counts.sum() == 4096 * 6 and counts.max() <= 4096
        idx = routes_from_counts(counts, 4096, 6, seed)
        assert idx.shape == (4096, 6)
        assert (np.bincount(idx[idx >= 0], minlength=256) == counts).all()
        s = np.sort(idx, axis=1)
        assert ((np.diff(s, axis=1) != 0) | (s[:, 1:] < 0)).all()  # distinct experts per token
    # a deficit becomes -1 entries (tokens routed to fewer than k experts)
    idx = routes_from_counts(np.array([3, 3, 2]), 4, 2, 0)
    assert (idx == -1).sum() == 0 and np.bincount(idx.ravel(), minlength=3).tolist() == [3, 3, 2]
    idx = routes_from_counts(np.array([2, 1]), 4, 2, 0)
    assert (idx == -1).sum() == 5


def test_placements_and_count_routing():
    from deepep_slingshot_b200.harness.routing import greedy_placement, make_routing, route_matrix
    load = np.array([10, 1, 1, 1, 9, 1, 1, 1], dtype=np.float64)
    perm = greedy_placement(load, 4)
    assert sorted(perm.tolist()) == list(range(8))
    assert (perm[0] // 4) != (perm[4] // 4)  # the two hot experts land on different ranks
    a = make_routing('zipf1.1', 0, 8, 512, 256, 8, 0)
    b = make_routing('zipf1.1_greedy', 0, 8, 512, 256, 8, 0)
    assert a.shape == b.shape == (512, 8)
    # greedy placement balances the group-wide expert load (assignments of every rank's tokens)
    def group_load(name):
        tot = np.zeros(8, dtype=np.int64)
        for r in range(8):
            t = make_routing(name, r, 8, 512, 256, 8, 0).numpy()
            tot += np.bincount(t[t >= 0] // 32, minlength=8)
        return tot
    la, lb = group_load('zipf1.1'), group_load('zipf1.1_greedy')
    assert la.sum() == lb.sum() and lb.max() / lb.mean() < la.max() / la.mean()
    assert route_matrix(b.numpy(), 8, 256).sum() > 0


def _write_results(d, world=2, fail_rank=None, drop_timing=None, sources=None):
    import json as _json
    for r in range(world):
        man = {'kind': 'manifest', 'rank': r, 'world': world, 'sources': sources[r] if sources else {'a.py': 'x'}}
        (d / f'manifest-rank{r}.jsonl').write_text(_json.dumps(man) + '\n')
        case = {'model': 'qwen3', 'tokens_per_rank': 512, 'dispatch_dtype': 'fp8', 'routing': 'mixed', 'seed': 0}
        cor = dict(case, kind='correctness', passed=(r != fail_rank))
        (d / f'correctness-rank{r}.jsonl').write_text(_json.dumps(cor) + '\n')
        lines = []
        for op in ('dispatch', 'cached_dispatch', 'combine'):
            if drop_timing == (r, op):
                continue
            lines.append(_json.dumps(dict(case, kind='timing', op=op, ranks=world, bytes=100, rank_max_us=[10.0, 11.0],
                                          max_host_us_per_iteration=5.0)))
        (d / f'timings-rank{r}.jsonl').write_text('\n'.join(lines) + '\n')


def test_validate_results(tmp_path):
    from deepep_slingshot_b200.harness.summarize import summarize_dir
    from deepep_slingshot_b200.harness.validate import validate
    good = tmp_path / 'good'
    good.mkdir()
    _write_results(good)
    summarize_dir(str(good))
    assert validate(str(good), ranks=2) == []
    bad = tmp_path / 'bad'
    bad.mkdir()
    _write_results(bad, fail_rank=1, drop_timing=(0, 'combine'), sources=[{'a.py': 'x'}, {'a.py': 'y'}])
    summarize_dir(str(bad))
    probs = validate(str(bad), ranks=2)
    text = '\n'.join(probs)
    assert 'source hashes differ' in text and 'correctness failed' in text
    assert validate(str(tmp_path / 'missing')) != []


def test_kernel_summary_aggregates_device_events():
    import torch
    from deepep_slingshot_b200.harness.profile_capture import kernel_summary

    class Ev:
        def __init__(self, name, dev, t):
            self.name, self.device_type, self.device_time_total = name, dev, t

    cuda, cpu = torch.autograd.DeviceType.CUDA, torch.autograd.DeviceType.CPU
    rows = kernel_summary([Ev('pull', cuda, 30.0), Ev('pull', cuda, 10.0), Ev('combine', cuda, 60.0),
                           Ev('python', cpu, 999.0)], steps=2)
    assert [r['kernel'] for r in rows] == ['combine', 'pull']
    assert rows[1]['calls'] == 2 and rows[1]['mean_us'] == 20.0 and rows[1]['per_step_us'] == 20.0
    assert abs(rows[0]['share'] - 0.6) < 1e-9


def test_ladder_stops_and_resumes(tmp_path):
    from deepep_slingshot_b200.harness.ladder import load_state, run_ladder
    gates = [{'name': 'a', 'args': []}, {'name': 'b', 'args': []}, {'name': 'c', 'args': []}]
    calls = []
    outcome = {'a': [], 'b': ['bad'], 'c': []}

    def fake(gate, d):
        calls.append(gate['name'])
        return outcome[gate['name']]
    out = str(tmp_path / 'ladder')
    assert not run_ladder(out, fake, gates)
    assert calls == ['a', 'b'] and load_state(out + '/ladder_state.json')['failed'] == 'b'
    assert not run_ladder(out, fake, gates)          # refuses to run without a resume reason
    assert calls == ['a', 'b']
    outcome['b'] = []
    assert run_ladder(out, fake, gates, resume_reason='fixed the notify wait')
    assert calls == ['a', 'b', 'b', 'c']             # passed gates are skipped
    st = load_state(out + '/ladder_state.json')
    assert st['passed'] == ['a', 'b', 'c'] and st['resumes'][0]['reason'] == 'fixed the notify wait'


_TOPO = """\tGPU0\tGPU1\tGPU2\tNIC0\tCPU Affinity\tNUMA Affinity\tGPU NUMA ID
GPU0\t X \tNV18\tNV18\tSYS\t0-55\t0\t\tN/A
GPU1\tNV18\t X \tNV18\tSYS\t0-55\t0\t\tN/A
GPU2\tNV18\tNV18\t X \tNODE\t56-111\t1\t\tN/A
NIC0\tSYS\tSYS\tNODE\t X \t\t\t\t

Legend:

  X    = Self
  NV#  = Connection traversing a bonded set of # NVLinks
"""


def test_box_probe_topology_and_cpu_collect(tmp_path):
    from deepep_slingshot_b200.harness import box_probe
    m = box_probe.parse_topo_matrix(_TOPO)
    assert sorted(m) == ['GPU0', 'GPU1', 'GPU2']
    assert m['GPU0'] == {'GPU0': 'X', 'GPU1': 'NV18', 'GPU2': 'NV18'}
    assert m['GPU2']['GPU1'] == 'NV18'
    assert box_probe.parse_topo_matrix('') == {}
    (tmp_path / 'MEASURED_PEAKS.json').write_text('{"hbm_gbs": 1.0}')
    info = box_probe.collect(bandwidth=True, repo_root=str(tmp_path))  # CPU box: no GPUs, no failure
    assert info['measured_peaks'] == {'hbm_gbs': 1.0}
    assert isinstance(info['gpus'], list) and isinstance(info['peer_access'], list)
    assert box_probe.main(['--out', str(tmp_path / 'box.json')]) == 0
    assert (tmp_path / 'box.json').exists()


def test_ladder_counterbalanced_repeat(tmp_path):
    """A repeat gate must reproduce the earlier gate's medians within its tolerance."""
    import csv
    from deepep_slingshot_b200.harness.ladder import GATES, compare_summaries, run_ladder
    names = [g['name'] for g in GATES]
    assert names.index('perf_4k_repeat') > names.index('perf_4k')
    assert any('--drop-every' in g['args'] for g in GATES) and any('16384' in g['args'] for g in GATES)

    def write(d, medians):
        os.makedirs(d, exist_ok=True)
        with open(os.path.join(d, 'summary.csv'), 'w', newline='') as f:
            w = csv.DictWriter(f, fieldnames=['model', 'tokens_per_rank', 'ranks', 'dispatch_dtype', 'routing', 'seed',
                                              'op', 'median_rank_max_us'])
            w.writeheader()
            for (op, m) in medians.items():
                w.writerow(dict(model='v4flash', tokens_per_rank=4096, ranks=8, dispatch_dtype='fp8', routing='mixed',
                                seed=0, op=op, median_rank_max_us=m))
    a, b = str(tmp_path / 'a'), str(tmp_path / 'b')
    write(a, {'dispatch': 100.0, 'combine': 200.0})
    write(b, {'dispatch': 104.0, 'combine': 195.0})
    assert compare_summaries(a, b, 0.1) == []
    write(b, {'dispatch': 130.0, 'combine': 195.0})
    assert len(compare_summaries(a, b, 0.1)) == 1
    write(b, {'dispatch': 100.0})
    assert 'different cases' in compare_summaries(a, b, 0.1)[0]
    assert 'missing summary' in compare_summaries(a, str(tmp_path / 'none'), 0.1)[0]

    gates = [{'name': 'p', 'args': []}, {'name': 'r', 'args': [], 'compare_with': 'p', 'max_rel_diff': 0.1}]
    out = str(tmp_path / 'ladder')
    medians = {'p': {'dispatch': 100.0}, 'r': {'dispatch': 150.0}}

    def fake(gate, d):
        write(d, medians[gate['name']])
        return []
    assert not run_ladder(out, fake, gates)            # the repeat is 50% off: fails closed
    medians['r'] = {'dispatch': 103.0}
    assert run_ladder(out, fake, gates, resume_reason='quiet box')


def test_bench_report(tmp_path):
    from deepep_slingshot_b200.harness import report
    line1 = {'metric': 'm', 'value': 496.6, 'n_gpus': 1, 'vs_baseline': 0.676, 'dispatch_gbps_per_rank': 333.7,
             'combine_gbps_per_rank': 666.0, 'dispatch_ms': 0.0919, 'combine_ms': 0.0884, 'll_dispatch_us': 24.7,
             'll_combine_us': 34.8, 'moe_tokens_per_s': 79000.0, 'moe_ms_per_step': 51.8, 'moe_roofline_fraction': 0.27,
             'moe_roofline_ms': {'compute': 4.4, 'nvlink': 0.0, 'hbm': 13.7, 'bound': 13.7},
             'e2e': {'value': 80.0, 'ms_per_step': 1.1, 'h2d_bytes_per_step': 59113472, 'schedule': 'pipelined',
                     'serial_value': 39.8},
             'clocks': {'sm_mhz': 1965.0, 'sm_max_mhz': 1965.0, 'reasons': []}}
    line8 = dict(line1, value=4091.0, n_gpus=8,
                 moe_roofline_rank={'rank': 2, 'expert_rows': 41932.0, 'expert_rows_mean': 32768.0,
                                    'remote_tokens_in': 21852.0, 'remote_tokens_out': 17853.0})
    f = tmp_path / 'b.json'
    f.write_text('NCCL version 2.28\n' + json.dumps(line1) + '\n' + json.dumps(line8) + '\nnot json {\n'
                 + json.dumps({'impl': 'reference', 'unavailable': 'not installable'}) + '\n')
    recs = report.load_lines([str(f)])
    assert len(recs) == 3
    rows = report.summarize(recs[0], {'hbm_gbs': 6558.4, 'bf16_tflops': 1650.1})
    text = '\n'.join(rows)
    assert '0.676' in text and '0.46 of published 726' in text and '3.12x faster' in text
    assert 'HBM 13.7' in text and 'serial 39.8' in text and 'reasons: none' in text
    assert 'unavailable' in report.summarize(recs[2])[0]
    assert 'rank 2: 41932 expert rows' in '\n'.join(report.summarize(recs[1]))
    sync = '\n'.join(report.summarize(dict(line1, n_gpus=2, dispatch_ms=0.694, dispatch_nosync_ms=0.149,
                                            dispatch_synced_alone_ms=0.2)))
    assert 'step interval 694.0 µs, synced alone 200.0 µs, without the CPU sync 149.0 µs' in sync
    sc = '\n'.join(report.scaling(recs))
    assert '| 8 | 4091.0 | 511.4 | 1.03 |' in sc
    assert report.main([str(f), '--peaks', str(tmp_path / 'missing.json')]) == 0


def test_bench_reference_arm_prints_one_line_per_job():
    """`bench.py --impl reference` exits 0 with one `unavailable` JSON line from rank 0 only (the
    driver launches it under torchrun like the own arm)."""
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    outs = {}
    for rank in ('0', '1'):
        env = dict(os.environ, RANK=rank, WORLD_SIZE='2')
        r = subprocess.run([sys.executable, os.path.join(root, 'bench.py'), '--impl', 'reference', '--gpus', '2'],
                           cwd=root, env=env, capture_output=True, text=True, timeout=300)
        assert r.returncode == 0, r.stderr[-2000:]
        outs[rank] = [line for line in r.stdout.splitlines() if line.strip()]
    assert len(outs['0']) == 1 and outs['1'] == []
    rec = json.loads(outs['0'][0])
    assert rec['impl'] == 'reference' and rec['unavailable']


def test_ep_benchmark_nccl_arm_options():
    """`--impl nccl` times the NCCL all-to-all baseline on the same cases; the kernel-only options
    are refused before any process group or device is touched."""
    from deepep_slingshot_b200.harness import ep_benchmark
    for bad in (['--impl', 'nccl', '--sweep-sms', '8,16'], ['--impl', 'nccl', '--stall-us', '50']):
        with pytest.raises(SystemExit) as e:
            ep_benchmark.main(bad)
        assert e.value.code == 2


def _nccl_baseline_body(rank, world):
    import torch.distributed as dist
    from deepep_slingshot_b200 import ReferenceBuffer
    from deepep_slingshot_b200.parallel.nccl_baseline import NcclAllToAllEP
    from deepep_slingshot_b200.utils.gate import normal_routing
    N, H, E, K = 96 - 7 * rank, 256, 8 * world, 4
    g = torch.Generator().manual_seed(3 + rank)
    x = torch.randn((N, H), generator=g).to(torch.bfloat16)
    idx, w = normal_routing(N, E, K, generator=g)
    idx[5] = -1  # a token routed nowhere
    base, ref = NcclAllToAllEP(dist.group.WORLD), ReferenceBuffer(dist.group.WORLD)
    a, b = base.get_dispatch_layout(idx, E), ref.get_dispatch_layout(idx, E)
    assert torch.equal(a[0], b[0]) and torch.equal(a[2], b[2]) and torch.equal(a[3], b[3])
    for fp8 in (False, True):
        ox, oi, ow, ol, oh, _ = base.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E, quantize_fp8=fp8,
                                              expert_alignment=4)
        ex, ei, ew, el, eh, _ = ref.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E, quantize_fp8=fp8,
                                             expert_alignment=4)
        if fp8:
            assert torch.equal(ox[0].view(torch.uint8), ex[0].view(torch.uint8)) and torch.equal(ox[1], ex[1])
            ox, ex = ox[0], ex[0]
        else:
            assert torch.equal(ox, ex)
        assert torch.equal(oi, ei) and torch.equal(ow, ew) and ol == el
        assert torch.equal(oh[3], eh[3]) and torch.equal(oh[4], eh[4]) and torch.equal(oh[5], eh[5])
        cx, *_ = base.dispatch((x, None)[0], handle=oh)  # cached: same rows without the routing
        assert torch.equal(cx, ref.dispatch(x, handle=eh)[0])
        y = (torch.randn((ox.shape[0], H), generator=g)).to(torch.bfloat16)
        bias = torch.randn((N, H), generator=g).to(torch.bfloat16)
        o, o_w, _ = base.combine(y, oh, topk_weights=ow, bias=bias)
        e, e_w, _ = ref.combine(y, eh, topk_weights=ew, bias=bias)
        assert torch.allclose(o.float(), e.float(), atol=1e-2, rtol=1e-2) and torch.allclose(o_w, e_w, atol=1e-6)
    px, pi, *_ = base.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E, num_worst_tokens=N * world)
    assert px.shape[0] == N * world and bool((pi[oi.shape[0]:] == -1).all())


def test_nccl_baseline_matches_oracle_gloo():
    """The NCCL baseline arm is its own implementation; on gloo ranks it must return exactly what
    the oracle returns (receive order, handle fields, combine sums), so its timings compare."""
    from tests._dist import run_ranks
    run_ranks(_nccl_baseline_body, 2, 'gloo')


def test_host_spans_join_the_device_timeline():
    """Host spans (host clock) and device records (GPU clock minus the rank's offset) land on one
    timeline: a host call that starts 2 µs before a kernel appears 2 µs earlier."""
    import time
    from deepep_slingshot_b200.utils.trace import TRACE_DTYPE, HostSpans, to_chrome_trace
    spans = HostSpans()
    with spans.span('host.dispatch_call'):
        time.sleep(0.001)
    (name, hs, he), = spans.spans
    assert name == 'host.dispatch_call' and he - hs >= 1_000_000
    offset = 5_000_000_000  # GPU clock ahead of the host clock
    rec = np.zeros(1, dtype=TRACE_DTYPE)
    rec['start_ns'], rec['end_ns'], rec['event'] = hs + 2000 + offset, hs + 9000 + offset, 102
    tr = to_chrome_trace({0: rec}, {0: offset}, {0: spans.spans})
    by_name = {e['name']: e for e in tr['traceEvents']}
    assert by_name['host.dispatch_call']['ts'] == 0.0 and by_name['host.dispatch_call']['tid'] == 'host'
    assert by_name['dispatch.count']['ts'] == 2.0 and by_name['dispatch.count']['dur'] == 7.0


def test_trace_phase_table_splits_steps_at_host_spans():
    from deepep_slingshot_b200.harness.trace_capture import phase_table
    ev = [
        {'name': 'host.step', 'pid': 0, 'ts': 0.0, 'dur': 100.0},
        {'name': 'dispatch.count', 'pid': 0, 'ts': 10.0, 'dur': 5.0},
        {'name': 'dispatch.count', 'pid': 0, 'ts': 12.0, 'dur': 6.0},   # second block of the same phase
        {'name': 'host.step', 'pid': 0, 'ts': 200.0, 'dur': 100.0},
        {'name': 'dispatch.count', 'pid': 0, 'ts': 210.0, 'dur': 4.0},
        {'name': 'host.step', 'pid': 1, 'ts': 1.0, 'dur': 100.0},
        {'name': 'dispatch.pull', 'pid': 1, 'ts': 30.0, 'dur': 10.0},
    ]
    rows = {(l['rank'], l['step'], l['phase']): (l['start_us'], l['end_us']) for l in phase_table(ev)}
    assert rows[(0, 0, 'dispatch.count')] == (10.0, 18.0)
    assert rows[(0, 1, 'dispatch.count')] == (210.0, 214.0)
    assert rows[(1, 0, 'dispatch.pull')] == (30.0, 40.0)
    assert (0, 1, 'host.step') in rows and (1, 0, 'host.step') in rows
