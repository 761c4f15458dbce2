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
