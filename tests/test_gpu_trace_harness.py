"""GPU tests of the device trace ring (records, clock alignment, overflow detection) and of the
EP benchmark harness end to end (exact-reference checks, JSONL records, summary.csv)."""
import json
import os

import pytest
import torch
import torch.distributed as dist

from tests._dist import run_ranks
from tests.test_gpu_intranode import _make_inputs, _worlds

pytestmark = pytest.mark.gpu


def _trace_body(rank, world):
    from deepep_slingshot_b200 import Buffer
    from deepep_slingshot_b200.utils.trace import TraceOverflow, capture, gather_and_write, summarize
    N, H, E, K = 256, 1024, 32, 4
    buf = Buffer(dist.group.WORLD, num_nvl_bytes=Buffer.get_nvl_buffer_size_hint(N, H, world),
                 num_rdma_bytes=Buffer.get_low_latency_rdma_size_hint(32, H, world, E), low_latency_mode=True)
    x, idx, w = _make_inputs(rank, N, H, E, K, seed=1)

    def step():
        (rx, rs), ri, rw, _, h, _ = buf.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E, quantize_fp8=True)
        buf.combine(torch.zeros((rx.shape[0], H), dtype=torch.bfloat16, device='cuda'), h, topk_weights=rw)
        _, _, lh, _, hook = buf.low_latency_dispatch(x[:32].contiguous(), idx[:32].contiguous(), 32, E,
                                                     return_recv_hook=True)
        hook()
        y = torch.zeros((E // world, 32 * world, H), dtype=torch.bfloat16, device='cuda')
        _, _, chook = buf.low_latency_combine(y, idx[:32].contiguous(), w[:32].contiguous(), lh, return_recv_hook=True)
        chook()
        buf.barrier()

    rec, offset = capture(buf, step, iterations=2, group=dist.group.WORLD)
    events = set(int(e) for e in rec['event'])
    for ev in (100, 101, 102, 103, 104, 110, 120, 121, 122, 123, 130):
        assert ev in events, f'event {ev} missing'
    assert (rec['end_ns'] >= rec['start_ns']).all() and (rec['rank'] == rank).all()
    assert summarize(rec)['dispatch.pull']['count'] > 0
    trace = gather_and_write(rec, offset, None, dist.group.WORLD)
    assert {e['pid'] for e in trace['traceEvents']} == set(range(world))
    with pytest.raises(TraceOverflow):
        capture(buf, step, iterations=1, capacity=4, group=dist.group.WORLD)
    buf.check_error()


@pytest.mark.parametrize('world', _worlds())
def test_trace_ring(world):
    run_ranks(_trace_body, world, backend='nccl')


def _harness_body(rank, world, out):
    from deepep_slingshot_b200.harness.ep_benchmark import main
    routings = ['uniform', 'self'] if world == 1 else ['uniform', 'mixed', 'hot_rank']
    rc = main(['--models', 'qwen3', '--tokens', '512', '--dtype', 'fp8', 'bf16', '--routing', *routings,
               '--iters', '4', '--warmup', '2', '--out', out])
    assert rc == 0


@pytest.mark.parametrize('world', _worlds())
def test_ep_benchmark_harness(world, tmp_path):
    out = str(tmp_path / 'ep')
    run_ranks(_harness_body, world, backend='nccl', args=(out,))
    with open(os.path.join(out, 'summary.csv')) as f:
        lines = f.read().strip().splitlines()
    n_routings = 2 if world == 1 else 3
    from deepep_slingshot_b200.harness.ep_benchmark import TIMED_OPS
    assert len(lines) == 1 + n_routings * 2 * len(TIMED_OPS)  # routings x dtypes x ops
    for r in range(world):
        recs = [json.loads(l) for l in open(os.path.join(out, f'correctness-rank{r}.jsonl'))]
        assert recs and all(x['passed'] for x in recs)
        man = json.loads(open(os.path.join(out, f'manifest-rank{r}.jsonl')).readline())
        assert man['sources'] and man['world'] == world


def _bank_body(rank, world, out):
    from deepep_slingshot_b200.harness.ep_benchmark import main
    rc = main(['--models', 'qwen3', '--tokens', '512', '--dtype', 'fp8', '--routing', 'bank:hot8', 'bank:drift:greedy',
               'bank:dead', 'bank:saturated', '--iters', '2', '--warmup', '1', '--out', out])
    assert rc == 0


@pytest.mark.parametrize('world', _worlds())
def test_ep_benchmark_bank_routings(world, tmp_path):
    """The built-in count-table scenarios through dispatch / combine, each checked exactly against the
    oracle before it is timed (hot experts, rank-local drift with greedy placement, dead experts,
    experts chosen by every token)."""
    out = str(tmp_path / 'bank')
    run_ranks(_bank_body, world, backend='nccl', args=(out,))
    for r in range(world):
        recs = [json.loads(l) for l in open(os.path.join(out, f'correctness-rank{r}.jsonl'))]
        assert len({x['routing'] for x in recs}) == 4 and all(x['passed'] for x in recs)
