"""Small host-side utilities (CPU): comparison metrics, byte counts, unique rows, routing helpers,
event wrappers and the functional dispatch / combine references on a one-rank gloo group."""
import pytest
import torch

from deepep_slingshot_b200.utils import gate, math as epm
from deepep_slingshot_b200.utils.event import EventOverlap
from tests._dist import run_ranks


def test_math_helpers():
    x = torch.randn(64, 32)
    assert abs(epm.calc_diff(x, x)) < 1e-12
    assert epm.calc_diff(x, x + 1.0) > 1e-3
    assert epm.count_bytes(torch.zeros(4, dtype=torch.float32), (torch.zeros(2, dtype=torch.int64), None), []) == 32
    assert epm.safe_div(6, 3) == 2 and epm.safe_div(0, 0) == 0
    with pytest.raises(ZeroDivisionError):
        epm.safe_div(1, 0)
    assert epm.ceil_div(7, 2) == 4 and epm.align(7, 4) == 8
    u = torch.tensor([[3, 1, 3, -1], [2, 2, 2, 2], [-1, -1, -1, -1]])
    epm.inplace_unique(u, 4)
    assert u.tolist() == [[3, 1, -1, -1], [2, -1, -1, -1], [-1, -1, -1, -1]]


def test_routing_helpers():
    g = torch.Generator().manual_seed(0)
    idx, w = gate.hot_rank_routing(128, 32, 4, 4, hot_rank=2, generator=g)
    assert bool(((idx // 8) == 2).all()) and torch.allclose(w.sum(1), torch.ones(128))
    idx, w = gate.local_routing(128, 32, 4, 4, rank=1, generator=g)
    assert bool(((idx // 8) == 1).all())
    idx, w = gate.normal_routing(256, 32, 4, generator=g)
    gate.drop_tokens(idx, w, 0.25, generator=torch.Generator().manual_seed(1))
    dropped = idx < 0
    assert 0.15 < float(dropped.float().mean()) < 0.35
    assert bool((w[dropped] == 0).all())
    before = idx.clone()
    gate.drop_tokens(idx, w, 0.0)
    assert torch.equal(idx, before)


def test_event_overlap_without_event():
    ev = EventOverlap(None, (torch.zeros(1),))
    with ev:
        pass
    with ev(release_handle=True):
        pass
    with pytest.raises(RuntimeError):
        ev.current_stream_wait()


class _CountingEvent:
    def __init__(self):
        self.waits = 0

    def current_stream_wait(self):
        self.waits += 1


def test_event_overlap_joins_and_releases():
    native = _CountingEvent()
    ev = EventOverlap(native)
    with ev as inner:
        assert inner is ev
    assert native.waits == 1 and ev.event is native
    with ev(release_handle=True) as inner:
        assert inner is ev
    assert native.waits == 2 and ev.event is None
    with ev:  # nothing left to join
        pass
    assert native.waits == 2


def _refs_body(rank, world):
    import torch.distributed as dist
    from deepep_slingshot_b200.utils import refs
    g = torch.Generator().manual_seed(5 + rank)
    N, H, E, K = 16, 64, 8, 2
    x = torch.randn((N, H), generator=g)
    idx = torch.rand((N, E), generator=g).topk(K, dim=1).indices.to(torch.int64)
    idx[3] = -1
    w = torch.rand((N, K), generator=g)
    rx, ri, rw, gidx, per_rank = refs.dispatch(x, idx, w, N, E, dist.group.WORLD)
    assert int(per_rank.sum()) == rx.shape[0] and rx.shape[1] == H and gidx.shape[0] == rx.shape[0]
    if world == 1:  # every token with a valid expert arrives once; token 3 selected none
        assert rx.shape[0] == N - 1 and sorted(gidx.tolist()) == [t for t in range(N) if t != 3]
    y = refs.generate_pre_combine_data(torch.arange(N), N, K, H, seed=3)
    assert y.shape == (N, K, H) and y.dtype == torch.bfloat16
    again = refs.generate_pre_combine_data(torch.arange(N), N, K, H, seed=3)
    assert torch.equal(y, again)
    plain = refs.combine(y, idx, 1, world, E, reduce_in_local=False)
    acc = refs.ordered_accumulate(torch.where((idx >= 0).unsqueeze(-1), y, torch.zeros((), dtype=y.dtype)))
    assert torch.equal(plain, acc)
    assert float(plain[3].abs().max()) == 0.0  # a token with no expert combines to zero
    local = refs.combine(y, idx, 1, world, E, reduce_in_local=True)
    assert torch.allclose(local.float(), plain.float(), atol=5e-2)


@pytest.mark.parametrize('world', [1, 2])
def test_functional_refs_gloo(world):
    run_ranks(_refs_body, world, 'gloo')


def test_fast_rdma_atomic_check_without_nic(monkeypatch):
    import subprocess
    from deepep_slingshot_b200.utils.envs import check_fast_rdma_atomic_support

    class Out:
        def __init__(self, code, text):
            self.returncode, self.stdout = code, text
    monkeypatch.setattr(subprocess, 'run', lambda *a, **k: Out(0, "CA 'mlx5_0'\n\tCA type: MT4131\n"))
    assert check_fast_rdma_atomic_support()
    monkeypatch.setattr(subprocess, 'run', lambda *a, **k: Out(0, "\tCA type: MT4129\n"))
    assert not check_fast_rdma_atomic_support()
    monkeypatch.setattr(subprocess, 'run', lambda *a, **k: Out(1, ''))
    assert not check_fast_rdma_atomic_support()
