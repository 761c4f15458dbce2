"""Failure detection without any GPU fault (CPU, gloo ranks): a rank that dies between steps is
seen by its peer's heartbeat check before the next collective, a collective with a missing peer
ends with an error at the process group's timeout instead of hanging, and the error-page watcher
reports a code written by a (fake) failed kernel."""
import datetime
import os
import time
import traceback

import pytest
import torch
import torch.multiprocessing as mp

from tests._dist import free_port


def _peer_dies(rank, world, port, q):
    import torch.distributed as dist
    from deepep_slingshot_b200 import ReferenceBuffer
    from deepep_slingshot_b200.utils.health import Heartbeat
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    try:
        dist.init_process_group('gloo', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=4))
        store = dist.distributed_c10d._get_default_store()
        hb = Heartbeat(store, rank, world, interval=0.2)
        ref = ReferenceBuffer(dist.group.WORLD)
        x = torch.randn(16, 128)
        idx = torch.randint(0, 8, (16, 2))
        w = torch.rand(16, 2)
        ref.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=8)  # one good step
        dist.barrier()
        if rank == 1:
            hb.stop()
            q.put((rank, 'left'))
            os._exit(0)  # leaves between steps, nothing in flight
        time.sleep(1.5)
        stale = hb.stale_ranks(max_age=1.0)
        detected = stale == [1]
        t0 = time.time()
        try:
            ref.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=8)
            outcome = 'completed'
        except Exception as e:  # gloo reports the missing peer (timeout or closed connection)
            outcome = f'error after {time.time() - t0:.1f}s: {type(e).__name__}'
        q.put((rank, ('detected' if detected else f'not detected {stale}', outcome)))
        hb.stop()
        os._exit(0)
    except Exception:
        q.put((rank, traceback.format_exc()))
        os._exit(1)


def test_dead_peer_detected_and_collective_fails():
    ctx = mp.get_context('spawn')
    q = ctx.SimpleQueue()
    port = free_port()
    procs = [ctx.Process(target=_peer_dies, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    results = {}
    while not q.empty():
        r, v = q.get()
        results[r] = v
    for p in procs:
        if p.is_alive():
            p.kill()
    assert results.get(1) == 'left', results
    detected, outcome = results[0]
    assert detected == 'detected', results
    assert outcome.startswith('error after'), outcome


class _FakeRuntimeBuffer:
    """Stands in for a Buffer whose kernel reported a bounded-wait timeout after a few polls."""

    def __init__(self, after: int):
        self.polls, self.after = 0, after

    def get_error_state(self):
        self.polls += 1
        return (1, 3, 7, 0) if self.polls > self.after else (0, 0, 0, 0)


def test_error_watch_reports_code():
    from deepep_slingshot_b200.utils.health import ErrorWatch
    seen = []
    w = ErrorWatch(_FakeRuntimeBuffer(after=3), interval=0.01, on_error=seen.append)
    deadline = time.time() + 5
    while w.error is None and time.time() < deadline:
        time.sleep(0.01)
    w.stop()
    assert w.error == (1, 3, 7, 0) and seen == [(1, 3, 7, 0)]
    with pytest.raises(RuntimeError, match='code 1'):
        w.raise_if_error()


def test_heartbeat_single_process():
    import torch.distributed as dist
    from deepep_slingshot_b200.utils.health import Heartbeat
    store = dist.HashStore()
    hb = Heartbeat(store, 0, 2, interval=0.05)
    assert hb.stale_ranks(max_age=1.0) == [1]  # rank 1 never joined
    store.set('deepep_b200_hb/1', repr(time.time()))
    assert hb.stale_ranks(max_age=1.0) == []
    with pytest.raises(RuntimeError):
        store.set('deepep_b200_hb/1', repr(time.time() - 10))
        hb.require_alive(max_age=1.0)
    hb.stop()
