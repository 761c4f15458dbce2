"""GPU tests of the NVLink micro-probes (`harness/nvlink_probe.py`): the flag round trip returns a
finite latency, and the peer copy moves the exact bytes at every start alignment, with the widest
access the two addresses allow. At one GPU the probes run against the GPU's own mapping (the round
trip between two blocks of one launch)."""
import pytest
import torch
import torch.distributed as dist

from tests._dist import run_ranks

pytestmark = pytest.mark.gpu


def _worlds():
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    return [w for w in (1, 2) if w <= n] or [1]


def _body(rank, world):
    from deepep_slingshot_b200 import Buffer
    from deepep_slingshot_b200.harness import nvlink_probe
    buf = Buffer(dist.group.WORLD, num_nvl_bytes=64 << 20, num_gpu_timeout_secs=10, explicitly_destroy=True)
    lat = nvlink_probe.flag_latency(buf, iters=200)
    if rank == 0:
        assert all(0 < v < 1e6 for v in lat.values()), lat
    shift = 1 % world
    size = (1 << 20) + 12  # a ragged tail past the last whole vector
    g = torch.Generator(device='cuda').manual_seed(5 + rank)
    for off, vec in ((0, 16), (4, 4), (6, 2), (8, 8), (16, 16), (3, 1)):
        data = torch.randint(0, 256, (size + 64,), generator=g, device='cuda', dtype=torch.int32).to(torch.uint8)
        res = buf.runtime.probe_peer_copy(shift, size, off, True, 1, 64, data)  # my bytes into the peer's region
        assert int(res[-1]) == vec and res[0] > 0
        back = torch.zeros_like(data)
        # the same peer region read back: it holds what this rank stored there
        res = buf.runtime.probe_peer_copy(shift, size, off, False, 1, 64, back)
        assert int(res[-1]) == vec
        torch.cuda.synchronize()
        assert torch.equal(back[off:off + size], data[off:off + size]), off
        assert int(back[:off].sum()) == 0 and int(back[off + size:].sum()) == 0  # nothing outside the window
    rows = nvlink_probe.copy_sweep(buf, sizes=(4096, 1 << 20), offsets=(0, 8), store=True, reps=2)
    assert len(rows) == 4 and all(r['gbps'] > 0 for r in rows)
    m = nvlink_probe.peer_matrix(buf, bytes_=8 << 20, store=False, reps=2)
    assert len(m) == world and all(len(r) == world and all(v > 0 for v in r) for r in m)
    buf.destroy()


@pytest.mark.parametrize('world', _worlds())
def test_nvlink_probes(world):
    run_ranks(_body, world, backend='nccl')
