"""CPU (gloo) tests of the host-memory segments shared by the ranks of one box
(`parallel/host_memory.py`, `csrc/runtime/host_segment.cpp`), the hybrid CPU memory that holds the
elastic API's Engram storage: every rank creates its segment and maps every rank's, a write through
one rank's view is seen through every other rank's mapping, the Engram row rule read from the views
matches the gloo oracle (`ReferenceSideFeatures.engram_fetch`), and destroy unlinks the names.
"""
import os

import pytest
import torch
import torch.distributed as dist

from tests._dist import run_ranks


def _body(rank, world, entries, hidden):
    from deepep_slingshot_b200.parallel.host_memory import HostSegments, fetch_rows_reference
    from deepep_slingshot_b200.parallel.symmetric import ReferenceSideFeatures
    group = dist.group.WORLD
    nbytes = 2 << 20
    seg = HostSegments(group, nbytes)
    names = seg.names
    assert len(set(names)) == world and all(os.path.exists('/dev/shm' + n) for n in names)
    g = torch.Generator().manual_seed(17 + rank)
    storage = torch.randn((entries, hidden), generator=g).to(torch.bfloat16)
    seg.view(rank)[:storage.numel() * 2].copy_(storage.view(torch.uint8).flatten())
    dist.barrier()
    for r in range(world):  # every rank's bytes through this rank's mapping of them
        got = seg.view(r)[:entries * hidden * 2].view(torch.bfloat16).view(entries, hidden)
        want = torch.randn((entries, hidden), generator=torch.Generator().manual_seed(17 + r)).to(torch.bfloat16)
        assert torch.equal(got, want)
    ref = ReferenceSideFeatures(group)
    ref.engram_write(storage)
    idx = torch.randint(-3, entries * world + 3, (200,), generator=g, dtype=torch.int32)
    out = fetch_rows_reference(idx, [seg.view(r) for r in range(world)], entries, hidden)
    valid = (idx >= 0) & (idx < entries * world)
    expect = ref.engram_fetch(torch.where(valid, idx, torch.zeros_like(idx)))()
    assert torch.equal(out[valid], expect[valid]) and torch.count_nonzero(out[~valid]) == 0
    seg.destroy()
    dist.barrier()
    assert not any(os.path.exists('/dev/shm' + n) for n in names)


@pytest.mark.skipif(not os.path.isdir('/dev/shm'), reason='POSIX shared memory is not mounted')
@pytest.mark.parametrize('world', [1, 2, 3])
def test_host_segments_shared_between_ranks(world):
    run_ranks(_body, world, backend='gloo', args=(64, 256))


def test_host_segment_name_rules():
    from deepep_slingshot_b200._ext import require_ext
    _C = require_ext()
    with pytest.raises(Exception):
        _C.HostSegment('no-leading-slash', 4096, True)
    with pytest.raises(Exception):
        _C.HostSegment('/deepep_b200_missing_segment_for_test', 4096, False)  # opening what does not exist
    s = _C.HostSegment('/deepep_b200_unit_test_%d' % os.getpid(), 8192, True)
    try:
        v = s.host_view(0, 8192)
        v.fill_(7)
        assert int(s.host_view(4096, 16).sum()) == 7 * 16
        with pytest.raises(Exception):
            s.host_view(8000, 400)
    finally:
        s.destroy()
    assert not os.path.exists('/dev/shm/deepep_b200_unit_test_%d' % os.getpid())
