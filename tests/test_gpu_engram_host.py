"""GPU test of the elastic API's Engram storage in host memory (hybrid mode, `num_cpu_bytes`):
every rank's storage lives in its shared host segment, the fetch kernel reads the segments through
their CUDA registrations, and the rows must equal both the concatenated storage and the fetch from
GPU-resident storage. Out-of-range indices give zero rows and a bounds report.

This path has not run on a B200 yet: the file is skipped until DEEPEP_B200_TEST_NEW_KERNELS=1.
"""
import os

import pytest
import torch
import torch.distributed as dist

from tests._dist import run_ranks

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(os.environ.get('DEEPEP_B200_TEST_NEW_KERNELS', '0') != '1',
                       reason='first B200 run pending (set DEEPEP_B200_TEST_NEW_KERNELS=1)'),
]


def _worlds():
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    return [w for w in (1, 2, 4, 8) if w <= n] or [1]


def _body(rank, world):
    from deepep_slingshot_b200 import ElasticBuffer
    from deepep_slingshot_b200.ops.gemm import op_error_state
    entries, hidden = 500, 1024
    _, cpu_bytes = ElasticBuffer.get_engram_storage_size_hint(entries, hidden, 1024)
    host = ElasticBuffer(dist.group.WORLD, num_max_tokens_per_rank=256, hidden=hidden, num_cpu_bytes=cpu_bytes,
                         explicitly_destroy=True)
    gpu = ElasticBuffer(dist.group.WORLD, num_max_tokens_per_rank=256, hidden=hidden, explicitly_destroy=True)

    def storage_of(r):
        gen = torch.Generator().manual_seed(77 + r)
        return torch.randn((entries, hidden), generator=gen).to(torch.bfloat16)
    for buf in (host, gpu):
        buf.engram_write(storage_of(rank).cuda())
    full = torch.cat([storage_of(r) for r in range(world)]).cuda()
    gen = torch.Generator().manual_seed(5 + rank)
    idx = torch.randint(0, entries * world, (777,), generator=gen, dtype=torch.int32).cuda()
    out_host = host.engram_fetch(idx)()
    out_gpu = gpu.engram_fetch(idx)()
    torch.cuda.synchronize()
    assert torch.equal(out_host, full[idx.long()]) and torch.equal(out_host, out_gpu)
    # a fresh write is what the next fetch sees
    host.engram_write((storage_of(rank) * 2).cuda())
    out2 = host.engram_fetch(idx)()
    torch.cuda.synchronize()
    assert torch.equal(out2, (full.float() * 2).to(torch.bfloat16)[idx.long()])
    op_error_state(True)
    bad = torch.tensor([-1, entries * world, 3], dtype=torch.int32, device='cuda')
    out3 = host.engram_fetch(bad)()
    torch.cuda.synchronize()
    assert torch.count_nonzero(out3[:2]) == 0 and torch.equal(out3[2], (full[3].float() * 2).to(torch.bfloat16))
    assert op_error_state(True)[0] != 0  # the bounds report
    dist.barrier()
    host.destroy()
    gpu.destroy()


@pytest.mark.parametrize('world', _worlds())
def test_engram_storage_in_host_memory(world):
    run_ranks(_body, world, backend='nccl')
