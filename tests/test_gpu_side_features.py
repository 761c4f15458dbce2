"""GPU tests of the elastic API's experimental side features: pipeline send/recv on the ring, AGRS
all-gather sessions (copy engines) and Engram fetch (peer loads), each against values every rank
can compute on its own."""
import pytest
import torch
import torch.distributed as dist

from tests._dist import run_ranks
from tests.test_gpu_intranode import _worlds

pytestmark = pytest.mark.gpu


def _payload(src: int, it: int, nbytes: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(1000 * src + it)
    return torch.randint(0, 256, (nbytes,), generator=g, dtype=torch.uint8).cuda()


def _side_body(rank, world):
    from deepep_slingshot_b200 import ElasticBuffer
    from deepep_slingshot_b200.parallel.symmetric import ring_neighbours
    buf = ElasticBuffer(dist.group.WORLD, num_max_tokens_per_rank=64, hidden=256, num_topk=2, num_gpu_timeout_secs=20)
    prev, nxt = ring_neighbours(rank, world)

    # ---- pipeline ring: two sends in flight, then the receives; odd sizes use the byte tail
    buf.pp_set_config(1 << 20, 2)
    sizes = [1001, 65536, 1 << 20, 48, 300000]
    for it, nb in enumerate(sizes):
        buf.pp_send(_payload(rank, it, nb), nxt)
        if it % 2 == 1 or it == len(sizes) - 1:
            for j in ([it - 1, it] if it % 2 == 1 else [it]):
                got = torch.empty(sizes[j], dtype=torch.uint8, device='cuda')
                buf.pp_recv(got, prev)
                torch.cuda.synchronize()
                assert torch.equal(got, _payload(prev, j, sizes[j])), f'pp payload {j} from {prev}'
    # reverse direction
    buf.pp_send(_payload(rank, 99, 4096), prev)
    got = torch.empty(4096, dtype=torch.uint8, device='cuda')
    buf.pp_recv(got, nxt)
    torch.cuda.synchronize()
    assert torch.equal(got, _payload(nxt, 99, 4096))

    # ---- AGRS: single, batched and in-place all-gathers over two sessions
    buf.agrs_set_config(32 << 20, 8)
    for session in range(2):
        with buf.agrs_new_session():
            x = torch.full((33, 64), float(rank + 10 * session), dtype=torch.float32, device='cuda')
            g, hook = buf.all_gather(x)
            hook()
            exp = torch.stack([torch.full((33, 64), float(r + 10 * session), device='cuda') for r in range(world)])
            assert g.shape == (world, 33, 64) and torch.equal(g, exp)
            a = torch.arange(1000, device='cuda', dtype=torch.int32) + rank
            b = torch.ones((7, 9), device='cuda', dtype=torch.bfloat16) * (rank + 1)
            ga, gb, hook = buf.all_gather([a, b])
            hook()
            for r in range(world):
                assert torch.equal(ga[r], torch.arange(1000, device='cuda', dtype=torch.int32) + r)
                assert torch.equal(gb[r], torch.ones((7, 9), device='cuda', dtype=torch.bfloat16) * (r + 1))
            t = buf.agrs_get_inplace_tensor((128, 256), torch.bfloat16)
            t.copy_(torch.full((128, 256), float(rank - 3), device='cuda'))
            gt, hook = buf.all_gather(t)
            hook()
            for r in range(world):
                assert torch.equal(gt[r].float(), torch.full((128, 256), float(r - 3), device='cuda'))
            torch.cuda.synchronize()

    # ---- Engram: every rank publishes rows; any rank fetches any global entry
    entries, hidden = 500, 1024
    def storage_of(r):
        gen = torch.Generator().manual_seed(77 + r)
        return torch.randn((entries, hidden), generator=gen).to(torch.bfloat16)
    buf.engram_write(storage_of(rank).cuda())
    full = torch.cat([storage_of(r) for r in range(world)]).cuda()
    gen = torch.Generator().manual_seed(5 + rank)
    idx = torch.randint(0, entries * world, (777,), generator=gen, dtype=torch.int32).cuda()
    out = buf.engram_fetch(idx)()
    torch.cuda.synchronize()
    assert torch.equal(out, full[idx.long()])
    buf._engram.check_error()
    dist.barrier()


@pytest.mark.parametrize('world', _worlds())
def test_side_features(world):
    run_ranks(_side_body, world, backend='nccl')
