"""CPU (gloo, world 2) tests of the side-feature oracle (pipeline ring, all-gather, Engram fetch)
and of the ring-direction rule shared with the GPU implementation."""
import torch
import torch.distributed as dist

from tests._dist import run_ranks


def _oracle_body(rank, world):
    from deepep_slingshot_b200.parallel.symmetric import ReferenceSideFeatures, ring_neighbours
    ref = ReferenceSideFeatures(dist.group.WORLD)
    prev, nxt = ring_neighbours(rank, world)
    # ring: even ranks send first to avoid a blocking-send cycle
    x = torch.arange(10, dtype=torch.float32) + 100 * rank
    got = torch.empty(10)
    if rank % 2 == 0:
        ref.pp_send(x, nxt)
        ref.pp_recv(got, prev)
    else:
        ref.pp_recv(got, prev)
        ref.pp_send(x, nxt)
    assert torch.equal(got, torch.arange(10, dtype=torch.float32) + 100 * prev)
    g = ref.all_gather(torch.full((3, 4), float(rank)))
    assert g.shape == (world, 3, 4) and all(torch.equal(g[r], torch.full((3, 4), float(r))) for r in range(world))
    ref.engram_write(torch.full((5, 8), float(rank)))
    out = ref.engram_fetch(torch.tensor([0, 9, 5, -1, 10], dtype=torch.int32))()
    assert out[:, 0].tolist() == [0.0, 1.0, 1.0, 0.0, 0.0]


def test_side_oracle_gloo():
    run_ranks(_oracle_body, 2)


def test_ring_neighbours():
    from deepep_slingshot_b200.parallel.symmetric import ring_neighbours
    assert ring_neighbours(0, 1) == (0, 0)
    assert ring_neighbours(0, 2) == (1, 1)
    assert ring_neighbours(0, 8) == (7, 1) and ring_neighbours(7, 8) == (6, 0)
