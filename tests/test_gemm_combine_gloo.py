"""CPU (gloo) checks of the down projection -> combine index rules, restated in torch in
`parallel/gemm_combine.py` (`row_destinations`, `exchange_reference`, `reduce_reference`).

Over the oracle's own dispatch, the slots that the row destinations select, reduced with every
source's own routing, must equal `ReferenceBuffer.combine` in its expanded weighted mode (the unfused
composition the fused path replaces). Rows hold small integers and the weights are 1/2 or 1, so every
partial sum is exact in bf16 and the two orders of summation agree bit for bit. Some tokens are
routed nowhere (all -1) or partly (-1 selections), and the ranks hold different token counts.
"""
import pytest
import torch
import torch.distributed as dist

from tests._dist import run_ranks


def _row_map(recv_topk_idx: torch.Tensor, num_local_experts: int, alignment: int):
    """The permute's (received token, k) -> row map: 128-aligned block per local expert, rows in
    (token, k) order; returns (row_map [num_recv, K] int32, rows)."""
    num_recv, K = recv_topk_idx.shape
    counts = [int((recv_topk_idx == e).sum()) for e in range(num_local_experts)]
    offsets = [0]
    for c in counts:
        offsets.append(offsets[-1] + (c + alignment - 1) // alignment * alignment)
    row_map = torch.full((num_recv, K), -1, dtype=torch.int32)
    fill = [0] * num_local_experts
    for j in range(num_recv):
        for k in range(K):
            e = int(recv_topk_idx[j, k])
            if e >= 0:
                row_map[j, k] = offsets[e] + fill[e]
                fill[e] += 1
    return row_map, max(offsets[-1], 1)


def _body(rank, world, N, H, E, K):
    from deepep_slingshot_b200 import ReferenceBuffer
    from deepep_slingshot_b200.parallel.gemm_combine import exchange_reference, reduce_reference, row_destinations
    from deepep_slingshot_b200.utils import gate
    group = dist.group.WORLD
    ref = ReferenceBuffer(group)
    g = torch.Generator().manual_seed(31 + rank)
    n = N - 3 * rank
    x = torch.randn((n, H), generator=g).to(torch.bfloat16)
    idx, _ = gate.normal_routing(n, E, K, generator=g)
    idx[torch.rand(idx.shape, generator=g) < 0.15] = -1
    idx[: max(1, n // 10)] = -1  # tokens routed nowhere
    w = torch.where(torch.rand(idx.shape, generator=g) < 0.5, 0.5, 1.0).float()
    rx, ridx, rw, _, h, _ = ref.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E)
    row_map, rows = _row_map(ridx, E // world, 128)
    y = torch.randint(-2, 3, (rows, H), generator=g).to(torch.bfloat16)
    dest = row_destinations(row_map, h[3], h[0], rank, rows)
    assert dest.shape == (rows,) and int((dest >= 0).sum()) == int((row_map >= 0).sum())
    slots = exchange_reference(group, y, dest, n, K)
    out = reduce_reference(slots, idx, w)
    expect, _, _ = ref.combine(y, h, row_map=row_map, row_weights=rw)
    assert out.shape == (n, H) and out.dtype == torch.bfloat16
    assert torch.equal(out, expect), (out.float() - expect.float()).abs().max()
    # unweighted: plain sum of the token's expert rows
    expect_u, _, _ = ref.combine(y, h, row_map=row_map)
    assert torch.equal(reduce_reference(slots, idx, None), expect_u)


@pytest.mark.parametrize('world', [1, 2, 3])
def test_gemm_combine_index_rules_match_the_oracle_combine(world):
    run_ranks(_body, world, backend='gloo', args=(48, 256, 12, 4))


def test_row_destination_words():
    from deepep_slingshot_b200.parallel.gemm_combine import MAX_SLOTS, SLOT_BITS, row_destinations
    # 3 ranks; this is rank 1, receiving 2 tokens from rank 0, none from rank 1, 3 from rank 2
    rank_prefix_matrix = torch.tensor([[0, 2, 0], [0, 2, 0], [0, 5, 0]], dtype=torch.int32)
    recv_src_idx = torch.tensor([4, 9, 0, 1, 7], dtype=torch.int32)
    row_map = torch.tensor([[0, -1], [-1, 1], [2, 3], [-1, -1], [-1, 4]], dtype=torch.int32)
    dest = row_destinations(row_map, recv_src_idx, rank_prefix_matrix, rank=1, rows=6)
    K = 2
    want = [(0 << SLOT_BITS) | (4 * K + 0), (0 << SLOT_BITS) | (9 * K + 1), (2 << SLOT_BITS) | (0 * K + 0),
            (2 << SLOT_BITS) | (0 * K + 1), (2 << SLOT_BITS) | (7 * K + 1), -1]
    assert dest.tolist() == want
    assert MAX_SLOTS == 1 << 24
