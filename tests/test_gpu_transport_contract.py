"""The transport contract the EP kernels rely on, checked over NVLink peer memory on the GPU.

Restates the reference's backend device tests for this library's primitives:
  * multi-producer signalling (backend/tests/gin_producer_stress.cu:10-63): many warps add to one
    flag in a peer's memory with sys-scope release reductions; the owner's bounded wait sees the
    exact total;
  * window bounds (backend/tests/gin_bounds.cu:9-28): the window rule every indexed peer access uses
    (`in_window`), evaluated on isolated cases only, so no out-of-range address is ever accessed;
  * guard bytes around receive regions (backend/tests/gin_smoke.cu:17-48): the parts of the staging
    and combine regions a dispatch + combine must not write keep a byte pattern;
  * receive capacity: a dispatch into `num_worst_tokens` rows fewer than it receives reports
    kErrCapacity before writing any row, which the host raises as an exception;
  * per-destination counts above 65535 (the count step's 32-bit counters).
None of these faults a GPU or leaves a kernel waiting: every wait is bounded and every bad index is
rejected before an access.
"""
import pytest
import torch
import torch.distributed as dist

from tests._dist import run_ranks
from tests.test_gpu_intranode import _make_inputs, _worlds

pytestmark = pytest.mark.gpu


def _rule(i, c, w):
    return 0 if (i >= 0 and c >= 0 and w >= 0 and c <= w and i <= w - c) else 11


def test_window_rule_on_device():
    from deepep_slingshot_b200._ext import require_ext
    big = (1 << 62)
    cases = [(0, 1, 1), (0, 0, 0), (1, 1, 1), (-1, 1, 10), (9, 1, 10), (10, 1, 10), (10, 0, 10), (5, 6, 10),
             (5, 5, 10), (big, big, big), (big, 1, big), (-big, 1, 10), (3, -1, 10), (0, 1, -5), (7, big, 10),
             ((1 << 63) - 1, 1, (1 << 63) - 1), (0, (1 << 63) - 1, (1 << 63) - 1)]
    t = torch.tensor(cases, dtype=torch.int64, device='cuda')
    codes = require_ext().window_check(t).cpu().tolist()
    assert codes == [_rule(*c) for c in cases]


def _signal_body(rank, world):
    from deepep_slingshot_b200 import Buffer
    buf = Buffer(dist.group.WORLD, num_nvl_bytes=Buffer.get_nvl_buffer_size_hint(128, 1024, world),
                 num_gpu_timeout_secs=10)
    for blocks, warps, rounds in ((1, 1, 1), (64, 8, 16), (132, 32, 8)):
        status, seen = buf.transport_selftest(blocks, warps, rounds)
        assert (status, seen) == (0, blocks * warps * rounds), (blocks, warps, rounds, status, seen)
    buf.check_error()


@pytest.mark.parametrize('world', _worlds())
def test_multi_producer_signal(world):
    run_ranks(_signal_body, world, 'nccl')


def _guard_body(rank, world):
    from deepep_slingshot_b200 import Buffer, ReferenceBuffer
    from deepep_slingshot_b200._ext import require_ext
    N, H, E, K = 200, 1024, 16, 4
    size = Buffer.get_nvl_buffer_size_hint(2 * N, H, world)
    buf = Buffer(dist.group.WORLD, num_nvl_bytes=size, num_gpu_timeout_secs=20)
    ref = ReferenceBuffer(dist.group.WORLD)
    L = require_ext().normal_layout(size, H, world)
    region = buf.get_local_buffer_tensor(torch.uint8)
    x, idx, w = _make_inputs(rank, N, H, E, K)
    ntpr = ref.get_dispatch_layout(idx, E)[0]
    sent_rows = int(ntpr.sum())  # rows of my tokens that come back into my combine region
    row = 2 * H
    guards = [  # (start, end) byte ranges nobody may write in this dispatch + combine
        (L['staging_off'] + N * L['record_bytes'], L['staging_off'] + L['capacity'] * L['record_bytes']),
        (L['combine_off'] + sent_rows * row, L['combine_off'] + L['capacity'] * world * row),
    ]
    for a, b in guards:
        region[a:b] = 0xA5
    torch.cuda.synchronize()
    dist.barrier()
    for it in range(2):
        rx, ri, rw, _, h, _ = buf.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E, quantize_fp8=(it == 1))
        if it == 1:
            rx = rx[0].float().to(torch.bfloat16)
        out, _, _ = buf.combine(rx.contiguous(), h, topk_weights=rw)
        torch.cuda.synchronize()
        for a, b in guards:
            assert bool((region[a:b] == 0xA5).all()), (it, a, b)
    buf.check_error()


@pytest.mark.parametrize('world', _worlds())
def test_guard_bytes_around_receive_regions(world):
    run_ranks(_guard_body, world, 'nccl')


def _capacity_body(rank, world):
    from deepep_slingshot_b200 import Buffer
    N, H, E, K = 256, 512, 16, 4
    group = dist.group.WORLD
    buf = Buffer(group, num_nvl_bytes=Buffer.get_nvl_buffer_size_hint(N, H, world), num_gpu_timeout_secs=10,
                 explicitly_destroy=True)
    x, idx, w = _make_inputs(rank, N, H, E, K)
    # every rank receives at least one row of each of its own tokens routed to it; 8 rows of room is
    # far below what normal routing delivers, so every rank's pull reports the capacity error
    buf.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E, num_worst_tokens=8)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match='capacity'):
        buf.check_error()
    assert buf.get_error_state()[0] == 10
    dist.barrier()
    buf.destroy()
    buf2 = Buffer(group, num_nvl_bytes=Buffer.get_nvl_buffer_size_hint(N, H, world), num_gpu_timeout_secs=10)
    rx, *_ = buf2.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E)
    torch.cuda.synchronize()
    buf2.check_error()


@pytest.mark.parametrize('world', _worlds()[:2])
def test_capacity_error_raises(world):
    run_ranks(_capacity_body, world, 'nccl')


def _many_tokens_body(rank, world):
    from deepep_slingshot_b200 import Buffer, ReferenceBuffer
    N, H, E, K = 70000, 128, 8 * world, 1
    buf = Buffer(dist.group.WORLD, num_nvl_bytes=Buffer.get_nvl_buffer_size_hint(N, H, world), num_gpu_timeout_secs=30)
    ref = ReferenceBuffer(dist.group.WORLD)
    g = torch.Generator().manual_seed(rank)
    x = torch.randn((N, H), generator=g).to(torch.bfloat16).cuda()
    idx = torch.zeros((N, K), dtype=torch.int64).cuda()  # every token to expert 0 of rank 0: 70000 > 65535
    w = torch.ones((N, K)).cuda()
    rx, ri, rw, lst, h, _ = buf.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E)
    ex, ei, ew, elst, eh, _ = ref.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E)
    torch.cuda.synchronize()
    assert rx.shape == ex.shape and torch.equal(rx, ex) and lst == elst
    assert torch.equal(h[5], eh[5])  # send_head positions beyond 65535
    out, _, _ = buf.combine(rx, h)
    eo, _, _ = ref.combine(ex, eh)
    torch.cuda.synchronize()
    assert torch.equal(out, eo)


@pytest.mark.parametrize('world', _worlds()[:2])
def test_per_destination_count_above_16_bits(world):
    run_ranks(_many_tokens_body, world, 'nccl')
