"""GPU test of the low-latency combine in zero-copy mode: the expert outputs are written into the
registered send buffer (`get_next_low_latency_combine_buffer`) and combined with `zero_copy=True`;
the result must equal the copying combine's.
"""
import pytest
import torch
import torch.distributed as dist

from tests._dist import run_ranks

pytestmark = pytest.mark.gpu


def _zero_copy_body(rank, world, N, H, E, K):
    from deepep_slingshot_b200 import Buffer
    group = dist.group.WORLD
    buf = Buffer(group, num_rdma_bytes=Buffer.get_low_latency_rdma_size_hint(N, H, world, E), low_latency_mode=True,
                 num_gpu_timeout_secs=20)
    E_l = E // world
    for it in range(3):
        g = torch.Generator(device='cuda').manual_seed(it * 10 + rank)
        x = torch.randn((N, H), device='cuda', generator=g).to(torch.bfloat16)
        idx = torch.rand((N, E), device='cuda', generator=g).topk(K, dim=1).indices.to(torch.int64)
        w = torch.rand((N, K), device='cuda', generator=g)
        y = torch.randn((E_l, world * N, H), device='cuda', generator=g).to(torch.bfloat16)
        _, cnt, h, _, _ = buf.low_latency_dispatch(x, idx, N, E, use_fp8=True)
        ref, _, _ = buf.low_latency_combine(y, idx, w, h)
        _, cnt2, h2, _, _ = buf.low_latency_dispatch(x, idx, N, E, use_fp8=True)
        send = buf.get_next_low_latency_combine_buffer(h2)
        # the same expert output for the same (source token, k), whatever slot it landed in
        def rows_by_src(hh):
            src_info, meta = hh[0], hh[7]
            return src_info, meta
        s1, m1 = rows_by_src(h)
        s2, m2 = rows_by_src(h2)
        for e in range(E_l):
            c = int(cnt[e])
            key1 = (m1[e, :c].long() * 1_000_000 + s1[e, :c].long())
            key2 = (m2[e, :c].long() * 1_000_000 + s2[e, :c].long())
            o1, o2 = torch.argsort(key1), torch.argsort(key2)
            send[e, o2] = y[e, o1]
        out, _, _ = buf.low_latency_combine(send, idx, w, h2, zero_copy=True)
        torch.cuda.synchronize()
        assert torch.equal(cnt, cnt2)
        assert torch.equal(out, ref)
    buf.check_error()


@pytest.mark.parametrize('world', [1, 2])
def test_low_latency_zero_copy_combine(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f'needs {world} GPUs')
    run_ranks(_zero_copy_body, world, 'nccl', args=(64, 512, 8 * world, 4))
