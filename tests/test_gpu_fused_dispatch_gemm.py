"""GPU tests of the normal-mode dispatch fused with the gate/up grouped FP8 GEMM
(`Buffer.dispatch_gemm`), against dispatch -> permute -> grouped_gemm_fp8 on the same inputs, and of
the MoE layer with the fused forward.
"""
import pytest
import torch
import torch.distributed as dist

from tests._dist import run_ranks

pytestmark = pytest.mark.gpu


def _fused_body(rank, world, N, H, E, K, n, pull_ctas):
    from deepep_slingshot_b200 import Buffer
    from deepep_slingshot_b200.ops.gemm import grouped_gemm_fp8, quantize_weights_fp8
    from deepep_slingshot_b200.ops.permute import permute
    from deepep_slingshot_b200.utils import gate
    group = dist.group.WORLD
    buf = Buffer(group, num_nvl_bytes=Buffer.get_nvl_buffer_size_hint(N, H, world), num_gpu_timeout_secs=20)
    E_l = E // world
    gw = torch.Generator().manual_seed(99 + rank)
    w = (torch.randn((E_l, n, H), generator=gw) * 0.05).to(torch.bfloat16).cuda()
    wq, ws = quantize_weights_fp8(w)
    ws = ws.contiguous()
    for it in range(3):
        g = torch.Generator().manual_seed(it * 10 + rank)
        x = torch.randn((N, H), generator=g).to(torch.bfloat16).cuda()
        idx, wts = gate.normal_routing(N, E, K, generator=g)
        idx, wts = idx.cuda(), wts.cuda().float()
        h, grp, handle = buf.dispatch_gemm(x, idx, wts, E, wq, ws, pull_ctas=pull_ctas)
        (rx, rs), ridx, rw, counts_list, ref_handle, _ = buf.dispatch(x, topk_idx=idx, topk_weights=wts, num_experts=E,
                                                                     quantize_fp8=True, expert_alignment=128)
        p = permute(rx, ridx, E_l, alignment=128, probs=rw, x_scales=rs)
        ref_h = grouped_gemm_fp8(p.x, p.scales, wq, ws, p.expert_offsets, p.expert_counts)
        torch.cuda.synchronize()
        assert torch.equal(grp['expert_offsets'], p.expert_offsets)
        assert torch.equal(grp['expert_counts'], p.expert_counts)
        assert grp['num_recv_tokens_per_expert_list'] == list(counts_list)
        assert torch.equal(handle[0], ref_handle[0]) and torch.equal(handle[3], ref_handle[3])
        assert torch.equal(handle[5], ref_handle[5])
        rm, ref_rm = grp['row_map'], p.row_map
        assert torch.equal(rm >= 0, ref_rm >= 0)
        assert torch.equal(grp['topk_weights'], rw)
        valid = rm >= 0
        got_rows, ref_rows = rm[valid].long(), ref_rm[valid].long()
        # same (received token, k) -> same operand bytes and the same GEMM row
        assert torch.equal(grp['x'][got_rows].view(torch.uint8), p.x[ref_rows].view(torch.uint8))
        assert torch.equal(grp['scales'][got_rows], p.scales[ref_rows])
        got_h, exp_h = h[got_rows].float(), ref_h[ref_rows].float()
        assert float((got_h - exp_h).abs().max()) <= 1e-2 * float(exp_h.abs().max()) + 1e-3
        # rows of every expert stay inside its aligned block
        off = grp['expert_offsets'].tolist()
        cnt = grp['expert_counts'].tolist()
        e_of = torch.searchsorted(grp['expert_offsets'][1:].long(), got_rows, right=True)
        starts = grp['expert_offsets'][e_of].long()
        assert bool(((got_rows - starts) < grp['expert_counts'][e_of].long()).all())
        assert sum(cnt) == int(valid.sum()) and off[-1] >= sum(cnt)
    buf.check_error()


@pytest.mark.parametrize('world', [1, 2])
@pytest.mark.parametrize('pull_ctas', [8, 32])
def test_dispatch_gemm_matches_unfused(world, pull_ctas):
    if torch.cuda.device_count() < world:
        pytest.skip(f'needs {world} GPUs')
    run_ranks(_fused_body, world, 'nccl', args=(512, 1024, 32, 8, 512, pull_ctas))


def _moe_fused_body(rank, world, *args):
    from deepep_slingshot_b200.models import moe as moe_mod
    from tests.test_gpu_moe import _moe_body
    moe_mod._FUSED_DISPATCH['enabled'] = True
    _moe_body(rank, world, *args, bwd='grouped')


@pytest.mark.parametrize('world', [1, 2])
def test_moe_layer_fused_dispatch(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f'needs {world} GPUs')
    run_ranks(_moe_fused_body, world, 'nccl', args=(256, 1024, 512, 16, 4))
