"""GPU tests of the tcgen05 grouped FP8 GEMM against an fp32 torch reference."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize('counts,n,k', [([200, 0, 130, 37], 256, 256), ([128], 128, 128), ([300, 257, 1, 640], 512, 1024),
                                        ([1000, 900, 1100, 512, 64, 700, 333, 800], 4096, 7168)])
def test_grouped_gemm_fp8(counts, n, k):
    from deepep_slingshot_b200.ops.gemm import (grouped_gemm_fp8, grouped_gemm_fp8_reference, op_error_state,
                                                quantize_weights_fp8)
    from deepep_slingshot_b200.utils.math import per_token_cast_to_fp8
    g = torch.Generator().manual_seed(len(counts) * 7 + n)
    E = len(counts)
    aligned = [(c + 127) // 128 * 128 for c in counts]
    offsets = torch.tensor([0] + list(torch.tensor(aligned).cumsum(0).tolist()), dtype=torch.int32).cuda()
    rows = int(offsets[-1]) + 128
    x = torch.randn((rows, k), generator=g).to(torch.bfloat16).cuda()
    a, sa = per_token_cast_to_fp8(x)
    w = (torch.randn((E, n, k), generator=g) * 0.02).cuda()
    b, sb = quantize_weights_fp8(w)
    cnt = torch.tensor(counts, dtype=torch.int32).cuda()
    op_error_state(clear=True)
    d = grouped_gemm_fp8(a, sa.contiguous(), b, sb.contiguous(), offsets, cnt, timeout_s=5.0)
    torch.cuda.synchronize()
    assert op_error_state()[0] == 0, op_error_state()
    ref = grouped_gemm_fp8_reference(a, sa, b, sb, offsets, cnt)
    for e in range(E):
        r0, r1 = int(offsets[e]), int(offsets[e]) + counts[e]
        if r1 > r0:
            got, exp = d[r0:r1].float(), ref[r0:r1]
            err = (got - exp).abs().max().item()
            assert err <= 2e-2 * exp.abs().max().item() + 1e-3, (e, err, exp.abs().max().item())


@pytest.mark.parametrize('E,n,k', [(3, 256, 384), (2, 4096, 7168)])
def test_quantize_weights_kernel_matches_torch(E, n, k):
    from deepep_slingshot_b200.ops.gemm import quantize_weights_fp8, quantize_weights_fp8_reference
    g = torch.Generator().manual_seed(E * n)
    w = (torch.randn((E, n, k), generator=g) * torch.rand((E, 1, 1), generator=g) * 0.1).to(torch.bfloat16).cuda()
    w[0, :128, :128] = 0  # an all-zero block takes the 1e-4 floor
    q, s = quantize_weights_fp8(w)
    rq, rs = quantize_weights_fp8_reference(w)
    torch.cuda.synchronize()
    assert torch.equal(s, rs)
    assert torch.equal(q.view(torch.uint8), rq.view(torch.uint8))
