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


@pytest.mark.parametrize('E,n,k,rows_per', [(3, 256, 512, [130, 0, 300]), (4, 2048, 7168, [256, 128, 37, 500])])
def test_grouped_gemm_bf16_dgrad(E, n, k, rows_per):
    """M-grouped bf16 tcgen05 GEMM (activation gradients) against an fp32 torch oracle."""
    from deepep_slingshot_b200.ops.gemm import grouped_gemm_bf16, grouped_gemm_bf16_reference
    g = torch.Generator().manual_seed(n + k)
    counts = torch.tensor(rows_per, dtype=torch.int32)
    aligned = (counts + 127) // 128 * 128
    offsets = torch.zeros(E + 1, dtype=torch.int32)
    offsets[1:] = aligned.cumsum(0)
    rows = int(offsets[-1])
    a = torch.randn((rows, k), generator=g).to(torch.bfloat16).cuda()
    b = (torch.randn((E, n, k), generator=g) * 0.05).to(torch.bfloat16).cuda()
    d = grouped_gemm_bf16(a, b, offsets.cuda(), counts.cuda())
    ref = grouped_gemm_bf16_reference(a, b, offsets, counts)
    torch.cuda.synchronize()
    for e in range(E):
        r0, r1 = int(offsets[e]), int(offsets[e]) + rows_per[e]
        if r1 > r0:
            assert torch.allclose(d[r0:r1].float(), ref[r0:r1], atol=2e-2, rtol=2e-2), (e, (d[r0:r1].float() - ref[r0:r1]).abs().max())


@pytest.mark.parametrize('m,n,rows_per', [(256, 384, [128, 0, 256, 64]), (2048, 7168, [512, 1024, 128])])
def test_grouped_gemm_bf16_wgrad(m, n, rows_per):
    """K-grouped bf16 tcgen05 GEMM (weight gradients) against an fp32 torch oracle; an expert with
    no rows gets a zero gradient."""
    from deepep_slingshot_b200.ops.gemm import grouped_gemm_bf16_wgrad, grouped_gemm_bf16_wgrad_reference
    g = torch.Generator().manual_seed(m + n)
    E = len(rows_per)
    offsets = torch.zeros(E + 1, dtype=torch.int32)
    offsets[1:] = torch.tensor(rows_per, dtype=torch.int32).cumsum(0)
    K = int(offsets[-1])
    a_t = torch.randn((m, K), generator=g).to(torch.bfloat16).cuda()
    b_t = (torch.randn((n, K), generator=g) * 0.05).to(torch.bfloat16).cuda()
    d = grouped_gemm_bf16_wgrad(a_t, b_t, offsets.cuda())
    ref = grouped_gemm_bf16_wgrad_reference(a_t, b_t, offsets)
    torch.cuda.synchronize()
    assert d.shape == (E, m, n)
    assert torch.allclose(d.float(), ref, atol=5e-2, rtol=2e-2), (d.float() - ref).abs().max()
