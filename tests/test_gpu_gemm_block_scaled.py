"""GPU tests of the block-scaled FP8 grouped GEMM (`grouped_gemm_fp8(..., ue8m0=True)`): with
power-of-two scales the tensor core applies them itself (kind::mxf8f6f4.block_scale). Checked against
the fp32 torch oracle with the same dequantisation, and against the promotion kernel on the same
inputs (the two differ only in the order of fp32 accumulation)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize('counts,n,k', [([128], 128, 128), ([200, 0, 130, 37], 256, 256),
                                        ([300, 257, 1, 640], 512, 1024),
                                        ([1000, 900, 1100, 512, 64, 700, 333, 800], 4096, 7168)])
def test_grouped_gemm_fp8_block_scaled(counts, n, k):
    from deepep_slingshot_b200.ops.gemm import (grouped_gemm_fp8, grouped_gemm_fp8_reference, op_error_state,
                                                quantize_weights_fp8)
    from deepep_slingshot_b200.utils.math import per_token_cast_to_fp8
    g = torch.Generator().manual_seed(len(counts) * 11 + n)
    E = len(counts)
    aligned = [(c + 127) // 128 * 128 for c in counts]
    offsets = torch.tensor([0] + list(torch.tensor(aligned).cumsum(0).tolist()), dtype=torch.int32).cuda()
    rows = int(offsets[-1])
    # activations with a spread of magnitudes per row and per 128-block, so the scales differ
    x = (torch.randn((rows, k), generator=g) * torch.exp2(torch.randint(-6, 6, (rows, k // 128), generator=g).float())
         .repeat_interleave(128, dim=1)).to(torch.bfloat16).cuda()
    a, sa = per_token_cast_to_fp8(x, round_scale=True)
    w = (torch.randn((E, n, k), generator=g) * 0.02).to(torch.bfloat16).cuda()
    b, sb = quantize_weights_fp8(w, round_scale=True)
    assert bool((torch.log2(sb) == torch.round(torch.log2(sb))).all())  # powers of two
    cnt = torch.tensor(counts, dtype=torch.int32).cuda()
    op_error_state(clear=True)
    d = grouped_gemm_fp8(a, sa.contiguous(), b, sb.contiguous(), offsets, cnt, timeout_s=5.0, ue8m0=True)
    dp = grouped_gemm_fp8(a, sa.contiguous(), b, sb.contiguous(), offsets, cnt, timeout_s=5.0)
    torch.cuda.synchronize()
    assert op_error_state()[0] == 0, op_error_state()
    ref = grouped_gemm_fp8_reference(a, sa, b, sb, offsets, cnt)
    for e in range(E):
        r0, r1 = int(offsets[e]), int(offsets[e]) + counts[e]
        if r1 > r0:
            got, exp, prom = d[r0:r1].float(), ref[r0:r1], dp[r0:r1].float()
            scale = exp.abs().max().item()
            assert (got - exp).abs().max().item() <= 2e-2 * scale + 1e-3, (e, (got - exp).abs().max().item(), scale)
            assert (got - prom).abs().max().item() <= 1e-2 * scale + 1e-3, (e, (got - prom).abs().max().item(), scale)


def test_weight_quantization_round_scale_matches_torch():
    from deepep_slingshot_b200.ops.gemm import quantize_weights_fp8, quantize_weights_fp8_reference
    g = torch.Generator().manual_seed(3)
    w = (torch.randn((2, 256, 384), generator=g) * 0.05).to(torch.bfloat16).cuda()
    q, s = quantize_weights_fp8(w, round_scale=True)
    rq, rs = quantize_weights_fp8_reference(w, round_scale=True)
    torch.cuda.synchronize()
    assert torch.equal(s, rs) and torch.equal(q.view(torch.uint8), rq.view(torch.uint8))
