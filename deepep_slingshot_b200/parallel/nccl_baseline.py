"""The NCCL all-to-all baseline (what the fused NVLink kernels are measured against).

Same API as `Buffer` for dispatch / combine / layout; data moves with
`torch.distributed.all_to_all_single` over NCCL and FP8 quantization is the torch version. This is
the "path that only calls NCCL all-to-all" that the benchmark names as the baseline, not the product.
"""
from .reference import ReferenceBuffer


class NcclAllToAllEP(ReferenceBuffer):
    """Dispatch / combine as `all_to_all_single` over NCCL with torch FP8 casts: the baseline the
    library is measured against, not the product."""
    pass
