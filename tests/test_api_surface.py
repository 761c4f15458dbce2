"""API surface parity (CPU): every public method of DeepEP's `Buffer` (v1) and `ElasticBuffer` (v2)
exists here with compatible leading parameters, and the package exports the same names."""
import inspect

import deepep_slingshot_b200 as ep

BUFFER_METHODS = [
    'barrier', 'capture', 'clean_low_latency_buffer', 'combine', 'destroy', 'dispatch', 'get_combine_config',
    'get_comm_stream', 'get_dispatch_config', 'get_dispatch_layout', 'get_local_buffer_tensor',
    'get_low_latency_rdma_size_hint', 'get_next_low_latency_combine_buffer', 'internode_combine',
    'internode_dispatch', 'is_sm90_compiled', 'low_latency_clean_mask_buffer', 'low_latency_combine',
    'low_latency_dispatch', 'low_latency_query_mask_buffer', 'low_latency_update_mask_buffer', 'set_num_sms',
]
ELASTIC_METHODS = [
    'agrs_get_inplace_tensor', 'agrs_new_session', 'agrs_set_config', 'all_gather', 'barrier', 'capture', 'combine',
    'create_agrs_session', 'destroy', 'destroy_agrs_session', 'dispatch', 'engram_fetch', 'engram_write',
    'get_agrs_buffer_size_hint', 'get_agrs_num_max_session_bytes', 'get_buffer_size_hint', 'get_comm_stream',
    'get_elastic_buffer_alignment', 'get_engram_storage_size_hint', 'get_logical_domain_size',
    'get_physical_domain_size', 'get_pp_buffer_size_hint', 'get_theoretical_num_qps', 'get_theoretical_num_sms',
    'pp_recv', 'pp_send', 'pp_set_config',
]
EXPORTS = ['Buffer', 'Config', 'ElasticBuffer', 'EPHandle', 'EventOverlap', 'topk_idx_t',
           'get_physical_domain_size', 'get_logical_domain_size']


def test_buffer_methods():
    missing = [m for m in BUFFER_METHODS if not hasattr(ep.Buffer, m)]
    assert not missing, missing


def test_elastic_methods():
    missing = [m for m in ELASTIC_METHODS if not hasattr(ep.ElasticBuffer, m)]
    assert not missing, missing


def test_exports():
    missing = [n for n in EXPORTS if not hasattr(ep, n)]
    assert not missing, missing


def test_leading_parameters():
    """Positional parameters callers pass without keywords keep DeepEP's order."""
    def params(f):
        return [p for p in inspect.signature(f).parameters if p != 'self']
    assert params(ep.Buffer.__init__)[:4] == ['group', 'num_nvl_bytes', 'num_rdma_bytes', 'low_latency_mode']
    assert params(ep.Buffer.dispatch)[:2] == ['x', 'handle']
    assert params(ep.Buffer.combine)[:3] == ['x', 'handle', 'topk_weights']
    assert params(ep.Buffer.get_dispatch_layout)[:2] == ['topk_idx', 'num_experts']
    assert params(ep.Buffer.low_latency_dispatch)[:4] == ['x', 'topk_idx', 'num_max_dispatch_tokens_per_rank',
                                                          'num_experts']
    assert params(ep.Buffer.low_latency_combine)[:4] == ['x', 'topk_idx', 'topk_weights', 'handle']
    assert params(ep.ElasticBuffer.dispatch)[:3] == ['x', 'topk_idx', 'topk_weights']
    assert params(ep.ElasticBuffer.combine)[:3] == ['x', 'handle', 'topk_weights']


def test_every_kernel_source_is_built():
    """setup.py compiles every .cu / .cpp source of the extension (a new kernel file cannot be left out)."""
    import glob
    import os
    import re
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    setup = open(os.path.join(root, 'setup.py')).read()
    listed = set(re.findall(r'"(kernels|runtime)", "([A-Za-z0-9_]+\.(?:cu|cpp))"', setup))
    csrc = os.path.join(root, 'deepep_slingshot_b200', 'csrc')
    on_disk = {(os.path.basename(os.path.dirname(p)), os.path.basename(p))
               for p in glob.glob(os.path.join(csrc, 'kernels', '*.cu')) + glob.glob(os.path.join(csrc, 'runtime', '*.cpp'))}
    assert on_disk <= listed, sorted(on_disk - listed)


def test_fused_entry_points_exist():
    from deepep_slingshot_b200 import Buffer
    from deepep_slingshot_b200.models import MoEFFN
    from deepep_slingshot_b200.ops import gemm, quant
    for name in ('dispatch_gemm', 'low_latency_dispatch_gemm', 'low_latency_gemm_combine'):
        assert callable(getattr(Buffer, name))
    assert callable(MoEFFN.forward_low_latency) and callable(MoEFFN.quantized_weights)
    assert callable(gemm.masked_grouped_gemm_fp8) and callable(gemm.grouped_gemm_bf16_wgrad_rows)
    assert callable(quant.swiglu_quant)


def test_gemm_combine_and_host_memory_entry_points():
    from deepep_slingshot_b200._ext import require_ext
    from deepep_slingshot_b200.models import MoEFFN
    from deepep_slingshot_b200.parallel.gemm_combine import GemmCombine
    from deepep_slingshot_b200.parallel.host_memory import HostSegments
    _C = require_ext()
    for name in ('gemm_combine_send', 'gemm_combine_reduce'):
        assert callable(getattr(_C.SymmetricRegion, name))
    assert callable(_C.engram_fetch_rows) and hasattr(_C, 'HostSegment')
    assert callable(GemmCombine.send) and callable(GemmCombine.reduce) and callable(HostSegments.device_ptrs)
    assert callable(MoEFFN.release)
    assert GemmCombine.size_hint(4096, 8, 7168) == 4096 * 8 * 7168 * 2
