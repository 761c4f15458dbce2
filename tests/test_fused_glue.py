"""Python glue of the fused paths, checked on CPU with fake runtimes (argument order, handle tuples,
and the decode layer's call sequence); the kernels themselves are tested on GPUs."""
import types

import torch

from deepep_slingshot_b200.parallel.buffer import Buffer


class _FakeRuntime:
    def __init__(self):
        self.calls = []

    def intranode_dispatch_gemm(self, *args):
        self.calls.append(('intranode_dispatch_gemm', args))
        send_head = torch.tensor([[0, -1], [1, 0]], dtype=torch.int32)
        return (torch.zeros(256, 128), torch.zeros(256, 128), torch.zeros(256, 1), torch.zeros(2, 2, dtype=torch.int32),
                torch.ones(2, 2), torch.tensor([0, 128, 256], dtype=torch.int32), torch.tensor([3, 1], dtype=torch.int32),
                torch.tensor([5, 6], dtype=torch.int32), [128, 128], 'rpm', 'spm', 'rrp', send_head)

    def low_latency_dispatch_gemm(self, *args):
        self.calls.append(('low_latency_dispatch_gemm', args))
        return 'out', 'rx', 'rs', 'count', 'src_info', 'src_meta', 1

    def low_latency_gemm_combine(self, *args):
        self.calls.append(('low_latency_gemm_combine', args))
        return 'combined'


def _buffer():
    b = Buffer.__new__(Buffer)
    b.runtime = _FakeRuntime()
    return b


def test_dispatch_gemm_handle_and_grouped():
    b = _buffer()
    x = torch.zeros(2, 128)
    h, grouped, handle = b.dispatch_gemm(x, 'idx', 'w', 16, 'wq', 'ws', round_scale=True, num_sms=7, pull_ctas=3)
    name, args = b.runtime.calls[0]
    assert name == 'intranode_dispatch_gemm' and args == (x, 'idx', 'w', 16, 'wq', 'ws', True, 7, 3)
    assert h.shape == (256, 128)
    assert handle[0] == 'rpm' and handle[1] == 'spm' and handle[2] == 'rrp'
    assert torch.equal(handle[3], torch.tensor([5, 6], dtype=torch.int32))
    assert torch.equal(handle[4], torch.tensor([[True, False], [True, True]]))
    assert torch.equal(handle[5], torch.tensor([[0, -1], [1, 0]], dtype=torch.int32))
    assert grouped['num_recv_tokens_per_expert_list'] == [128, 128]
    assert grouped['expert_offsets'].tolist() == [0, 128, 256] and grouped['expert_counts'].tolist() == [3, 1]
    # the combine reads (rpm, spm, _, recv_src_idx, _, send_head) from the same positions as dispatch()'s handle
    rpm, spm, _, src, _, sh = handle
    assert rpm == 'rpm' and spm == 'spm' and src is handle[3] and sh is handle[5]


def test_low_latency_gemm_paths_pass_the_handle_through():
    b = _buffer()
    x = torch.zeros(3, 128)
    out, count, handle, (rx, rs) = b.low_latency_dispatch_gemm(x, 'idx', 64, 16, 'wq', 'ws', None, False, 5)
    assert b.runtime.calls[0] == ('low_latency_dispatch_gemm', (x, 'idx', None, 64, 16, 'wq', 'ws', False, 5))
    assert (out, count, rx, rs) == ('out', 'count', 'rx', 'rs')
    # same layout as low_latency_dispatch's handle: (src_info, layout_range, max_tokens, hidden, experts, count, half, meta)
    assert handle == ('src_info', None, 64, 128, 16, 'count', 1, 'src_meta')
    res = b.low_latency_gemm_combine('aq', 'as', 'w2q', 'w2s', 'idx', 'wts', handle, num_sms=9)
    assert res == 'combined'
    assert b.runtime.calls[1] == ('low_latency_gemm_combine', ('aq', 'as', 'count', 'w2q', 'w2s', 'idx', 'wts', 1, 64, 16, 9))


def test_decode_layer_call_sequence(monkeypatch):
    """MoEFFN.forward_low_latency: fused dispatch + GEMM, masked SwiGLU on the returned counts, then
    the fused down projection + combine (or the unfused GEMM + combine)."""
    import deepep_slingshot_b200.models.moe as moe
    import deepep_slingshot_b200.ops.gemm as gemm_ops
    import deepep_slingshot_b200.ops.quant as quant_ops
    seen = []
    layer = types.SimpleNamespace(num_experts=16)
    layer.quantized_weights = lambda: ('w1q', 'w1s', 'w2q', 'w2s')

    class FakeBuf:
        def low_latency_dispatch_gemm(self, x, idx, maxT, E, wq, ws):
            seen.append(('dispatch_gemm', maxT, E, wq, ws))
            return 'h', 'counts', 'handle', None

        def low_latency_gemm_combine(self, aq, as_, wq, ws, idx, wts, handle):
            seen.append(('gemm_combine', aq, as_, wq, ws, handle))
            return 'out'

        def low_latency_combine(self, y, idx, wts, handle):
            seen.append(('combine', y, handle))
            return 'out2', None, None

    monkeypatch.setattr(quant_ops, 'swiglu_quant', lambda h, counts=None: seen.append(('swiglu', h, counts)) or ('a', 'aq', 'as'))
    monkeypatch.setattr(gemm_ops, 'masked_grouped_gemm_fp8', lambda *a: seen.append(('masked_gemm',) + a) or 'y')
    fwd = moe.MoEFFN.forward_low_latency.__wrapped__ if hasattr(moe.MoEFFN.forward_low_latency, '__wrapped__') \
        else moe.MoEFFN.forward_low_latency
    wts = torch.ones(2, 2)
    assert fwd(layer, FakeBuf(), 'x', 'idx', wts, 64) == 'out'
    assert [s[0] for s in seen] == ['dispatch_gemm', 'swiglu', 'gemm_combine']
    assert seen[0] == ('dispatch_gemm', 64, 16, 'w1q', 'w1s') and seen[1] == ('swiglu', 'h', 'counts')
    assert seen[2] == ('gemm_combine', 'aq', 'as', 'w2q', 'w2s', 'handle')
    seen.clear()
    assert fwd(layer, FakeBuf(), 'x', 'idx', wts, 64, fuse_combine=False) == 'out2'
    assert [s[0] for s in seen] == ['dispatch_gemm', 'swiglu', 'masked_gemm', 'combine']
    assert seen[2] == ('masked_gemm', 'aq', 'as', 'counts', 'w2q', 'w2s')
