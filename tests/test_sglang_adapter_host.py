"""Host-side tests of the SGLang adapter's buffer pool and dispatcher states (no GPU: the pooled
buffer is a fake that records calls)."""
import pytest
import torch

from deepep_slingshot_b200.integrations import sglang_dispatcher as sd


class _FakeHandle:
    num_recv_tokens_per_expert_list = [3, 1]


class _FakeBuffer:
    def __init__(self):
        self.destroyed = False
        self.calls = []

    def dispatch(self, x, **kw):
        self.calls.append(('dispatch', kw['num_sms'], kw['expert_alignment']))
        return x, None, None, _FakeHandle(), None

    def combine(self, x, handle, num_sms):
        self.calls.append(('combine', num_sms))
        return x * 2, None, None

    def destroy(self):
        self.destroyed = True


class _Group:
    def size(self):
        return 2


@pytest.fixture
def pool(monkeypatch):
    p = sd.BufferPool()
    monkeypatch.setattr(sd.DeepEPB200Normal, 'pool', p)
    monkeypatch.setattr(sd.DeepEPB200Normal, '_make_buffer', lambda self: _FakeBuffer())
    return p


def test_layers_share_one_buffer_and_release_it_last(pool):
    g = _Group()
    a, b = sd.DeepEPB200Normal(g, 64, 8), sd.DeepEPB200Normal(g, 64, 8)
    other = sd.DeepEPB200Normal(g, 128, 8)  # another hidden size: another entry
    assert a.buffer is b.buffer and other.buffer is not a.buffer and len(pool) == 2
    buf = a.buffer
    a.close()
    assert not buf.destroyed and len(pool) == 2
    b.close()
    assert buf.destroyed and len(pool) == 1
    other.close()
    assert len(pool) == 0
    a.close()  # closing twice is a no-op


def test_one_dispatch_in_flight_per_buffer(pool):
    g = _Group()
    a, b = sd.DeepEPB200Normal(g, 64, 8, expert_alignment=128), sd.DeepEPB200Normal(g, 64, 8)
    x = torch.ones(4, 64, dtype=torch.bfloat16)
    out = a._dispatch_core(x, None, None)
    assert out[3] == [3, 1] and a.state is sd._State.DISPATCHED
    with pytest.raises(RuntimeError, match='uncombined dispatch'):
        b._dispatch_core(x, None, None)
    with pytest.raises(RuntimeError, match='dispatched'):
        a._dispatch_core(x, None, None)  # a fresh dispatch before the combine
    with pytest.raises(RuntimeError, match='cannot close'):
        a.close()
    with pytest.raises(TypeError):
        a._combine_core(x.float())
    y, _ = a._combine_core(x)
    assert torch.equal(y, x * 2) and a.state is sd._State.IDLE
    b._dispatch_core(x, None, None)  # the buffer is free again
    b._combine_core(x)
    assert a.buffer.calls == [('dispatch', 64, 128), ('combine', 64), ('dispatch', 64, 1), ('combine', 64)]
    with pytest.raises(RuntimeError, match='idle'):
        b._combine_core(x)  # no dispatch to combine


def test_configuration_checks(pool, monkeypatch):
    g = _Group()
    with pytest.raises(NotImplementedError):
        sd.DeepEPB200Normal(g, 64, 8, async_finish=True)
    monkeypatch.setenv('DEEPEP_B200_SGLANG_SMS', '0')
    with pytest.raises(ValueError):
        sd.DeepEPB200Normal(g, 64, 8)
    monkeypatch.setenv('DEEPEP_B200_SGLANG_SMS', '24')
    monkeypatch.setenv('DEEPEP_B200_SGLANG_MAX_TOKENS', '8')
    d = sd.DeepEPB200Normal(g, 64, 8)
    with pytest.raises(ValueError, match='capacity'):
        d._dispatch_core(torch.ones(9, 64), None, None)
    with pytest.raises(NotImplementedError):
        d._dispatch_core(torch.ones(2, 64), None, None, previous_event=object())
    assert d.state is sd._State.IDLE and len(pool) == 0  # nothing leased by refused calls
