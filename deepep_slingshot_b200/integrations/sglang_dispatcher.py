"""Normal-mode token dispatcher for an SGLang-style MoE runner, backed by `ElasticBuffer`.

Capability parity with the reference's opt-in SGLang adapter (backend/sglang/deepep_v2_cxi.py:24-146):
SGLang's `_DeepEPDispatcherImplNormal` calls `_dispatch_core`, `_combine_core` and `close`, and the
expert runner applies the routing weights itself, so the combine is an unweighted sum.

Design here: every MoE layer of a model builds its own dispatcher, but the layers of one process
run one after another, so they share the symmetric buffer of their configuration. `BufferPool`
owns those buffers. A dispatcher takes a `Lease` on its configuration's entry when it first
dispatches and gives it back in `close()`; the entry's buffer is destroyed when its last lease is
returned. Each entry also records which lease has a dispatch in flight (between a fresh dispatch and
its combine), because the buffer's receive state belongs to that dispatch until the combine; any
other layer that dispatches on the entry meanwhile is refused. A dispatcher moves through the
states IDLE -> DISPATCHED -> IDLE and ends in CLOSED.

When SGLang is importable, `make_sglang_dispatcher_class` builds a subclass of its
`_DeepEPDispatcherImplNormal` that forwards to `DeepEPB200Normal`; without SGLang the standalone
object offers the same three methods.

Environment knobs: DEEPEP_B200_SGLANG_MAX_TOKENS (token capacity per rank, default 4096) and
DEEPEP_B200_SGLANG_SMS (SMs for dispatch/combine, default 64).
"""
import enum
import functools
import logging
import os
from dataclasses import dataclass, field
from typing import Dict, Hashable, Optional, Set

import torch
import torch.distributed as dist

logger = logging.getLogger(__name__)


@dataclass
class _PoolEntry:
    buffer: object
    leases: Set[int] = field(default_factory=set)
    in_flight: Optional[int] = None  # id of the lease whose dispatch is not combined yet


@dataclass(frozen=True)
class Lease:
    """A dispatcher's claim on one pool entry; `key` names the entry, `ident` the holder."""
    key: Hashable
    ident: int


class BufferPool:
    """Symmetric buffers shared by every dispatcher of one (group, hidden, capacity) configuration."""

    def __init__(self) -> None:
        self._entries: Dict[Hashable, _PoolEntry] = {}
        self._next_ident = 0

    def __len__(self) -> int:
        return len(self._entries)

    def lease(self, key: Hashable, make_buffer) -> Lease:
        entry = self._entries.get(key)
        if entry is None:
            entry = self._entries[key] = _PoolEntry(make_buffer())
        self._next_ident += 1
        entry.leases.add(self._next_ident)
        return Lease(key, self._next_ident)

    def buffer(self, lease: Lease):
        return self._entries[lease.key].buffer

    def begin_dispatch(self, lease: Lease) -> None:
        entry = self._entries[lease.key]
        if entry.in_flight is not None:
            raise RuntimeError('another layer has an uncombined dispatch on this shared buffer')
        entry.in_flight = lease.ident

    def end_dispatch(self, lease: Lease) -> None:
        entry = self._entries[lease.key]
        if entry.in_flight != lease.ident:
            raise RuntimeError('this layer has no dispatch in flight on its shared buffer')
        entry.in_flight = None

    def give_back(self, lease: Lease) -> None:
        entry = self._entries[lease.key]
        if entry.in_flight == lease.ident:
            raise RuntimeError('a lease cannot be returned while its dispatch is in flight')
        entry.leases.discard(lease.ident)
        if not entry.leases:
            del self._entries[lease.key]
            entry.buffer.destroy()


class _State(enum.Enum):
    IDLE = 'idle'
    DISPATCHED = 'dispatched'
    CLOSED = 'closed'


class DeepEPB200Normal:
    """Synchronous normal-mode dispatch / combine on a pooled `ElasticBuffer`."""

    pool = BufferPool()

    def __init__(self, group: dist.ProcessGroup, hidden_size: int, num_experts: int, expert_alignment: int = 1,
                 scales_col_major_ue8m0: bool = False, async_finish: bool = False):
        if async_finish:
            raise NotImplementedError('this adapter runs dispatch and combine synchronously')
        self.group = group
        self.hidden_size = hidden_size
        self.num_experts = num_experts
        self.expert_alignment = expert_alignment
        self.scales_col_major_ue8m0 = scales_col_major_ue8m0
        self.capacity = int(os.getenv('DEEPEP_B200_SGLANG_MAX_TOKENS', '4096'))
        self.num_sms = int(os.getenv('DEEPEP_B200_SGLANG_SMS', '64'))
        if self.capacity <= 0 or self.num_sms <= 0:
            raise ValueError(f'capacity ({self.capacity}) and SM count ({self.num_sms}) must be positive')
        self.state = _State.IDLE
        self.handle = None
        self._lease: Optional[Lease] = None

    @property
    def buffer(self):
        """The pooled `ElasticBuffer` of this configuration (leased on first use)."""
        if self._lease is None:
            key = (id(self.group), self.hidden_size, self.capacity)
            self._lease = self.pool.lease(key, self._make_buffer)
        return self.pool.buffer(self._lease)

    def _make_buffer(self):
        from ..parallel.elastic import ElasticBuffer
        logger.info('DeepEP B200 adapter: new shared buffer, group of %d, capacity %d, %d SMs',
                    self.group.size(), self.capacity, self.num_sms)
        return ElasticBuffer(self.group, num_max_tokens_per_rank=self.capacity, hidden=self.hidden_size,
                             allow_hybrid_mode=True, allow_multiple_reduction=True, prefer_overlap_with_compute=False,
                             num_cpu_timeout_secs=120, num_gpu_timeout_secs=60, explicitly_destroy=True)

    def _expect(self, state: _State, action: str) -> None:
        if self.state is not state:
            raise RuntimeError(f'cannot {action}: the dispatcher is {self.state.value}, not {state.value}')

    def _dispatch_core(self, x, topk_ids: torch.Tensor, topk_weights: torch.Tensor, previous_event=None):
        """x: bf16 `[T, hidden]` or an FP8 `(values, scales)` pair. Returns the received tokens, their
        local expert ids and weights, the per-expert received counts (aligned) and the event."""
        if previous_event is not None:
            raise NotImplementedError('this adapter does not take a previous event')
        self._expect(_State.IDLE, 'dispatch')
        rows = (x[0] if isinstance(x, tuple) else x).shape[0]
        if rows > self.capacity:
            raise ValueError(f'{rows} tokens exceed the adapter capacity of {self.capacity}')
        buffer = self.buffer
        # If the dispatch raises, the entry stays marked busy: the buffer's state after a failed
        # dispatch is unknown, so no other layer may use it (recovery needs a new process group).
        self.pool.begin_dispatch(self._lease)
        received, ids, weights, handle, event = buffer.dispatch(
            x, topk_idx=topk_ids, topk_weights=topk_weights, num_experts=self.num_experts,
            num_max_tokens_per_rank=self.capacity, expert_alignment=self.expert_alignment,
            num_sms=self.num_sms, do_cpu_sync=True, do_expand=False,
            use_tma_aligned_col_major_sf=self.scales_col_major_ue8m0)
        self.handle = handle
        self.state = _State.DISPATCHED
        return received, ids, weights, handle.num_recv_tokens_per_expert_list, event

    def _combine_core(self, x: torch.Tensor, previous_event=None):
        """Unweighted sum of the expert outputs (the runner already applied the routing weights)."""
        if previous_event is not None:
            raise NotImplementedError('this adapter does not take a previous event')
        self._expect(_State.DISPATCHED, 'combine')
        if x.dtype != torch.bfloat16:
            raise TypeError(f'combine expects bf16 expert outputs, got {x.dtype}')
        combined, _, event = self.buffer.combine(x, self.handle, num_sms=self.num_sms)
        self.handle = None
        self.pool.end_dispatch(self._lease)
        self.state = _State.IDLE
        return combined, event

    def close(self) -> None:
        if self.state is _State.CLOSED:
            return
        self._expect(_State.IDLE, 'close')
        if self._lease is not None:
            self.pool.give_back(self._lease)
            self._lease = None
        self.state = _State.CLOSED


@functools.lru_cache(maxsize=None)
def make_sglang_dispatcher_class():
    """Subclass of SGLang's `_DeepEPDispatcherImplNormal` using this library (needs SGLang); one
    class per process, so every layer's dispatcher has the same type."""
    from sglang.srt.layers.moe.token_dispatcher.deepep import _DeepEPDispatcherImplNormal  # noqa: F401

    class DeepEPB200SGLangNormal(_DeepEPDispatcherImplNormal):
        def __init__(self, async_finish=False, **kwargs):
            super().__init__(async_finish=False, **kwargs)
            self._impl = DeepEPB200Normal(self.group, self.hidden_size, self.num_experts,
                                          expert_alignment=128, async_finish=async_finish)

        def _dispatch_core(self, x, topk_ids, topk_weights, previous_event):
            return self._impl._dispatch_core(x, topk_ids, topk_weights, previous_event)

        def _combine_core(self, x, previous_event):
            return self._impl._combine_core(x, previous_event)

    return DeepEPB200SGLangNormal
