"""Normal-mode token dispatcher for an SGLang-style MoE runner, backed by `ElasticBuffer`.

The reference ships an opt-in SGLang adapter (backend/sglang/deepep_v2_cxi.py:24-146) that swaps the
normal-mode DeepEP dispatcher for a v2 `ElasticBuffer` one: synchronous only, a fixed token capacity
(>= 4096), one shared buffer per (group, hidden, capacity) across layers, one live dispatch per
buffer, routing weights applied by the expert runner (so combine is an unweighted sum). This module
keeps that contract for one NVLink domain. When SGLang is importable, `make_sglang_dispatcher_class`
builds a subclass of its `_DeepEPDispatcherImplNormal`; without SGLang, `DeepEPB200Normal` is a
standalone object with the same `_dispatch_core` / `_combine_core` / `close` methods.

Environment knobs: DEEPEP_B200_SGLANG_MAX_TOKENS (capacity, default 4096),
DEEPEP_B200_SGLANG_SMS (SMs for dispatch/combine, default 64).
"""
import functools
import logging
import os
from typing import Dict, Optional

import torch
import torch.distributed as dist

logger = logging.getLogger(__name__)


class DeepEPB200Normal:
    """Synchronous normal-mode dispatch/combine with a shared `ElasticBuffer` per configuration."""

    _buffers: Dict[tuple, dict] = {}

    def __init__(self, group: dist.ProcessGroup, hidden_size: int, num_experts: int, expert_alignment: int = 1,
                 scales_col_major_ue8m0: bool = False, async_finish: bool = False):
        if async_finish:
            raise NotImplementedError('the B200 normal-mode adapter is synchronous (no async overlap)')
        self.group = group
        self.hidden_size = hidden_size
        self.num_experts = num_experts
        self.expert_alignment = expert_alignment
        self.scales_col_major_ue8m0 = scales_col_major_ue8m0
        self.handle = None
        self._elastic = None
        self._buffer_key: Optional[tuple] = None
        self._capacity = int(os.getenv('DEEPEP_B200_SGLANG_MAX_TOKENS', '4096'))
        self._sms = int(os.getenv('DEEPEP_B200_SGLANG_SMS', '64'))
        if self._capacity < 4096 or self._sms <= 0 or self._sms % 2:
            raise ValueError('invalid adapter capacity / SM configuration')

    def _get_buffer(self):
        from ..parallel.elastic import ElasticBuffer
        if self._elastic is not None:
            return self._elastic
        key = (id(self.group), self.hidden_size, self._capacity)
        cached = self._buffers.get(key)
        if cached is not None:
            cached['references'] += 1
        else:
            buf = ElasticBuffer(self.group, num_max_tokens_per_rank=self._capacity, hidden=self.hidden_size,
                                allow_hybrid_mode=True, allow_multiple_reduction=True, prefer_overlap_with_compute=False,
                                num_cpu_timeout_secs=120, num_gpu_timeout_secs=60, explicitly_destroy=True)
            cached = {'buffer': buf, 'references': 1, 'owner': None}
            self._buffers[key] = cached
            logger.info('DeepEP B200 adapter: group=%d capacity=%d SMs=%d', self.group.size(), self._capacity, self._sms)
        self._elastic = cached['buffer']
        self._buffer_key = key
        return self._elastic

    def _dispatch_core(self, x, topk_ids: torch.Tensor, topk_weights: torch.Tensor, previous_event=None):
        """x: bf16 `[T, hidden]` or an FP8 `(values, scales)` pair. Returns (received, local expert ids,
        weights, per-expert received counts (aligned), event)."""
        if previous_event is not None:
            raise NotImplementedError('async event translation is not supported')
        if self.handle is not None:
            raise RuntimeError('the previous dispatch must be combined before a fresh dispatch')
        tensor = x[0] if isinstance(x, tuple) else x
        if tensor.shape[0] > self._capacity:
            raise ValueError('input exceeds the allocated token capacity')
        buffer = self._get_buffer()
        state = self._buffers[self._buffer_key]
        if state['owner'] is not None:
            raise RuntimeError('overlapping dispatches on one shared buffer are not supported')
        state['owner'] = self  # kept on failure: recovery needs a new process group
        received, ids, weights, handle, event = buffer.dispatch(
            x, topk_idx=topk_ids, topk_weights=topk_weights, num_experts=self.num_experts,
            num_max_tokens_per_rank=self._capacity, expert_alignment=self.expert_alignment, num_sms=self._sms,
            do_cpu_sync=True, do_expand=False, use_tma_aligned_col_major_sf=self.scales_col_major_ue8m0)
        self.handle = handle
        return received, ids, weights, handle.num_recv_tokens_per_expert_list, event

    def _combine_core(self, x: torch.Tensor, previous_event=None):
        """Unweighted sum of the expert outputs (the runner already applied the routing weights)."""
        if previous_event is not None or self.handle is None:
            raise RuntimeError('expected the live handle of a synchronous fresh dispatch')
        if x.dtype != torch.bfloat16:
            raise TypeError('combine expects bf16 expert outputs')
        combined, _, event = self._get_buffer().combine(x, self.handle, num_sms=self._sms)
        self.handle = None
        self._buffers[self._buffer_key]['owner'] = None
        return combined, event

    def close(self) -> None:
        if self.handle is not None:
            raise RuntimeError('cannot close the adapter with an uncombined dispatch')
        if self._elastic is None:
            return
        state = self._buffers[self._buffer_key]
        if state['owner'] is not None:
            raise RuntimeError('cannot destroy shared storage during a live dispatch')
        state['references'] -= 1
        if state['references'] == 0:
            state['buffer'].destroy()
            del self._buffers[self._buffer_key]
        self._elastic = None
        self._buffer_key = None


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
