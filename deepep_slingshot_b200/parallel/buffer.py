"""`Buffer`: the expert-parallel communication buffer (the reference's legacy v1 API) on B200.

API parity with [DE]deep_ep/buffers/legacy.py:14-713: constructor arguments, `set_num_sms`,
`capture`, size hints, `get_comm_stream`, `get_local_buffer_tensor`, `get_dispatch_config` /
`get_combine_config`, `get_dispatch_layout`, `dispatch` / `combine` (handles, cached mode,
`num_worst_tokens` for CUDA graphs, `previous_event` / `async_finish` / `allocate_on_comm_stream`),
`clean_low_latency_buffer`, `low_latency_dispatch` / `low_latency_combine` (`return_recv_hook`,
`use_fp8`, `round_scale`, `use_ue8m0`, `zero_copy`, `out`, statistics tensors), the shrink-mode
mask APIs and `get_next_low_latency_combine_buffer`.

Underneath is the C++ runtime `_C.Buffer` with hand-written sm_100a kernels that load and store
directly into peer GPUs' buffers over NVLink 5 / NVSwitch (see csrc/kernels/*.cu). Differences that
a caller can see:
  * one NVLink domain (1..8 ranks). `num_rdma_bytes` sizes the low-latency region (NVLink peer
    stores too); internode RDMA is not available on a single box and raises;
  * `dispatch(..., quantize_fp8=True)` fuses the 1x128 FP8 quantization into the dispatch;
  * the normal-mode region holds a fixed number of tokens per rank per call, derived from
    `num_nvl_bytes` (`Buffer.get_nvl_buffer_size_hint(num_max_tokens, hidden, num_ranks)`).
"""
import functools
import os
from typing import Optional, Tuple, Union

import torch
import torch.distributed as dist

from .._ext import require_ext
from ..utils import lifecycle
from ..utils.event import EventOverlap
from ..utils.runtime_guard import check_nccl_runtime
from ..utils.math import pack_ue8m0

topk_idx_t = torch.int64


def _default_timeout() -> float:
    return float(os.environ.get('DEEPEP_B200_GPU_TIMEOUT_SECS', '100'))


_NVTX = os.environ.get('DEEPEP_B200_NVTX', '0') == '1'


def nvtx_range(name: str):
    """Wrap an API method in an NVTX range named `name` when DEEPEP_B200_NVTX=1 (profiler timelines;
    the reference wraps its API calls the same way, backend/tests/profile_capture.py:11-62)."""
    def deco(fn):
        @functools.wraps(fn)
        def wrapper(*args, **kwargs):
            if not _NVTX:
                return fn(*args, **kwargs)
            torch.cuda.nvtx.range_push(name)
            try:
                return fn(*args, **kwargs)
            finally:
                torch.cuda.nvtx.range_pop()
        return wrapper
    return deco


class Config:
    """Performance config (the reference's `Config`, [DE]csrc/legacy/config.hpp:24-51)."""

    def __init__(self, num_sms: int = 20, num_max_nvl_chunked_send_tokens: int = 6,
                 num_max_nvl_chunked_recv_tokens: int = 256, num_max_rdma_chunked_send_tokens: int = 6,
                 num_max_rdma_chunked_recv_tokens: int = 256) -> None:
        self.num_sms = num_sms
        self.num_max_nvl_chunked_send_tokens = num_max_nvl_chunked_send_tokens
        self.num_max_nvl_chunked_recv_tokens = num_max_nvl_chunked_recv_tokens
        self.num_max_rdma_chunked_send_tokens = num_max_rdma_chunked_send_tokens
        self.num_max_rdma_chunked_recv_tokens = num_max_rdma_chunked_recv_tokens

    def get_nvl_buffer_size_hint(self, hidden_bytes: int, num_ranks: int, num_max_tokens: int = 4096) -> int:
        return require_ext().normal_region_size_for(num_max_tokens, max(hidden_bytes // 2, 128), num_ranks)

    def get_rdma_buffer_size_hint(self, hidden_bytes: int, num_ranks: int) -> int:
        return 0

    def __repr__(self) -> str:
        return f'Config(num_sms={self.num_sms})'


class Buffer:
    """Expert-parallel buffer over one NVLink 5 / NVSwitch domain (see module docstring)."""

    num_sms: int = 64

    def __init__(self, group: Optional[dist.ProcessGroup], num_nvl_bytes: int = 0, num_rdma_bytes: int = 0,
                 low_latency_mode: bool = False, num_qps_per_rank: int = 24,
                 allow_nvlink_for_low_latency_mode: bool = True, allow_mnnvl: bool = False,
                 explicitly_destroy: bool = False, enable_shrink: bool = False, comm=None,
                 num_gpu_timeout_secs: Optional[float] = None) -> None:
        _C = require_ext()
        if group is None:
            raise ValueError('a torch.distributed process group is required')
        check_nccl_runtime()
        used_before = lifecycle.snapshot()
        self.rank = group.rank()
        self.group = group
        self.group_size = group.size()
        self.num_nvl_bytes = num_nvl_bytes
        self.num_rdma_bytes = num_rdma_bytes
        self.low_latency_mode = low_latency_mode
        self.explicitly_destroy = explicitly_destroy
        self.enable_shrink = enable_shrink
        self.num_qps_per_rank = num_qps_per_rank
        timeout = _default_timeout() if num_gpu_timeout_secs is None else num_gpu_timeout_secs
        self.runtime = _C.Buffer(self.rank, self.group_size, num_nvl_bytes, num_rdma_bytes, low_latency_mode,
                                 explicitly_destroy, enable_shrink, timeout)

        def all_gather_object(obj):
            out = [None] * self.group_size
            dist.all_gather_object(out, obj, group)
            return out

        device_ids = all_gather_object(self.runtime.get_local_device_id())
        handles = all_gather_object(bytes(self.runtime.get_local_ipc_handle()))
        ll_local = bytes(self.runtime.get_local_ll_ipc_handle())
        ll_handles = all_gather_object(ll_local if len(ll_local) else None)
        self.runtime.sync(device_ids, handles, ll_handles)
        assert self.runtime.is_available()
        torch.cuda.synchronize()
        dist.barrier(group)
        lifecycle.record('create', 'Buffer', self, num_nvl_bytes + num_rdma_bytes, used_before)

    # ------------------------------------------------------------------ lifecycle / info
    def destroy(self) -> None:
        assert self.explicitly_destroy, '`explicitly_destroy` flag must be set'
        self.runtime.destroy()
        self.runtime = None
        lifecycle.record('destroy', 'Buffer', self)

    @staticmethod
    def is_sm90_compiled() -> bool:
        return False

    @staticmethod
    def is_sm100_compiled() -> bool:
        return True

    @staticmethod
    def set_num_sms(new_num_sms: int) -> None:
        assert new_num_sms % 2 == 0, 'The SM count must be even'
        Buffer.num_sms = new_num_sms

    @staticmethod
    def capture() -> EventOverlap:
        return EventOverlap(require_ext().EventHandle())

    @staticmethod
    def get_low_latency_rdma_size_hint(num_max_dispatch_tokens_per_rank: int, hidden: int, num_ranks: int,
                                       num_experts: int) -> int:
        return require_ext().ll_region_size_for(num_max_dispatch_tokens_per_rank, hidden, num_ranks, num_experts)

    @staticmethod
    def get_nvl_buffer_size_hint(num_max_tokens: int, hidden: int, num_ranks: int) -> int:
        return require_ext().normal_region_size_for(num_max_tokens, hidden, num_ranks)

    def get_comm_stream(self) -> torch.cuda.Stream:
        ts = self.runtime.get_comm_stream()
        return torch.cuda.Stream(stream_id=ts.stream_id, device_index=ts.device_index, device_type=ts.device_type)

    def get_local_buffer_tensor(self, dtype: torch.dtype, size: Optional[torch.Size] = None, offset: int = 0,
                                use_rdma_buffer: bool = False) -> torch.Tensor:
        tensor = self.runtime.get_local_buffer_tensor(dtype, offset, use_rdma_buffer)
        if size is None:
            return tensor
        assert tensor.numel() >= size.numel()
        return tensor[:size.numel()].view(size)

    def get_capacity(self, hidden: int) -> int:
        """Maximum tokens per rank per normal-mode call for this hidden size."""
        return self.runtime.get_capacity(hidden, 8)

    def transport_selftest(self, producer_blocks: int = 64, warps: int = 8, rounds: int = 16) -> Tuple[int, int]:
        """Multi-producer signalling check over NVLink (collective): producer_blocks x warps warps of
        every rank add 1 to the next rank's self-test flag `rounds` times with sys-scope release
        reductions, and every rank waits (bounded by the GPU timeout) for the exact total. Returns
        (status, value seen): status 0 exact, 1 more adds than sent, 2 the wait expired
        (capability of the reference's producer stress test, backend/tests/gin_producer_stress.cu)."""
        status, seen = self.runtime.selftest_signal_stress(producer_blocks, warps, rounds)
        return status, seen

    def check_error(self) -> None:
        """Raise if any kernel of this buffer reported a failed (timed-out) wait or bad index."""
        self.runtime.check_error()

    def get_error_state(self) -> Tuple[int, int, int, int]:
        return self.runtime.get_error_state()

    def clear_error(self) -> None:
        self.runtime.clear_error()

    def get_profile(self) -> dict:
        """Mean device milliseconds per phase (count / count_to_pull / pull / combine) since the last call,
        recorded only when the process runs with DEEPEP_B200_PROFILE=1 (diagnostics; adds events)."""
        return dict(self.runtime.get_profile())

    @nvtx_range('ep.barrier')
    def barrier(self, use_comm_stream: bool = True, with_cpu_sync: bool = False) -> None:
        self.runtime.barrier(use_comm_stream, with_cpu_sync)

    # ------------------------------------------------------------------ device trace ring
    def enable_trace(self, capacity: int = 1 << 20) -> None:
        """Start appending per-block kernel records (40 B each) to a device ring of `capacity`."""
        self.runtime.enable_trace(capacity)

    def disable_trace(self) -> None:
        self.runtime.disable_trace()

    def read_trace(self, reset: bool = True):
        """(decoded records, appended count); see `deepep_slingshot_b200.utils.trace`."""
        from ..utils.trace import decode
        raw, appended = self.runtime.read_trace(reset)
        return decode(raw), appended

    @staticmethod
    def _unpack_bias(bias):
        bias_0, bias_1 = None, None
        if isinstance(bias, torch.Tensor):
            bias_0 = bias
        elif isinstance(bias, tuple):
            assert len(bias) == 2
            bias_0, bias_1 = bias
        return bias_0, bias_1

    @staticmethod
    def get_dispatch_config(num_ranks: int) -> Config:
        assert 1 <= num_ranks <= 8, f'Unsupported number of EP ranks on one NVLink domain: {num_ranks}'
        return Config(Buffer.num_sms, 6, 256, 6, 128)

    @staticmethod
    def get_combine_config(num_ranks: int) -> Config:
        assert 1 <= num_ranks <= 8, f'Unsupported number of EP ranks on one NVLink domain: {num_ranks}'
        return Config(Buffer.num_sms, 4, 256, 6, 128)

    # ------------------------------------------------------------------ normal mode
    @nvtx_range('ep.get_dispatch_layout')
    def get_dispatch_layout(self, topk_idx: torch.Tensor, num_experts: int,
                            previous_event: Optional[EventOverlap] = None, async_finish: bool = False,
                            allocate_on_comm_stream: bool = False):
        """Per-rank / per-expert counts and `is_token_in_rank` (sm_100a kernel)."""
        num_tokens_per_rank, num_tokens_per_rdma_rank, num_tokens_per_expert, is_token_in_rank, event = \
            self.runtime.get_dispatch_layout(topk_idx, num_experts, getattr(previous_event, 'event', None),
                                             async_finish, allocate_on_comm_stream)
        return num_tokens_per_rank, num_tokens_per_rdma_rank, num_tokens_per_expert, is_token_in_rank, \
            EventOverlap(event)

    @nvtx_range('ep.dispatch')
    def dispatch(self, x: Union[torch.Tensor, Tuple[torch.Tensor, torch.Tensor]], handle: Optional[Tuple] = None,
                 num_tokens_per_rank: Optional[torch.Tensor] = None,
                 num_tokens_per_rdma_rank: Optional[torch.Tensor] = None,
                 is_token_in_rank: Optional[torch.Tensor] = None,
                 num_tokens_per_expert: Optional[torch.Tensor] = None,
                 topk_idx: Optional[torch.Tensor] = None, topk_weights: Optional[torch.Tensor] = None,
                 expert_alignment: int = 1, num_worst_tokens: int = 0, config: Optional[Config] = None,
                 previous_event: Optional[EventOverlap] = None, async_finish: bool = False,
                 allocate_on_comm_stream: bool = False, num_experts: Optional[int] = None,
                 quantize_fp8: bool = False, round_scale: bool = False, scales_col_major: bool = False):
        """Dispatch tokens to the ranks that own their experts.

        Returns `(recv_x | (recv_x_fp8, recv_scales), recv_topk_idx, recv_topk_weights,
        num_recv_tokens_per_expert_list, handle, event)`. Received rows are grouped by source rank and
        ordered by source token. `recv_topk_idx` holds local expert ids (-1 for experts of other ranks).
        With `num_worst_tokens > 0` there is no CPU sync (CUDA-graph compatible) and the list is empty.
        `quantize_fp8=True` quantizes bf16 `x` to FP8 e4m3 with 1x128 fp32 scales inside the dispatch.
        Handle: (rank_prefix_matrix, send_prefix_matrix, recv_rank_prefix, recv_src_idx,
        is_token_in_rank, send_head).
        """
        config = self.get_dispatch_config(self.group_size) if config is None else config
        x, x_scales = x if isinstance(x, tuple) else (x, None)
        prev = getattr(previous_event, 'event', None)
        if handle is not None:
            assert topk_idx is None and topk_weights is None
            rank_prefix_matrix, send_prefix_matrix, recv_rank_prefix, recv_src_idx, is_token_in_rank, send_head = handle
            out = self.runtime.intranode_dispatch(
                x, x_scales, None, None, None, 0, rank_prefix_matrix, send_prefix_matrix, recv_src_idx, send_head,
                expert_alignment, 0, quantize_fp8, round_scale, scales_col_major, None, config.num_sms, prev,
                async_finish, allocate_on_comm_stream)
            recv_x, recv_scales, event = out[0], out[1], out[11]
            return (recv_x, recv_scales) if recv_scales is not None else recv_x, None, None, None, None, \
                EventOverlap(event)
        if num_experts is None:
            assert num_tokens_per_expert is not None, 'pass num_tokens_per_expert (or num_experts)'
            num_experts = num_tokens_per_expert.numel()
        (recv_x, recv_scales, recv_topk_idx, recv_topk_weights, num_recv_tokens_per_expert_list, rank_prefix_matrix,
         send_prefix_matrix, recv_rank_prefix, recv_src_idx, send_head, _, event) = self.runtime.intranode_dispatch(
            x, x_scales, topk_idx, topk_weights, is_token_in_rank, num_experts, None, None, None, None,
            expert_alignment, num_worst_tokens, quantize_fp8, round_scale, scales_col_major, None, config.num_sms,
            prev, async_finish, allocate_on_comm_stream)
        if is_token_in_rank is None:
            if async_finish:
                # Nothing waited for the comm stream (no CPU sync with num_worst_tokens): derive the mask
                # there, after the kernels that write send_head, and return an event that covers it.
                comm = self.get_comm_stream()
                with torch.cuda.stream(comm):
                    is_token_in_rank = send_head >= 0
                    event = require_ext().EventHandle()
                is_token_in_rank.record_stream(torch.cuda.current_stream())
            else:
                is_token_in_rank = send_head >= 0
        handle = (rank_prefix_matrix, send_prefix_matrix, recv_rank_prefix, recv_src_idx, is_token_in_rank, send_head)
        return (recv_x, recv_scales) if recv_scales is not None else recv_x, recv_topk_idx, recv_topk_weights, \
            num_recv_tokens_per_expert_list, handle, EventOverlap(event)

    @nvtx_range('ep.dispatch_gemm')
    def dispatch_gemm(self, x: torch.Tensor, topk_idx: torch.Tensor, topk_weights: torch.Tensor, num_experts: int,
                      weights: torch.Tensor, weight_scales: torch.Tensor, round_scale: bool = False, num_sms: int = 0,
                      pull_ctas: int = 0):
        """FP8 dispatch whose receive feeds the gate/up grouped GEMM in the same launch.

        The stage and notify steps are `dispatch(..., quantize_fp8=True, expert_alignment=128)`'s.
        Then one persistent kernel pulls every received token, writes it once per local expert it
        selected into an expert-grouped, 128-aligned FP8 operand, and runs the grouped FP8 GEMM with
        `weights [E_local, n, hidden]` (e4m3, 128x128 `weight_scales`) tile by tile as the rows land;
        `pull_ctas` CTAs pull first and then join the GEMM (default: 32).

        Returns `(h, grouped, handle)`: `h [rows, n]` bf16 (rows of expert e at
        `grouped['expert_offsets'][e]`, valid for the first `grouped['expert_counts'][e]` of them),
        `grouped` with `x` / `scales` (the FP8 operand and its 1x128 scales), `row_map [num_recv, K]`
        (operand row of (received token, k), -1 if not local), `topk_weights [num_recv, K]` (local),
        `expert_offsets`, `expert_counts` and the aligned `num_recv_tokens_per_expert_list`; `handle`
        is the one `combine` takes.
        """
        (h, a, a_scales, row_map, recv_w, offsets, counts, recv_src_idx, per_expert, rank_prefix_matrix,
         send_prefix_matrix, recv_rank_prefix, send_head) = self.runtime.intranode_dispatch_gemm(
            x, topk_idx, topk_weights, num_experts, weights, weight_scales, round_scale, num_sms, pull_ctas)
        handle = (rank_prefix_matrix, send_prefix_matrix, recv_rank_prefix, recv_src_idx, send_head >= 0, send_head)
        grouped = {'x': a, 'scales': a_scales, 'row_map': row_map, 'topk_weights': recv_w, 'expert_offsets': offsets,
                   'expert_counts': counts, 'num_recv_tokens_per_expert_list': per_expert}
        return h, grouped, handle

    @nvtx_range('ep.combine')
    def combine(self, x: torch.Tensor, handle: Tuple, topk_weights: Optional[torch.Tensor] = None,
                bias: Union[torch.Tensor, Tuple[torch.Tensor, torch.Tensor], None] = None,
                config: Optional[Config] = None, previous_event: Optional[EventOverlap] = None,
                async_finish: bool = False, allocate_on_comm_stream: bool = False,
                row_map: Optional[torch.Tensor] = None, row_weights: Optional[torch.Tensor] = None):
        """Sum (without weights) every rank's row of each token back on its source rank (+ bias);
        also returns the summed top-k weights. Returns `(combined_x, combined_topk_weights, event)`
        ([DE]deep_ep/buffers/legacy.py:408-455).

        Weighted expanded mode (this library's addition, the MoE layer's combine): with `row_map`
        (int32 [num_recv, K], the grouped row of each (received token, top-k slot) or -1, as `permute`
        returns it) `x` is the expert-grouped output with one row per (received token, local expert).
        Each rank first reduces a token's local rows in fp32 with the factors `row_weights` (fp32
        [num_recv, K], typically the received top-k weights; None sums them), casts to bf16 and pushes
        that one row; the source rank then sums the ranks' rows in fp32 (+ bias) and casts to bf16.
        The top-k weighted reduction, the bf16 casts and the exchange are one kernel; no unpermute pass
        runs and only one row per (token, rank) crosses NVLink."""
        config = self.get_combine_config(self.group_size) if config is None else config
        rank_prefix_matrix, send_prefix_matrix, _, recv_src_idx, _, send_head = handle
        bias_0, bias_1 = Buffer._unpack_bias(bias)
        recv_x, recv_topk_weights, event = self.runtime.intranode_combine(
            x, topk_weights, bias_0, bias_1, rank_prefix_matrix, send_prefix_matrix, send_head, recv_src_idx, config.num_sms,
            getattr(previous_event, 'event', None), async_finish, allocate_on_comm_stream, row_map, row_weights)
        return recv_x, recv_topk_weights, EventOverlap(event)

    def internode_dispatch(self, *args, **kwargs):
        raise NotImplementedError('internode (RDMA) dispatch needs a multi-node fabric; one B200 box is one NVLink domain')

    def internode_combine(self, *args, **kwargs):
        raise NotImplementedError('internode (RDMA) combine needs a multi-node fabric; one B200 box is one NVLink domain')

    # ------------------------------------------------------------------ low-latency mode
    def clean_low_latency_buffer(self, num_max_dispatch_tokens_per_rank: int, hidden: int, num_experts: int) -> None:
        self.runtime.clean_low_latency_buffer(num_max_dispatch_tokens_per_rank, hidden, num_experts)

    @nvtx_range('ep.low_latency_dispatch')
    def low_latency_dispatch(self, x: torch.Tensor, topk_idx: torch.Tensor, num_max_dispatch_tokens_per_rank: int,
                             num_experts: int, cumulative_local_expert_recv_stats: Optional[torch.Tensor] = None,
                             dispatch_wait_recv_cost_stats: Optional[torch.Tensor] = None, use_fp8: bool = True,
                             round_scale: bool = False, use_ue8m0: bool = False, async_finish: bool = False,
                             return_recv_hook: bool = False):
        """Low-latency dispatch into a per-expert padded layout `[E_local, R * max_tokens, hidden]`.

        Valid rows of local expert e are `[0, recv_count[e])`. The returned tensors are views of the
        registered buffer (two halves alternate): at most two results may be alive at once. With
        `return_recv_hook=True` only the send phase runs; call the hook before using the results.
        """
        (recv_x, recv_scales, recv_count, src_info, src_meta, layout_range, half, event,
         hook) = self.runtime.low_latency_dispatch(x, topk_idx, cumulative_local_expert_recv_stats,
                                                   dispatch_wait_recv_cost_stats, num_max_dispatch_tokens_per_rank,
                                                   num_experts, use_fp8, round_scale, use_ue8m0, async_finish,
                                                   return_recv_hook)
        handle = (src_info, layout_range, num_max_dispatch_tokens_per_rank, x.size(1), num_experts, recv_count, half,
                  src_meta)
        if use_fp8 and use_ue8m0:
            # Packed UE8M0 scales [E_local, slots, hidden/512] int32, column-major in the last two dims.
            e_l, slots, nb = recv_scales.shape
            packed = torch.empty((e_l, nb // 4, slots), dtype=torch.int32, device=x.device).transpose(1, 2)

            def _fill():
                packed.copy_(pack_ue8m0(recv_scales.contiguous()))

            if hook is not None:
                raw_hook = hook

                def hook():
                    raw_hook()
                    _fill()
            elif async_finish:
                # The dispatch ran on the comm stream and nothing waited for it: pack there, after it,
                # and hand back an event that also covers the packing.
                comm = self.get_comm_stream()
                packed.record_stream(comm)
                with torch.cuda.stream(comm):
                    _fill()
                    event = require_ext().EventHandle()  # recorded on the comm stream, after the packing
            else:
                _fill()
            recv = (recv_x, packed)
        else:
            recv = (recv_x, recv_scales) if use_fp8 else recv_x
        tensors_to_record = (x, topk_idx, recv_x, recv_scales, recv_count, src_info, layout_range,
                             cumulative_local_expert_recv_stats)
        return recv, recv_count, handle, EventOverlap(event, tensors_to_record if async_finish else None), hook

    @nvtx_range('ep.low_latency_dispatch_gemm')
    def low_latency_dispatch_gemm(self, x: torch.Tensor, topk_idx: torch.Tensor, num_max_dispatch_tokens_per_rank: int,
                                  num_experts: int, weights: torch.Tensor, weight_scales: torch.Tensor,
                                  cumulative_local_expert_recv_stats: Optional[torch.Tensor] = None,
                                  round_scale: bool = False, num_sms: int = 0):
        """FP8 low-latency dispatch straight into the first expert GEMM.

        The send phase is `low_latency_dispatch(..., use_fp8=True, return_recv_hook=True)`; instead of
        the hook, one masked grouped FP8 GEMM kernel (tcgen05) prefetches `weights` into L2 while the
        tokens cross NVLink, waits for every rank, takes the per-expert counts and computes
        `out[e, m] = x_e[m] @ weights[e]^T` for the received rows. `weights [E_local, n, hidden]` e4m3 with
        128x128 scales `weight_scales [E_local, n/128, hidden/128]` (`ops.gemm.quantize_weights_fp8`).

        Returns `(out [E_local, R * max_tokens, n] bf16 (rows < recv_count[e] valid), recv_count, handle,
        (recv_x, recv_scales))`; the handle is the one `low_latency_combine` takes (its layout range is
        not computed). Not available in shrink mode.
        """
        out, recv_x, recv_scales, recv_count, src_info, src_meta, half = self.runtime.low_latency_dispatch_gemm(
            x, topk_idx, cumulative_local_expert_recv_stats, num_max_dispatch_tokens_per_rank, num_experts, weights,
            weight_scales, round_scale, num_sms)
        handle = (src_info, None, num_max_dispatch_tokens_per_rank, x.size(1), num_experts, recv_count, half, src_meta)
        return out, recv_count, handle, (recv_x, recv_scales)

    @nvtx_range('ep.low_latency_gemm_combine')
    def low_latency_gemm_combine(self, x: torch.Tensor, x_scales: torch.Tensor, weights: torch.Tensor,
                                 weight_scales: torch.Tensor, topk_idx: torch.Tensor, topk_weights: torch.Tensor,
                                 handle: tuple, num_sms: int = 0) -> torch.Tensor:
        """Down projection and low-latency combine in two launches: a masked grouped FP8 GEMM over the
        dispatch's per-expert layout (`x [E_local, R * max_tokens, k]` e4m3 with 1x128 `x_scales`,
        `weights [E_local, hidden, k]` e4m3 with 128x128 `weight_scales`) whose epilogue stores each
        output row straight into its source rank's combine slot over NVLink, then the combine's
        receive (top-k weighted reduction). Returns the combined `[num_tokens, hidden]` bf16. `handle`
        is the dispatch's (`low_latency_dispatch` or `low_latency_dispatch_gemm`). Not available in
        shrink mode."""
        src_info, _, num_max_dispatch_tokens_per_rank, hidden, num_experts, recv_count, half, _ = handle
        return self.runtime.low_latency_gemm_combine(x, x_scales, recv_count, weights, weight_scales, topk_idx, topk_weights,
                                                     half, num_max_dispatch_tokens_per_rank, num_experts, num_sms)

    @nvtx_range('ep.low_latency_combine')
    def low_latency_combine(self, x: torch.Tensor, topk_idx: torch.Tensor, topk_weights: torch.Tensor, handle: tuple,
                            use_logfmt: bool = False, zero_copy: bool = False, async_finish: bool = False,
                            return_recv_hook: bool = False, out: Optional[torch.Tensor] = None,
                            combine_wait_recv_cost_stats: Optional[torch.Tensor] = None):
        """Low-latency combine: top-k WEIGHTED reduction back on the source rank (bf16 output)."""
        src_info, layout_range, num_max_dispatch_tokens_per_rank, hidden, num_experts, recv_count, half, _ = handle
        combined_x, event, hook = self.runtime.low_latency_combine(
            x, topk_idx, topk_weights, recv_count, half, combine_wait_recv_cost_stats, num_max_dispatch_tokens_per_rank,
            num_experts, use_logfmt, zero_copy, async_finish, return_recv_hook, out)
        tensors_to_record = (x, topk_idx, topk_weights, src_info, layout_range, combined_x)
        return combined_x, EventOverlap(event, tensors_to_record if async_finish else None), hook

    def low_latency_update_mask_buffer(self, rank_to_mask: int, mask: bool = False) -> None:
        self.runtime.low_latency_update_mask_buffer(rank_to_mask, mask)

    def low_latency_query_mask_buffer(self, mask_status: torch.Tensor) -> None:
        self.runtime.low_latency_query_mask_buffer(mask_status)

    def low_latency_clean_mask_buffer(self) -> None:
        self.runtime.low_latency_clean_mask_buffer()

    def get_next_low_latency_combine_buffer(self, handle: object) -> torch.Tensor:
        src_info, layout_range, num_max_dispatch_tokens_per_rank, hidden, num_experts = handle[:5]
        return self.runtime.get_next_low_latency_combine_buffer(num_max_dispatch_tokens_per_rank, hidden, num_experts)
