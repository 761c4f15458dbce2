"""`ElasticBuffer` / `EPHandle`: the reference's v2 API ([DE]deep_ep/buffers/elastic.py:24-928) on B200.

One NVLink domain: the logical and physical domains are (1 scale-out rank, R scale-up ranks); the
hybrid (RDMA + NVLink) mode, QPs and service levels are accepted and have no effect. Dispatch and
combine run on the same sm_100a NVLink kernels as `Buffer` (pull-dispatch from the sources' staging,
push-combine + fp32 reduce), with the layout computed inside the dispatch (no separate layout call).
"""
import math
import os
from contextlib import contextmanager
from typing import Optional, Tuple, Union

import torch
import torch.distributed as dist

from .._ext import require_ext
from ..utils.event import EventOverlap
from ..utils.envs import get_nvlink_gbs
from ..utils.math import align
from ..ops.permute import permute
from .buffer import Buffer, nvtx_range


def _native_event(previous_event):
    """The native event of `previous_event` (an `EventOverlap`, as dispatch / combine return, or the
    native event itself), or None."""
    return getattr(previous_event, 'event', previous_event)


@contextmanager
def _no_stream_change():
    yield


def _record_on_current_stream(*objs) -> None:
    """`record_stream` every tensor reachable from `objs` (tuples, lists, EPHandle attributes) on the
    current stream: they were allocated on the comm stream and are used on this one."""
    cur = torch.cuda.current_stream()
    seen = set()

    def walk(o):
        if isinstance(o, torch.Tensor):
            if id(o) not in seen:
                seen.add(id(o))
                o.record_stream(cur)
        elif isinstance(o, (tuple, list)):
            for x in o:
                walk(x)
        elif isinstance(o, EPHandle):
            for x in vars(o).values():
                walk(x)

    for o in objs:
        walk(o)


class EPHandle:
    """Routing state returned by `ElasticBuffer.dispatch`, reusable as a cached handle and consumed by
    `combine` (fields follow [DE]deep_ep/buffers/elastic.py:24-87)."""

    def __init__(self, do_expand: bool, num_experts: int, expert_alignment: int, num_max_tokens_per_rank: int,
                 num_sms: int, topk_idx: torch.Tensor, num_recv_tokens_per_expert_list: list,
                 psum_num_recv_tokens_per_scaleup_rank: torch.Tensor, psum_num_recv_tokens_per_expert: torch.Tensor,
                 recv_src_metadata: torch.Tensor, legacy_handle: tuple):
        self.do_expand = do_expand
        self.num_experts = num_experts
        self.expert_alignment = expert_alignment
        self.num_max_tokens_per_rank = num_max_tokens_per_rank
        self.num_sms = num_sms
        self.topk_idx = topk_idx
        self.num_recv_tokens_per_expert_list = num_recv_tokens_per_expert_list
        self.psum_num_recv_tokens_per_scaleup_rank = psum_num_recv_tokens_per_scaleup_rank
        self.psum_num_recv_tokens_per_expert = psum_num_recv_tokens_per_expert
        self.recv_src_metadata = recv_src_metadata
        self.dst_buffer_slot_idx = legacy_handle[5]
        self.token_metadata_at_forward = None
        self.channel_linked_list = None
        self.legacy_handle = legacy_handle
        self.num_recv_tokens = recv_src_metadata.shape[0]


class ElasticBuffer:
    """Elastic EP buffer (v2 API) over one NVLink 5 / NVSwitch domain."""

    def __init__(self, group: dist.ProcessGroup, num_bytes: Optional[int] = None, num_cpu_bytes: int = 0,
                 num_max_tokens_per_rank: int = 0, hidden: int = 0, num_topk: int = 0, use_fp8_dispatch: bool = False,
                 deterministic: bool = False, allow_hybrid_mode: bool = True, allow_multiple_reduction: bool = True,
                 prefer_overlap_with_compute: bool = True, sl_idx: int = 3, num_allocated_qps: int = 0,
                 num_cpu_timeout_secs: int = 300, num_gpu_timeout_secs: int = 100,
                 explicitly_destroy: bool = False) -> None:
        _C = require_ext()
        self.group = group
        self.rank_idx = group.rank()
        self.num_ranks = group.size()
        self.allow_hybrid_mode = allow_hybrid_mode
        self.allow_multiple_reduction = allow_multiple_reduction
        self.prefer_overlap_with_compute = prefer_overlap_with_compute
        self.deterministic = deterministic
        if num_bytes is None:
            num_bytes = self.get_buffer_size_hint(group, num_max_tokens_per_rank, hidden, num_topk, use_fp8_dispatch)
        if os.environ.get('EP_BUFFER_DEBUG', 0):
            print(f'Initializing EP elastic buffer with {num_bytes} bytes at rank {self.rank_idx}/{self.num_ranks}')
        self.num_bytes = num_bytes
        self.num_max_tokens_per_rank = num_max_tokens_per_rank
        self.num_allocated_qps = num_allocated_qps or 17
        self.explicitly_destroy = explicitly_destroy
        self._buffer = Buffer(group, num_nvl_bytes=num_bytes, num_rdma_bytes=0, explicitly_destroy=explicitly_destroy,
                              num_gpu_timeout_secs=num_gpu_timeout_secs)
        # Hybrid CPU memory: one shared host segment per rank, mapped by every rank (Engram storage).
        self.num_cpu_bytes = int(num_cpu_bytes) if allow_hybrid_mode else 0
        self.num_gpu_timeout_secs = num_gpu_timeout_secs
        self._host = None
        if self.num_cpu_bytes > 0:
            if self.num_cpu_bytes % self.get_elastic_buffer_alignment():
                raise ValueError('num_cpu_bytes must be a multiple of get_elastic_buffer_alignment() (2 MiB)')
            from .host_memory import HostSegments
            self._host = HostSegments(group, self.num_cpu_bytes)
        self.runtime = self._buffer.runtime
        self.num_scaleout_ranks, self.num_scaleup_ranks = 1, self.num_ranks
        self.scaleout_rank_idx, self.scaleup_rank_idx = 0, self.rank_idx
        self.num_rdma_ranks, self.num_nvlink_ranks = 1, self.num_ranks
        torch.cuda.synchronize()
        group.barrier()

    def destroy(self) -> None:
        assert self.explicitly_destroy
        for region in self.__dict__.get('_side_regions', {}).values():
            region.destroy()
        self.__dict__['_side_regions'] = {}
        if getattr(self, '_host', None) is not None:
            self._host.destroy()
            self._host = None
        if self._buffer is not None:
            self._buffer.destroy()
            self._buffer = None
            self.runtime = None

    @staticmethod
    def get_buffer_size_hint(group: dist.ProcessGroup, num_max_tokens_per_rank: int, hidden: int, num_topk: int = 0,
                             use_fp8_dispatch: bool = False, allow_hybrid_mode: bool = True,
                             allow_multiple_reduction: bool = True) -> int:
        return require_ext().normal_region_size_for(max(num_max_tokens_per_rank, 1), max(hidden, 128), group.size())

    @staticmethod
    def get_elastic_buffer_alignment() -> int:
        return 2 << 20

    # Size hints of the experimental side features (their regions: [64 KiB control | data], 2 MiB
    # aligned; the reference carves the same features out of its one symmetric window).
    @staticmethod
    def get_engram_storage_size_hint(num_entries: int, hidden: int, num_max_tokens_per_rank: int,
                                     dtype: torch.dtype = torch.bfloat16) -> Tuple[int, int]:
        """(fetch receive bytes, storage bytes), each 2 MiB aligned. Rows are bf16 here; the fetched
        rows land in a fresh tensor. The storage lives in a GPU region, or, with `num_cpu_bytes` set
        to the storage bytes (hybrid mode), in each rank's shared host segment."""
        row = align(hidden * dtype.itemsize, 32)
        a = ElasticBuffer.get_elastic_buffer_alignment()
        return align(row * num_max_tokens_per_rank, a), align(64 * 1024 + row * num_entries, a)

    @staticmethod
    def get_pp_buffer_size_hint(num_max_tensor_bytes: int, num_max_inflight_tensors: int) -> int:
        """Bytes of the pipeline region: a receive slot ring per neighbour (two neighbours)."""
        slot = align(num_max_tensor_bytes, 128)
        return align(64 * 1024 + 2 * slot * num_max_inflight_tensors, ElasticBuffer.get_elastic_buffer_alignment())

    @staticmethod
    def get_agrs_num_max_session_bytes(group: dist.ProcessGroup, shapes, dtype: torch.dtype) -> int:
        """Session bytes that all-gathers of these local shapes use (each gathered tensor 32-byte aligned)."""
        if not isinstance(shapes[0], (tuple, list, torch.Size)):
            shapes = (shapes,)
        return sum(align(group.size() * math.prod(s) * dtype.itemsize, 32) for s in shapes)

    @staticmethod
    def get_agrs_buffer_size_hint(group: dist.ProcessGroup, num_max_session_bytes: int) -> int:
        return align(64 * 1024 + num_max_session_bytes, ElasticBuffer.get_elastic_buffer_alignment())

    def barrier(self, use_comm_stream: bool = True, with_cpu_sync: bool = False) -> None:
        self._buffer.barrier(use_comm_stream, with_cpu_sync)

    @staticmethod
    def capture():
        return require_ext().EventHandle()

    def get_comm_stream(self) -> torch.cuda.Stream:
        return self._buffer.get_comm_stream()

    def get_physical_domain_size(self) -> Tuple[int, int]:
        return 1, self.num_ranks

    def get_logical_domain_size(self) -> Tuple[int, int]:
        return 1, self.num_ranks

    def get_theoretical_num_sms(self, num_experts: int, num_topk: int, num_scaleout_topk: int = 0,
                                rdma_gbs: float = 0, nvlink_gbs: float = 0, sm_read_gbs: float = 200,
                                sm_write_gbs: float = 50) -> int:
        """SM count for the NVLink kernels from a bandwidth model: each SM sustains about `sm_write_gbs`
        of NVLink traffic; size the grid so the link (not the SMs) is the bottleneck, with 25% headroom."""
        if self.num_ranks == 1:
            return torch.cuda.get_device_properties('cuda').multi_processor_count // 2
        nvlink_gbs = nvlink_gbs or get_nvlink_gbs()
        remote_fraction = 1 - 1 / self.num_ranks
        num_sms = math.ceil(nvlink_gbs * remote_fraction / sm_write_gbs * 1.25)
        num_sms = align(max(num_sms, 8), 2)
        if not self.prefer_overlap_with_compute:
            num_sms = max(num_sms, 64)
        return min(num_sms, torch.cuda.get_device_properties('cuda').multi_processor_count)

    def get_theoretical_num_qps(self, num_sms: int) -> int:
        return min(num_sms, 8 + 1)

    @nvtx_range('ep.elastic.dispatch')
    def dispatch(self, x: Union[torch.Tensor, Tuple[torch.Tensor, torch.Tensor]],
                 topk_idx: Optional[torch.Tensor] = None, topk_weights: Optional[torch.Tensor] = None,
                 cumulative_local_expert_recv_stats: Optional[torch.Tensor] = None, num_experts: Optional[int] = None,
                 num_max_tokens_per_rank: Optional[int] = None, expert_alignment: Optional[int] = None,
                 num_sms: int = 0, num_qps: int = 0, previous_event=None, previous_event_before_epilogue=None,
                 async_with_compute_stream: bool = False, allocate_on_comm_stream: bool = False,
                 handle: Optional[EPHandle] = None, do_handle_copy: bool = True, do_cpu_sync: Optional[bool] = None,
                 do_expand: bool = False, use_tma_aligned_col_major_sf: bool = False, quantize_fp8: bool = False,
                 round_scale: bool = False):
        """v2 dispatch ([DE]deep_ep/buffers/elastic.py:708-855): returns
        `(recv_x, recv_topk_idx, recv_topk_weights, EPHandle, EventOverlap)`.

        With `async_with_compute_stream` the kernels and the post-processing run on the comm stream and
        the returned event covers both. `do_expand` sizes its expanded outputs from the received row
        count, which the host reads, so with `do_expand` the call waits for the comm stream before it
        returns even in the asynchronous mode (the event is then already complete)."""
        x, sf = x if isinstance(x, tuple) else (x, None)
        if handle is not None:
            assert topk_idx is None and topk_weights is None
            assert not do_cpu_sync, 'Cannot do CPU sync with cached handle'
            num_experts = num_experts or handle.num_experts
            num_sms = num_sms or handle.num_sms
            prev = _native_event(previous_event)
            rpm, spm, rrp, src_idx, itir, send_head = handle.legacy_handle
            out = self.runtime.intranode_dispatch(
                x, sf, None, None, None, 0, rpm, spm, src_idx, send_head, handle.expert_alignment, 0, quantize_fp8,
                round_scale, use_tma_aligned_col_major_sf and not handle.do_expand, None, num_sms, prev,
                async_with_compute_stream, allocate_on_comm_stream)
            rx, rs, event = out[0], out[1], out[11]
            if handle.do_expand:
                if async_with_compute_stream:
                    # as in the fresh dispatch: expand after the kernels, on the comm stream
                    with torch.cuda.stream(self.get_comm_stream()):
                        rx, rs = self._expand_rows(rx, rs, handle)
                        event = require_ext().EventHandle()
                    _record_on_current_stream(rx, rs)
                else:
                    rx, rs = self._expand_rows(rx, rs, handle)
            recv_x = (rx, rs) if rs is not None else rx
            return recv_x, None, None, handle, EventOverlap(event)
        assert topk_idx is not None and num_experts is not None
        num_topk = topk_idx.shape[1]
        num_sms = self.get_theoretical_num_sms(num_experts, num_topk) if num_sms == 0 else num_sms
        num_max_tokens_per_rank = num_max_tokens_per_rank or self.num_max_tokens_per_rank or x.shape[0]
        expert_alignment = expert_alignment or 1
        do_cpu_sync = True if do_cpu_sync is None else do_cpu_sync
        num_worst = 0 if do_cpu_sync else num_max_tokens_per_rank * self.num_ranks
        # The handle's copy of the routing is taken on the caller's stream, before the call returns, so a
        # later in-place write to `topk_idx` on that stream cannot reach the cached handle (in the
        # asynchronous mode the post-processing below runs later, on the comm stream).
        handle_topk_idx = topk_idx.clone() if do_handle_copy else topk_idx
        (recv_x, recv_sf, recv_topk_idx, recv_topk_weights, per_expert_list, rpm, spm, rrp, src_idx, send_head,
         per_expert_dev, event) = self.runtime.intranode_dispatch(
            x, sf, topk_idx, topk_weights, None, num_experts, None, None, None, None, expert_alignment, num_worst,
            quantize_fp8, round_scale, use_tma_aligned_col_major_sf, cumulative_local_expert_recv_stats, num_sms,
            _native_event(previous_event), async_with_compute_stream, allocate_on_comm_stream)
        # Asynchronous mode: nothing has waited for the comm stream, so everything below, which reads the
        # pulled rows and their metadata, runs there after the kernels, and the returned event is
        # recorded after it; the outputs are then marked for use on the caller's stream.
        comm = self.get_comm_stream() if async_with_compute_stream else None
        with (torch.cuda.stream(comm) if comm is not None else _no_stream_change()):
            is_token_in_rank = send_head >= 0
            legacy = (rpm, spm, rrp, src_idx, is_token_in_rank, send_head)
            # source metadata: [global source token index, source rank]
            num_rows = src_idx.shape[0]
            src_rank = torch.searchsorted(rrp[1:].to(torch.int64),
                                          torch.arange(num_rows, device=src_idx.device, dtype=torch.int64), right=True)
            src_rank = src_rank.clamp_(max=self.num_ranks - 1).to(torch.int32)
            recv_src_metadata = torch.stack([src_rank * num_max_tokens_per_rank + src_idx, src_rank], dim=1)
            psum_expert = per_expert_dev.cumsum(0).to(torch.int32)
            ep_handle = EPHandle(do_expand, num_experts, expert_alignment, num_max_tokens_per_rank, num_sms,
                                 handle_topk_idx, per_expert_list, rrp[1:], psum_expert,
                                 recv_src_metadata, legacy)
            if do_expand:
                # Expanded layout: one row per (received token, local expert), grouped by expert with every
                # group padded to `expert_alignment` (the permute kernels). recv_src_metadata gains the row
                # of each top-k slot (-1 if not local); psum per expert = aligned start + unpadded count.
                E_l = num_experts // self.num_ranks
                ep_handle.recv_topk_idx_local = recv_topk_idx
                # padding rows are zeroed, so the expanded outputs are fully defined (two calls with the
                # same inputs return the same bytes, and a grouped GEMM may run over whole groups)
                perm = permute(recv_x, recv_topk_idx, E_l, alignment=expert_alignment, probs=recv_topk_weights,
                               x_scales=recv_sf.contiguous() if recv_sf is not None else None, zero_padding=True)
                ep_handle.row_map = perm.row_map
                ep_handle.expert_offsets = perm.expert_offsets
                ep_handle.recv_src_metadata = torch.cat([recv_src_metadata, perm.row_map], dim=1)
                ep_handle.psum_num_recv_tokens_per_expert = (perm.expert_offsets[:-1] + perm.expert_counts).to(torch.int32)
                ep_handle.num_recv_tokens_per_expert_list = perm.expert_counts.tolist() if do_cpu_sync else []
                rows = int(perm.expert_offsets[-1].item())
                recv_x = perm.x[:rows]
                recv_sf = perm.scales[:rows] if perm.scales is not None else None
                if recv_sf is not None and use_tma_aligned_col_major_sf:
                    recv_sf = recv_sf.t().contiguous().t()
                recv_topk_weights = perm.probs[:rows] if perm.probs is not None else None
            if comm is not None:
                event = require_ext().EventHandle()
        out_x = (recv_x, recv_sf) if recv_sf is not None else recv_x
        if comm is not None:
            _record_on_current_stream(out_x, recv_topk_idx, recv_topk_weights, ep_handle)
        return out_x, recv_topk_idx, recv_topk_weights, ep_handle, EventOverlap(event)

    @staticmethod
    def _expand_rows(rx, rs, handle):
        """Cached-mode expansion with the handle's grouped layout."""
        E_l = handle.expert_offsets.numel() - 1
        perm = permute(rx, handle.recv_topk_idx_local, E_l, alignment=handle.expert_alignment,
                       x_scales=rs.contiguous() if rs is not None else None, zero_padding=True)
        rows = int(handle.expert_offsets[-1].item())
        return perm.x[:rows], (perm.scales[:rows] if perm.scales is not None else None)

    @nvtx_range('ep.elastic.combine')
    def combine(self, x: torch.Tensor, handle: EPHandle, topk_weights: Optional[torch.Tensor] = None,
                bias: Union[torch.Tensor, Tuple[torch.Tensor, torch.Tensor], None] = None, num_sms: int = 0,
                num_qps: int = 0, previous_event=None, previous_event_before_epilogue=None,
                async_with_compute_stream: bool = False, allocate_on_comm_stream: bool = False):
        num_sms = handle.num_sms if num_sms == 0 else num_sms
        row_map = None
        if handle.do_expand:
            # One row per (token, local expert): the combine kernel sums each token's rows on the
            # sender before the exchange (weights already applied by the caller, as in the reference's
            # expanded combine, [DE]deep_ep/include/deep_ep/impls/combine.cuh), then across ranks.
            x = x.contiguous()
            row_map = handle.row_map
            topk_weights = None
        rpm, spm, _, src_idx, _, send_head = handle.legacy_handle
        bias_0, bias_1 = Buffer._unpack_bias(bias)
        combined_x, combined_w, event = self.runtime.intranode_combine(
            x, topk_weights, bias_0, bias_1, rpm, spm, send_head, src_idx, num_sms, _native_event(previous_event),
            async_with_compute_stream, allocate_on_comm_stream, row_map, None)
        return combined_x, combined_w, EventOverlap(event)

    # ------------------------------------------------------------------ experimental side features
    # Engram storage, pipeline send/recv and AGRS all-gather sessions ([DE]deep_ep/buffers/elastic.py:
    # 433-572). Each feature owns a symmetric CUDA-IPC region that its (collective) configuration call
    # allocates; see `parallel/symmetric.py` and `csrc/runtime/symmetric.cpp`.
    def _side_region(self, name: str, data_bytes: int):
        from .symmetric import SymmetricRegion
        regions = self.__dict__.setdefault('_side_regions', {})
        sizes = [None] * self.num_ranks
        dist.all_gather_object(sizes, int(data_bytes), self.group)
        need = max(sizes)
        region = regions.get(name)
        if region is None or region.data_bytes < need:
            if region is not None:
                region.destroy()
            region = SymmetricRegion(self.group, need)
            regions[name] = region
        return region.runtime

    def engram_write(self, storage: torch.Tensor) -> None:
        """(Experimental) Publish this rank's Engram storage `[num_entries, hidden]` bf16 (collective;
        barriers before and after). Entry `i` of the group lives on rank `i // num_entries`. With
        `num_cpu_bytes` (hybrid mode) the storage lives in this rank's shared host segment, as in
        the reference; otherwise in a GPU region."""
        assert storage.dtype == torch.bfloat16 and storage.dim() == 2
        shapes = [None] * self.num_ranks
        dist.all_gather_object(shapes, tuple(storage.shape), self.group)
        assert all(s == shapes[0] for s in shapes), 'every rank must hold the same number of Engram entries'
        if self._host is not None:
            nbytes = storage.numel() * storage.element_size()
            if nbytes > self.num_cpu_bytes:
                raise ValueError(f'Engram storage of {nbytes} bytes exceeds num_cpu_bytes ({self.num_cpu_bytes})')
            if (storage.shape[1] * 2) % 16:
                raise ValueError('Engram hidden * 2 bytes must be a multiple of 16')
            torch.cuda.synchronize()
            dist.barrier(self.group)  # earlier fetches by peers have finished reading the old storage
            self._host.view(self.rank_idx)[:nbytes].copy_(storage.contiguous().view(torch.uint8).flatten())
            dist.barrier(self.group)  # every rank's storage is in place
            self._engram_host = (int(storage.shape[0]), int(storage.shape[1]))
            return
        self._engram = self._side_region('engram', storage.numel() * storage.element_size())
        self._engram.engram_write(storage.contiguous())

    def engram_fetch(self, indices: torch.Tensor, num_qps: int = 0):
        """(Experimental) Fetch rows by global entry index (int32 `[num_tokens]`). GPU storage: the
        peer reads run on the region's copy stream and the returned hook joins it. Host storage
        (hybrid mode): the kernel reads the ranks' host segments on the current stream. The hook
        returns `[num_tokens, hidden]` bf16."""
        if getattr(self, '_engram_host', None) is not None:
            entries, hidden = self._engram_host
            out = require_ext().engram_fetch_rows(indices.to(torch.int32).contiguous(), self._host.device_ptrs(), entries,
                                                  hidden, 0, float(self.num_gpu_timeout_secs))
            return lambda: out
        assert getattr(self, '_engram', None) is not None, 'call engram_write first'
        return self._engram.engram_fetch(indices.to(torch.int32).contiguous(), 0)

    def pp_set_config(self, num_max_tensor_bytes: int, num_max_inflight_tensors: int) -> None:
        """(Experimental) Size the pipeline ring: `num_max_inflight_tensors` receive slots of
        `num_max_tensor_bytes` per neighbour (collective; includes a barrier). A send waits for a free
        slot; with one or two ranks the previous and next rank are the same and share one ring."""
        slot = align(num_max_tensor_bytes, 128)
        self._pp = self._side_region('pp', 2 * slot * num_max_inflight_tensors)
        self._pp.pp_set_config(num_max_tensor_bytes, num_max_inflight_tensors)

    def pp_send(self, t: torch.Tensor, dst_rank_idx: int, num_sms: int = 0) -> None:
        """(Experimental) Send `t` to the previous or next rank of the ring (TMA stores into its slot)."""
        assert getattr(self, '_pp', None) is not None, 'call pp_set_config first'
        self._pp.pp_send(t, dst_rank_idx, num_sms)

    def pp_recv(self, t: torch.Tensor, src_rank_idx: int, num_sms: int = 0) -> None:
        """(Experimental) Receive into `t` from the previous or next rank of the ring."""
        assert getattr(self, '_pp', None) is not None, 'call pp_set_config first'
        self._pp.pp_recv(t, src_rank_idx, num_sms)

    def agrs_set_config(self, num_max_session_bytes: int, num_max_all_gathers_per_session: int) -> None:
        """(Experimental) Size the AGRS session buffer (collective; includes a barrier)."""
        self._agrs = self._side_region('agrs', align(num_max_session_bytes, 32))
        self._agrs.agrs_set_config(num_max_session_bytes, num_max_all_gathers_per_session)

    def create_agrs_session(self) -> None:
        assert getattr(self, '_agrs', None) is not None, 'call agrs_set_config first'
        self._agrs.create_agrs_session()

    def destroy_agrs_session(self) -> None:
        """End the session: after this rank's compute stream, signal every peer and wait for theirs
        (on the copy stream), so the next session may overwrite the buffer."""
        self._agrs.destroy_agrs_session()

    @contextmanager
    def agrs_new_session(self, enabled: bool = True):
        if not enabled:
            yield
            return
        self.create_agrs_session()
        try:
            yield
        finally:
            self.destroy_agrs_session()

    def agrs_get_inplace_tensor(self, shapes, dtype: torch.dtype):
        """Tensor(s) in this rank's slot of the next all-gather: filling them in place saves the local
        copy. One shape, or a sequence of shapes (batched)."""
        batched = isinstance(shapes[0], (tuple, list, torch.Size))
        if not batched:
            shapes = (shapes,)
        nbytes = [math.prod(s) * dtype.itemsize for s in shapes]
        raw = self._agrs.agrs_get_inplace_tensor(nbytes)
        out = tuple(r.view(dtype).view(tuple(s)) for r, s in zip(raw, shapes))
        return out if batched else out[0]

    def all_gather(self, t):
        """All-gather inside an AGRS session on the copy engines (one cudaMemcpyAsync per peer and
        tensor, no SMs). Returns `(gathered, hook)` (or `(*gathered, hook)` for a sequence): each
        gathered tensor is `[num_ranks, *t.shape]` in the session buffer; `hook()` makes the current
        stream wait for every peer's copy."""
        single = isinstance(t, torch.Tensor)
        tensors = (t,) if single else tuple(t)
        raw, hook = self._agrs.all_gather([x.contiguous() for x in tensors])
        out = tuple(r.view(x.dtype).view(self.num_ranks, *x.shape) for r, x in zip(raw, tensors))
        return (out[0], hook) if single else (*out, hook)
