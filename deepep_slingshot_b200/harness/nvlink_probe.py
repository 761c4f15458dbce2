"""NVLink micro-probes over a normal-mode `Buffer`: flag round-trip latency per peer, the copy
bandwidth of peer stores and peer loads over a size x alignment sweep, and the per-pair bandwidth
matrix with every rank copying at once.

    torchrun --nproc-per-node N -m deepep_slingshot_b200.harness.nvlink_probe --out probe.json

The reference qualifies its NIC transport with raw probes before any EP gate (offset / size /
alignment and latency probes: harness/pipeline_1101/offset_probe.cu, harness/runner/burst_probe.cu).
On one NVSwitch box the transport is peer loads and stores plus release/acquire flags, so the
questions become: what does one flag round trip cost across the switch, how fast do peer stores and
peer loads move data at each size and start alignment, and does every pair reach the same bandwidth
under full load. One GPU runs the same probes against its own mapping (local HBM, and the
round trip between two blocks of one launch), which checks the plumbing but measures no link.
"""
import argparse
import json
import statistics
from typing import Dict, List, Sequence

import torch
import torch.distributed as dist

DEFAULT_SIZES = (4 << 10, 64 << 10, 1 << 20, 16 << 20, 128 << 20)
DEFAULT_OFFSETS = (0, 4, 8, 16, 64)


def flag_latency(buf, iters: int = 2000) -> Dict[int, float]:
    """Mean flag round-trip ns between rank 0 and every other rank (one GPU: key 0). Collective."""
    world = buf.group_size
    peers = [0] if world == 1 else list(range(1, world))
    out = {}
    for p in peers:
        out[p] = buf.runtime.probe_flag_latency(p, iters)
    return out


def _gbps(bytes_: int, ms: Sequence[float]) -> float:
    return bytes_ / (statistics.median(ms) * 1e-3) / 1e9


def copy_sweep(buf, sizes: Sequence[int] = DEFAULT_SIZES, offsets: Sequence[int] = DEFAULT_OFFSETS,
               store: bool = True, reps: int = 5, blocks: int = 0, shift: int = 1) -> List[dict]:
    """GB/s of this rank's copy to / from rank (rank + shift) % world per (size, start offset), every
    rank copying at once. Collective."""
    world = buf.group_size
    shift = shift % world
    blocks = blocks or 2 * torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    local = torch.empty(max(sizes) + max(offsets), dtype=torch.uint8, device='cuda').random_(0, 255)
    rows = []
    for size in sizes:
        for off in offsets:
            res = buf.runtime.probe_peer_copy(shift, size, off, store, reps, blocks, local)
            ms, vec = res[:-1], int(res[-1])
            rows.append({'bytes': size, 'offset': off, 'access_bytes': vec, 'direction': 'store' if store else 'load',
                         'peer_shift': shift, 'gbps': _gbps(size, ms), 'median_us': statistics.median(ms) * 1e3})
    return rows


def peer_matrix(buf, bytes_: int = 256 << 20, store: bool = True, reps: int = 3, blocks: int = 0) -> List[List[float]]:
    """[src][dst] GB/s: for every shift d, each rank r copies to (r + d) % world at the same time.
    Collective; every rank returns the whole matrix."""
    world = buf.group_size
    blocks = blocks or 2 * torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    local = torch.empty(bytes_, dtype=torch.uint8, device='cuda').random_(0, 255)
    mine = [0.0] * world
    for d in range(world):
        res = buf.runtime.probe_peer_copy(d, bytes_, 0, store, reps, blocks, local)
        mine[(buf.rank + d) % world] = _gbps(bytes_, res[:-1])
    rows = [None] * world
    dist.all_gather_object(rows, mine, group=buf.group)
    return rows


def main() -> None:
    p = argparse.ArgumentParser(description=__doc__.split('\n')[0])
    p.add_argument('--out', default='')
    p.add_argument('--iters', type=int, default=2000)
    p.add_argument('--matrix-bytes', type=int, default=256 << 20)
    args = p.parse_args()
    import os
    local_rank = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local_rank)
    dist.init_process_group('nccl', device_id=torch.device('cuda', local_rank))
    from deepep_slingshot_b200 import Buffer
    # the region past the control block must hold the largest copy plus its offset
    need = max(args.matrix_bytes, max(DEFAULT_SIZES) + max(DEFAULT_OFFSETS)) + (16 << 20)
    hint = max(Buffer.get_nvl_buffer_size_hint(4096, 7168, dist.get_world_size()), need)
    buf = Buffer(dist.group.WORLD, num_nvl_bytes=hint, num_gpu_timeout_secs=10, explicitly_destroy=True)
    report = {'world': buf.group_size,
              'flag_round_trip_ns': flag_latency(buf, args.iters),
              'store_sweep': copy_sweep(buf, store=True),
              'load_sweep': copy_sweep(buf, store=False),
              'store_matrix_gbps': peer_matrix(buf, args.matrix_bytes, store=True),
              'load_matrix_gbps': peer_matrix(buf, args.matrix_bytes, store=False)}
    if buf.rank == 0:
        text = json.dumps(report, indent=1)
        print(text)
        if args.out:
            with open(args.out, 'w') as f:
                f.write(text)
    buf.destroy()
    dist.destroy_process_group()


if __name__ == '__main__':
    main()
