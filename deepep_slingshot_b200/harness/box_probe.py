"""Box probe: what an EP group on this machine can rely on, recorded before any benchmark.

    python -m deepep_slingshot_b200.harness.box_probe --out box.json [--bandwidth]

Records (JSON): host, library versions (torch, CUDA, NCCL, driver), every GPU (name, memory, SMs,
compute capability), the peer-access matrix, `nvidia-smi topo -m` parsed into a link matrix, the
NVLink status lines, multicast (NVLS) support per GPU through the CUDA driver attribute, and the
driver-written measured peaks when present. With `--bandwidth` it also times a 256 MiB copy between
every ordered GPU pair with CUDA events (best of 5, GB/s per direction). Everything here only reads
settings; nothing is changed. The reference probes its transport before its gates with raw NIC
probes (harness/runner/burst_probe.cu, harness/pipeline_1101/offset_probe.cu) and a preflight
(harness/runner/preflight.sh); on one NVLink box the questions are peer access, link type, NVLS and
per-pair bandwidth.
"""
import argparse
import json
import os
import re
import socket
import subprocess
import sys
from typing import Dict, List, Optional


def _run(cmd: List[str]) -> Optional[str]:
    try:
        out = subprocess.run(cmd, capture_output=True, text=True, timeout=30)
    except (OSError, subprocess.TimeoutExpired):
        return None
    return out.stdout if out.returncode == 0 else None


def parse_topo_matrix(text: str) -> Dict[str, Dict[str, str]]:
    """`nvidia-smi topo -m` -> {gpu: {peer: link}} over the GPU rows and columns (link names such as
    X, NV18, NODE, SYS, PIX). Rows for NICs and the legend are ignored."""
    lines = [ln.rstrip() for ln in text.splitlines() if ln.strip()]
    header = None
    matrix: Dict[str, Dict[str, str]] = {}
    for ln in lines:
        cells = ln.split()
        if header is None:
            if cells and re.fullmatch(r'GPU\d+', cells[0]):
                header = [c for c in cells if re.fullmatch(r'GPU\d+', c)]
            continue
        if not cells or not cells[0].startswith('GPU') or not cells[0][3:].isdigit():
            if cells and cells[0].startswith('Legend'):
                break
            continue
        links = cells[1:1 + len(header)]
        if len(links) == len(header):
            matrix[cells[0]] = dict(zip(header, links))
    return matrix


def multicast_supported(device: int) -> Optional[bool]:
    """CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED through cuda-python (None when unavailable)."""
    try:
        import cuda.bindings.driver as drv
    except ImportError:
        return None
    try:
        err, = drv.cuInit(0)
        if err != drv.CUresult.CUDA_SUCCESS:
            return None
        err, dev = drv.cuDeviceGet(device)
        if err != drv.CUresult.CUDA_SUCCESS:
            return None
        err, val = drv.cuDeviceGetAttribute(drv.CUdevice_attribute.CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, dev)
        return bool(val) if err == drv.CUresult.CUDA_SUCCESS else None
    except Exception:
        return None


def peer_copy_gbs(src: int, dst: int, nbytes: int = 256 << 20, repeats: int = 5) -> float:
    """Best-of-`repeats` GB/s of one `nbytes` copy from GPU `src` to GPU `dst` (CUDA events on dst)."""
    import torch
    a = torch.empty(nbytes, dtype=torch.uint8, device=f'cuda:{src}')
    b = torch.empty(nbytes, dtype=torch.uint8, device=f'cuda:{dst}')
    best = float('inf')
    with torch.cuda.device(dst):
        for _ in range(repeats + 1):
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize(src)
            torch.cuda.synchronize(dst)
            start.record()
            b.copy_(a, non_blocking=True)
            end.record()
            end.synchronize()
            best = min(best, start.elapsed_time(end) / 1e3)
    del a, b
    return nbytes / best / 1e9


def collect(bandwidth: bool = False, repo_root: Optional[str] = None) -> dict:
    """Everything the probe records, as a dict (see the module docstring)."""
    import torch
    info = {'host': socket.gethostname(), 'torch': torch.__version__, 'cuda': torch.version.cuda,
            'nccl': None, 'driver': None, 'gpus': [], 'peer_access': [], 'topology': {}, 'nvlink_status': None,
            'measured_peaks': None}
    try:
        info['nccl'] = '.'.join(map(str, torch.cuda.nccl.version()))
    except Exception:
        pass
    smi = _run(['nvidia-smi', '--query-gpu=driver_version', '--format=csv,noheader'])
    if smi:
        info['driver'] = smi.splitlines()[0].strip()
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    for i in range(n):
        p = torch.cuda.get_device_properties(i)
        info['gpus'].append({'index': i, 'name': p.name, 'memory_bytes': p.total_memory, 'sms': p.multi_processor_count,
                             'capability': f'{p.major}.{p.minor}', 'multicast': multicast_supported(i)})
    info['peer_access'] = [[i == j or torch.cuda.can_device_access_peer(i, j) for j in range(n)] for i in range(n)]
    topo = _run(['nvidia-smi', 'topo', '-m'])
    if topo:
        info['topology'] = parse_topo_matrix(topo)
    info['nvlink_status'] = _run(['nvidia-smi', 'nvlink', '--status'])
    root = repo_root or os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    peaks = os.path.join(root, 'MEASURED_PEAKS.json')
    if os.path.exists(peaks):
        with open(peaks) as f:
            info['measured_peaks'] = json.load(f)
    if bandwidth and n > 1:
        info['peer_copy_gbs'] = [[None if i == j else round(peer_copy_gbs(i, j), 1) for j in range(n)] for i in range(n)]
    return info


def main(argv=None) -> int:
    p = argparse.ArgumentParser()
    p.add_argument('--out', default=None)
    p.add_argument('--bandwidth', action='store_true', help='time a peer copy between every ordered GPU pair')
    args = p.parse_args(argv)
    info = collect(args.bandwidth)
    text = json.dumps(info, indent=1)
    if args.out:
        with open(args.out, 'w') as f:
            f.write(text + '\n')
    print(text)
    n = len(info['gpus'])
    if n and not all(all(row) for row in info['peer_access']):
        print('WARNING: not every GPU pair has peer access; an EP group must be one NVLink domain', file=sys.stderr)
    return 0


if __name__ == '__main__':
    sys.exit(main())
