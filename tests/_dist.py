"""Helpers to run a test body on N local ranks (gloo on CPU, NCCL on GPUs) as child processes."""
import os
import socket
import traceback

import torch
import torch.multiprocessing as mp


def free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _worker(rank, world, port, backend, fn, args, errq):
    import datetime
    import torch.distributed as dist
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    os.environ['NCCL_NVLS_ENABLE'] = os.environ.get('NCCL_NVLS_ENABLE', '0')
    try:
        kw = dict(backend=backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
        if backend == 'nccl':
            torch.cuda.set_device(rank)
            kw['device_id'] = torch.device('cuda', rank)
        dist.init_process_group(**kw)
        fn(rank, world, *args)
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        errq.put((rank, traceback.format_exc()))
        raise


def run_ranks(fn, world: int, backend: str = 'gloo', args=()):
    ctx = mp.get_context('spawn')
    errq = ctx.SimpleQueue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, backend, fn, args, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    for p in procs:
        if p.is_alive():
            p.kill()
            errors.append((-1, 'rank process timed out'))
    bad = [p.exitcode for p in procs if p.exitcode != 0]
    if errors or bad:
        raise AssertionError(f'ranks failed (exit codes {bad}):\n' + '\n'.join(f'[rank {r}] {e}' for r, e in errors))
