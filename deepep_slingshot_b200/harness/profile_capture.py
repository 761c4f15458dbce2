"""torch.profiler capture of the EP step with NVTX ranges around the API calls, and a per-kernel
summary (the reference's `profile_capture.py`: torch.profiler + NVTX + kernel summaries).

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m deepep_slingshot_b200.harness.profile_capture \
        --tokens 4096 --hidden 7168 --experts 256 --topk 8 --steps 5 --out prof_ep8

Each operation (fresh dispatch with its layout, cached dispatch, combine, dispatch + combine cycle)
is profiled on its own, every call inside an `ep/<operation>/iteration<i>` range. Every rank writes,
per operation, `kernels-<op>-rank{r}.csv` (kernel, calls, total µs, mean µs, share of device time),
the Chrome trace `<op>-rank{r}.json` and `<op>-rank{r}-summary.json` (the case, with input and route
hashes); `harness.analyze_profiles` turns them into span/union/gap/overlap figures. Profiled numbers
are for shares and timelines, not benchmark values.
"""
import argparse
import csv
import datetime
import json
import os
from collections import defaultdict
from typing import Iterable, List

import torch
import torch.distributed as dist


def kernel_summary(events: Iterable, steps: int = 1) -> List[dict]:
    """Aggregate profiler events of the CUDA device by kernel name (sorted by total time)."""
    total = defaultdict(float)
    calls = defaultdict(int)
    for e in events:
        if getattr(e, 'device_type', None) != torch.autograd.DeviceType.CUDA:
            continue
        t = getattr(e, 'device_time_total', None)
        if t is None:
            t = getattr(e, 'cuda_time_total', 0.0)
        total[e.name] += float(t)
        calls[e.name] += 1
    grand = sum(total.values()) or 1.0
    rows = [{'kernel': k, 'calls': calls[k], 'total_us': round(v, 2), 'mean_us': round(v / calls[k], 2),
             'per_step_us': round(v / max(steps, 1), 2), 'share': round(v / grand, 4)} for k, v in total.items()]
    return sorted(rows, key=lambda r: -r['total_us'])


OPERATIONS = ('dispatch', 'cached_dispatch', 'combine', 'cycle')


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument('--tokens', type=int, default=4096)
    p.add_argument('--hidden', type=int, default=7168)
    p.add_argument('--experts', type=int, default=256)
    p.add_argument('--topk', type=int, default=8)
    p.add_argument('--steps', type=int, default=5)
    p.add_argument('--warmup', type=int, default=3)
    p.add_argument('--ops', nargs='+', default=list(OPERATIONS), choices=OPERATIONS)
    p.add_argument('--out', default='prof_out')
    args = p.parse_args(argv)
    from .. import Buffer
    from ..parallel import buffer as buffer_mod
    from ..utils import gate
    from ..utils.testing import hash_tensor
    buffer_mod._NVTX = True  # NVTX ranges around every API call for this capture
    owns = not dist.is_initialized()
    if owns:
        local = int(os.environ.get('LOCAL_RANK', '0'))
        torch.cuda.set_device(local)
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=120), device_id=torch.device('cuda', local))
    rank, world = dist.get_rank(), dist.get_world_size()
    N, H, E, K = args.tokens, args.hidden, args.experts, args.topk
    g = torch.Generator().manual_seed(1234 + rank)
    x = torch.randn((N, H), generator=g).to(torch.bfloat16).cuda()
    idx, w = gate.normal_routing(N, E, K, generator=g)
    idx, w = idx.cuda(), w.cuda()
    buf = Buffer(dist.group.WORLD, num_nvl_bytes=Buffer.get_nvl_buffer_size_hint(N, H, world))
    y_all = torch.randn((N * world, H), generator=g).to(torch.bfloat16).cuda()
    case = {'tokens': N, 'hidden': H, 'experts': E, 'topk': K, 'world': world, 'dtype': 'fp8',
            'input_sha256': hash_tensor(x), 'route_sha256': hash_tensor(idx)}

    def fresh():
        ntpr, _, ntpe, itir, _ = buf.get_dispatch_layout(idx, E)
        return buf.dispatch(x, num_tokens_per_rank=ntpr, is_token_in_rank=itir, num_tokens_per_expert=ntpe,
                            topk_idx=idx, topk_weights=w, quantize_fp8=True)

    (rx, _), _, rw, _, handle, _ = fresh()
    y = y_all[:rx.shape[0]]

    def cached():
        buf.dispatch(x, handle=handle, quantize_fp8=True)

    def comb():
        buf.combine(y, handle, topk_weights=rw)

    def cycle():
        (cx, _), _, cw, _, h, _ = fresh()
        buf.combine(y_all[:cx.shape[0]], h, topk_weights=cw)

    fns = {'dispatch': fresh, 'cached_dispatch': cached, 'combine': comb, 'cycle': cycle}
    os.makedirs(args.out, exist_ok=True)
    acts = [torch.profiler.ProfilerActivity.CPU, torch.profiler.ProfilerActivity.CUDA]
    for op in args.ops:
        fn = fns[op]
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        with torch.profiler.profile(activities=acts) as prof:
            for i in range(args.steps):
                with torch.profiler.record_function(f'ep/{op}/iteration{i}'):
                    fn()
                    torch.cuda.synchronize()
        rows = kernel_summary(prof.events(), args.steps)
        with open(os.path.join(args.out, f'kernels-{op}-rank{rank}.csv'), 'w', newline='') as f:
            wr = csv.DictWriter(f, fieldnames=['kernel', 'calls', 'total_us', 'mean_us', 'per_step_us', 'share'])
            wr.writeheader()
            wr.writerows(rows)
        prof.export_chrome_trace(os.path.join(args.out, f'{op}-rank{rank}.json'))
        with open(os.path.join(args.out, f'{op}-rank{rank}-summary.json'), 'w') as f:
            json.dump({'operation': op, 'rank': rank, 'profiled_iterations': args.steps, 'case': case}, f)
        if rank == 0:
            print(f'-- {op}')
            for r in rows[:8]:
                print(f"{r['share']:6.1%} {r['per_step_us']:9.1f} us/step  {r['kernel'][:90]}")
        dist.barrier()
    if owns:
        dist.destroy_process_group()


if __name__ == '__main__':
    main()
