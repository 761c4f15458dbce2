"""Where the MoE layer's training step spends its device time: torch.profiler over forward +
backward steps of `models.MoEFFN` (the bench's config: hidden 7168, inter 2048, 256 experts, top-8,
Zipf(1.1) routing), per-kernel totals with shares, plus each phase's device time from CUDA events.

    python -m deepep_slingshot_b200.harness.moe_profile --out moe_prof              # 1 GPU
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m deepep_slingshot_b200.harness.moe_profile

Every rank writes `moe-kernels-rank{r}.csv` (kernel, calls, total µs, mean µs, per step, share);
rank 0 prints the top kernels and writes `moe-phases.json` (forward / backward ms per step, max over
ranks). Profiled numbers are shares, not benchmark values (the bench times the step unprofiled).
"""
import argparse
import csv
import datetime
import json
import os

import torch
import torch.distributed as dist


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument('--tokens', type=int, default=4096)
    p.add_argument('--hidden', type=int, default=7168)
    p.add_argument('--inter', type=int, default=2048)
    p.add_argument('--experts', type=int, default=256)
    p.add_argument('--topk', type=int, default=8)
    p.add_argument('--steps', type=int, default=3)
    p.add_argument('--warmup', type=int, default=2)
    p.add_argument('--out', default='moe_prof')
    args = p.parse_args(argv)
    from .. import Buffer
    from ..models import MoEFFN
    from ..utils import gate
    from .profile_capture import kernel_summary
    owns = not dist.is_initialized()
    if owns:
        local = int(os.environ.get('LOCAL_RANK', '0'))
        os.environ.setdefault('MASTER_ADDR', '127.0.0.1')
        os.environ.setdefault('MASTER_PORT', '29561')
        os.environ.setdefault('RANK', '0')
        os.environ.setdefault('WORLD_SIZE', '1')
        torch.cuda.set_device(local)
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=300), device_id=torch.device('cuda', local))
    rank, world = dist.get_rank(), dist.get_world_size()
    N, H, I, E, K = args.tokens, args.hidden, args.inter, args.experts, args.topk
    buf = Buffer(dist.group.WORLD, num_nvl_bytes=Buffer.get_nvl_buffer_size_hint(N, H, world))
    g = torch.Generator().manual_seed(4321)
    layer = MoEFFN(buf, H, I, E, K, init_std=0.02, generator=g)
    x = torch.randn((N, H), generator=g).to(torch.bfloat16).cuda().requires_grad_(True)
    idx, w = gate.zipf_routing(N, E, K, s=1.1, generator=torch.Generator().manual_seed(77 + rank))
    idx, w = idx.cuda(), w.cuda().requires_grad_(True)
    gout = torch.randn((N, H), generator=g).to(torch.bfloat16).cuda()

    def step(times=None):
        layer.zero_grad(set_to_none=True)  # as the bench's step: gradients written once, not accumulated
        x.grad = None
        w.grad = None
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record()
        out = layer(x, idx, w)
        e1.record()
        out.backward(gout)
        e2.record()
        if times is not None:
            torch.cuda.synchronize()
            times.append((e0.elapsed_time(e1), e1.elapsed_time(e2)))

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    times = []
    for _ in range(args.steps):
        step(times)
    t = torch.tensor([[f, b] for f, b in times], dtype=torch.float64, device='cuda')
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    fwd_ms, bwd_ms = (t.mean(0)).tolist()
    dist.barrier()
    acts = [torch.profiler.ProfilerActivity.CPU, torch.profiler.ProfilerActivity.CUDA]
    with torch.profiler.profile(activities=acts) as prof:
        for _ in range(args.steps):
            step()
        torch.cuda.synchronize()
    rows = kernel_summary(prof.events(), args.steps)
    os.makedirs(args.out, exist_ok=True)
    with open(os.path.join(args.out, f'moe-kernels-rank{rank}.csv'), 'w', newline='') as f:
        wr = csv.DictWriter(f, fieldnames=['kernel', 'calls', 'total_us', 'mean_us', 'per_step_us', 'share'])
        wr.writeheader()
        wr.writerows(rows)
    if rank == 0:
        with open(os.path.join(args.out, 'moe-phases.json'), 'w') as f:
            json.dump({'world': world, 'forward_ms': fwd_ms, 'backward_ms': bwd_ms, 'tokens_per_rank': N,
                       'hidden': H, 'inter': I, 'experts': E, 'topk': K}, f, indent=1)
        print(f'forward {fwd_ms:.2f} ms, backward {bwd_ms:.2f} ms per step (max over ranks, unprofiled)')
        for r in rows[:20]:
            print(f"{r['share']:6.1%} {r['per_step_us']:10.1f} us/step  {r['kernel'][:100]}")
    dist.barrier()
    if owns:
        dist.destroy_process_group()


if __name__ == '__main__':
    main()
