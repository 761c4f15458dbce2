"""Capture a multi-rank device timeline of normal-mode dispatch + combine steps.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m deepep_slingshot_b200.harness.trace_capture \
        --tokens 4096 --hidden 7168 --experts 256 --topk 8 --steps 3 --out trace_ep8

Every rank runs warm-up steps, then `--steps` traced steps (layout + FP8 dispatch + combine, the
benchmark's step) with the device trace ring on and its host calls recorded as spans on the same
clock (`host.step`, `host.dispatch_call`, `host.combine_call`), so the timeline shows when each
rank's host issued and returned from its calls against its kernels and the peers'. Results are checked on the traced steps against the
untraced ones. Rank 0 writes `trace.json` (Chrome / Perfetto timeline: one process per rank, kernel
blocks as threads, all ranks on the host clock) and prints, per step and rank, when each phase
started and ended relative to the step's first record on any rank, which shows inter-rank skew.
Traced timings are for timelines only, never for benchmark numbers.
"""
import argparse
import contextlib
import datetime
import json
import os

import torch
import torch.distributed as dist


def phase_table(events):
    """Chrome-trace events -> one record per (rank, step, phase) with the phase's first start and last
    end (µs, across the phase's blocks). A rank's steps are split at its `host.step` spans (host
    clock, which the device records are aligned to); events before the first span get step -1."""
    by_rank = {}
    for e in events:
        by_rank.setdefault(e['pid'], []).append(e)
    lines = []
    for r, es in sorted(by_rank.items()):
        step_starts = sorted(e['ts'] for e in es if e['name'] == 'host.step')
        phases = {}
        for e in es:
            s = sum(1 for t in step_starts if t <= e['ts'] + 1e-6) - 1
            lo, hi = phases.get((s, e['name']), (1e30, -1e30))
            phases[(s, e['name'])] = (min(lo, e['ts']), max(hi, e['ts'] + e['dur']))
        for (s, name), (lo, hi) in sorted(phases.items()):
            lines.append({'rank': r, 'step': s, 'phase': name, 'start_us': round(lo, 1), 'end_us': round(hi, 1)})
    return lines


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument('--tokens', type=int, default=4096)
    p.add_argument('--hidden', type=int, default=7168)
    p.add_argument('--experts', type=int, default=256)
    p.add_argument('--topk', type=int, default=8)
    p.add_argument('--steps', type=int, default=3)
    p.add_argument('--warmup', type=int, default=3)
    p.add_argument('--num-sms', type=int, default=0)
    p.add_argument('--out', default='trace_out')
    args = p.parse_args(argv)
    from .. import Buffer
    from ..utils import gate
    from ..utils.trace import HostSpans, capture, gather_and_write
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
    cfg = Buffer.get_dispatch_config(world)
    if args.num_sms:
        cfg.num_sms = args.num_sms
    y = torch.randn((N * world, H), generator=g).to(torch.bfloat16).cuda()
    outs = []

    spans = HostSpans()
    tracing = {'on': False}

    def step():
        with (spans.span('host.step') if tracing['on'] else contextlib.nullcontext()):
            with (spans.span('host.dispatch_call') if tracing['on'] else contextlib.nullcontext()):
                ntpr, _, ntpe, itir, _ = buf.get_dispatch_layout(idx, E)
                (rx, rs), ri, rw, _, h, _ = buf.dispatch(x, num_tokens_per_rank=ntpr, is_token_in_rank=itir,
                                                         num_tokens_per_expert=ntpe, topk_idx=idx, topk_weights=w,
                                                         config=cfg, quantize_fp8=True)
            with (spans.span('host.combine_call') if tracing['on'] else contextlib.nullcontext()):
                out, _, _ = buf.combine(y[:rx.shape[0]], h, topk_weights=rw, config=cfg)
        outs.append(out)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    expected = outs[-1].clone()
    outs.clear()

    def check():
        torch.cuda.synchronize()
        assert torch.equal(outs[-1], expected), 'traced step differs from the untraced result'

    dist.barrier()
    tracing['on'] = True
    rec, offset = capture(buf, step, iterations=args.steps, group=dist.group.WORLD, check=check)
    tracing['on'] = False
    os.makedirs(args.out, exist_ok=True)
    trace = gather_and_write(rec, offset, os.path.join(args.out, 'trace.json'), dist.group.WORLD, spans)
    if rank == 0:
        lines = phase_table(trace['traceEvents'])
        with open(os.path.join(args.out, 'phases.jsonl'), 'w') as f:
            for l in lines:
                f.write(json.dumps(l) + '\n')
        for s in sorted({l['step'] for l in lines}):
            print(f'--- step {s}')
            names = sorted({l['phase'] for l in lines if l['step'] == s},
                           key=lambda n: min(l['start_us'] for l in lines if l['step'] == s and l['phase'] == n))
            for n in names:
                row = [l for l in lines if l['step'] == s and l['phase'] == n]
                print(f'{n:32s} ' + ' '.join(f"r{l['rank']}:{l['start_us']:.0f}-{l['end_us']:.0f}" for l in row))
    dist.barrier()
    if owns:
        dist.destroy_process_group()


if __name__ == '__main__':
    main()
