"""EP benchmark with an exact reference: correctness before timing, per case.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m deepep_slingshot_b200.harness.ep_benchmark \
        --models v4flash qwen3 minimax deepseek_v3 --routing uniform mixed skew2 hot_rank --dtype fp8 bf16 \
        --out ep_results

For every (model, tokens, dtype, routing, seed) case each rank:
  1. builds its routing (`harness.routing`), inputs and routing weights;
  2. checks a fresh dispatch against `ReferenceBuffer` (NCCL all_to_all_single): received payload
     and FP8 scales byte for byte, top-k ids, weights, source indices and the 128-aligned
     per-expert counts; then the combine (float rows within tolerance, integer-valued rows
     exactly) and the cached dispatch (byte for byte against the fresh one);
  3. times fresh dispatch, cached dispatch, combine and the full cycle (fresh dispatch + combine)
     with CUDA events after an L2 flush, taking the per-iteration max over ranks.
Records: `manifest-rank{r}.jsonl` (source hashes, versions, environment), `correctness-rank{r}.jsonl`,
`timings-rank{r}.jsonl`; rank 0 writes `summary.csv` and `repeatability.json` (`harness.summarize`).
Model shapes follow the reference's benchmark (backend/tests/ep_benchmark.py:19) plus DeepSeek-V3 and
a Mixtral-style small-expert-count shape (hidden 4096, 8 experts, top-2), swept as
`--models mixtral --dtype bf16 --routing uniform --tokens 128 512 2048 8192`.
`--impl nccl` runs the same cases through the NCCL all-to-all baseline (`parallel.nccl_baseline`);
`python -m deepep_slingshot_b200.harness.compare <ours_dir> <nccl_dir>` then pairs the two runs case by
case (same inputs, routes and placement) and prints the speedup at every point.
"""
import argparse
import datetime
import hashlib
import json
import os
import platform
import socket
import sys
import time

import torch
import torch.distributed as dist

MODELS = {'v4flash': (4096, 256, 6), 'qwen3': (4096, 128, 8), 'minimax': (3072, 256, 8),
          'deepseek_v3': (7168, 256, 8), 'mixtral': (4096, 8, 2)}
# The operations every case times, in order; summary.csv has one row per (case, op).
TIMED_OPS = ('dispatch', 'cached_dispatch', 'combine', 'cycle')


def dispatch_bytes(num_recv: int, hidden: int, num_topk: int, fp8: bool) -> int:
    """DeepEP v2 logical bytes of a dispatch: received rows x (row + scales + int64 ids + fp32 weights)."""
    row = hidden if fp8 else 2 * hidden
    scales = (hidden // 128) * 4 if fp8 else 0
    return num_recv * (row + scales + 8 * num_topk + 4 * num_topk)


def combine_bytes(num_recv: int, hidden: int, num_topk: int) -> int:
    """DeepEP v2 logical bytes of a combine: received rows x (bf16 row + fp32 top-k weights)."""
    return num_recv * (2 * hidden + 4 * num_topk)


def source_hashes() -> dict:
    """SHA-256 of every source file of the package (the manifest's code identity)."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out = {}
    for d, _, files in os.walk(root):
        for f in sorted(files):
            if f.endswith(('.py', '.cu', '.cuh', '.cpp', '.hpp', '.h')):
                p = os.path.join(d, f)
                with open(p, 'rb') as fh:
                    out[os.path.relpath(p, root)] = hashlib.sha256(fh.read()).hexdigest()
    return out


def manifest(args) -> dict:
    """This rank's manifest record: world, host, versions, environment knobs, source hashes."""
    return {'kind': 'manifest', 'rank': dist.get_rank(), 'world': dist.get_world_size(), 'host': socket.gethostname(),
            'time': datetime.datetime.utcnow().isoformat() + 'Z', 'argv': sys.argv, 'python': platform.python_version(),
            'torch': torch.__version__, 'cuda': torch.version.cuda,
            'nccl': '.'.join(map(str, torch.cuda.nccl.version())) if torch.cuda.is_available() else None,
            'gpu': torch.cuda.get_device_name() if torch.cuda.is_available() else None,
            'env': {k: v for k, v in os.environ.items() if k.startswith(('DEEPEP_', 'NCCL_', 'CUDA_', 'EP_'))},
            'sources': source_hashes(), 'impl': getattr(args, 'impl', 'ours')}


class _Jsonl:
    def __init__(self, path):
        self.f = open(path, 'a')

    def write(self, rec):
        self.f.write(json.dumps(rec) + '\n')
        self.f.flush()


def _check_equal(name, a, b):
    if not torch.equal(a, b):
        raise AssertionError(f'{name} mismatch')


def run_case(buf, ref, model, tokens, dtype, routing, seed, args, logs):
    """One (model, tokens, dtype, routing, seed) case: correctness against the oracle, then timings."""
    from ..utils.testing import bench, hash_tensor, rank_max
    from .routing import make_routing
    rank, R = dist.get_rank(), dist.get_world_size()
    H, E, K = MODELS[model]
    fp8 = dtype == 'fp8'
    idx = make_routing(routing, rank, R, tokens, E, K, seed).cuda()
    g = torch.Generator(device='cuda').manual_seed(seed * 1000 + rank)
    w = torch.rand((tokens, K), device='cuda', generator=g)
    w = torch.where(idx < 0, torch.zeros_like(w), w)
    w = w / w.sum(1, keepdim=True).clamp_min(1e-6)
    if args.drop_every > 0:
        # Dropped tokens (the reference's CXI_EP_DROP_EVERY, backend/tests/ep_benchmark.py:158-162):
        # every n-th token selects no expert at all.
        idx[::args.drop_every] = -1
        w[::args.drop_every] = 0
    x = torch.randn((tokens, H), device='cuda', generator=g).to(torch.bfloat16)
    case = {'model': model, 'hidden': H, 'experts': E, 'topk': K, 'tokens_per_rank': tokens, 'ranks': R,
            'dispatch_dtype': dtype, 'combine_dtype': 'bf16', 'routing': routing, 'seed': seed,
            'route_sha256': hash_tensor(idx), 'input_sha256': hash_tensor(x), 'alignment': 128,
            'num_sms': args.num_sms or getattr(buf, 'num_sms', 0), 'flush_l2': True, 'drop_every': args.drop_every,
            'impl': getattr(args, 'impl', 'ours')}

    # ---- correctness (fresh dispatch, then combine)
    kw = dict(topk_idx=idx, topk_weights=w, num_experts=E, expert_alignment=128)
    if fp8:
        kw['quantize_fp8'] = True
    rx, ri, rw, counts, handle, _ = buf.dispatch(x, **kw)
    ex, ei, ew, ecounts, ehandle, _ = ref.dispatch(x, **kw)
    torch.cuda.synchronize()
    num_recv = (rx[0] if fp8 else rx).shape[0]
    y = torch.randn((num_recv, H), device='cuda', generator=g).to(torch.bfloat16)
    error = None
    try:
        if fp8:
            _check_equal('payload', rx[0].view(torch.uint8), ex[0].view(torch.uint8))
            _check_equal('scales', rx[1], ex[1])
        else:
            _check_equal('payload', rx.view(torch.uint8), ex.view(torch.uint8))
        _check_equal('expert ids', ri, ei)
        _check_equal('weights', rw, ew)
        _check_equal('source ids', handle[3], ehandle[3].to(handle[3].dtype))
        if list(counts) != list(ecounts):
            raise AssertionError('padded per-expert counts mismatch')
    except AssertionError as e:
        error = str(e)
    # combine is collective: every rank runs it even after a local dispatch mismatch
    cx, cw, _ = buf.combine(y, handle, topk_weights=rw)
    ecx, ecw, _ = ref.combine(y, ehandle, topk_weights=ew)
    # cached dispatch (the handle's layout, no count exchange) reproduces the fresh one byte for byte
    crx = buf.dispatch(x, handle=handle, quantize_fp8=True)[0] if fp8 else buf.dispatch(x, handle=handle)[0]
    # integer-valued rows: every partial sum is exact in fp32 and bf16, so the combine must equal the
    # oracle's exactly, whatever the order of its reduction
    yi = torch.randint(-4, 5, (num_recv, H), device='cuda', generator=g).to(torch.bfloat16)
    ix, _, _ = buf.combine(yi, handle)
    eix, _, _ = ref.combine(yi, ehandle)
    torch.cuda.synchronize()
    if error is None and not torch.allclose(cx.float(), ecx.float(), atol=2e-2, rtol=2e-2):
        error = 'combine output mismatch'
    if error is None:
        try:
            if fp8:
                _check_equal('cached dispatch payload', crx[0].view(torch.uint8), rx[0].view(torch.uint8))
                _check_equal('cached dispatch scales', crx[1], rx[1])
            else:
                _check_equal('cached dispatch payload', crx.view(torch.uint8), rx.view(torch.uint8))
            _check_equal('integer combine', ix, eix)
        except AssertionError as e:
            error = str(e)
    ok = torch.tensor([0 if error else 1], device='cuda')
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if int(ok.item()) == 0:
        raise AssertionError(error or 'a peer rank failed its correctness check')
    logs['correctness'].write({'kind': 'correctness', **case, 'num_recv': num_recv, 'passed': True})

    # ---- timing (rank-max per iteration)
    def fresh():
        buf.dispatch(x, **kw)

    def cached():
        buf.dispatch(x, handle=handle, quantize_fp8=fp8) if fp8 else buf.dispatch(x, handle=handle)

    def comb():
        buf.combine(y, handle, topk_weights=rw)

    def cycle():  # a full step: fresh dispatch, then the combine of its handle
        h = buf.dispatch(x, **kw)[4]
        buf.combine(y, h, topk_weights=rw)

    ops = {'dispatch': (fresh, dispatch_bytes(num_recv, H, K, fp8)),
           'cached_dispatch': (cached, dispatch_bytes(num_recv, H, K, fp8)),
           'combine': (comb, combine_bytes(num_recv, H, K)),
           'cycle': (cycle, dispatch_bytes(num_recv, H, K, fp8) + combine_bytes(num_recv, H, K))}
    assert tuple(ops) == TIMED_OPS
    result = {}
    for op, (fn, nbytes) in ops.items():
        dist.barrier()
        host = []

        def timed():
            t0 = time.perf_counter()
            fn()
            host.append((time.perf_counter() - t0) * 1e6)
        _, _, _, times = bench(timed, num_warmups=args.warmup, num_tests=args.iters, flush_l2=True)
        local_us = [t * 1e6 for t in times[1:]]
        rmax_us = rank_max(local_us)
        host_max = rank_max([max(host[args.warmup:] or [0.0])])[0]
        bytes_max = rank_max([float(nbytes)])[0]
        rec = {'kind': 'timing', 'rank': dist.get_rank(), **case, 'op': op, 'bytes': nbytes, 'local_us': local_us,
               'rank_max_us': rmax_us,
               'max_host_us_per_iteration': host_max, 'bytes_rank_max': bytes_max}
        logs['timings'].write(rec)
        result[op] = rec
    if args.stall_us is not None:
        result['stall'] = _stall_loop(buf, fresh, comb, args, case, logs)
    if args.sweep_sms:
        result['sweep'] = _sms_sweep(buf, fresh, comb, ops, args, case, logs)
    return case, result


def _sms_sweep(buf, dispatch_fn, combine_fn, ops, args, case, logs):
    """Time dispatch and combine for each SM count of `--sweep-sms` (DeepEP's tuning sweep); the
    rank-max median per op and the best setting are recorded."""
    from ..utils.testing import bench, rank_max
    saved = type(buf).num_sms
    best = {}
    rows = []
    try:
        for sms in args.sweep_sms:
            type(buf).num_sms = sms
            row = {'num_sms': sms}
            for op, fn in (('dispatch', dispatch_fn), ('combine', combine_fn)):
                _, _, _, times = bench(fn, num_warmups=2, num_tests=max(4, args.iters // 2), flush_l2=True)
                med = sorted(rank_max([t * 1e6 for t in times[1:]]))[len(times[1:]) // 2]
                gbps = ops[op][1] / (med * 1e-6) / 1e9
                row[op + '_us'], row[op + '_gbps'] = med, gbps
                if op not in best or med < best[op]['us']:
                    best[op] = {'num_sms': sms, 'us': med, 'gbps': gbps}
            rows.append(row)
    finally:
        type(buf).num_sms = saved
    rec = {'kind': 'sweep', **case, 'rows': rows, 'best': best}
    logs['timings'].write(rec)
    if dist.get_rank() == 0:
        for op, b in best.items():
            print(f"[ep_benchmark] best {op}: {b['num_sms']} SMs, {b['us']:.1f} us, {b['gbps']:.0f} GB/s per rank", flush=True)
    return rec


def _stall_loop(buf, dispatch_fn, combine_fn, args, case, logs):
    """Dispatch -> GPU stall of `--stall-us` (standing in for the expert GEMMs) -> combine, looped;
    per-op device times averaged after a 20% ramp, max over ranks (the reference's stall ablation,
    tests/elastic/test_ep_stall.py:206-258)."""
    from ..utils.testing import rank_max
    n = args.stall_iters
    clock_mhz = torch.cuda.get_device_properties(torch.cuda.current_device()).clock_rate / 1e3
    cycles = int(args.stall_us * clock_mhz)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(n)]
    buf.barrier()
    torch.cuda.synchronize()
    for i in range(n):
        ev[i][0].record()
        dispatch_fn()
        ev[i][1].record()
        if cycles > 0:
            torch.cuda._sleep(cycles)
        ev[i][2].record()
        combine_fn()
        ev[i][3].record()
    torch.cuda.synchronize()
    warm = n // 5
    d_us = sum(ev[i][0].elapsed_time(ev[i][1]) for i in range(warm, n)) / max(1, n - warm) * 1e3
    c_us = sum(ev[i][2].elapsed_time(ev[i][3]) for i in range(warm, n)) / max(1, n - warm) * 1e3
    d_max, c_max = rank_max([d_us, c_us])
    rec = {'kind': 'stall', **case, 'stall_us': args.stall_us, 'iters': n, 'dispatch_us': d_max, 'combine_us': c_max}
    logs['timings'].write(rec)
    return rec


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.split('\n')[0])
    p.add_argument('--models', nargs='+', choices=list(MODELS), default=['v4flash', 'qwen3', 'minimax'])
    p.add_argument('--tokens', nargs='+', type=int, default=[4096])
    p.add_argument('--dtype', nargs='+', choices=['fp8', 'bf16'], default=['fp8'])
    p.add_argument('--routing', nargs='+', default=['uniform', 'mixed'])
    p.add_argument('--seeds', nargs='+', type=int, default=[0])
    p.add_argument('--drop-every', type=int, default=0, help='every n-th token selects no expert (0: none)')
    p.add_argument('--iters', type=int, default=20)
    p.add_argument('--warmup', type=int, default=5)
    p.add_argument('--num-sms', type=int, default=0)
    p.add_argument('--out', default='ep_results')
    p.add_argument('--spool', action='store_true',
                   help='write the journals to local memory (/dev/shm) and let an independent copier process '
                        'move them to --out, so written records survive a hung or killed run')
    p.add_argument('--impl', choices=['ours', 'nccl'], default='ours',
                   help="'nccl': the same cases through all_to_all_single over NCCL with torch FP8 casts (the "
                        "baseline; pair two result directories with harness.compare)")
    p.add_argument('--stall-us', type=float, default=None,
                   help='also run dispatch -> GPU stall -> combine loops (expert-compute stand-in)')
    p.add_argument('--stall-iters', type=int, default=200)
    p.add_argument('--sweep-sms', type=lambda v: [int(x) for x in v.split(',')], default=None,
                   help='comma-separated SM counts to time dispatch / combine with (tuning sweep)')
    args = p.parse_args(argv)
    if args.impl == 'nccl' and (args.sweep_sms or args.stall_us is not None):
        p.error('--sweep-sms and --stall-us time this library\'s kernels only (not --impl nccl)')

    from .. import Buffer, ReferenceBuffer
    from .summarize import summarize_dir
    owns_group = not dist.is_initialized()
    if owns_group:
        rank = int(os.environ.get('RANK', '0'))
        world = int(os.environ.get('WORLD_SIZE', '1'))
        local = int(os.environ.get('LOCAL_RANK', '0'))
        torch.cuda.set_device(local)
        os.environ.setdefault('MASTER_ADDR', '127.0.0.1')
        os.environ.setdefault('MASTER_PORT', '29561')
        dist.init_process_group('nccl', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device('cuda', local))
    rank, world = dist.get_rank(), dist.get_world_size()
    os.makedirs(args.out, exist_ok=True)
    copier = spool_dir = None
    if args.spool:
        from ..utils import result_spool
        spool_dir = result_spool.default_spool_dir(f'{os.path.basename(os.path.abspath(args.out))}-rank{rank}-{os.getpid()}')
        copier = result_spool.start_copier(spool_dir, args.out)
        logs = {k: result_spool.SpoolWriter(spool_dir, f'{k}-rank{rank}.jsonl') for k in ('manifest', 'correctness', 'timings')}
    else:
        logs = {k: _Jsonl(os.path.join(args.out, f'{k}-rank{rank}.jsonl')) for k in ('manifest', 'correctness', 'timings')}
    logs['manifest'].write(manifest(args))
    max_tokens = max(args.tokens)
    max_hidden = max(MODELS[m][0] for m in args.models)
    if args.impl == 'nccl':
        from ..parallel.nccl_baseline import NcclAllToAllEP
        buf = NcclAllToAllEP(dist.group.WORLD)
    else:
        buf = Buffer(dist.group.WORLD, num_nvl_bytes=Buffer.get_nvl_buffer_size_hint(max_tokens, max_hidden, world))
        if args.num_sms:
            Buffer.set_num_sms(args.num_sms)
    ref = ReferenceBuffer(dist.group.WORLD)
    failures = 0
    for model in args.models:
        for tokens in args.tokens:
            for dtype in args.dtype:
                for routing in args.routing:
                    for seed in args.seeds:
                        try:
                            case, res = run_case(buf, ref, model, tokens, dtype, routing, seed, args, logs)
                            if rank == 0:
                                line = ', '.join(f"{op} {sorted(r['rank_max_us'])[len(r['rank_max_us']) // 2]:.1f} us"
                                                 for op, r in res.items() if op not in ('stall', 'sweep'))
                                if 'stall' in res:
                                    line += (f", with {args.stall_us:g} us stall: dispatch {res['stall']['dispatch_us']:.1f} us"
                                             f" combine {res['stall']['combine_us']:.1f} us")
                                print(f'[ep_benchmark] {model} T={tokens} {dtype} {routing} seed {seed}: {line}', flush=True)
                        except (AssertionError, ValueError) as e:
                            failures += 1
                            logs['correctness'].write({'kind': 'correctness', 'model': model, 'tokens_per_rank': tokens,
                                                       'dispatch_dtype': dtype, 'routing': routing, 'seed': seed,
                                                       'passed': False, 'error': str(e)})
                            if rank == 0:
                                print(f'[ep_benchmark] {model} {dtype} {routing} seed {seed}: FAILED: {e}', flush=True)
    torch.cuda.synchronize()
    if copier is not None:  # every record reaches --out before the summary reads it
        result_spool.finish(spool_dir)
        copier.wait(timeout=120)
    dist.barrier()
    if rank == 0:
        summarize_dir(args.out)
    if owns_group:
        dist.destroy_process_group()
    return 1 if failures else 0


if __name__ == '__main__':
    sys.exit(main())
