"""Headline benchmark: DeepSeek-V3-shape normal-mode dispatch + combine over NVLink on N B200s,
plus the low-latency decode dispatch / combine latencies.

Config (the headline DeepSeek-V3 EP config): per rank 4096 tokens, hidden 7168, bf16 activations ~N(0,1),
256 experts (256/N per rank), top-8 from N(0,1) router logits with softmax weights; dispatch in
FP8 e4m3 with per-token 1x128 fp32 scales (quantization fused into the dispatch), combine in bf16.
One step = get_dispatch_layout + dispatch + combine (fresh, CPU-synced receive counts).

Byte definition (DeepEP v2 "logical bandwidth", local traffic included): dispatch bytes per
received token = FP8 row + fp32 scales + int64 top-k ids + fp32 top-k weights; combine bytes per
received token = bf16 row + fp32 top-k weights. `value` is the job aggregate: the sum over ranks of
those bytes divided by the step time (max over ranks). The published per-rank SM100 EP8 figures
(726 GB/s dispatch, 740 GB/s combine) combine into 735.1 GB/s per rank for a full cycle;
`vs_baseline` divides `value` by 735.1 x N.

Low-latency (config 3): 128 tokens/rank, hidden 7168, 256 experts, top-8 (uniform logits), FP8
dispatch with `return_recv_hook`, weighted bf16 combine; reported as device microseconds per
dispatch (send + hook) and per combine (send + hook), max over ranks, median over iterations.

Timing: CUDA events on the launching stream per step, L2 flushed (a 256 MiB write) before every
timed step, barrier + synchronize on both sides, max over ranks. SM clocks are sampled with
nvidia-smi during the timed region. `--impl reference` runs the unmodified reference through its
own public API when `import deep_ep` from baseline/_ref succeeds; otherwise it prints why it is
unavailable (the missing install or the import error). `--impl nccl` times the NCCL all-to-all
baseline (`parallel.nccl_baseline`) on the same step.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = 'dispatch/combine NVLink GB/s (normal) + LL dispatch/combine us, 8xB200'
BASELINE_CYCLE_GBPS_PER_RANK = 735.1
# Outcome of the offline install into baseline/_ref (pip reports the root as not installable; the
# vendored DeepEP v2 source does not compile here): printed when baseline/_ref is absent.
REFERENCE_INSTALL_OUTCOME = ('the offline install failed: the reference root has no setup.py/pyproject.toml '
                             '("not installable"), and its vendored DeepEP v2 source fails to build against NCCL '
                             '2.28.9 (no GIN/LSA device API: ncclCommProperties, ncclGetLsaDevicePointer) and '
                             'NVSHMEM IBGDA (missing infiniband/mlx5dv.h)')


def reference_module():
    """(deep_ep module, None) when the unmodified reference imports from baseline/_ref, else (None,
    the reason it is unavailable): a missing install or the actual import error."""
    ref_dir = os.path.join(ROOT, 'baseline', '_ref')
    if not os.path.isdir(ref_dir):
        return None, 'baseline/_ref is absent; ' + REFERENCE_INSTALL_OUTCOME
    sys.path.insert(0, ref_dir)
    try:
        import deep_ep
    except Exception as exc:  # report the real error, whatever the failing import raises
        return None, f'import deep_ep from baseline/_ref failed: {exc!r}'
    return deep_ep, None


def parse():
    p = argparse.ArgumentParser()
    p.add_argument('--gpus', type=int, default=1)
    p.add_argument('--steps', type=int, default=20)
    p.add_argument('--warmup', type=int, default=5)
    p.add_argument('--impl', default='ours', choices=['ours', 'reference', 'nccl'])
    p.add_argument('--tokens', type=int, default=4096)
    p.add_argument('--hidden', type=int, default=7168)
    p.add_argument('--experts', type=int, default=256)
    p.add_argument('--topk', type=int, default=8)
    p.add_argument('--num-sms', type=int, default=0)
    p.add_argument('--ll-tokens', type=int, default=128)
    p.add_argument('--no-ll', action='store_true')
    p.add_argument('--no-e2e', action='store_true')
    p.add_argument('--no-moe', action='store_true')
    p.add_argument('--moe-steps', type=int, default=3)
    p.add_argument('--moe-fused-dispatch', action='store_true',
                   help='MoE forward with the dispatch receive fused into the gate/up GEMM (Buffer.dispatch_gemm)')
    p.add_argument('--moe-fused-combine', action='store_true',
                   help='MoE forward with the down projection sending its rows into the combine slots '
                        '(parallel.gemm_combine) instead of grouped GEMM -> combine')
    p.add_argument('--ll-moe', action='store_true',
                   help='also time the decode MoE layer (MoEFFN.forward_low_latency) at the low-latency shape')
    p.add_argument('--check', action='store_true', help='verify against the torch oracle before timing')
    return p.parse_args()


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
              'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
              'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, device: int):
        # nvidia-smi numbers GPUs in PCI order whatever CUDA_VISIBLE_DEVICES says: name this process's
        # GPU by its PCI bus id (the CUDA index only when the bus id is unknown).
        from deepep_slingshot_b200.utils.numa import pci_bus_id
        self.device = pci_bus_id(device) or str(device)
        self.proc = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile('w+', suffix='.csv', delete=False)
            self.proc = subprocess.Popen(['nvidia-smi', f'--query-gpu={self.FIELDS}', '--format=csv,noheader,nounits',
                                          '-lms', '200', '-i', self.device], stdout=self.file,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': ['unsampled']}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        mhz, max_mhz, reasons = [], None, set()
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        for line in self.file.read().splitlines():
            f = [c.strip() for c in line.split(',')]
            if len(f) < 9:
                continue
            try:
                mhz.append(float(f[1]))
                max_mhz = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == 'active':
                    reasons.add(n)
        os.unlink(self.file.name)
        return {'sm_mhz': statistics.median(mhz) if mhz else None, 'sm_max_mhz': max_mhz,
                'reasons': sorted(reasons), 'samples': len(mhz)}


def init(args):
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    assert world == args.gpus, f'--gpus {args.gpus} but WORLD_SIZE={world}'
    os.environ.setdefault('MASTER_ADDR', '127.0.0.1')
    os.environ.setdefault('MASTER_PORT', str(29600 + os.getpid() % 1000))
    torch.cuda.set_device(local)
    # Run (and allocate pinned inputs) on the CPUs next to this GPU, before NCCL starts its threads.
    from deepep_slingshot_b200.utils.numa import bind_process_to_gpu
    cpus = bind_process_to_gpu(local)
    args.host_cpus = f'{len(cpus)} CPUs local to the GPU (NVML affinity)' if cpus else 'process affinity unchanged'
    import datetime
    dist.init_process_group('nccl', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=300),
                            device_id=torch.device('cuda', local))
    return rank, world, local


def moe_roofline_seconds(rows: float, hidden: int, inter: int, local_experts: int, world: int, num_recv: float,
                         bf16_flops: float = 1650.1e12, hbm_bytes_per_s: float = 6558.4e9,
                         nvlink_bytes_per_s: float = 770e9, remote_in: float = None, remote_out: float = None) -> dict:
    """Lower bounds of one MoE training step (forward + backward) on one rank, in seconds:
    compute (FP8 forward at 2x the measured bf16 peak, bf16 backward at the measured peak) over the
    rank's `rows` expert rows; NVLink per direction: the forward dispatch (FP8 rows + scales) and
    combine (bf16 rows) and their bf16 mirrors in the backward, for the `remote_in` tokens this rank
    receives from other ranks and the `remote_out` tokens it sends to them (both default to
    (world - 1) / world of `num_recv`); and HBM: every local expert weight element moves at least
    8 bytes per step (bf16 master read + FP8 write by the quantization, FP8 read by the forward
    GEMMs, bf16 read by the input-gradient GEMMs, bf16 weight gradient write). The rank can be no
    faster than the largest of the three."""
    fwd_flops = 6.0 * rows * hidden * inter
    bwd_flops = 12.0 * rows * hidden * inter
    t_compute = fwd_flops / (2 * bf16_flops) + bwd_flops / bf16_flops
    remote = (world - 1) / world * num_recv
    r_in = remote if remote_in is None else remote_in
    s_out = remote if remote_out is None else remote_out
    fp8_row, bf16_row = hidden + hidden // 128 * 4, 2 * hidden
    # forward: dispatch in / out (FP8), combine out / in (bf16); backward: the same tokens in bf16 both ways
    bytes_in = r_in * fp8_row + s_out * bf16_row + (r_in + s_out) * bf16_row
    bytes_out = s_out * fp8_row + r_in * bf16_row + (r_in + s_out) * bf16_row
    t_comm = max(bytes_in, bytes_out) / nvlink_bytes_per_s
    weight_elems = local_experts * 3.0 * hidden * inter
    t_hbm = 8.0 * weight_elems / hbm_bytes_per_s
    return {'compute': t_compute, 'nvlink': t_comm, 'hbm': t_hbm, 'bound': max(t_compute, t_comm, t_hbm)}


def moe_route_loads(topk_idx: torch.Tensor, num_experts: int, world: int):
    """This rank's contribution to every destination rank under a routing `topk_idx [N, K]` (-1 =
    dropped): expert rows (one per (token, k) whose expert lives there) and tokens (one per token with
    at least one expert there)."""
    per_rank = num_experts // world
    valid = topk_idx >= 0
    dest = torch.where(valid, topk_idx // per_rank, torch.zeros_like(topk_idx))
    hit = torch.zeros((topk_idx.shape[0], world), dtype=torch.int64, device=topk_idx.device)
    hit.scatter_add_(1, dest, valid.long())
    return hit.sum(0), (hit > 0).sum(0)


def moe_step_roofline(rows_to, tokens_from, hidden: int, inter: int, local_experts: int, **peaks) -> dict:
    """Roofline of one MoE step for a routing: `rows_to[d]` expert rows rank d computes,
    `tokens_from[s][d]` tokens rank s sends to rank d. Each rank's bound uses its own rows and its own
    remote traffic; the exchanges are synchronous, so the step is bounded by the slowest rank (under
    a skewed routing the rank that holds the popular experts, not the average rank)."""
    world = len(rows_to)
    worst = None
    for d in range(world):
        r_in = sum(tokens_from[s][d] for s in range(world) if s != d)
        s_out = sum(tokens_from[d][s] for s in range(world) if s != d)
        b = moe_roofline_seconds(rows_to[d], hidden, inter, local_experts, world, 0, remote_in=r_in, remote_out=s_out,
                                 **peaks)
        if worst is None or b['bound'] > worst['bound']:
            worst = dict(b, rank=d, rows=float(rows_to[d]), remote_in=float(r_in), remote_out=float(s_out))
    return worst


def max_over_ranks(values):
    t = torch.tensor(values, dtype=torch.float64, device='cuda')
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def min_over_ranks(v):
    t = torch.tensor([float(v)], dtype=torch.float64, device='cuda')
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return t.item()


def sum_over_ranks(v):
    t = torch.tensor([float(v)], dtype=torch.float64, device='cuda')
    dist.all_reduce(t)
    return t.item()


def main():
    args = parse()
    deep_ep = None
    if args.impl == 'reference':
        deep_ep, reason = reference_module()
        if deep_ep is None:
            if int(os.environ.get('RANK', '0')) == 0:  # one line per job, also under torchrun
                print(json.dumps({'impl': 'reference', 'unavailable': reason}))
            return 0
    rank, world, local = init(args)
    from deepep_slingshot_b200 import Buffer
    from deepep_slingshot_b200.utils import gate
    N, H, E, K = args.tokens, args.hidden, args.experts, args.topk
    E_l = E // world
    g = torch.Generator().manual_seed(1234 + rank)
    x = torch.randn((N, H), generator=g).to(torch.bfloat16).cuda()
    idx, w = gate.normal_routing(N, E, K, generator=g)
    idx, w = idx.cuda(), w.cuda()
    # One rank: every byte is a local HBM copy, use every SM. Several ranks: NVLink-bound, 64 SMs
    # (measured: 32-64 CTAs of the pull pipeline already reach ~745 GB/s from a peer).
    num_sms = args.num_sms or (torch.cuda.get_device_properties(local).multi_processor_count if world == 1 else Buffer.num_sms)
    cfg = Buffer.get_dispatch_config(world)
    cfg.num_sms = num_sms
    nvl_bytes = Buffer.get_nvl_buffer_size_hint(N, H, world)
    ll_bytes = 0 if args.no_ll else Buffer.get_low_latency_rdma_size_hint(args.ll_tokens, H, world, E)

    cast = None  # the reference arm quantizes with its own cast, then dispatches the FP8 pair
    if args.impl == 'nccl':
        from deepep_slingshot_b200.parallel.nccl_baseline import NcclAllToAllEP
        buf = NcclAllToAllEP(dist.group.WORLD)
    elif args.impl == 'reference':
        # the unmodified reference through its own public API (stock code path, its own configs)
        from deep_ep.utils.math import per_token_cast_to_fp8 as cast
        buf = deep_ep.Buffer(dist.group.WORLD, num_nvl_bytes=nvl_bytes, num_rdma_bytes=0)
        cfg = deep_ep.Buffer.get_dispatch_config(world)
    else:
        buf = Buffer(dist.group.WORLD, num_nvl_bytes=nvl_bytes, num_rdma_bytes=ll_bytes, low_latency_mode=ll_bytes > 0)
    y_full = torch.randn((N * world, H), generator=g).to(torch.bfloat16).cuda()
    state = {}

    def layout_and_dispatch(xb, ids, wts):
        """get_dispatch_layout + FP8 dispatch of bf16 tokens through the arm's public API (ours and
        the NCCL baseline quantize inside the dispatch; the reference casts first with its own op)."""
        ntpr, _, ntpe, itir, _ = buf.get_dispatch_layout(ids, E)
        xin, kw = (cast(xb), {}) if cast is not None else (xb, {'quantize_fp8': True})
        return buf.dispatch(xin, num_tokens_per_rank=ntpr, is_token_in_rank=itir, num_tokens_per_expert=ntpe,
                            topk_idx=ids, topk_weights=wts, config=cfg, **kw)

    host_times = []  # DEEPEP_B200_BENCH_HOST_TIMES=1: host seconds spent in the dispatch and combine calls

    def step():
        t0 = time.perf_counter()
        (rx, rs), ri, rw, lst, h, _ = layout_and_dispatch(x, idx, w)
        t1 = time.perf_counter()
        state['mid'].record()
        out, out_w, _ = buf.combine(y_full[:rx.shape[0]], h, topk_weights=rw, config=cfg)
        t2 = time.perf_counter()
        host_times.append((t1 - t0, t2 - t1))
        state['num_recv'] = rx.shape[0]
        return out

    if args.check and args.impl != 'reference':
        from deepep_slingshot_b200 import ReferenceBuffer
        ref = ReferenceBuffer(dist.group.WORLD)
        (rx, rs), ri, rw, lst, h, _ = buf.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E, quantize_fp8=True)
        (ex, es), ei, ew, el, eh, _ = ref.dispatch(x, topk_idx=idx, topk_weights=w, num_experts=E, quantize_fp8=True)
        assert torch.equal(rx.view(torch.uint8), ex.view(torch.uint8)) and torch.equal(rs, es) and lst == el
        o, _, _ = buf.combine(y_full[:rx.shape[0]], h)
        eo, _, _ = ref.combine(y_full[:rx.shape[0]], eh)
        assert torch.allclose(o.float(), eo.float(), atol=1e-2, rtol=1e-2)
        del ref

    flush = torch.empty(256 << 20, dtype=torch.uint8, device='cuda')
    for _ in range(args.warmup):
        state['mid'] = torch.cuda.Event(enable_timing=True)
        step()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()

    from deepep_slingshot_b200.utils.nvlink_counters import NvlinkCounters
    links = NvlinkCounters(local)  # read-only NVML per-link data counters
    sampler = ClockSampler(local)
    sampler.start()
    link_before = links.read()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    mids = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        flush.zero_()
        state['mid'] = mids[i]
        starts[i].record()
        step()
        ends[i].record()
    torch.cuda.synchronize()
    link_after = links.read()
    clocks = sampler.stop()
    dist.barrier()
    torch.cuda.synchronize()
    t_disp = [starts[i].elapsed_time(mids[i]) for i in range(args.steps)]
    t_comb = [mids[i].elapsed_time(ends[i]) for i in range(args.steps)]
    t_step = [starts[i].elapsed_time(ends[i]) for i in range(args.steps)]
    t_disp, t_comb, t_step = max_over_ranks(t_disp), max_over_ranks(t_comb), max_over_ranks(t_step)
    ms_step = sum(t_step) / len(t_step)
    ms_disp = sum(t_disp) / len(t_disp)
    ms_comb = sum(t_comb) / len(t_comb)
    num_recv = state['num_recv']
    disp_bytes = num_recv * (H + H // 128 * 4 + K * 8 + K * 4)
    comb_bytes = num_recv * (2 * H + K * 4)
    total_disp = sum_over_ranks(disp_bytes)
    total_comb = sum_over_ranks(comb_bytes)
    value = (total_disp + total_comb) / (ms_step * 1e-3) / 1e9
    disp_gbps_rank = disp_bytes / (ms_disp * 1e-3) / 1e9
    comb_gbps_rank = comb_bytes / (ms_comb * 1e-3) / 1e9
    # Bytes that crossed this GPU's NVLinks per step (the GPU's own link counters, protocol overhead
    # included) beside the algorithmic remote bytes: rows received from other ranks in the dispatch
    # and pushed back to them in the combine (local rows never touch a link).
    own_rows = int(((idx // E_l) == rank).any(dim=1).sum())
    remote_rows = num_recv - own_rows
    ok = link_before is not None and link_after is not None
    moved = link_after - link_before if ok else None
    # every rank joins the same reductions; -1 marks a rank without counters
    tx, rx, payload = max_over_ranks([moved.tx_bytes / args.steps if ok else -1.0, moved.rx_bytes / args.steps if ok else -1.0,
                                      remote_rows * ((H + H // 128 * 4 + K * 8 + K * 4) + (2 * H + K * 4))])
    ok_all = min_over_ranks(1.0 if ok else 0.0) > 0
    nvlink = ({'tx_bytes_per_step_max_rank': tx, 'rx_bytes_per_step_max_rank': rx,
               'remote_payload_bytes_per_step_max_rank': payload,
               'source': 'NVML per-link data counters, read before and after the timed steps'} if ok_all else
              {'counters': 'unavailable (NVML NVLink byte counters not supported on every rank)'})

    # The same dispatch without the CPU sync on the received counts (`num_worst_tokens`: outputs sized
    # for the worst case, the CUDA-graph-compatible mode), timed the same way: it shows what the
    # host round trip of the synced dispatch costs.
    nosync = {}
    if args.impl == 'ours':
        worst = N * world
        ntpr, _, ntpe, itir, _ = buf.get_dispatch_layout(idx, E)
        for _ in range(args.warmup):
            buf.dispatch(x, num_tokens_per_rank=ntpr, is_token_in_rank=itir, num_tokens_per_expert=ntpe, topk_idx=idx,
                         topk_weights=w, config=cfg, quantize_fp8=True, num_worst_tokens=worst)
        torch.cuda.synchronize()
        dist.barrier()
        t_ns = []
        for i in range(args.steps):
            flush.zero_()
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record()
            buf.dispatch(x, num_tokens_per_rank=ntpr, is_token_in_rank=itir, num_tokens_per_expert=ntpe, topk_idx=idx,
                         topk_weights=w, config=cfg, quantize_fp8=True, num_worst_tokens=worst)
            s1.record()
            t_ns.append((s0, s1))
        torch.cuda.synchronize()
        t_ns = max_over_ranks([a.elapsed_time(b) for a, b in t_ns])
        ms_ns = sum(t_ns) / len(t_ns)
        # The CPU-synced dispatch timed the same way (dispatches back to back, no combine between
        # them): against the step's dispatch interval it separates the host round trip itself from
        # the coupling of the ranks' host loops through the combine.
        dist.barrier()
        t_sa = []
        for i in range(args.steps):
            flush.zero_()
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record()
            buf.dispatch(x, num_tokens_per_rank=ntpr, is_token_in_rank=itir, num_tokens_per_expert=ntpe, topk_idx=idx,
                         topk_weights=w, config=cfg, quantize_fp8=True)
            s1.record()
            t_sa.append((s0, s1))
        torch.cuda.synchronize()
        t_sa = max_over_ranks([a.elapsed_time(b) for a, b in t_sa])
        nosync = {'dispatch_nosync_ms': ms_ns, 'dispatch_nosync_gbps_per_rank': disp_bytes / (ms_ns * 1e-3) / 1e9,
                  'dispatch_nosync_note': 'num_worst_tokens = tokens x ranks: no CPU sync on the received counts',
                  'dispatch_synced_alone_ms': sum(t_sa) / len(t_sa)}

    # ---------------------------------------------------------------- low-latency
    ll = {}
    if not args.no_ll and args.impl == 'ours':
        T = args.ll_tokens
        gl = torch.Generator().manual_seed(99 + rank)
        lx = torch.randn((T, H), generator=gl).to(torch.bfloat16).cuda()
        lidx, lw = gate.uniform_routing(T, E, K, generator=gl)
        lidx, lw = lidx.cuda(), lw.cuda()
        ly = torch.randn((E_l, world * T, H), generator=gl).to(torch.bfloat16).cuda()
        iters = max(args.steps, 20)

        def ll_dispatch():
            recv, cnt, hh, _, hook = buf.low_latency_dispatch(lx, lidx, T, E, use_fp8=True, return_recv_hook=True)
            hook()
            return hh

        def ll_combine(hh):
            out, _, chook = buf.low_latency_combine(ly, lidx, lw, hh, return_recv_hook=True)
            chook()
            return out

        def time_ll(run_d, run_c, n):
            d_us, c_us = [], []
            for i in range(n):
                e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
                dist.barrier()
                torch.cuda.synchronize()
                e0.record()
                hh = run_d()
                e1.record()
                run_c(hh)
                e2.record()
                torch.cuda.synchronize()
                d_us.append(e0.elapsed_time(e1) * 1e3)
                c_us.append(e1.elapsed_time(e2) * 1e3)
            return max_over_ranks(d_us), max_over_ranks(c_us)

        time_ll(ll_dispatch, ll_combine, args.warmup)
        eager_d, eager_c = time_ll(ll_dispatch, ll_combine, iters)
        # CUDA-graph replay (how decode runs): device time without host launch gaps
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            hh = ll_dispatch()
            ll_combine(hh)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        dist.barrier()
        gd, gc = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(gd):
            ghh = ll_dispatch()
        with torch.cuda.graph(gc):
            ll_combine(ghh)
        torch.cuda.synchronize()
        dist.barrier()
        time_ll(lambda: gd.replay(), lambda _: gc.replay(), args.warmup)
        d_us, c_us = time_ll(lambda: gd.replay(), lambda _: gc.replay(), iters)
        del gd, gc
        ll = {'ll_dispatch_us': statistics.median(d_us), 'll_combine_us': statistics.median(c_us),
              'll_timing': 'CUDA-graph replay, device time, max over ranks, median over iterations',
              'll_eager_dispatch_us': statistics.median(eager_d), 'll_eager_combine_us': statistics.median(eager_c),
              'll_config': {'tokens_per_rank': T, 'hidden': H, 'experts': E, 'topk': K, 'fp8_dispatch': True,
                            'return_recv_hook': True, 'routing': 'uniform logits'}}

    # ---------------------------------------------------------------- MoE layer forward + backward (config 4)
    moe = {}
    if not args.no_moe and args.impl == 'ours':
        from deepep_slingshot_b200.models import MoEFFN
        from deepep_slingshot_b200.models import moe as _moe_mod
        inter = 2048
        _moe_mod._FUSED_DISPATCH['enabled'] = args.moe_fused_dispatch
        _moe_mod._FUSED_COMBINE['enabled'] = args.moe_fused_combine
        gm = torch.Generator().manual_seed(4321)
        layer = MoEFFN(buf, H, inter, E, K, config=cfg, init_std=0.02, generator=gm)
        mx = torch.randn((N, H), generator=gm).to(torch.bfloat16).cuda().requires_grad_(True)
        midx, mw = gate.zipf_routing(N, E, K, s=1.1, generator=torch.Generator().manual_seed(77 + rank))
        midx, mw = midx.cuda(), mw.cuda().requires_grad_(True)
        gout = torch.randn((N, H), generator=gm).to(torch.bfloat16).cuda()

        def moe_step():
            # A training step starts from cleared gradients (optimizer.zero_grad(set_to_none=True), the
            # PyTorch default): backward writes each gradient once instead of adding it to the last step's.
            layer.zero_grad(set_to_none=True)
            mx.grad = None
            mw.grad = None
            out = layer(mx, midx, mw)
            out.backward(gout)
            return out

        for _ in range(2):
            moe_step()
        torch.cuda.synchronize()
        dist.barrier()
        mts = []
        for _ in range(args.moe_steps):
            flush.zero_()
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a0.record()
            moe_step()
            a1.record()
            torch.cuda.synchronize()
            mts.append(a0.elapsed_time(a1))
        mts = max_over_ranks(mts)
        ms_moe = sum(mts) / len(mts)
        # The routing's load per rank: expert rows each rank computes, tokens each pair of ranks exchanges.
        rows_to, tok_to = moe_route_loads(midx, E, world)
        rows_all = rows_to.double().cuda()
        dist.all_reduce(rows_all)
        tok_mat = torch.zeros((world, world), dtype=torch.float64, device='cuda')
        tok_mat[rank] = tok_to.double().cuda()
        dist.all_reduce(tok_mat)
        # measured peaks (MEASURED_PEAKS.json): cuBLAS bf16 burst, STREAM-style copy; FP8 counted at 2x bf16
        roof = moe_step_roofline(rows_all.tolist(), tok_mat.tolist(), H, inter, E // world)
        moe = {'moe_tokens_per_s': N * world / (ms_moe * 1e-3), 'moe_ms_per_step': ms_moe,
               'moe_roofline_fraction': roof['bound'] / (ms_moe * 1e-3),
               'moe_roofline_ms': {k: roof[k] * 1e3 for k in ('compute', 'nvlink', 'hbm', 'bound')},
               'moe_roofline_rank': {'rank': roof['rank'], 'expert_rows': roof['rows'],
                                     'expert_rows_mean': float(rows_all.mean()), 'remote_tokens_in': roof['remote_in'],
                                     'remote_tokens_out': roof['remote_out']},
               'moe_config': {'tokens_per_rank': N, 'hidden': H, 'inter': inter, 'experts': E, 'topk': K,
                              'routing': 'zipf s=1.1', 'grads': 'set to None before every step (zero_grad(set_to_none=True))',
                              'forward': 'fp8 block-scaled tcgen05 grouped GEMMs' +
                              (', dispatch receive fused into the gate/up GEMM' if args.moe_fused_dispatch else '') +
                              (', down projection sends its rows into the combine slots (fused combine)'
                               if args.moe_fused_combine and not args.moe_fused_dispatch else '') +
                              (', power-of-two (UE8M0) scales applied by the MMA' if _moe_mod._UE8M0['enabled'] else
                               ', fp32 scales promoted per 128-deep K block'),
                              'backward': {'tcgen05_mn': 'bf16 tcgen05 grouped GEMMs on MN-major operands (no transposes), '
                                                         'fused SwiGLU and unpermute backward kernels',
                                           'tcgen05': 'bf16 tcgen05 grouped GEMMs on transposed (K-major) operands',
                                           'grouped': 'bf16 torch grouped GEMMs (library stand-in, A/B only)',
                                           'loop': 'bf16 per-expert torch matmuls (stand-in)'}.get(_moe_mod._BWD['mode'],
                                                                                              _moe_mod._BWD['mode']),
                              'roofline': ('slowest rank of max(its fp8 fwd at 2x bf16 peak + bf16 bwd at measured '
                                           '1650 TFLOP/s over its expert rows, its NVLink bytes per direction at 770 GB/s, '
                                           '8 bytes per local weight element per step at measured 6558 GB/s HBM)')}}
        layer.release()
        del layer
        torch.cuda.empty_cache()

    # ---------------------------------------------------------------- decode MoE layer (opt-in)
    if args.ll_moe and not args.no_ll and args.impl == 'ours':
        from deepep_slingshot_b200.models import MoEFFN
        dlayer = MoEFFN(buf, H, 2048, E, K, config=cfg, init_std=0.02, generator=torch.Generator().manual_seed(2468))
        lwf = lw.float().contiguous()
        for _ in range(args.warmup):
            dlayer.forward_low_latency(buf, lx, lidx, lwf, T)
        torch.cuda.synchronize()
        dist.barrier()
        dts = []
        for _ in range(iters):
            d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            d0.record()
            dlayer.forward_low_latency(buf, lx, lidx, lwf, T)
            d1.record()
            torch.cuda.synchronize()
            dts.append(d0.elapsed_time(d1) * 1e3)
        dts = max_over_ranks(dts)
        ll.update({'ll_moe_forward_us': statistics.median(dts),
                   'll_moe_config': {'tokens_per_rank': T, 'hidden': H, 'inter': 2048, 'experts': E, 'topk': K,
                                     'path': 'fused LL dispatch + masked gate/up GEMM, masked SwiGLU requant, '
                                             'masked down GEMM with the combine send as its epilogue, weighted combine'}})
        del dlayer
        torch.cuda.empty_cache()

    # ---------------------------------------------------------------- end to end through the public API
    e2e = None
    if not args.no_e2e:
        hx = torch.empty((N, H), dtype=torch.bfloat16, pin_memory=True)
        hx.copy_(x.cpu())
        hidx = idx.cpu().pin_memory()
        hw = w.cpu().pin_memory()
        hy = torch.empty(1, dtype=torch.float32, pin_memory=True)
        e_steps = max(3, args.steps // 2)
        ts = []
        for i in range(args.warmup + e_steps):
            dist.barrier()
            torch.cuda.synchronize()
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            t0.record()
            dx = hx.cuda(non_blocking=True)
            didx = hidx.cuda(non_blocking=True)
            dw = hw.cuda(non_blocking=True)
            (rx, rs), ri, rw, lst, h, _ = layout_and_dispatch(dx, didx, dw)
            out, _, _ = buf.combine(y_full[:rx.shape[0]], h, topk_weights=rw, config=cfg)
            hy.copy_(out.float().sum().view(1), non_blocking=True)
            t1.record()
            t1.synchronize()
            _ = hy.item()
            if i >= args.warmup:
                ts.append(t0.elapsed_time(t1))
        ts = max_over_ranks(ts)
        ms_serial = sum(ts) / len(ts)
        e2e_bytes = total_disp + total_comb

        def e2e_pipelined(n_steps):
            # A loader's schedule: step i + 1's inputs are copied from pinned memory on a copy
            # stream while step i runs (two device input buffers), every step's result is copied
            # back, and one CUDA-event region spans all steps (their copies included).
            copy = torch.cuda.Stream()
            comp = torch.cuda.current_stream()
            bufs = [(torch.empty((N, H), dtype=torch.bfloat16, device='cuda'), torch.empty(hidx.shape, dtype=hidx.dtype,
                     device='cuda'), torch.empty(hw.shape, dtype=hw.dtype, device='cuda')) for _ in range(2)]
            copied = [torch.cuda.Event() for _ in range(2)]
            freed = [torch.cuda.Event() for _ in range(2)]
            hys = torch.empty(n_steps, dtype=torch.float32, pin_memory=True)

            def issue_copy(i):
                b = bufs[i % 2]
                with torch.cuda.stream(copy):
                    if i >= 2:
                        copy.wait_event(freed[i % 2])  # step i - 2 has read this buffer
                    b[0].copy_(hx, non_blocking=True)
                    b[1].copy_(hidx, non_blocking=True)
                    b[2].copy_(hw, non_blocking=True)
                    copied[i % 2].record(copy)

            dist.barrier()
            torch.cuda.synchronize()
            p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            p0.record(comp)
            copy.wait_stream(comp)
            issue_copy(0)
            for i in range(n_steps):
                if i + 1 < n_steps:
                    issue_copy(i + 1)
                comp.wait_event(copied[i % 2])
                dx, didx, dw = bufs[i % 2]
                (rx, rs), ri, rw, lst, h, _ = layout_and_dispatch(dx, didx, dw)
                freed[i % 2].record(comp)  # the dispatch (synchronous) has consumed the inputs
                out, _, _ = buf.combine(y_full[:rx.shape[0]], h, topk_weights=rw, config=cfg)
                hys[i:i + 1].copy_(out.float().sum().view(1), non_blocking=True)
            p1.record(comp)
            p1.synchronize()
            _ = hys.tolist()
            return p0.elapsed_time(p1) / n_steps

        ms_pipe = None
        try:
            e2e_pipelined(max(1, args.warmup))
            ms_pipe = e2e_pipelined(e_steps)
        except Exception as exc:  # keep the serial number if the pipelined schedule cannot run
            print(f'[bench] pipelined e2e unavailable: {exc!r}', file=sys.stderr, flush=True)
        ok = torch.tensor([1 if ms_pipe is not None else 0], device='cuda')
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        h2d = hx.numel() * 2 + hidx.numel() * 8 + hw.numel() * 4
        if int(ok.item()) == 1:
            ms_pipe = max_over_ranks([ms_pipe])[0]
            e2e = {'value': e2e_bytes / (ms_pipe * 1e-3) / 1e9, 'unit': 'GB/s', 'ms_per_step': ms_pipe,
                   'h2d_bytes_per_step': h2d, 'd2h_bytes_per_step': 4,
                   'schedule': 'pipelined: next step inputs copied on a copy stream during the current step',
                   'serial_value': e2e_bytes / (ms_serial * 1e-3) / 1e9, 'serial_ms_per_step': ms_serial}
        else:
            e2e = {'value': e2e_bytes / (ms_serial * 1e-3) / 1e9, 'unit': 'GB/s', 'ms_per_step': ms_serial,
                   'h2d_bytes_per_step': h2d, 'd2h_bytes_per_step': 4,
                   'schedule': 'serial: each step copies, runs and reads back alone'}

    if rank == 0:
        line = {
            'metric': METRIC, 'value': value, 'unit': 'GB/s', 'n_gpus': world, 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': ms_step, 'higher_is_better': True, 'scaling': 'weak',
            'vs_baseline': value / (BASELINE_CYCLE_GBPS_PER_RANK * world), 'dtype': 'bf16',
            'data': 'synthetic (random bf16 activations ~N(0,1), N(0,1) router logits, seeded)',
            'impl': args.impl,
            'config': {'model': 'DeepSeek-V3 MoE dispatch/combine (hidden 7168, 256 experts, top-8)',
                       'global_batch': N * world, 'seq_len': N, 'tokens_per_rank': N,
                       'parallelism': f'ep{world}', 'dispatch_dtype': 'fp8_e4m3 1x128 (fused quantization)',
                       'combine_dtype': 'bf16', 'num_sms': num_sms, 'l2': 'flushed before every timed step',
                       'host_cpus': getattr(args, 'host_cpus', None),
                       'byte_definition': 'DeepEP v2 logical bytes incl. local traffic, summed over ranks',
                       'transport': ('one GPU: every byte is a local HBM copy, none crosses NVLink' if world == 1
                                     else 'NVLink peer loads (dispatch) and stores (combine)'),
                       'baseline': f'{BASELINE_CYCLE_GBPS_PER_RANK} GB/s per rank x n_gpus (published SM100 EP8 726/740)'},
            'dispatch_ms': ms_disp, 'combine_ms': ms_comb, **nosync,
            'dispatch_gbps_per_rank': disp_gbps_rank, 'combine_gbps_per_rank': comb_gbps_rank,
            'num_recv_tokens_rank0': num_recv,
            'clocks': clocks,
            'nvlink': nvlink,
            # this library's kernels per timed step: layout, dispatch count, stage + pull, combine
            'gpu_launches': args.steps * 4 if args.impl == 'ours' else 0,
        }
        if os.environ.get('DEEPEP_B200_PROFILE') == '1' and hasattr(buf, 'get_profile'):
            line['kernel_profile_rank0'] = buf.get_profile()
        if os.environ.get('DEEPEP_B200_BENCH_HOST_TIMES') == '1':
            timed = host_times[args.warmup:args.warmup + args.steps]
            line['host_us_rank0'] = {'dispatch_call': 1e6 * sum(a for a, _ in timed) / len(timed),
                                     'combine_call': 1e6 * sum(b for _, b in timed) / len(timed)}
        line.update(ll)
        line.update(moe)
        if e2e is not None:
            line['e2e'] = e2e
        print(json.dumps(line), flush=True)
    dist.barrier()
    if hasattr(buf, 'runtime') and getattr(buf, 'explicitly_destroy', False):
        buf.destroy()
    dist.destroy_process_group()
    return 0


if __name__ == '__main__':
    sys.exit(main())
