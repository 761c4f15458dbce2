"""Small single-GPU workloads that launch every sm_100a kernel of the library once.

Used to profile kernels in isolation (for example with Nsight Compute, filtering on the NVTX range
`profile`): each workload first runs once as a warm-up outside the range, then once inside it.

    python -m deepep_slingshot_b200.utils.kernel_workloads [--only name,name] [--tokens 4096] [--time 20]

With `--time R` each workload is also timed: R repetitions, each bracketed by CUDA events on the
current stream after a 256 MB write that evicts L2, median reported in microseconds.
Workloads (names for `--only`): layout, dispatch (count + stage/pull), combine, combine_expanded
(weighted expanded combine, needs dispatch), low_latency, ll_logfmt, cast, quantize_weights,
grouped_gemm, grouped_gemm_ue8m0 (power-of-two scales, block-scaled MMA), swiglu_quant (needs grouped_gemm), permute, barrier, masked_gemm, ll_dispatch_gemm,
bf16_gemm, bf16_mn, bf16_wgrad, fused_dispatch_gemm (standalone stage + count + fused receive/GEMM),
moe_backward_ops (needs dispatch and grouped_gemm), transport_checks, ll_clean, side_features (PP,
AGRS, Engram), gemm_combine (down projection whose epilogue sends into the combine slots, and the
source-side reduce), gemm_then_combine (the same down projection unfused: grouped GEMM, then the
weighted expanded combine).
The default set is every workload.

Sizes default to inputs larger than L2 for the bandwidth-bound kernels while keeping the whole
process within a few GB of device memory.
"""
import argparse
import datetime
import socket

import torch
import torch.distributed as dist


def _init_single_rank():
    if dist.is_initialized():
        return
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        port = s.getsockname()[1]
    torch.cuda.set_device(0)
    dist.init_process_group('nccl', init_method=f'tcp://127.0.0.1:{port}', rank=0, world_size=1,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device('cuda', 0))


def build(args):
    from deepep_slingshot_b200 import Buffer
    from deepep_slingshot_b200.ops import gemm, permute, quant
    from deepep_slingshot_b200.utils import gate
    from deepep_slingshot_b200._ext import require_ext
    N, H, E, K = args.tokens, args.hidden, args.experts, args.topk
    g = torch.Generator().manual_seed(0)
    x = torch.randn((N, H), generator=g).to(torch.bfloat16).cuda()
    idx, w = gate.normal_routing(N, E, K, generator=g)
    idx, w = idx.cuda(), w.cuda()
    T = args.ll_tokens
    E_ll = args.ll_experts
    buf = Buffer(dist.group.WORLD, num_nvl_bytes=Buffer.get_nvl_buffer_size_hint(N, H, 1),
                 num_rdma_bytes=Buffer.get_low_latency_rdma_size_hint(T, H, 1, E_ll), low_latency_mode=True)
    lx = x[:T].contiguous()
    lidx, lw = gate.uniform_routing(T, E_ll, K, generator=g)
    lidx, lw = lidx.cuda(), lw.cuda()
    ly = torch.randn((E_ll, T, H), generator=g).to(torch.bfloat16).cuda()
    y_recv = torch.randn((N, H), generator=g).to(torch.bfloat16).cuda()  # world 1: at most N rows arrive
    state = {}

    def layout():
        state['layout'] = buf.get_dispatch_layout(idx, E)

    def dispatch():
        ntpr, _, ntpe, itir, _ = state['layout']
        state['disp'] = buf.dispatch(x, num_tokens_per_rank=ntpr, is_token_in_rank=itir, num_tokens_per_expert=ntpe,
                                     topk_idx=idx, topk_weights=w, quantize_fp8=True)

    def combine():
        (rx, rs), ri, rw, _, h, _ = state['disp']
        state['comb'] = buf.combine(y_recv[:rx.shape[0]], h, topk_weights=rw)

    def ll():
        recv, cnt, hh, _, hook = buf.low_latency_dispatch(lx, lidx, T, E_ll, use_fp8=True, return_recv_hook=True)
        hook()
        out, _, chook = buf.low_latency_combine(ly, lidx, lw, hh, return_recv_hook=True)
        chook()

    def cast():
        q, s = quant.per_token_cast_to_fp8(x)
        quant.per_token_cast_back(q, s)

    rows_per, n1, k1, e_g = args.gemm_rows, 2 * args.inter, H, args.gemm_experts
    ga, gsa = quant.per_token_cast_to_fp8(torch.randn((rows_per * e_g, k1), generator=g).to(torch.bfloat16).cuda())
    gb, gsb = gemm.quantize_weights_fp8((torch.randn((e_g, n1, k1), generator=g) * 0.02).cuda())
    gsb = gsb.contiguous()
    goff = torch.arange(0, e_g + 1, dtype=torch.int32, device='cuda') * rows_per
    gcnt = torch.full((e_g,), rows_per, dtype=torch.int32, device='cuda')

    def grouped_gemm():
        state['h'] = gemm.grouped_gemm_fp8(ga, gsa, gb, gsb, goff, gcnt)

    # the same shape with power-of-two scales on the block-scaled MMA path
    ga_r, gsa_r = quant.per_token_cast_to_fp8(torch.randn((rows_per * e_g, k1), generator=g).to(torch.bfloat16).cuda(),
                                              round_scale=True)
    gb_r, gsb_r = gemm.quantize_weights_fp8((torch.randn((e_g, n1, k1), generator=g) * 0.02).cuda(), round_scale=True)
    gsb_r = gsb_r.contiguous()

    def grouped_gemm_ue8m0():
        gemm.grouped_gemm_fp8(ga_r, gsa_r, gb_r, gsb_r, goff, gcnt, ue8m0=True)

    def swiglu():
        require_ext().swiglu_quant(state['h'], False)

    def perm():
        p = permute.permute(x, idx[:, :K], E, alignment=128, probs=w)
        permute.unpermute(p.x, p.row_map, w)

    def barrier():
        buf.barrier()

    def quantize_weights():
        gemm.quantize_weights_fp8(wq_src)

    wq_src = (torch.randn((e_g, n1, k1), generator=g) * 0.02).to(torch.bfloat16).cuda()

    # combine in the weighted expanded mode: the grouped rows of the dispatch's tokens
    def combine_expanded():
        (rx, rs), ri, rw, _, h, _ = state['disp']
        if 'perm' not in state:
            state['perm'] = permute.permute(rx, ri, E, alignment=128, probs=rw, x_scales=rs, zero_padding=True)
            state['y_exp'] = torch.randn((state['perm'].x.shape[0], H), generator=g).to(torch.bfloat16).cuda()
        pm = state['perm']
        buf.combine(state['y_exp'], h, row_map=pm.row_map, row_weights=rw)

    # down projection with the combine send as its epilogue, then the source-side reduce (its own
    # FP8 dispatch over 8 experts: square [8, hidden, hidden] weights stay under a GB)
    def gc_setup():
        if 'gc' not in state:
            from ..parallel.gemm_combine import GemmCombine
            e2 = 8
            idx2, w2 = gate.normal_routing(N, e2, K, generator=g)
            idx2, w2 = idx2.cuda(), w2.cuda()
            (rx2, rs2), ri2, rw2, _, h2, _ = buf.dispatch(x, topk_idx=idx2, topk_weights=w2, num_experts=e2,
                                                          quantize_fp8=True)
            p2 = permute.permute(rx2, ri2, e2, alignment=128, probs=rw2, x_scales=rs2, zero_padding=True)
            wd, wds = gemm.quantize_weights_fp8((torch.randn((e2, H, H), device='cuda') * 0.02).to(torch.bfloat16))
            state['gc'] = (GemmCombine(dist.group.WORLD, N, K, H), p2, wd, wds.contiguous(), h2, idx2, w2, rw2)
        return state['gc']

    def gemm_combine():
        gc, p2, wd, wds, h2, idx2, w2, _ = gc_setup()
        gc.send(p2.x, p2.scales, wd, wds, p2.expert_offsets, p2.expert_counts, p2.row_map, h2, keep_local=False)
        gc.reduce(idx2, w2)

    # the same down projection unfused: grouped GEMM, then the weighted expanded combine
    def gemm_then_combine():
        _, p2, wd, wds, h2, _, _, rw2 = gc_setup()
        y2 = gemm.grouped_gemm_fp8(p2.x, p2.scales, wd, wds, p2.expert_offsets, p2.expert_counts)
        buf.combine(y2, h2, row_map=p2.row_map, row_weights=rw2)

    def ll_logfmt():
        recv, cnt, hh, _, hook = buf.low_latency_dispatch(lx, lidx, T, E_ll, use_fp8=True, return_recv_hook=True)
        hook()
        out, _, chook = buf.low_latency_combine(ly, lidx, lw, hh, use_logfmt=True, return_recv_hook=True)
        chook()

    slots = T  # world 1: the low-latency layout has num_ranks * max_tokens slots per expert
    n_small = 512  # weights generated on the device, kept to a few GB
    mw1, mw1s = gemm.quantize_weights_fp8((torch.randn((E_ll, n_small, H), device='cuda') * 0.02).to(torch.bfloat16))
    mw1s = mw1s.contiguous()
    mx, msx = quant.per_token_cast_to_fp8(torch.randn((E_ll * slots, H), generator=g).to(torch.bfloat16).cuda())
    mcnt = torch.full((E_ll,), min(slots, max(1, T * K // E_ll)), dtype=torch.int32, device='cuda')

    def masked_gemm():
        gemm.masked_grouped_gemm_fp8(mx.view(E_ll, slots, H), msx.view(E_ll, slots, H // 128), mcnt, mw1, mw1s)

    def ll_dispatch_gemm():
        out, cnt, hh, _ = buf.low_latency_dispatch_gemm(lx, lidx, T, E_ll, mw1, mw1s)
        buf.low_latency_combine(ly, lidx, lw, hh)

    bw = (torch.randn((e_g, k1, n1), generator=g) * 0.02).to(torch.bfloat16).cuda()  # [E, k, n] as it lies
    bk = bw.transpose(1, 2).contiguous()                                              # [E, n, k]
    ba = torch.randn((rows_per * e_g, k1), generator=g).to(torch.bfloat16).cuda()
    bg = torch.randn((rows_per * e_g, n1), generator=g).to(torch.bfloat16).cuda()

    def bf16_gemm():
        gemm.grouped_gemm_bf16(ba, bk, goff, gcnt)

    def bf16_mn():
        gemm.grouped_gemm_bf16(ba, bw, goff, gcnt, b_mn_major=True)

    def bf16_wgrad():
        gemm.grouped_gemm_bf16_wgrad_rows(bg, ba, goff)

    fw, fws = gemm.quantize_weights_fp8((torch.randn((E, n_small, H), device='cuda') * 0.02).to(torch.bfloat16))
    fws = fws.contiguous()

    def fused_dispatch_gemm():
        h, grp, hnd = buf.dispatch_gemm(x, idx, w.float().contiguous(), E, fw, fws)
        buf.combine(y_recv[:hnd[3].shape[0]], hnd, topk_weights=grp['topk_weights'])

    # MoE backward helpers on the grouped layout of the dispatch workload's tokens
    def moe_backward_ops():
        (rx, rs), ri, rw, _, h, _ = state['disp']
        if 'perm' not in state:
            combine_expanded()
        pm = state['perm']
        R = int(pm.expert_offsets[-1])
        g_y = torch.zeros((R, H), dtype=torch.bfloat16, device='cuda')
        permute.unpermute_backward(y_recv[:rx.shape[0]], pm.row_map, rw, state['y_exp'][:R], g_y)
        quant.swiglu_backward(state['h'], state['h'][:, :n1 // 2].contiguous())
        permute.zero_group_padding([pm.x, pm.scales], pm.expert_offsets, pm.expert_counts)

    probe_src = torch.randint(0, 256, ((32 << 20) + 64,), generator=g, dtype=torch.int32).to(torch.uint8).cuda()

    def transport_checks():
        buf.transport_selftest(64, 8, 16)
        require_ext().window_check(torch.tensor([[0, 1, 1], [5, 6, 10]], dtype=torch.int64, device='cuda'))
        buf.runtime.sample_clock()  # the trace clock alignment's %globaltimer read
        buf.runtime.probe_flag_latency(0, 100)  # NVLink micro-probes against this GPU's own mapping
        buf.runtime.probe_peer_copy(0, 32 << 20, 0, True, 1, 296, probe_src)

    def ll_clean():
        buf.clean_low_latency_buffer(T, H, E_ll)

    from deepep_slingshot_b200 import ElasticBuffer
    side = {}

    def side_features():
        if not side:
            side['buf'] = ElasticBuffer(dist.group.WORLD, num_max_tokens_per_rank=64, hidden=256, num_topk=2)
            side['buf'].pp_set_config(8 << 20, 2)
            side['buf'].agrs_set_config(32 << 20, 4)
            side['buf'].engram_write(torch.randn((4096, 1024), generator=g).to(torch.bfloat16).cuda())
            side['payload'] = torch.randint(0, 256, (8 << 20,), generator=g, dtype=torch.uint8).cuda()
            side['idx'] = torch.randint(0, 4096, (2048,), generator=g, dtype=torch.int32).cuda()
        sb = side['buf']
        sb.pp_send(side['payload'], 0)
        got = torch.empty_like(side['payload'])
        sb.pp_recv(got, 0)
        with sb.agrs_new_session():
            gathered, hook = sb.all_gather(side['payload'][:1 << 20].view(torch.int32))
            hook()
        sb.engram_fetch(side['idx'])()

    work = {'layout': layout, 'dispatch': dispatch, 'combine': combine, 'low_latency': ll, 'cast': cast,
            'grouped_gemm': grouped_gemm, 'grouped_gemm_ue8m0': grouped_gemm_ue8m0, 'swiglu_quant': swiglu, 'permute': perm, 'barrier': barrier}
    work.update({'quantize_weights': quantize_weights, 'combine_expanded': combine_expanded, 'll_logfmt': ll_logfmt,
                 'masked_gemm': masked_gemm, 'll_dispatch_gemm': ll_dispatch_gemm, 'bf16_gemm': bf16_gemm,
                 'bf16_mn': bf16_mn, 'bf16_wgrad': bf16_wgrad, 'fused_dispatch_gemm': fused_dispatch_gemm,
                 'moe_backward_ops': moe_backward_ops, 'transport_checks': transport_checks, 'll_clean': ll_clean,
                 'side_features': side_features, 'gemm_combine': gemm_combine,
                 'gemm_then_combine': gemm_then_combine})
    return work


def main():
    p = argparse.ArgumentParser()
    p.add_argument('--only', default='')
    p.add_argument('--tokens', type=int, default=4096)
    p.add_argument('--hidden', type=int, default=7168)
    p.add_argument('--experts', type=int, default=256)
    p.add_argument('--topk', type=int, default=8)
    p.add_argument('--inter', type=int, default=2048)
    p.add_argument('--ll-tokens', type=int, default=128)
    p.add_argument('--ll-experts', type=int, default=64)
    p.add_argument('--gemm-rows', type=int, default=1024)
    p.add_argument('--gemm-experts', type=int, default=4)
    p.add_argument('--time', type=int, default=0, help='timed repetitions per workload (0: profile pass only)')
    args = p.parse_args()
    _init_single_rank()
    work = build(args)
    wanted = set(args.only.split(',')) if args.only else set(work)
    names = [n for n in work if n in wanted]
    for n in names:  # warm-up outside the profiled range
        work[n]()
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push('profile')
    for n in names:
        work[n]()
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    print('kernel workloads done:', ','.join(names))
    if args.time > 0:
        flush = torch.empty(256 << 20, dtype=torch.uint8, device='cuda')
        for n in names:
            ts = []
            for _ in range(args.time):
                flush.fill_(1)
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda.synchronize()
                s.record()
                work[n]()
                e.record()
                torch.cuda.synchronize()
                ts.append(s.elapsed_time(e) * 1e3)
            ts.sort()
            print(f'time {n}: median {ts[len(ts) // 2]:.1f} us, min {ts[0]:.1f} us')
    dist.destroy_process_group()


if __name__ == '__main__':
    main()
