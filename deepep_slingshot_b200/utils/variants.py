"""Kernel variant table: every sm_100a kernel entry of the extension, its resources as built, and the
rule that selects it at run time.

The reference compiles kernel variants on demand (its JIT keys a compiled variant by template
arguments and rejects one whose ptxas report shows local-memory use). This library compiles every
variant ahead of time for sm_100a; the build (`setup.py`) records each entry's ptxas report
(registers, barriers, static shared memory, stack, spill stores / loads) in
`deepep_slingshot_b200/kernel_variants.json`, and a spill fails the build. This module joins that
record with the selection rules below.

    python -m deepep_slingshot_b200.utils.variants          # one line per kernel entry
"""
import json
import os
import re
from typing import Dict, List, Optional

TABLE = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), 'kernel_variants.json')

# kernel base name -> how an instance is chosen at run time (template arguments or launch switches)
SELECTION: Dict[str, str] = {
    'dispatch_layout_kernel': 'get_dispatch_layout',
    'dispatch_count_kernel': 'normal dispatch, fresh or cached handle (a cached handle with the concurrent stage skips it)',
    'dispatch_stage_kernel': 'DEEPEP_B200_DISPATCH_STAGE=concurrent (default) and the fused dispatch + GEMM; chunk counters at GPU scope with DEEPEP_B200_STAGE_SIGNAL_SCOPE=gpu',
    'dispatch_pull_kernel': 'normal dispatch; stage warps inside it with DEEPEP_B200_DISPATCH_STAGE=warps',
    'combine_kernel': '<false>: rows per received token; <true>: expanded rows (combine(..., row_map=...)), weighted on the sender',
    'barrier_kernel': 'Buffer.barrier',
    'read_globaltimer_kernel': 'trace clock alignment',
    'll_dispatch_kernel': 'low_latency_dispatch',
    'll_combine_kernel': '<false>: bf16 send; <true>: LogFMT-10 send (use_logfmt=True)',
    'll_clean_kernel': 'clean_low_latency_buffer',
    'per_token_cast_to_fp8_kernel': 'ops.quant.per_token_cast_to_fp8',
    'per_token_cast_back_kernel': 'ops.quant.per_token_cast_back',
    'quantize_weights_fp8_kernel': 'ops.gemm.quantize_weights_fp8',
    'swiglu_quant_kernel': 'ops.quant.swiglu_quant',
    'grouped_gemm_fp8_kernel': '<256, *>: N % 256 == 0 (default), <128, *>: otherwise or DEEPEP_B200_GEMM_BN=128; '
                               '<*, true>: GemmCombine.send (the combine send as the epilogue)',
    'gc_row_dest_kernel': 'GemmCombine.send (destination of every operand row)',
    'gc_reduce_kernel': 'GemmCombine.reduce (source-side top-k weighted sum of the combine slots)',
    'grouped_gemm_fp8_bs_kernel': 'grouped_gemm_fp8(..., ue8m0=True) (power-of-two scales, block-scaled MMA)',
    'grouped_gemm_fp8_pair_kernel': 'N % 256 == 0 (CTA pairs, cta_group::2) and DEEPEP_B200_GEMM_PAIR=1 (<16>: 16 epilogue '
                                    'warps) or =2 (<8>: 8 epilogue warps, pipelined promotion)',
    'grouped_gemm_bf16_kernel': '<A MN-major, B MN-major>: operand layouts of grouped_gemm_bf16 / _wgrad_rows',
    'masked_gemm_fp8_kernel': 'ops.gemm.masked_grouped_gemm_fp8, low_latency_dispatch_gemm, low_latency_gemm_combine',
    'fused_dispatch_gemm_kernel': 'Buffer.dispatch_gemm (DEEPEP_B200_MOE_FUSED_DISPATCH=1 in the MoE layer)',
    'permute_count_kernel': 'ops.permute.permute',
    'permute_scan_kernel': 'ops.permute.permute',
    'permute_rowmap_kernel': 'ops.permute.permute',
    'permute_copy_kernel': 'ops.permute.permute',
    'permute_zero_padding_kernel': 'permute(..., zero_padding=True)',
    'unpermute_kernel': 'ops.permute.unpermute',
    'unpermute_backward_kernel': '<8>: top-k <= 8, <16>: top-k <= 16',
    'swiglu_backward_kernel': 'ops.quant.swiglu_backward',
    'zero_group_padding_kernel': 'ops.permute.zero_group_padding',
    'signal_stress_kernel': 'Buffer.transport_selftest',
    'window_check_kernel': 'window_check (transport contract tests)',
    'flag_pingpong_kernel': 'harness.nvlink_probe.flag_latency',
    'probe_copy_kernel': 'harness.nvlink_probe.copy_sweep / peer_matrix',
    'pp_copy_kernel': 'ElasticBuffer pp_send / pp_recv',
    'signal_wait_kernel': 'AGRS sessions, PP',
    'engram_fetch_kernel': 'ElasticBuffer engram_fetch',
}


def parse_ptxas(log: str, csrc_root: str = '') -> Dict[str, List[dict]]:
    """{source (relative to `csrc_root`): [kernel entry records]} from the `ptxas -v` lines of a build
    log. ninja prints each command with its output; an entry's lines follow the nvcc command that
    compiled its translation unit. Records: mangled name, arch, stack, spill stores / loads,
    registers, barriers, static shared memory."""
    out: Dict[str, List[dict]] = {}
    source, entry = None, None
    for line in log.splitlines():
        m = re.search(r"nvcc .* -c (?:-c )?(\S+\.cu) -o ", line)
        if m:
            path = m.group(1)
            source = os.path.relpath(path, csrc_root) if csrc_root and os.path.isabs(path) else path
            out.setdefault(source, [])
            continue
        m = re.search(r"Compiling entry function '([^']+)' for '(sm_\w+)'", line)
        if m and source is not None:
            entry = {'mangled': m.group(1), 'arch': m.group(2)}
            out[source].append(entry)
            continue
        if entry is None:
            continue
        m = re.search(r"(\d+) bytes stack frame, (\d+) bytes spill stores, (\d+) bytes spill loads", line)
        if m:
            entry.update(stack=int(m.group(1)), spill_stores=int(m.group(2)), spill_loads=int(m.group(3)))
            continue
        m = re.search(r"Used (\d+) registers(?:, used (\d+) barriers)?(?:, (\d+) bytes smem)?", line)
        if m:
            entry.update(registers=int(m.group(1)), barriers=int(m.group(2) or 0), smem_static=int(m.group(3) or 0))
            entry = None
    return out


def base_name(demangled: str) -> str:
    """`ep::grouped_gemm_fp8_kernel<256>(...)` -> `grouped_gemm_fp8_kernel`."""
    head = demangled.split('(', 1)[0]
    head = re.sub(r'<.*>$', '', head)
    return head.split('::')[-1].replace('void ', '').strip()


def load(path: Optional[str] = None) -> List[dict]:
    """Every kernel entry of the last build: source, name, resources, selection rule. Raises
    FileNotFoundError before the extension was built."""
    with open(path or TABLE) as f:
        table = json.load(f)
    rows = []
    for src, entries in table['sources'].items():
        for e in entries:
            r = dict(e, source=src, base=base_name(e.get('name', e['mangled'])))
            r['selected_by'] = SELECTION.get(r['base'], '')
            rows.append(r)
    return rows


def main() -> None:
    rows = load()
    print(f"{'kernel':70s} {'regs':>5s} {'smem':>6s} {'stack':>5s} {'spill':>5s}  selected by")
    for r in sorted(rows, key=lambda r: (r['source'], r['name'])):
        spill = r.get('spill_stores', 0) + r.get('spill_loads', 0)
        print(f"{r['name'][:70]:70s} {r.get('registers', 0):5d} {r.get('smem_static', 0):6d} {r.get('stack', 0):5d} "
              f"{spill:5d}  {r['selected_by']}")


if __name__ == '__main__':
    main()
