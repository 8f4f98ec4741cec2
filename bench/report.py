"""Aggregate a results directory into summary.md and ops.csv (reference: bench/report.py).

Reads ``ops_ep*.jsonl`` (bench/bench_ops.py), ``transport_ep*.jsonl``, ``baselines_ep*.jsonl``,
``moe_ep*.jsonl``, ``gemm.jsonl`` and ``headline_*.jsonl`` (the JSON lines of bench.py).

python bench/report.py results/<run_id>
"""
from __future__ import annotations

import csv
import json
import sys
from pathlib import Path


def load(run: Path, prefix: str) -> list[dict]:
    rows = []
    for path in sorted(run.glob(f'{prefix}_ep*.jsonl')):
        rows += [json.loads(line) for line in path.read_text().splitlines() if line.strip()]
    return rows


def med(d):
    return d['median_us'] if d else None


def fmt(v):
    if v is None:
        return '-'
    if isinstance(v, float):
        return f'{v:.4g}' if abs(v) < 10 else f'{v:.2f}'
    return str(v)


def table(header, rows):
    out = ['| ' + ' | '.join(header) + ' |', '|' + '---|' * len(header)]
    out += ['| ' + ' | '.join(fmt(c) for c in r) + ' |' for r in rows]
    return '\n'.join(out)


def main():
    run = Path(sys.argv[1])
    ops, tr, bl = load(run, 'ops'), load(run, 'transport'), load(run, 'baselines')
    env = json.loads((run / 'env.json').read_text()) if (run / 'env.json').exists() else {}
    parts = [f'# deepep_trn_b200 benchmark: {run.name}', '', f'- env: {env}', '',
             'Device time (CUDA events), max over ranks, median of rounds. Logical bytes follow deep_ep '
             '(normal: received rows x H x 2; LL: selected experts x H x 2).', '']
    if ops:
        rows = [[r['mode'], r['preset'], r['ep'], r['tokens'], r['routing'], r.get('fp8'), r['check'],
                 med(r['send_us']), med(r['back_us']), med(r['both_us']), med(r['send_latency_us']),
                 med(r['back_latency_us']), r['gbps_per_rank']['both'], r['rows']['imbalance']]
                for r in sorted(ops, key=lambda r: (r['mode'], r['preset'], r['ep'], r['tokens'], r['routing']))]
        parts += ['## Ops', '', table(['mode', 'preset', 'EP', 'T/rank', 'routing', 'fp8', 'check', 'dispatch us',
                                       'combine us', 'd+c us', 'latency d us', 'latency c us', 'GB/s/rank d+c',
                                       'imbalance'], rows), '']
        with open(run / 'ops.csv', 'w', newline='') as f:
            w = csv.writer(f)
            w.writerow(['mode', 'preset', 'ep', 'tokens', 'routing', 'fp8', 'check', 'dispatch_us', 'combine_us',
                        'dc_us', 'gbps_rank_dc'])
            for r in ops:
                w.writerow([r['mode'], r['preset'], r['ep'], r['tokens'], r['routing'], r.get('fp8'), r['check'],
                            med(r['send_us']), med(r['back_us']), med(r['both_us']), r['gbps_per_rank']['both']])
    if tr:
        rows = [[r['ep'], r['engine'], r['chunk'], r['mib_per_peer'], med(r['device_us']), r['gbps_per_gpu']]
                for r in tr]
        parts += ['## NVLink engines (all-to-all, every rank to every peer at once)', '',
                  table(['EP', 'engine', 'bytes/transfer', 'MiB/peer', 'us', 'off-rank GB/s per GPU'], rows), '']
    if bl:
        rows = [[r['op'], r['preset'], r['ep'], r['tokens'], med(r.get('device_us')), med(r.get('latency_us')),
                 r.get('error', '')] for r in bl]
        parts += ['## NCCL collective baselines', '',
                  table(['op', 'preset', 'EP', 'T/rank', 'pipelined us', 'latency us', 'error'], rows), '']
    heads = []
    for path in sorted(run.glob('headline_*.jsonl')):
        heads += [json.loads(line) for line in path.read_text().splitlines() if line.startswith('{')]
    if heads:
        rows = []
        for r in sorted(heads, key=lambda r: (r.get('impl', ''), r.get('n_gpus', 0), r.get('dtype', ''))):
            ll, nc, e2e = r.get('ll') or {}, r.get('nccl') or {}, r.get('e2e') or {}
            roof = (r.get('roofline') or {}).get('of_measured_770')
            rows.append([r.get('impl'), r.get('n_gpus'), r.get('dtype'), r.get('check'), r.get('ms_per_step'),
                         r.get('value'), r.get('per_gpu_gbps'), r.get('offrank_gbps_per_gpu'), roof,
                         nc.get('ms_per_step'), r.get('vs_baseline'), ll.get('dispatch_fp8_plus_combine_us'),
                         (nc.get('ll') or {}).get('dispatch_fp8_plus_combine_us'), e2e.get('value'),
                         (r.get('clocks') or {}).get('sm_mhz')])
        parts += ['## Headline (`bench.py`: 4096 tokens per rank, H=7168, top-8 of 256; LL at 128 tokens)', '',
                  table(['impl', 'GPUs', 'dtype', 'check', 'ms/step', 'GB/s (sum)', 'GB/s/GPU', 'off-rank GB/s/GPU',
                         'of 770', 'NCCL ms/step', 'vs NCCL', 'LL us', 'NCCL LL us', 'e2e GB/s', 'SM MHz'], rows), '']
    moe = load(run, 'moe')
    if moe:
        rows = []
        for r in moe:
            for impl in ('ours', 'nccl'):
                if impl in r:
                    rows.append([r.get('pass_', 'forward+backward'), r['ep'], r['experts'], r['tokens'],
                                 r.get('dispatch_dtype', 'bf16'), r.get('expert_gemm_dtype', 'bf16'), impl,
                                 r[impl]['ms_per_step'], r[impl]['tokens_per_s'], r[impl]['expert_tflops_per_rank']])
        parts += ['## MoE layer (`bench/bench_moe.py`)', '',
                  table(['pass', 'EP', 'experts', 'T/rank', 'dispatch', 'expert GEMMs', 'impl', 'ms/step', 'tokens/s',
                         'expert TFLOP/s/rank'], rows), '']
    gemm_file = run / 'gemm.jsonl'
    if gemm_file.exists():
        recs = [json.loads(line) for line in gemm_file.read_text().splitlines() if line.startswith('{')]
        rows = [[k, v['ms'], v['tflops']] for r in recs for k, v in r.items() if isinstance(v, dict) and 'tflops' in v]
        parts += ['## Grouped GEMM (`bench/bench_gemm.py`)', '', table(['GEMM', 'ms', 'TFLOP/s'], rows), '']
    (run / 'summary.md').write_text('\n'.join(parts))
    print(f'wrote {run / "summary.md"}')


if __name__ == '__main__':
    main()
