"""Dispatch / combine benchmark over (mode, model preset, tokens per rank, routing, fp8).

Each case is an ``OpPlan``: the three calls to time (send = dispatch, back = combine,
both = dispatch then combine), a check that identity experts give back what the
sources sent, the logical and wire bytes of the case, and the rows each rank
receives. ``measure`` times every call back to back and with a synchronisation after
each call (see ``harness.device_stats``), records the first call's host time and the
per-stage device times of the Buffer's stage timer, and derives GB/s and the load
spread over the EP group. One JSON line per case goes to ``ops_ep<R>.jsonl``.

torchrun --nnodes 1 --nproc-per-node 8 --master-addr 127.0.0.1 bench/bench_ops.py --modes normal,low_latency
"""
from __future__ import annotations

import json
from dataclasses import dataclass, field
from typing import Callable

from harness import PRESETS, ROUTINGS, BenchGroup, cli, device_stats, env_record, gbps, ints, make_routing, wall_once, \
    words, write_jsonl

import torch

from deepep_trn_b200.utils.profiling import timer


@dataclass
class OpPlan:
    send: Callable
    back: Callable
    both: Callable
    ok: bool
    logical: tuple[int, int]       # (dispatch, combine) bytes per rank as the reference counts them
    wire: tuple[int, int]          # bytes per rank that cross the transport
    rows: int                      # rows (normal) or (token, expert) pairs (low latency) received
    first_s: dict = field(default_factory=dict)


def normal_plan(bg, buf, x, idx, w, E, fp8) -> OpPlan:
    H = x.shape[1]
    ntr, _, nte, itr, _ = buf.get_dispatch_layout(idx, E)
    layout = dict(topk_idx=idx, topk_weights=w, num_tokens_per_rank=ntr, is_token_in_rank=itr,
                  num_tokens_per_expert=nte, use_fp8=fp8)
    send = lambda: buf.dispatch(x, **layout)
    res, t_send = wall_once(bg, send)
    rx, handle = res[0], res[4]
    if fp8:
        from deepep_trn_b200.ops.quant import dequantize_fp8
        rx = dequantize_fp8(*rx)
    back = lambda: buf.combine(rx, handle)
    (y, _, _), t_back = wall_once(bg, back)

    def both():
        r = send()
        return buf.combine(rx if fp8 else r[0], r[4])
    want = (x.float() * itr.sum(1, keepdim=True)).to(torch.bfloat16)
    ok = torch.equal(y, want) if not fp8 else torch.allclose(y.float(), want.float(), rtol=0.07, atol=0.05)
    n = int(handle.recv_counts.sum())
    row = H + H // 32 if fp8 else 2 * H
    return OpPlan(send, back, both, bool(ok), (n * 2 * H, n * 2 * H), (n * row, n * 2 * H), n,
                  {'dispatch': round(t_send, 4), 'combine': round(t_back, 4)})


def low_latency_plan(bg, buf, x, idx, w, E, fp8) -> OpPlan:
    T, H = x.shape
    R = buf.group_size
    send = lambda: buf.low_latency_dispatch(x, idx, T, E, use_fp8=fp8)
    res, t_send = wall_once(bg, send)
    recv, counts, handle = res[0], res[1], res[2]
    xin = (recv[0].float() * recv[1].repeat_interleave(128, -1)) if fp8 else recv.float()
    xin = xin.to(torch.bfloat16)
    back = lambda: buf.low_latency_combine(xin, idx, w, handle)
    (y, _, _), t_back = wall_once(bg, back)

    def both():
        r = send()
        return buf.low_latency_combine(xin, idx, w, r[2])
    want = x.float() * (w * (idx >= 0)).sum(-1, keepdim=True)
    ok = torch.allclose(y.float(), want, rtol=0.07 if fp8 else 1e-2, atol=0.05 if fp8 else 1e-3)
    pairs = int((idx >= 0).sum())
    owner = torch.where(idx >= 0, idx // (E // R), -1)
    ranks = int(sum((owner == r).any(1).sum() for r in range(R)))
    row = H + H // 32 if fp8 else 2 * H
    return OpPlan(send, back, both, bool(ok), (pairs * 2 * H, pairs * 2 * H), (ranks * row, pairs * 2 * H),
                  int(counts.sum()), {'dispatch': round(t_send, 4), 'combine': round(t_back, 4)})


def stage_times(bg, fn, calls=3) -> dict:
    """Per-stage device time of the Buffer's stage timer, max over ranks."""
    timer.enabled, timer.use_cuda_events = True, bg.device.type == 'cuda'
    timer.sync = None if bg.device.type == 'cuda' else bg.sync
    timer.reset()
    for _ in range(calls):
        fn()
    bg.sync()
    mine = timer.per_call_us(calls)
    timer.enabled = timer.use_cuda_events = False
    timer.reset()
    all_ranks = bg.gather(mine)
    return {k: round(max(d.get(k, 0.0) for d in all_ranks), 2) for k in sorted({k for d in all_ranks for k in d})}


def measure(bg, args, plan: OpPlan) -> dict:
    rec = {'first_call_s': plan.first_s}
    for name in ('send', 'back', 'both'):
        fn = getattr(plan, name)
        rec[f'{name}_us'] = device_stats(bg, fn, args.rounds, args.iters)
        rec[f'{name}_latency_us'] = device_stats(bg, fn, args.rounds, args.iters, each=True)
    rec['stages_us'] = {'send': stage_times(bg, plan.send), 'back': stage_times(bg, plan.back)}
    group = bg.over_group({'ok': plan.ok, 'rows': plan.rows, 'logical': plan.logical, 'wire': plan.wire})
    rows = [g['rows'] for g in group]
    mean_rows = sum(rows) / len(rows)
    rec['check'] = 'PASS' if all(g['ok'] for g in group) else 'FAIL'
    rec['rows'] = {'min': min(rows), 'max': max(rows), 'imbalance': round(max(rows) / max(mean_rows, 1e-9), 3)}
    avg = lambda key, i: sum(g[key][i] for g in group) / len(group)
    rec['bytes_per_rank'] = {'logical': [avg('logical', 0), avg('logical', 1)], 'wire': [avg('wire', 0), avg('wire', 1)]}
    lg = rec['bytes_per_rank']['logical']
    rec['gbps_per_rank'] = {'send': gbps(lg[0], rec['send_us']['median_us']),
                            'back': gbps(lg[1], rec['back_us']['median_us']),
                            'both': gbps(lg[0] + lg[1], rec['both_us']['median_us'])}
    return rec


def main():
    p = cli(__doc__)
    p.add_argument('--modes', type=words, default=['normal', 'low_latency'])
    p.add_argument('--routings', type=words, default=['random'])
    p.add_argument('--fp8', type=ints, default=[0])
    args = p.parse_args()
    bg = BenchGroup(args.backend, args.ep)
    if bg.rank == 0:
        args.out_dir.mkdir(parents=True, exist_ok=True)
        (args.out_dir / 'env.json').write_text(json.dumps(env_record(), indent=2))
    M = max(args.tokens)
    H, E = max(PRESETS[n][0] for n in args.presets), max(PRESETS[n][1] for n in args.presets)
    extra = dict(hidden=H, num_experts=E, topk=8, num_max_dispatch_tokens_per_rank=min(M, 256)) \
        if args.backend == 'nvlink' else {}
    buf = bg.new_buffer(M, **extra)
    for mode in args.modes:
        for preset in args.presets:
            H, E, K = PRESETS[preset]
            for T in args.tokens:
                if mode == 'low_latency' and T > 256:
                    continue
                for routing in args.routings:
                    for fp8 in map(bool, args.fp8):
                        if fp8 and mode == 'normal' and args.backend != 'nvlink':
                            continue
                        seed = 104729 * T + 17 * bg.rank + ROUTINGS.index(routing)
                        idx, w = make_routing(routing, T, E, K, bg.ep, bg.ep_rank, seed)
                        x = torch.randn(T, H, generator=torch.Generator().manual_seed(seed)).to(torch.bfloat16)
                        x, idx, w = x.to(bg.device), idx.to(bg.device), w.to(bg.device)
                        make = normal_plan if mode == 'normal' else low_latency_plan
                        rec = dict(bench='ops', mode=mode, preset=preset, hidden=H, experts=E, topk=K, ep=bg.ep,
                                   tokens=T, routing=routing, fp8=fp8, backend=args.backend)
                        rec.update(measure(bg, args, make(bg, buf, x, idx, w, E, fp8)))
                        if bg.rank == 0:
                            write_jsonl(args.out_dir / f'ops_ep{bg.ep}.jsonl', rec)
                            print(f"[ops] {mode} {preset} ep={bg.ep} T={T} {routing} fp8={int(fp8)} {rec['check']}: "
                                  f"send/back/both {rec['send_us']['median_us']}/{rec['back_us']['median_us']}/"
                                  f"{rec['both_us']['median_us']} us, {rec['gbps_per_rank']['both']} GB/s per rank, "
                                  f"imbalance {rec['rows']['imbalance']}", flush=True)
    buf.destroy()
    bg.close()


if __name__ == '__main__':
    main()
