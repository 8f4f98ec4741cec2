"""DeepEP-style op benchmark: normal (dispatch / combine) and low-latency modes.

For every (mode, preset, tokens, routing) case: a correctness check with identity
experts, first-call time, device time of dispatch, combine and dispatch+combine
(pipelined and per-call latency), the stage breakdown, bytes (logical, wire) and
the load imbalance. Same case structure as the reference's bench/bench_ops.py.

torchrun --nnodes 1 --nproc-per-node 8 --master-addr 127.0.0.1 bench/bench_ops.py --modes normal,low_latency
"""
from common import PRESETS, ROUTINGS, Ctx, append_jsonl, base_parser, csv_list, env_record, gbps, make_routing

import torch

from deepep_trn_b200.utils.profiling import timer


def breakdown(ctx, call, calls: int) -> dict:
    timer.enabled, timer.use_cuda_events = True, ctx.device.type == 'cuda'
    timer.sync = ctx.sync if ctx.device.type != 'cuda' else None
    timer.reset()
    for _ in range(calls):
        call()
    ctx.sync()
    mine = timer.per_call_us(calls)
    timer.enabled, timer.use_cuda_events = False, False
    timer.reset()
    everyone = ctx.gather(mine)
    stages = sorted({k for d in everyone for k in d})
    return {s: round(max(d.get(s, 0.0) for d in everyone), 2) for s in stages}


def bench_case(ctx, args, buf, mode, preset, T, routing, fp8):
    H, E, K = PRESETS[preset]
    R = ctx.ep
    seed = 7919 * T + 31 * ctx.rank + ROUTINGS.index(routing)
    idx, w = make_routing(routing, T, E, K, R, ctx.ep_rank, seed)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(seed)).to(torch.bfloat16)
    d_x, d_idx, d_w = x.to(ctx.device), idx.to(ctx.device), w.to(ctx.device)
    measure = lambda call, sync_each=False: ctx.measure(call, args.rounds, args.iters, sync_each)
    if mode == 'normal':
        ntr, _, nte, itr, _ = buf.get_dispatch_layout(d_idx, E)

        def dispatch():
            return buf.dispatch(d_x, topk_idx=d_idx, topk_weights=d_w, num_tokens_per_rank=ntr,
                                is_token_in_rank=itr, num_tokens_per_expert=nte, use_fp8=fp8)

        out, first_d = ctx.first_call(dispatch)
        recv_x, handle = out[0], out[4]
        if fp8:
            from deepep_trn_b200.utils.codec import dequantize_fp8_1x128
            recv_bf = dequantize_fp8_1x128(*recv_x).to(torch.bfloat16)
        else:
            recv_bf = recv_x

        def combine():
            return buf.combine(recv_bf, handle)

        (combined, _, _), first_c = ctx.first_call(combine)

        def both():
            r = dispatch()
            return buf.combine(recv_bf if fp8 else r[0], r[4])

        ref = (x.float() * itr.cpu().sum(1, keepdim=True)).to(torch.bfloat16)
        if fp8:
            passed = bool(torch.allclose(combined.cpu().float(), ref.float(), rtol=0.07, atol=0.05))
        else:
            passed = bool(torch.equal(combined.cpu(), ref))
        recv_rows = int(handle.recv_counts.sum())
        row_bytes = H * (1 if fp8 else 2) + (H // 128 * 4 if fp8 else 0)
        logical_d = logical_c = recv_rows * H * 2
        wire_d, wire_c = recv_rows * row_bytes, recv_rows * H * 2
        load = recv_rows
    else:
        def dispatch():
            return buf.low_latency_dispatch(d_x, d_idx, T, E, use_fp8=fp8)

        out, first_d = ctx.first_call(dispatch)
        recv_x, handle = out[0], out[2]
        EL = E // R
        y = torch.randn(EL, R * T, H, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16).to(ctx.device)

        def combine():
            return buf.low_latency_combine(y, d_idx, d_w, handle)

        _, first_c = ctx.first_call(combine)

        def both():
            r = dispatch()
            return buf.low_latency_combine(y, d_idx, d_w, r[2])

        # correctness: identity experts on the received rows
        xin = recv_x[0].float() * recv_x[1].repeat_interleave(128, -1) if fp8 else recv_x.float()
        (got, _, _) = buf.low_latency_combine(xin.to(torch.bfloat16), d_idx, d_w, handle)
        ref = x.float() * (w * (idx >= 0)).sum(-1, keepdim=True)
        passed = bool(torch.allclose(got.cpu().float(), ref, rtol=0.07 if fp8 else 1e-2, atol=0.05 if fp8 else 1e-3))
        selections = int((idx >= 0).sum())
        logical_d = logical_c = selections * H * 2
        rank_rows = int((torch.zeros(T, R, dtype=torch.bool).scatter_(
            1, torch.where(idx >= 0, idx // (E // R), torch.zeros_like(idx)), idx >= 0)).sum())
        wire_d = rank_rows * (H + H // 32 if fp8 else 2 * H)
        wire_c = selections * H * 2
        load = int(out[1].sum())
    record = dict(
        bench='ops', mode=mode, preset=preset, hidden=H, experts=E, topk=K, ep=R, tokens=T, routing=routing,
        fp8=fp8, backend=ctx.backend, check=dict(passed=passed),
        first_call_s=dict(dispatch=round(first_d, 4), combine=round(first_c, 4)),
        device_us=dict(dispatch=measure(dispatch), combine=measure(combine), dispatch_combine=measure(both)),
        latency_us=dict(dispatch=measure(dispatch, True), combine=measure(combine, True)),
        breakdown_us=dict(dispatch=breakdown(ctx, dispatch, 3), combine=breakdown(ctx, combine, 3)),
    )
    peers = ctx.peer_values(dict(ld=logical_d, lc=logical_c, wd=wire_d, wc=wire_c, load=load, passed=passed))
    mean = lambda k: sum(p[k] for p in peers) / len(peers)
    record['check']['passed'] = all(p['passed'] for p in peers)
    loads = [p['load'] for p in peers]
    record['recv_load'] = dict(min=min(loads), max=max(loads), mean=round(sum(loads) / len(loads), 1),
                               imbalance=round(max(loads) / max(sum(loads) / len(loads), 1e-9), 3))
    record['bytes_per_rank'] = dict(logical_dispatch=mean('ld'), logical_combine=mean('lc'),
                                    wire_dispatch=mean('wd'), wire_combine=mean('wc'))
    b, d = record['bytes_per_rank'], record['device_us']
    record['gbps_per_rank'] = dict(dispatch=gbps(b['logical_dispatch'], d['dispatch']['median_us']),
                                   combine=gbps(b['logical_combine'], d['combine']['median_us']),
                                   dispatch_combine=gbps(b['logical_dispatch'] + b['logical_combine'],
                                                         d['dispatch_combine']['median_us']))
    return record


def main():
    p = base_parser(__doc__)
    p.add_argument('--modes', type=csv_list(str), default=['normal', 'low_latency'])
    p.add_argument('--routings', type=csv_list(str), default=['random'])
    p.add_argument('--fp8', type=csv_list(int), default=[0])
    args = p.parse_args()
    ctx = Ctx(args.backend, args.ep)
    if ctx.rank == 0:
        args.out_dir.mkdir(parents=True, exist_ok=True)
        (args.out_dir / 'env.json').write_text(__import__('json').dumps(env_record(), indent=2))
    maxT = max(args.tokens)
    H, E, K = max(PRESETS[p][0] for p in args.presets), max(PRESETS[p][1] for p in args.presets), 8
    buf = ctx.buffer(maxT, hidden=H, num_experts=E, topk=K, num_max_dispatch_tokens_per_rank=maxT) \
        if args.backend == 'nvlink' else ctx.buffer(maxT)
    for mode in args.modes:
        for preset in args.presets:
            for T in args.tokens:
                for routing in args.routings:
                    for fp8 in args.fp8:
                        if fp8 and args.backend != 'nvlink' and mode == 'normal':
                            continue
                        if mode == 'low_latency' and T > 256:
                            continue
                        rec = bench_case(ctx, args, buf, mode, preset, T, routing, bool(fp8))
                        if ctx.rank == 0:
                            append_jsonl(args.out_dir / f'ops_ep{ctx.ep}.jsonl', rec)
                            d = rec['device_us']
                            print(f"[ops] {mode} {preset} ep={ctx.ep} T={T} {routing} fp8={fp8}: "
                                  f"check={'PASS' if rec['check']['passed'] else 'FAIL'} "
                                  f"d/c/d+c={d['dispatch']['median_us']}/{d['combine']['median_us']}/"
                                  f"{d['dispatch_combine']['median_us']}us "
                                  f"GB/s/rank d+c={rec['gbps_per_rank']['dispatch_combine']} "
                                  f"imbalance={rec['recv_load']['imbalance']}", flush=True)
    buf.destroy()
    ctx.finish()


if __name__ == '__main__':
    main()
