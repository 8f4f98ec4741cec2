#!/usr/bin/env python
"""Headline benchmark: normal-mode dispatch + combine NVLink GB/s at 4096 tokens per rank
(H=7168, top-8 of 256 experts, bf16), plus low-latency fp8 dispatch + bf16 combine latency
at 128 tokens per rank (CUDA graph).

    python bench.py --gpus N --steps K --warmup W [--impl ours|reference|nccl]

For N > 1 launch under torchrun (one rank per GPU); rank 0 prints one JSON line.

Timing: W untimed warm-up steps, then exactly K steps between a barrier and a
device synchronisation on both sides; each step is timed with CUDA events on the
launching stream after an untimed L2 flush (a 256 MiB write), and the total is the
max over ranks. ``value`` is the whole-job aggregate: the sum over ranks of the bytes
each rank receives in dispatch and in combine, divided by the max-over-ranks step
time (``per_gpu_gbps`` = value / N). ``offrank_gbps_per_gpu`` counts only rows that
cross NVLink, and ``roofline`` divides it by the link bandwidth (900 GB/s nominal per
direction, 770 GB/s measured peer copy on this pool).

``e2e`` is the same metric through the public API with, inside every timed step, the
step's inputs copied from pinned host memory and the combined result copied back to
pinned host memory.

Arms:
  ours       deepep_trn_b200 Buffer, backend 'nvlink' (sm_100a kernels over peer memory).
             The same run also measures the NCCL build of the same semantics on the same
             inputs (``nccl``); ``vs_baseline`` is value / that NCCL value, the B200
             comparison point the baseline document names.
  nccl       deepep_trn_b200 Buffer, backend 'nccl' (reference semantics + NCCL all_to_all_single)
  reference  the unmodified reference (baseline/_ref/deep_ep_trn) through its public API and its
             stock CPU/gloo transport (its NKI transport needs a Trainium device)
"""
from __future__ import annotations

import argparse
import json
import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch
import torch.distributed as dist

METRIC = 'dispatch+combine NVLink GB/s/GPU (4096 tok) & LL µs (128 tok), 1/2/4/8 B200'
LINK_NOMINAL_GBPS = 900.0   # NVLink 5 per direction per GPU
LINK_MEASURED_GBPS = 770.0  # peer copy per direction measured on this pool


def parse():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument('--gpus', type=int, default=1)
    p.add_argument('--steps', type=int, default=20)
    p.add_argument('--warmup', type=int, default=5)
    p.add_argument('--impl', choices=['ours', 'nccl', 'reference'], default='ours')
    p.add_argument('--tokens', type=int, default=4096)
    p.add_argument('--hidden', type=int, default=7168)
    p.add_argument('--experts', type=int, default=256)
    p.add_argument('--topk', type=int, default=8)
    p.add_argument('--ll-tokens', type=int, default=128)
    p.add_argument('--no-ll', action='store_true')
    p.add_argument('--no-e2e', action='store_true')
    p.add_argument('--no-nccl', action='store_true', help='skip the NCCL comparison arm of --impl ours')
    p.add_argument('--fp8', action='store_true', help='quantise to fp8 1x128 inside dispatch (config 3)')
    p.add_argument('--profile', action='store_true', help='print a per-kernel breakdown (torch.profiler) to stderr')
    p.add_argument('--trace', action='store_true', help='print device phase timestamps of one step per rank')
    p.add_argument('--no-combine-weights', action='store_true', help='combine without the top-k weight channel')
    return p.parse_args()


def init_dist():
    if 'RANK' not in os.environ:
        os.environ.update(RANK='0', WORLD_SIZE='1', LOCAL_RANK='0', MASTER_ADDR='127.0.0.1')
        with socket.socket() as s:
            s.bind(('127.0.0.1', 0))
            os.environ['MASTER_PORT'] = str(s.getsockname()[1])
    local = int(os.environ.get('LOCAL_RANK', 0))
    torch.cuda.set_device(local)
    timeout = timedelta(seconds=int(os.environ.get('B200EP_PG_TIMEOUT', '300')))
    dist.init_process_group('nccl', timeout=timeout, device_id=torch.device('cuda', local))
    return dist.get_rank(), dist.get_world_size(), local


def make_inputs(args, rank):
    from deepep_trn_b200.utils.testing import randn_router
    g = torch.Generator().manual_seed(1234 + rank)
    x = torch.randn(args.tokens, args.hidden, generator=g).to(torch.bfloat16)
    idx, w = randn_router(args.tokens, args.experts, args.topk, seed=99 + rank)
    return x, idx, w


def ref_buffer(group, M):
    ref = ROOT / 'baseline' / '_ref'
    if not (ref / 'deep_ep_trn').exists():
        return None, 'reference not installed under baseline/_ref'
    sys.path.insert(0, str(ref))
    from deep_ep_trn import Buffer as RefBuffer
    return RefBuffer(group, backend='gloo', num_max_tokens_per_rank=M), None


def make_step(args, buf, E, use_fp8):
    def step(x, idx, w):
        ntr, _, nte, itr, _ = buf.get_dispatch_layout(idx, E)
        kw = dict(topk_idx=idx, topk_weights=w, num_tokens_per_rank=ntr, is_token_in_rank=itr,
                  num_tokens_per_expert=nte)
        if use_fp8:
            kw['use_fp8'] = True
        rx, ridx, rw, per_expert, handle, _ = buf.dispatch(x, **kw)
        if use_fp8:
            from deepep_trn_b200.ops.quant import dequantize_fp8   # the identity expert reads fp8 in
            rx = dequantize_fp8(*rx)
        out, ow, _ = buf.combine(rx, handle, topk_weights=None if args.no_combine_weights else rw)
        return out, ow, handle, itr
    return step


def time_steps(step, steps, warmup, control, clocks=None):
    """ms per step: CUDA events around each step (L2 flushed before it), max over ranks."""
    from deepep_trn_b200.utils.benchutil import DeviceTimer, max_over_ranks
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier(group=control)
    timer = DeviceTimer()
    if clocks is not None:
        clocks.__enter__()
    torch.cuda.synchronize()
    dist.barrier(group=control)
    for _ in range(steps):
        timer.run(step)
    torch.cuda.synchronize()
    dist.barrier(group=control)
    if clocks is not None:
        clocks.__exit__(None, None, None)
    return max_over_ranks(timer.total_ms()) / steps


def time_pipelined(step, host_inputs, out_shape, dev, steps, warmup, control):
    """ms per step of the serving loop: every step uploads its inputs from pinned host memory
    (copy stream), runs on the compute stream, and downloads its result into pinned host
    memory (a second copy stream). Two input and output buffers let step i+1's upload and
    step i's download run while step i or i+1 computes, as a serving engine would run it.
    The whole loop is timed between events on the compute stream; max over ranks."""
    from deepep_trn_b200.utils.benchutil import L2_FLUSH_BYTES, max_over_ranks
    comp = torch.cuda.current_stream()
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    nb = 2
    dins = [tuple(torch.empty_like(h, device=dev) for h in host_inputs) for _ in range(nb)]
    outs = [torch.empty(out_shape, dtype=torch.bfloat16).pin_memory() for _ in range(nb)]
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    landed = [torch.cuda.Event() for _ in range(nb)]
    used = [torch.cuda.Event() for _ in range(nb)]

    def loop(n):
        start = torch.cuda.Event(enable_timing=True)
        start.record(comp)
        up.wait_event(start)
        for i in range(n):
            b = i % nb
            with torch.cuda.stream(up):
                if i >= nb:
                    up.wait_event(used[b])          # step i - 2 no longer reads these inputs
                for d, h in zip(dins[b], host_inputs):
                    d.copy_(h, non_blocking=True)
                landed[b].record(up)
            comp.wait_event(landed[b])
            flush.fill_(1)
            o, *_ = step(*dins[b])
            used[b].record(comp)
            with torch.cuda.stream(down):
                down.wait_event(used[b])
                outs[b].copy_(o, non_blocking=True)
                o.record_stream(down)
        comp.wait_stream(down)
        stop = torch.cuda.Event(enable_timing=True)
        stop.record(comp)
        stop.synchronize()
        return start.elapsed_time(stop)

    loop(warmup)
    torch.cuda.synchronize()
    dist.barrier(group=control)
    ms = loop(steps)
    torch.cuda.synchronize()
    dist.barrier(group=control)
    return max_over_ranks(ms) / steps


def main():
    args = parse()
    from deepep_trn_b200.utils.benchutil import ClockSampler, log, max_over_ranks, sum_over_ranks
    rank, world, local = init_dist()
    dev = torch.device('cuda', local)
    control = dist.new_group(backend='gloo')
    if args.impl == 'reference':
        buf, why = ref_buffer(control, args.tokens)
        if buf is None:
            if rank == 0:
                print(json.dumps({'impl': 'reference', 'unavailable': why}), flush=True)
            dist.destroy_process_group()
            return
    else:
        from deepep_trn_b200 import Buffer
        buf = Buffer(dist.group.WORLD, backend='nvlink' if args.impl == 'ours' else 'nccl',
                     num_max_tokens_per_rank=args.tokens, hidden=args.hidden, num_experts=args.experts,
                     topk=args.topk, num_max_dispatch_tokens_per_rank=args.ll_tokens)
    E, H = args.experts, args.hidden
    x_h, idx_h, w_h = make_inputs(args, rank)
    x, idx, w = x_h.to(dev), idx_h.to(dev), w_h.to(dev)
    use_fp8 = args.fp8 and args.impl == 'ours'
    step = make_step(args, buf, E, use_fp8)

    # ---- correctness gate: identity combine returns x * ranks_visited exactly
    out, ow, handle, itr = step(x, idx, w)
    torch.cuda.synchronize()
    ref = (x.float() * itr.sum(1, keepdim=True)).to(torch.bfloat16)
    ok = bool(torch.equal(out, ref)) if not use_fp8 else bool(torch.allclose(out.float(), ref.float(), rtol=0.07, atol=0.05))
    ok = max_over_ranks(0.0 if ok else 1.0) == 0.0
    recv_rows = int(handle.recv_counts.sum()) if handle.recv_counts is not None else int(itr.sum())
    own = int(itr[:, rank].sum()) if itr.shape[1] > rank else 0   # rows this rank sends to itself
    bytes_rank = 2 * recv_rows * H * 2          # dispatch + combine, bf16 rows received
    offrank_bytes_rank = 2 * (recv_rows - own) * H * 2

    clocks = ClockSampler(local)
    ms_step = time_steps(lambda: step(x, idx, w), args.steps, args.warmup, control, clocks)
    agg_bytes = sum_over_ranks(bytes_rank)
    value = agg_bytes / (ms_step * 1e-3) / 1e9
    offrank_per_gpu = sum_over_ranks(offrank_bytes_rank) / world / (ms_step * 1e-3) / 1e9

    if args.profile:
        profile_steps(lambda: step(x, idx, w), 'normal d+c', rank)
    if args.trace and args.impl == 'ours':
        buf._engine.barrier()   # a device barrier: its exit stamp lines up the ranks' clocks
        for _ in range(3):
            step(x, idx, w)
        tr = buf.device_trace()
        everyone = [None] * world
        dist.all_gather_object(everyone, (rank, tr), group=control)
        if rank == 0:
            for r, t in everyone:
                log(f'device trace rank {r}: ' + ' '.join(f'{k}={v}' for k, v in t.items() if k != 'abs.raw'))
            log_aligned(everyone)

    # ---- end to end through the public API: pinned H2D of inputs, D2H of the combined result
    e2e = None
    if not args.no_e2e:
        xp, ip, wp = x_h.pin_memory(), idx_h.pin_memory(), w_h.pin_memory()
        e2e_ms = time_pipelined(step, (xp, ip, wp), (args.tokens, H), dev, args.steps,
                                max(1, args.warmup // 2), control)
        bi = xp.numel() * 2 + ip.numel() * 8 + wp.numel() * 4
        bo = args.tokens * H * 2
        e2e = {'value': round(agg_bytes / (e2e_ms * 1e-3) / 1e9, 2), 'unit': 'GB/s (sum over GPUs)',
               'ms_per_step': round(e2e_ms, 4), 'h2d_bytes_per_step': bi, 'd2h_bytes_per_step': bo,
               'timing': 'whole loop of K steps between CUDA events on the compute stream (max over ranks) / K; '
                         "each step's inputs copied host->device on a copy stream and its result device->host "
                         'on another, double-buffered so step i+1 uploads while step i downloads; L2 flushed '
                         'before every step inside the timed loop'}

    # ---- low-latency: fp8 dispatch + bf16 combine of 128 tokens (CUDA-graph replay for ours)
    ll = None
    if not args.no_ll and args.impl in ('ours', 'nccl'):
        ll = bench_ll(args, buf, rank, dev, control, graph=args.impl == 'ours')
        if args.trace and args.impl == 'ours':
            tr = ll.pop('_trace', None) or {}
            everyone = [None] * world
            dist.all_gather_object(everyone, (rank, tr), group=control)
            if rank == 0:
                for r, t in everyone:
                    log(f'device trace rank {r}: ' + ' '.join(f'{k}={v}' for k, v in t.items()))

    # ---- the NCCL build of the same semantics, same inputs, same process group
    nccl = None
    if args.impl == 'ours' and not args.no_nccl:
        from deepep_trn_b200 import Buffer
        torch.cuda.synchronize()
        nbuf = Buffer(dist.group.WORLD, backend='nccl', num_max_tokens_per_rank=args.tokens)
        nstep = make_step(args, nbuf, E, False)
        o2, *_ = nstep(x, idx, w)
        torch.cuda.synchronize()
        nccl_ok = max_over_ranks(0.0 if torch.equal(o2, ref) else 1.0) == 0.0
        nms = time_steps(lambda: nstep(x, idx, w), args.steps, args.warmup, control)
        nccl = {'value': round(agg_bytes / (nms * 1e-3) / 1e9, 2), 'ms_per_step': round(nms, 4),
                'check': 'PASS' if nccl_ok else 'FAIL'}
        if ll is not None:
            nccl['ll'] = bench_ll(args, nbuf, rank, dev, control, graph=False, hook=False)
        del nbuf

    summaries = [None] * world
    dist.all_gather_object(summaries, clocks.summary(), group=control)
    clk = ClockSampler.merge(summaries)
    # layout, dispatch, combine per step (+ the fp8 dequantisation of the identity expert)
    launches = (4 if use_fp8 else 3) * args.steps if args.impl == 'ours' else 0
    if rank == 0:
        rec = {
            'metric': METRIC, 'value': round(value, 2), 'unit': 'GB/s (sum over GPUs)', 'n_gpus': world,
            'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': round(ms_step, 4),
            'higher_is_better': True, 'scaling': 'weak',
            'vs_baseline': round(value / nccl['value'], 3) if nccl else None,
            'dtype': 'fp8-dispatch/bf16-combine' if use_fp8 else 'bf16',
            'data': 'synthetic: randn bf16 tokens, randn router logits -> top-8 of 256 (softmax weights), seeded per rank',
            'config': {'model': 'deepseek-v3 MoE layer comms (H=7168, E=256, top-8)',
                       'global_batch': args.tokens * world, 'seq_len': args.tokens,
                       'parallelism': f'ep{world}', 'tokens_per_rank': args.tokens,
                       'l2': 'flushed before every timed step (256 MiB write, untimed)',
                       'step': 'get_dispatch_layout + dispatch + combine (identity expert)'},
            'per_gpu_gbps': round(value / world, 2), 'offrank_gbps_per_gpu': round(offrank_per_gpu, 2),
            'offrank_gbps_sum': round(offrank_per_gpu * world, 2),
            'roofline': {'of_nominal_900': round(offrank_per_gpu / LINK_NOMINAL_GBPS, 3),
                         'of_measured_770': round(offrank_per_gpu / LINK_MEASURED_GBPS, 3)} if world > 1 else None,
            'check': 'PASS' if ok else 'FAIL', 'impl': args.impl, 'clocks': clk, 'e2e': e2e,
            'gpu_launches': launches, 'll': ll, 'nccl': nccl,
        }
        print(json.dumps(rec), flush=True)
    if hasattr(buf, 'destroy'):
        buf.destroy()
    dist.barrier(group=control)
    dist.destroy_process_group()


def log_aligned(everyone):
    """The last step's phase stamps of every rank on one time line (us): each rank's clock is
    shifted so that the device barrier before the traced steps exits at the same moment."""
    from deepep_trn_b200.utils.benchutil import log
    names = {0: 'd.start', 9: 'd.free', 10: 'd.grid_bar', 1: 'd.scanned', 4: 'd.cta0_pushed',
             7: 'd.cta0_published', 2: 'd.counts_in', 3: 'd.notified', 5: 'd.cta0_recvd', 6: 'd.end',
             16: 'c.start', 17: 'c.cta0_pushed', 20: 'c.cta0_published', 18: 'c.cta0_reduced', 19: 'c.end'}
    base = None
    for r, t in everyone:
        raw = t.get('abs.raw') or []
        if len(raw) < 21 or not raw[15]:
            return
        rel = {n: (raw[i] - raw[15]) / 1e3 for i, n in names.items() if raw[i]}
        if base is None:
            base = rel['d.start']
        log(f'aligned rank {r}: ' + ' '.join(f'{n}={v - base:.1f}' for n, v in sorted(rel.items(), key=lambda kv: kv[1])))


def profile_steps(fn, label, rank, n=3):
    from torch.profiler import ProfilerActivity, profile
    from deepep_trn_b200.utils.benchutil import log
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(n):
            fn()
        torch.cuda.synchronize()
    if rank == 0:
        log(f'---- kernel breakdown: {label} ({n} steps, profiler timings, not bench numbers)')
        log(prof.key_averages().table(sort_by='cuda_time_total', row_limit=15))


def _events_us(fn, iters):
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st.record()
    for _ in range(iters):
        fn()
    en.record()
    torch.cuda.synchronize()
    return st.elapsed_time(en) * 1e3 / iters


def _capture(fn):
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
        out = fn()
    torch.cuda.current_stream().wait_stream(s)
    return g, out


def bench_ll(args, buf, rank, dev, control, graph: bool = True, hook: bool = True):
    """fp8 low-latency dispatch + bf16 combine of ``--ll-tokens`` tokens.

    * ``dispatch_fp8_plus_combine_us``: one dispatch and one combine (CUDA-graph replays for
      the NVLink kernels; plain host-synchronised calls for the NCCL build), max over ranks.
    * ``check``: identity experts (each expert returns its dequantised input) must give
      ``x * sum_k w_k`` within the fp8 rounding bound, on every rank.
    * ``hook_overlap``: a 2048x7168 @ 7168x7168 bf16 GEMM (the dummy compute of config 4)
      placed between dispatch's send and its receive hook, against the same GEMM after the
      receive; both captured as CUDA graphs.
    """
    from deepep_trn_b200.utils.benchutil import max_over_ranks
    from deepep_trn_b200.utils.testing import randn_router
    T, E, H, K = args.ll_tokens, args.experts, args.hidden, args.topk
    R = dist.get_world_size()
    g = torch.Generator().manual_seed(77 + rank)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(dev)
    idx, w = randn_router(T, E, K, seed=55 + rank, device=dev)
    y = torch.randn(E // R, R * T, H, generator=g).to(torch.bfloat16).to(dev)

    def ll_step():
        rx, cnt, h, _, _ = buf.low_latency_dispatch(x, idx, T, E, use_fp8=True)
        out, _, _ = buf.low_latency_combine(y, idx, w, h)
        return out

    # correctness: identity experts
    (q, s), cnt, h, _, _ = buf.low_latency_dispatch(x, idx, T, E, use_fp8=True)
    deq = (q.float() * s.float().repeat_interleave(128, -1)).to(torch.bfloat16)
    got, _, _ = buf.low_latency_combine(deq, idx, w, h)
    torch.cuda.synchronize()
    want = x.float() * (w * (idx >= 0)).sum(-1, keepdim=True)
    good = bool(torch.allclose(got.float(), want, rtol=0.07, atol=0.05))
    check = 'PASS' if max_over_ranks(0.0 if good else 1.0) == 0.0 else 'FAIL'

    for _ in range(3):
        ll_step()
    torch.cuda.synchronize()
    if not graph:
        dist.barrier(group=control)
        us = max_over_ranks(_events_us(ll_step, 20))
        return {'tokens_per_rank': T, 'dispatch_fp8_plus_combine_us': round(us, 2), 'cuda_graph': False,
                'check': check}
    if args.profile:
        profile_steps(ll_step, 'low-latency fp8 d + bf16 c', rank)
    gr, _ = _capture(ll_step)
    for _ in range(5):
        gr.replay()
    torch.cuda.synchronize()
    dist.barrier(group=control)
    us = max_over_ranks(_events_us(gr.replay, 50))
    del gr
    trace = {k: v for k, v in buf.device_trace().items() if k.startswith('ll.')} if args.trace else None
    res = {'tokens_per_rank': T, 'dispatch_fp8_plus_combine_us': round(us, 2), 'cuda_graph': True,
           'launches_per_iter': 4, 'check': check}
    if trace is not None:
        res['_trace'] = trace   # phase stamps of the last plain replay (printed, not reported)
    if hook:
        a = torch.randn(2048, H, generator=g).to(torch.bfloat16).to(dev)
        b = torch.randn(H, H, generator=g).to(torch.bfloat16).to(dev) * 0.01

        def overlapped():
            _, _, h2, _, rh = buf.low_latency_dispatch(x, idx, T, E, use_fp8=True, return_recv_hook=True)
            c = a @ b   # compute while the rows travel
            rh()
            out, _, ch = buf.low_latency_combine(y, idx, w, h2, return_recv_hook=True)
            ch()
            return c, out

        def serial():
            _, _, h2, _, _ = buf.low_latency_dispatch(x, idx, T, E, use_fp8=True)
            c = a @ b
            out, _, _ = buf.low_latency_combine(y, idx, w, h2)
            return c, out

        times = {}
        for name, fn in (('serial', serial), ('hooked', overlapped)):
            fn()
            torch.cuda.synchronize()
            gg, _ = _capture(fn)
            for _ in range(3):
                gg.replay()
            torch.cuda.synchronize()
            dist.barrier(group=control)
            times[name] = max_over_ranks(_events_us(gg.replay, 20))
            del gg
            if args.trace and trace is not None:
                trace.update({f'{name}.{k}': v for k, v in buf.device_trace().items() if k.startswith('ll.')})
        gemm_us = max_over_ranks(_events_us(lambda: a @ b, 20))
        res['hook_overlap'] = {'gemm': '2048x7168 @ 7168x7168 bf16', 'gemm_us': round(gemm_us, 2),
                               'serial_us': round(times['serial'], 2), 'hooked_us': round(times['hooked'], 2),
                               'saved_us': round(times['serial'] - times['hooked'], 2)}
    buf.check()
    return res


if __name__ == '__main__':
    main()
