#!/usr/bin/env python
"""Headline benchmark: normal-mode dispatch + combine NVLink GB/s at 4096 tokens per rank
(H=7168, top-8 of 256 experts, bf16), plus low-latency fp8 dispatch + bf16 combine latency
at 128 tokens per rank (CUDA graph).

    python bench.py --gpus N --steps K --warmup W [--impl ours|reference|nccl]

For N > 1 launch under torchrun (one rank per GPU); rank 0 prints one JSON line.

Timing: W untimed warm-up steps, then exactly K steps between a barrier and a
device synchronisation on both sides; each step is timed with CUDA events on the
launching stream after an untimed L2 flush (a 256 MiB write), and the total is
the max over ranks. ``value`` is the whole-job aggregate: the sum over ranks of
the bytes each rank receives in dispatch and in combine, divided by the max-over-
ranks step time. The ``e2e`` number repeats the measurement through the public
API with the step's inputs copied from pinned host memory and the combined result
copied back to pinned host memory inside the timed region.

Arms:
  ours       deepep_trn_b200 Buffer, backend 'nvlink' (sm_100a kernels over peer memory)
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
    p.add_argument('--fp8', action='store_true', help='quantise to fp8 1x128 inside dispatch (config 3)')
    p.add_argument('--profile', action='store_true', help='print a per-kernel breakdown (torch.profiler) to stderr')
    p.add_argument('--trace', action='store_true', help='print device phase timestamps of one step per rank')
    p.add_argument('--no-combine-weights', action='store_true', help='combine without the top-k weight channel')
    return p.parse_args()


def init_dist(backend: str):
    if 'RANK' not in os.environ:
        os.environ.update(RANK='0', WORLD_SIZE='1', LOCAL_RANK='0', MASTER_ADDR='127.0.0.1')
        with socket.socket() as s:
            s.bind(('127.0.0.1', 0))
            os.environ['MASTER_PORT'] = str(s.getsockname()[1])
    local = int(os.environ.get('LOCAL_RANK', 0))
    torch.cuda.set_device(local)
    timeout = timedelta(seconds=int(os.environ.get('B200EP_PG_TIMEOUT', '300')))
    if backend == 'nccl':
        dist.init_process_group('nccl', timeout=timeout, device_id=torch.device('cuda', local))
    else:
        dist.init_process_group('gloo', timeout=timeout)
    return dist.get_rank(), dist.get_world_size(), local


def make_inputs(args, rank, dev):
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


def main():
    args = parse()
    from deepep_trn_b200.utils.benchutil import ClockSampler, DeviceTimer, env_record, log, max_over_ranks, sum_over_ranks
    rank, world, local = init_dist('nccl')
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
    x_h, idx_h, w_h = make_inputs(args, rank, dev)
    x, idx, w = x_h.to(dev), idx_h.to(dev), w_h.to(dev)
    use_fp8 = args.fp8 and args.impl == 'ours'

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

    # ---- correctness gate: identity combine returns x * ranks_visited exactly
    out, ow, handle, itr = step(x, idx, w)
    torch.cuda.synchronize()
    ref = (x.float() * itr.sum(1, keepdim=True)).to(torch.bfloat16)
    ok = bool(torch.equal(out, ref)) if not use_fp8 else bool(torch.allclose(out.float(), ref.float(), rtol=0.07, atol=0.05))
    ok = max_over_ranks(0.0 if ok else 1.0) == 0.0
    recv_rows = int(handle.recv_counts.sum()) if handle.recv_counts is not None else int(itr.sum())
    bytes_rank = 2 * recv_rows * H * 2  # dispatch + combine, bf16 rows received
    own = int(handle.recv_counts[rank]) if (handle.recv_counts is not None and handle.recv_counts.numel() > rank) else 0
    offrank_bytes_rank = 2 * (recv_rows - own) * H * 2

    for _ in range(args.warmup):
        step(x, idx, w)
    torch.cuda.synchronize()
    dist.barrier(group=control)
    timer = DeviceTimer()
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize()
        dist.barrier(group=control)
        for _ in range(args.steps):
            timer.run(lambda: step(x, idx, w))
        torch.cuda.synchronize()
        dist.barrier(group=control)
    total_ms = max_over_ranks(timer.total_ms())
    ms_step = total_ms / args.steps
    agg_bytes = sum_over_ranks(bytes_rank)
    value = agg_bytes / (ms_step * 1e-3) / 1e9
    offrank = sum_over_ranks(offrank_bytes_rank) / (ms_step * 1e-3) / 1e9

    if args.profile:
        profile_steps(lambda: step(x, idx, w), 'normal d+c', rank)
    if args.trace and args.impl == 'ours':
        for _ in range(3):
            step(x, idx, w)
        tr = buf.device_trace()
        everyone = [None] * world
        dist.all_gather_object(everyone, (rank, tr), group=control)
        if rank == 0:
            for r, t in everyone:
                log(f'device trace rank {r}: ' + ' '.join(f'{k}={v}' for k, v in t.items()))

    # ---- end to end through the public API: pinned H2D of inputs, D2H of the combined result
    e2e = None
    if not args.no_e2e:
        xp, ip, wp = x_h.pin_memory(), idx_h.pin_memory(), w_h.pin_memory()
        outp = torch.empty(args.tokens, H, dtype=torch.bfloat16).pin_memory()
        xd, idd, wd = torch.empty_like(x), torch.empty_like(idx), torch.empty_like(w)

        def e2e_step():
            xd.copy_(xp, non_blocking=True)
            idd.copy_(ip, non_blocking=True)
            wd.copy_(wp, non_blocking=True)
            o, *_ = step(xd, idd, wd)
            outp.copy_(o, non_blocking=True)

        for _ in range(max(1, args.warmup // 2)):
            e2e_step()
        torch.cuda.synchronize()
        dist.barrier(group=control)
        t2 = DeviceTimer()
        for _ in range(args.steps):
            t2.run(e2e_step)
        torch.cuda.synchronize()
        dist.barrier(group=control)
        e2e_ms = max_over_ranks(t2.total_ms()) / args.steps
        bi = xp.numel() * 2 + ip.numel() * 8 + wp.numel() * 4
        bo = outp.numel() * 2
        e2e = {'value': round(agg_bytes / (e2e_ms * 1e-3) / 1e9, 2), 'unit': 'GB/s (sum over GPUs)',
               'ms_per_step': round(e2e_ms, 4), 'h2d_bytes_per_step': bi, 'd2h_bytes_per_step': bo}

    # ---- low-latency: fp8 dispatch + bf16 combine of 128 tokens, CUDA-graph replay
    ll = None
    if not args.no_ll and args.impl in ('ours', 'nccl'):
        ll = bench_ll(args, buf, rank, dev, control, graph=args.impl == 'ours')

    summaries = [None] * world
    dist.all_gather_object(summaries, clocks.summary(), group=control)
    clk = ClockSampler.merge(summaries)
    # layout, prepare, pull, combine per step (+ the fp8 dequantisation of the identity expert)
    launches = (5 if use_fp8 else 4) * args.steps if args.impl == 'ours' else 0
    if rank == 0:
        rec = {
            'metric': METRIC, 'value': round(value, 2), 'unit': 'GB/s (sum over GPUs)', 'n_gpus': world,
            'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': round(ms_step, 4),
            'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None,
            'dtype': 'fp8-dispatch/bf16-combine' if use_fp8 else 'bf16',
            'data': 'synthetic: randn bf16 tokens, randn router logits -> top-8 of 256 (softmax weights), seeded per rank',
            'config': {'model': 'deepseek-v3 MoE layer comms (H=7168, E=256, top-8)',
                       'global_batch': args.tokens * world, 'seq_len': args.tokens,
                       'parallelism': f'ep{world}', 'tokens_per_rank': args.tokens,
                       'l2': 'flushed before every timed step (256 MiB write, untimed)',
                       'step': 'get_dispatch_layout + dispatch + combine (identity expert)'},
            'per_gpu_gbps': round(value / world, 2), 'offrank_gbps_sum': round(offrank, 2),
            'check': 'PASS' if ok else 'FAIL', 'impl': args.impl, 'clocks': clk, 'e2e': e2e,
            'gpu_launches': launches, 'll': ll,
        }
        print(json.dumps(rec), flush=True)
    if hasattr(buf, 'destroy'):
        buf.destroy()
    dist.barrier(group=control)
    dist.destroy_process_group()


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


def bench_ll(args, buf, rank, dev, control, graph: bool = True):
    """fp8 low-latency dispatch + bf16 combine of ``--ll-tokens`` tokens. The NVLink kernels are
    timed as CUDA-graph replays; the NCCL build (host-synchronised split sizes) as plain calls."""
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

    for _ in range(3):
        ll_step()
    torch.cuda.synchronize()
    if not graph:
        dist.barrier(group=control)
        iters = 20
        st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        st.record()
        for _ in range(iters):
            ll_step()
        en.record()
        torch.cuda.synchronize()
        us = max_over_ranks(st.elapsed_time(en) * 1e3 / iters)
        return {'tokens_per_rank': T, 'dispatch_fp8_plus_combine_us': round(us, 2), 'cuda_graph': False}
    if args.profile:
        profile_steps(ll_step, 'low-latency fp8 d + bf16 c', rank)
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s), torch.cuda.graph(graph, stream=s):
        ll_step()
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(5):
        graph.replay()
    torch.cuda.synchronize()
    dist.barrier(group=control)
    iters = 50
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st.record()
    for _ in range(iters):
        graph.replay()
    en.record()
    torch.cuda.synchronize()
    us = max_over_ranks(st.elapsed_time(en) * 1e3 / iters)
    del graph
    buf.check()
    return {'tokens_per_rank': T, 'dispatch_fp8_plus_combine_us': round(us, 2), 'cuda_graph': True,
            'launches_per_iter': 4}


if __name__ == '__main__':
    main()
