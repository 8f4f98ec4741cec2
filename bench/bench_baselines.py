"""Collective baselines an EP MoE layer could use instead of dispatch / combine (NCCL).

Same op set as the reference's bench/bench_baselines.py, device-resident on the
EP group, timed with CUDA events (max over ranks):

  all_reduce        [R*T, H]            all-expert MoE path
  all_gather        [T, H] -> [R*T, H]
  reduce_scatter    [R*T, H] -> [T, H]
  ag_rs             all_gather + reduce_scatter
  all_to_all_single [R*T, H]            capacity-padded dispatch, no routing

torchrun --nnodes 1 --nproc-per-node 8 --master-addr 127.0.0.1 bench/bench_baselines.py
"""
from harness import PRESETS, BenchGroup, cli, device_stats, write_jsonl

import torch
import torch.distributed as dist


def main():
    args = cli(__doc__).parse_args()
    if args.backend == 'gloo':
        raise SystemExit('baselines run over NCCL on the GPUs')
    ctx = BenchGroup('nccl', args.ep)
    g, R = ctx.group, ctx.ep

    def ops(T, H):
        dev = ctx.device
        a = torch.randn(R * T, H, device=dev).to(torch.bfloat16)
        b = torch.randn(T, H, device=dev).to(torch.bfloat16)
        out_big, out_small = torch.empty_like(a), torch.empty_like(b)
        return {
            'all_reduce': lambda: dist.all_reduce(a, group=g),
            'all_gather': lambda: dist.all_gather_into_tensor(out_big, b, group=g),
            'reduce_scatter': lambda: dist.reduce_scatter_tensor(out_small, a, group=g),
            'ag_rs': lambda: (dist.all_gather_into_tensor(out_big, b, group=g),
                              dist.reduce_scatter_tensor(out_small, a, group=g)),
            'all_to_all_single': lambda: dist.all_to_all_single(out_big, a, group=g),
        }

    for preset in args.presets:
        H = PRESETS[preset][0]
        for T in args.tokens:
            for name, fn in ops(T, H).items():
                rec = dict(bench='baseline', op=name, preset=preset, hidden=H, ep=R, tokens=T)
                try:
                    rec['device_us'] = device_stats(ctx, fn, args.rounds, args.iters)
                    rec['latency_us'] = device_stats(ctx, fn, args.rounds, args.iters, each=True)
                except Exception as exc:  # an unsupported collective is a result, not a crash
                    rec['error'] = f'{type(exc).__name__}: {str(exc).splitlines()[0][:300]}'
                if ctx.rank == 0:
                    write_jsonl(args.out_dir / f'baselines_ep{R}.jsonl', rec)
                    val = (f"{rec['device_us']['median_us']}us latency={rec['latency_us']['median_us']}us"
                           if 'device_us' in rec else rec['error'])
                    print(f'[baseline] {name} {preset} ep={R} T={T}: {val}', flush=True)
    ctx.close()


if __name__ == '__main__':
    main()
