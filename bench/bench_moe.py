"""MoE layer forward + backward, the fused path against NCCL + cuBLAS.

Per rank: T tokens, H=7168, 256 experts top-8 with Zipf-skewed routing (router
logits plus a log(1/r) bias over a seeded expert permutation), SwiGLU experts with
intermediate 2048, weights ~N(0, 0.02) (bf16). One step = forward + backward of
the layer (dx and every weight gradient). Device time with CUDA events, max over
ranks, L2 flushed between steps.

torchrun --nnodes 1 --nproc-per-node 8 --master-addr 127.0.0.1 bench/bench_moe.py
"""
from harness import BenchGroup, cli, write_jsonl

import json

import torch
import torch.distributed as dist

from deepep_trn_b200.utils.benchutil import DeviceTimer, max_over_ranks


def zipf_bias(E: int, seed: int = 12345) -> torch.Tensor:
    perm = torch.randperm(E, generator=torch.Generator().manual_seed(seed))
    bias = torch.empty(E)
    bias[perm] = -torch.log(torch.arange(1, E + 1, dtype=torch.float32))
    return bias


def main():
    p = cli(__doc__)
    p.add_argument('--hidden', type=int, default=7168)
    p.add_argument('--inter', type=int, default=2048)
    p.add_argument('--experts', type=int, default=256)
    p.add_argument('--topk', type=int, default=8)
    p.add_argument('--steps', type=int, default=5)
    p.add_argument('--warmup', type=int, default=3)
    p.add_argument('--impls', default='ours,nccl')
    p.add_argument('--breakdown', action='store_true', help='per-phase device time of the fused layer')
    p.add_argument('--fp8', action='store_true', help='fused layer: forward dispatch in fp8 e4m3 + 1x128 scales '
                   '(with --forward-only also fp8 block-scaled expert GEMMs)')
    p.add_argument('--forward-only', action='store_true', help='inference: forward under torch.no_grad()')
    p.set_defaults(tokens=[4096])
    args = p.parse_args()
    T = args.tokens[0]
    ctx = BenchGroup('nccl', args.ep)
    from deepep_trn_b200 import Buffer
    from deepep_trn_b200.models.moe import MoELayer
    from deepep_trn_b200.models.moe_baseline import BaselineMoELayer
    H, I, E, K = args.hidden, args.inter, args.experts, args.topk
    dev = ctx.device
    results = {}
    params = None   # the first layer's parameters, copied into the others
    for impl in args.impls.split(','):
        buf = Buffer(ctx.group, backend='nvlink' if impl == 'ours' else 'nccl', num_max_tokens_per_rank=T,
                     hidden=H, num_experts=E, topk=K)
        layer = (MoELayer(buf, H, I, E, K, device=dev, init_std=0.02, seed=7, fp8_dispatch=args.fp8,
                          fp8_experts=args.fp8 and args.forward_only) if impl == 'ours'
                 else BaselineMoELayer(buf, H, I, E, K, device=dev))
        with torch.no_grad():
            if params is None:
                if impl != 'ours':
                    src = MoELayer(buf, H, I, E, K, device=dev, init_std=0.02, seed=7)
                    for n in ('w1', 'w2', 'router'):
                        getattr(layer, n).copy_(getattr(src, n))
                    del src
                # router scale: x ~ N(0, 1) and |Wr| ~ 1/sqrt(H) give logits ~ N(0, 1)
                layer.router.mul_(1.0 / (0.02 * H ** 0.5))
                layer.router_bias.copy_(zipf_bias(E).to(dev))
                params = {n: getattr(layer, n).detach() for n in ('router', 'w1', 'w2', 'router_bias')}
            else:
                for n, v in params.items():
                    getattr(layer, n).copy_(v)
        x = torch.randn(T, H, generator=torch.Generator().manual_seed(100 + ctx.rank)).to(torch.bfloat16).to(dev)
        x.requires_grad_()
        dy = torch.randn(T, H, generator=torch.Generator().manual_seed(200 + ctx.rank)).to(torch.bfloat16).to(dev)

        def step():
            if args.forward_only:
                with torch.no_grad():
                    return layer(x)
            x.grad = None
            for prm in layer.parameters():
                prm.grad = None
            y = layer(x)
            y.backward(dy)
            return y

        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        dist.barrier(group=ctx.meta)
        timer = DeviceTimer()
        for _ in range(args.steps):
            timer.run(step)
        ms = max_over_ranks(timer.total_ms()) / args.steps
        per_step = [round(st.elapsed_time(en), 3) for st, en in timer.events]
        # expert GEMMs per rank on average: forward 6*P*H*I, backward twice that
        flops = (6.0 if args.forward_only else 18.0) * T * K * H * I
        results[impl] = dict(ms_per_step=round(ms, 3), tokens_per_s=round(T * ctx.ep / (ms * 1e-3), 1),
                             expert_tflops_per_rank=round(flops / (ms * 1e-3) / 1e12, 1), steps_ms_rank0=per_step)
        if args.breakdown and impl == 'ours':
            from deepep_trn_b200.utils.profiling import timer
            timer.reset()
            timer.enabled, timer.use_cuda_events = True, True
            for _ in range(3):
                step()
            torch.cuda.synchronize()
            per = timer.per_call_us(3)
            timer.enabled = False
            allr = ctx.gather({k: round(v, 1) for k, v in per.items() if k.startswith('moe.')})
            results[impl]['breakdown_us'] = {k: [r[k] for r in allr] for k in allr[0]}
        buf.destroy()
        del layer
        torch.cuda.empty_cache()
    rec = dict(bench='moe', ep=ctx.ep, tokens=T, hidden=H, inter=I, experts=E, topk=K, routing='zipf',
               dispatch_dtype='fp8-e4m3-1x128' if args.fp8 else 'bf16',
               expert_gemm_dtype='fp8-e4m3-1x128-block-scaled' if (args.fp8 and args.forward_only) else 'bf16',
               pass_='forward' if args.forward_only else 'forward+backward', **results)
    if 'ours' in results and 'nccl' in results:
        rec['speedup_vs_nccl_cublas'] = round(results['nccl']['ms_per_step'] / results['ours']['ms_per_step'], 3)
    if ctx.rank == 0:
        write_jsonl(args.out_dir / f'moe_ep{ctx.ep}.jsonl', rec)
        print(json.dumps(rec), flush=True)
    ctx.close()


if __name__ == '__main__':
    main()
