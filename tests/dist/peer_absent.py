"""A peer that never joins an op: the waiting rank's kernels must give up after the
buffer's timeout and report it, leaving the GPU context usable.

Two ranks on two GPUs, NVLink backend with a 1 s device wait budget. Rank 1 skips
the op (it stays alive, with its heap mapped, and launches nothing); rank 0 runs
it. Cases:

    normal   rank 0's dispatch raises DeviceError (the prepare kernel's bounded wait
             for rank 1's counts ran out and wrote the status page)
    ll       rank 0's low-latency dispatch completes on the device with an error
             status; ``Buffer.check()`` raises DeviceError

Afterwards rank 0 checks that its context still works (a local op and a
synchronize), both ranks meet on the gloo control group and tear down. No GPU
fault, trap or unbounded wait is involved: every wait in the kernels is bounded.
The reference raises on the same conditions from the host (its collectives time
out through NEURON_RT_EXEC_TIMEOUT, scripts/env_trn2.sh:3).
"""
from __future__ import annotations

import argparse
import os
import sys
import time
from datetime import timedelta
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[2]))

import torch
import torch.distributed as dist


def main():
    p = argparse.ArgumentParser()
    p.add_argument('--case', choices=['normal', 'll'], required=True)
    args = p.parse_args()
    local = int(os.environ.get('LOCAL_RANK', 0))
    torch.cuda.set_device(local)
    dist.init_process_group('nccl', timeout=timedelta(seconds=60), device_id=torch.device('cuda', local))
    control = dist.new_group(backend='gloo')
    rank = dist.get_rank()
    from deepep_trn_b200 import Buffer
    from deepep_trn_b200.parallel.engine_nvlink import DeviceError
    T, H, E, K, M = 32, 256, 16, 4, 64
    buf = Buffer(dist.group.WORLD, backend='nvlink', num_max_tokens_per_rank=M, hidden=H, num_experts=E, topk=K,
                 num_max_dispatch_tokens_per_rank=M, timeout_s=1.0)
    g = torch.Generator().manual_seed(rank)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).cuda()
    idx = torch.rand(T, E, generator=g).topk(K, dim=-1).indices.cuda()
    w = torch.rand(T, K, generator=g).cuda()
    dist.barrier(group=control)
    if rank == 0:
        t0 = time.perf_counter()
        err = None
        try:
            if args.case == 'normal':
                ntr, _, nte, itr, _ = buf.get_dispatch_layout(idx, E)
                buf.dispatch(x, topk_idx=idx, topk_weights=w, num_tokens_per_rank=ntr, is_token_in_rank=itr,
                             num_tokens_per_expert=nte)
            else:
                buf.low_latency_dispatch(x, idx, M, E, use_fp8=False)
                torch.cuda.synchronize()
                buf.check()
        except DeviceError as e:
            err = e
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        y = (x.float() * 2).sum()  # the context is still usable
        torch.cuda.synchronize()
        ok = err is not None and torch.isfinite(y).item()
        print(f'RANK=0 DETECTED={type(err).__name__ if err else None} after {dt:.2f}s: {err}', flush=True)
        if ok:
            print('PEER_ABSENT_PASS', flush=True)
    dist.barrier(group=control)  # rank 1 kept its heap mapped until rank 0's kernels were done
    buf.destroy()
    dist.destroy_process_group()


if __name__ == '__main__':
    main()
