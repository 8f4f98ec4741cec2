"""Transport probe: the edge cases of the exchange in one run, reported as data.

Rank 0 sends nothing (T = 0); the last rank sends its full capacity, every token to
every rank; the others route randomly. Each rank checks the rows it receives against
an oracle gathered over a gloo control group (bitwise, in (source rank, source token)
order) and the identity combine against ``x * ranks_visited``, then prints
``PROBE {json}`` with the outcome and exits non-zero on a mismatch. Counterpart of the
reference's tools/probe_transport.py:33-53 (an empty and a full peer, compared with
gloo-gathered send data, JSON status); the subject here is the NVLink kernels' handling
of zero counts and full capacity rather than the Neuron runtime's accepted slot shapes.

torchrun --nnodes 1 --nproc-per-node 2 --master-addr 127.0.0.1 bench/probe_transport.py --backend nvlink
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import traceback
from datetime import timedelta
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import torch
import torch.distributed as dist


def main() -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument('--backend', choices=['nvlink', 'nccl', 'gloo'], default='nvlink')
    p.add_argument('--max-tokens', type=int, default=64)
    p.add_argument('--hidden', type=int, default=512)
    p.add_argument('--experts', type=int, default=16)
    p.add_argument('--topk', type=int, default=4)
    args = p.parse_args()
    timeout = timedelta(seconds=int(os.environ.get('B200EP_PG_TIMEOUT', '120')))
    if args.backend == 'gloo':
        dist.init_process_group('gloo', timeout=timeout)
        dev = torch.device('cpu')
    else:
        local = int(os.environ.get('LOCAL_RANK', 0))
        torch.cuda.set_device(local)
        dist.init_process_group('nccl', timeout=timeout, device_id=torch.device('cuda', local))
        dev = torch.device('cuda', local)
    control = dist.new_group(backend='gloo')
    rank, R = dist.get_rank(), dist.get_world_size()
    from deepep_trn_b200 import Buffer
    from deepep_trn_b200.utils.layout import rank_of_expert
    M, H, E, K = args.max_tokens, args.hidden, args.experts, args.topk
    EL = E // R
    record = dict(rank=rank, ranks=R, backend=args.backend, max_tokens=M, hidden=H)
    ok = True
    try:
        buf = Buffer(dist.group.WORLD, backend=args.backend, num_max_tokens_per_rank=M)
        g = torch.Generator().manual_seed(17 + rank)
        if rank == 0 and R > 1:
            T, idx = 0, torch.zeros(0, K, dtype=torch.int64)                        # empty peer
        elif rank == R - 1:
            T = M                                                                     # full peer
            # every token visits every rank: its first min(K, R) experts sit on distinct ranks
            k = torch.arange(K)
            idx = torch.stack([(k % R) * EL + (k // R) % EL] * T)   # distinct ids, rank k % R first
        else:
            T = M // 2
            idx = torch.rand(T, E, generator=g).topk(K, dim=-1).indices
        x = torch.randn(T, H, generator=g).to(torch.bfloat16)
        w = torch.rand(T, K, generator=g)
        record['tokens'] = T
        ntr, _, nte, itr, _ = buf.get_dispatch_layout(idx.to(dev), E)
        rx, ridx, rw, per_expert, handle, _ = buf.dispatch(
            x.to(dev), topk_idx=idx.to(dev), topk_weights=w.to(dev), num_tokens_per_rank=ntr,
            is_token_in_rank=itr, num_tokens_per_expert=nte)
        everyone = [None] * R
        dist.all_gather_object(everyone, (x, idx), group=control)
        exp = []
        for px, pidx in everyone:
            rows = (rank_of_expert(pidx, E, R) == rank).any(1).nonzero().flatten() if pidx.numel() else \
                torch.zeros(0, dtype=torch.int64)
            exp.append(px[rows])
        exp = torch.cat(exp)
        got = rx.cpu()
        record['recv_rows'] = int(got.shape[0])
        record['recv_match'] = bool(got.shape == exp.shape and torch.equal(got.view(torch.int16), exp.view(torch.int16)))
        out, _, _ = buf.combine(rx, handle)
        ref = (x.float() * itr.cpu().sum(1, keepdim=True)).to(torch.bfloat16)
        record['combine_match'] = bool(torch.equal(out.cpu(), ref))
        buf.check()
        ok = record['recv_match'] and record['combine_match']
        buf.destroy()
    except Exception as exc:  # noqa: BLE001 - the probe reports failures as data
        record['error'] = f'{type(exc).__name__}: {exc}'
        record['trace'] = traceback.format_exc(limit=3)
        ok = False
    record['status'] = 'pass' if ok else 'fail'
    print('PROBE ' + json.dumps(record), flush=True)
    dist.barrier(group=control)
    dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == '__main__':
    sys.exit(main())
