"""Host-made failures on CPU ranks (gloo): every case must end in an exception on the
ranks that can see the failure, never in a hang.

    config    ranks construct the Buffer with different capacities -> ValueError on
              every rank at construction (one all-gather of the configuration)
    exit      the last rank leaves before the dispatch -> the survivors' dispatch
              raises (the closed connection or the short process-group timeout)
    counts    one rank's handle has corrupted receive counts -> a combine count
              mismatch (RuntimeError) on the ranks whose rows went missing

Each rank prints ``RANK=<r> DETECTED=<exception type>`` (or ``UNDETECTED``) and
exits 0; the pytest wrapper checks the lines. The reference checks the same
conditions by raising (deep_ep_trn/buffer.py:158-160, 244-245, 255-256; the
count check of transport/base.py:48-50).
"""
from __future__ import annotations

import argparse
import os
import sys
from datetime import timedelta
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[2]))

import torch
import torch.distributed as dist


def report(rank: int, exc) -> None:
    # a leading newline keeps the line whole when ranks' outputs interleave
    print(f'\nRANK={rank} DETECTED={type(exc).__name__};' if exc is not None else f'\nRANK={rank} UNDETECTED;',
          flush=True)


def main():
    p = argparse.ArgumentParser()
    p.add_argument('--case', choices=['config', 'exit', 'counts'], required=True)
    args = p.parse_args()
    dist.init_process_group('gloo', timeout=timedelta(seconds=float(os.environ.get('B200EP_PG_TIMEOUT', '20'))))
    torch.set_num_threads(1)
    rank, world = dist.get_rank(), dist.get_world_size()
    from deepep_trn_b200 import Buffer
    T, H, E, K = 16, 64, 4 * world, 2
    g = torch.Generator().manual_seed(rank)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    idx = torch.rand(T, E, generator=g).topk(K, dim=-1).indices
    w = torch.rand(T, K, generator=g)

    if args.case == 'config':
        err = None
        try:
            Buffer(dist.group.WORLD, backend='gloo', num_max_tokens_per_rank=32 * (1 + (rank == 1)))
        except ValueError as e:
            err = e
        report(rank, err)
        dist.barrier()
        dist.destroy_process_group()
        return

    buf = Buffer(dist.group.WORLD, backend='gloo', num_max_tokens_per_rank=32)
    ntr, _, nte, itr, _ = buf.get_dispatch_layout(idx, E)
    if args.case == 'exit':
        dist.barrier()
        if rank == world - 1:
            print(f'RANK={rank} LEAVING', flush=True)
            os._exit(0)  # between steps: nothing of this rank is in flight
        err = None
        try:
            buf.dispatch(x, topk_idx=idx, topk_weights=w, num_tokens_per_rank=ntr, is_token_in_rank=itr,
                         num_tokens_per_expert=nte)
        except Exception as e:  # noqa: BLE001 - the test reports whichever error the survivors see
            err = e
        report(rank, err)
        os._exit(0)  # the group is broken; skip its teardown

    # counts: rank 0 claims one row fewer from its first non-empty source
    rx, ridx, rw, _, handle, _ = buf.dispatch(x, topk_idx=idx, topk_weights=w, num_tokens_per_rank=ntr,
                                              is_token_in_rank=itr, num_tokens_per_expert=nte)
    y = rx
    if rank == 0:
        src = int(torch.nonzero(handle.recv_counts > 0)[0])
        handle.recv_counts = handle.recv_counts.clone()
        handle.recv_counts[src] -= 1
        y = rx[:-1]
    err = None
    try:
        buf.combine(y, handle)
    except RuntimeError as e:
        err = e
    report(rank, err)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == '__main__':
    main()
