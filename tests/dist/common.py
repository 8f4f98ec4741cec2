"""Shared setup of the torchrun scenario tests (reference: tests/dist/common.py of deep_ep_trn).

Run under torchrun. ``--backend gloo`` keeps every tensor on the CPU (the
oracle semantics); ``--backend nvlink`` / ``nccl`` put them on ``cuda:LOCAL_RANK``.
The oracle data always travels over a separate gloo control group, so it is
independent of the path under test.
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

from deepep_trn_b200.utils.testing import (bitwise_equal, expert_scale, make_routing,  # noqa: F401
                                           strided_ep_groups)

KINDS = ('balanced', 'random', 'hot_rank0', 'ragged', 'masked')


def parse_args(description: str):
    p = argparse.ArgumentParser(description=description)
    p.add_argument('--backend', choices=['nvlink', 'nccl', 'gloo'], default='gloo')
    p.add_argument('--ep', type=int, default=0, help='EP group size (0 = world)')
    p.add_argument('--tokens', type=int, default=24)
    p.add_argument('--max-tokens', type=int, default=32)
    p.add_argument('--hidden', type=int, default=256)
    p.add_argument('--experts', type=int, default=32)
    p.add_argument('--topk', type=int, default=4)
    p.add_argument('--kinds', default=','.join(KINDS))
    p.add_argument('--fp8', type=int, default=1)
    p.add_argument('--graph', type=int, default=0)
    return p.parse_args()


def init(backend: str):
    timeout = timedelta(seconds=int(os.environ.get('B200EP_PG_TIMEOUT', '120')))
    if backend == 'gloo':
        dist.init_process_group('gloo', timeout=timeout)
    else:
        torch.cuda.set_device(int(os.environ.get('LOCAL_RANK', 0)))
        dist.init_process_group('nccl', timeout=timeout, device_id=torch.device('cuda', torch.cuda.current_device()))
    torch.set_num_threads(1)
    return dist.get_rank(), dist.get_world_size(), dist.new_group(backend='gloo')


def make_buffer(backend: str, ep: int, max_tokens: int, **kw):
    from deepep_trn_b200 import Buffer
    rank, world = dist.get_rank(), dist.get_world_size()
    ep = ep or world
    groups = strided_ep_groups(world, ep)
    mine = peers = None
    for ranks in groups:  # every rank creates every group, in the same order
        g = dist.new_group(ranks=ranks, backend='gloo' if backend == 'gloo' else 'nccl')
        if rank in ranks:
            mine, peers = g, ranks
    buf = Buffer(mine, backend=backend, replica_groups=groups, num_max_tokens_per_rank=max_tokens, **kw)
    return buf, peers


def gather_peers(obj, peers, control):
    everyone = [None] * dist.get_world_size()
    dist.all_gather_object(everyone, (dist.get_rank(), obj), group=control)
    data = dict(everyone)
    return [data[p] for p in peers]


def device(backend: str):
    return torch.device('cpu') if backend == 'gloo' else torch.device('cuda', torch.cuda.current_device())


def finish(control, buf=None):
    dist.barrier(group=control)
    if buf is not None:
        buf.destroy()
    dist.destroy_process_group()
