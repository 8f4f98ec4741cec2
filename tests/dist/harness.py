"""Process-group plumbing for the torchrun scenario scripts in this directory.

A ``Scenario`` owns everything a script needs besides the checks themselves:

* the command line (``backend`` plus the shape flags every scenario understands),
* the world process group (gloo on CPU ranks, NCCL with one GPU per rank otherwise)
  and a separate gloo group that carries oracle data, so the oracle never travels
  over the path under test,
* the EP groups: the world split into strided groups of ``--ep`` ranks (TP x EP
  layouts such as ``[[0, 2], [1, 3]]``), built in the same order on every rank,
* ``share(obj)``: the objects of every rank of this rank's EP group, in group order,
* ``dev(t)`` / ``host(t)``: move tensors to the backend's device and back.

Scripts end with ``sc.done(tag)``, which meets every rank, tears the buffer and the
process group down and prints ``<tag>_PASS`` on rank 0.
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

from deepep_trn_b200.utils.testing import strided_ep_groups

ROUTING_KINDS = 'balanced,random,hot_rank0,ragged,masked'


class Scenario:
    def __init__(self, doc: str, extra=None):
        cli = argparse.ArgumentParser(description=doc)
        cli.add_argument('--backend', choices=['nvlink', 'nccl', 'gloo'], default='gloo')
        cli.add_argument('--ep', type=int, default=0, help='ranks per EP group (0: the whole world)')
        for flag, default in (('tokens', 24), ('max-tokens', 32), ('hidden', 256), ('experts', 32), ('topk', 4),
                              ('fp8', 1), ('graph', 0)):
            cli.add_argument(f'--{flag}', type=int, default=default)
        cli.add_argument('--kinds', default=ROUTING_KINDS)
        if extra is not None:
            extra(cli)
        self.args = cli.parse_args()
        self.backend = self.args.backend
        wait = timedelta(seconds=int(os.environ.get('B200EP_PG_TIMEOUT', '120')))
        if self.backend == 'gloo':
            dist.init_process_group('gloo', timeout=wait)
            self.device = torch.device('cpu')
        else:
            torch.cuda.set_device(int(os.environ.get('LOCAL_RANK', 0)))
            self.device = torch.device('cuda', torch.cuda.current_device())
            dist.init_process_group('nccl', timeout=wait, device_id=self.device)
        torch.set_num_threads(1)
        self.rank, self.world = dist.get_rank(), dist.get_world_size()
        self.oracle_group = dist.new_group(backend='gloo')
        self.layout = strided_ep_groups(self.world, self.args.ep or self.world)
        self.group = None
        self.members: list[int] = []
        for ranks in self.layout:
            g = dist.new_group(ranks=ranks, backend='gloo' if self.backend == 'gloo' else 'nccl')
            if self.rank in ranks:
                self.group, self.members = g, list(ranks)
        self.buf = None

    def buffer(self, **kw):
        from deepep_trn_b200 import Buffer
        self.buf = Buffer(self.group, backend=self.backend, replica_groups=self.layout,
                          num_max_tokens_per_rank=self.args.max_tokens, **kw)
        return self.buf

    def share(self, obj) -> list:
        """``obj`` of every member of this rank's EP group, in group order (over the gloo group)."""
        got = [None] * self.world
        dist.all_gather_object(got, (self.rank, obj), group=self.oracle_group)
        by_rank = dict(got)
        return [by_rank[r] for r in self.members]

    def all_ok(self, ok: bool) -> bool:
        """True on every rank iff ``ok`` holds on every rank."""
        return all(self.share_world(bool(ok)))

    def share_world(self, obj) -> list:
        got = [None] * self.world
        dist.all_gather_object(got, obj, group=self.oracle_group)
        return got

    def dev(self, t):
        return t.to(self.device) if isinstance(t, torch.Tensor) else tuple(x.to(self.device) for x in t)

    @staticmethod
    def host(t):
        return t.cpu() if isinstance(t, torch.Tensor) else tuple(x.cpu() for x in t)

    def log(self, msg: str) -> None:
        print(f'RANK={self.rank} {msg}', flush=True)

    def done(self, tag: str) -> None:
        dist.barrier(group=self.oracle_group)
        if self.buf is not None:
            self.buf.destroy()
        dist.destroy_process_group()
        if self.rank == 0:
            print(f'{tag}_PASS backend={self.backend} ep={len(self.members)}', flush=True)
