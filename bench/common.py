"""Shared benchmark plumbing: presets, distributed context, device timing, byte accounting.

Same presets and routing kinds as the reference's bench/common.py:35-40; timing is on
the device (CUDA events on the launching stream, max over ranks) instead of host
wall-clock, because every op here is device-resident.

    pipelined: calls issued back to back, one event pair around N calls (throughput)
    latency:   a synchronisation after every call (what a decode step waiting on each
               layer's communication sees)
"""
from __future__ import annotations

import argparse
import os
import statistics
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import torch
import torch.distributed as dist

from deepep_trn_b200.utils.benchutil import append_jsonl, env_record, max_over_ranks  # noqa: F401
from deepep_trn_b200.utils.testing import make_routing, strided_ep_groups  # noqa: F401

# (hidden, num_experts, top_k)
PRESETS = {
    'qwen3-30b-a3b': (2048, 128, 8),
    'qwen3-235b-a22b': (4096, 128, 8),
    'deepseek-v3': (7168, 256, 8),
}
ROUTINGS = ('random', 'balanced', 'zipf', 'hot_rank0')  # kinds that keep T fixed


def csv_list(kind):
    return lambda s: [kind(v) for v in s.split(',') if v]


def base_parser(description: str) -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=description)
    p.add_argument('--backend', choices=['nvlink', 'nccl', 'gloo'], default='nvlink')
    p.add_argument('--ep', type=int, default=0, help='EP group size (0 = world)')
    p.add_argument('--presets', type=csv_list(str), default=['deepseek-v3'])
    p.add_argument('--tokens', type=csv_list(int), default=[128, 512, 4096], help='tokens per rank')
    p.add_argument('--rounds', type=int, default=5)
    p.add_argument('--iters', type=int, default=20)
    p.add_argument('--out-dir', type=Path, default=ROOT / 'results' / 'adhoc')
    return p


class Ctx:
    """Process-wide distributed state for one EP layout."""

    def __init__(self, backend: str, ep: int):
        self.backend = backend
        timeout = timedelta(seconds=int(os.environ.get('B200EP_PG_TIMEOUT', '300')))
        if backend == 'gloo':
            dist.init_process_group('gloo', timeout=timeout)
            self.device = torch.device('cpu')
        else:
            local = int(os.environ.get('LOCAL_RANK', 0))
            torch.cuda.set_device(local)
            dist.init_process_group('nccl', timeout=timeout, device_id=torch.device('cuda', local))
            self.device = torch.device('cuda', local)
        self.rank, self.world = dist.get_rank(), dist.get_world_size()
        self.control = dist.new_group(backend='gloo')
        self.ep = ep or self.world
        self.groups = strided_ep_groups(self.world, self.ep)
        for ranks in self.groups:  # every rank creates every group, in order
            g = dist.new_group(ranks=ranks, backend='gloo' if backend == 'gloo' else 'nccl')
            if self.rank in ranks:
                self.ep_group, self.peers = g, ranks
        self.ep_rank = self.peers.index(self.rank)

    def buffer(self, num_max_tokens_per_rank: int, **kw):
        from deepep_trn_b200 import Buffer
        return Buffer(self.ep_group, backend=self.backend, num_max_tokens_per_rank=num_max_tokens_per_rank, **kw)

    def sync(self):
        if self.device.type == 'cuda':
            torch.cuda.synchronize()

    def gather(self, obj):
        out = [None] * self.world
        dist.all_gather_object(out, obj, group=self.control)
        return out

    def peer_values(self, obj):
        data = dict(self.gather((self.rank, obj)))
        return [data[p] for p in self.peers]

    def measure(self, call, rounds: int, iters: int, sync_each: bool = False) -> dict:
        """Median/min/max over rounds of the per-call time, max over ranks, device-timed."""
        for _ in range(2):
            call()
        self.sync()
        per_round = []
        for _ in range(rounds):
            dist.barrier(group=self.control)
            if self.device.type == 'cuda':
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                for _ in range(iters):
                    call()
                    if sync_each:
                        torch.cuda.synchronize()
                e.record()
                e.synchronize()
                us = s.elapsed_time(e) * 1e3 / iters
            else:
                import time
                t0 = time.perf_counter()
                for _ in range(iters):
                    call()
                us = (time.perf_counter() - t0) * 1e6 / iters
            per_round.append(max(self.gather(us)))
        return dict(median_us=round(statistics.median(per_round), 2), min_us=round(min(per_round), 2),
                    max_us=round(max(per_round), 2), iters=iters, rounds=rounds)

    def first_call(self, call):
        import time
        t0 = time.perf_counter()
        out = call()
        self.sync()
        return out, max(self.gather(time.perf_counter() - t0))

    def finish(self):
        dist.barrier(group=self.control)
        dist.destroy_process_group()


def gbps(num_bytes: float, us: float) -> float:
    return round(num_bytes / (us * 1e-6) / 1e9, 3) if us > 0 else 0.0
