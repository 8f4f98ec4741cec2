"""Plumbing of the torchrun benchmark scripts in this directory.

* ``PRESETS``: (hidden, experts, top-k) of the model shapes the suite sweeps; the same
  three models as the reference suite, so its published rows have counterparts here.
* ``cli``: the flags every script shares (backend, EP size, presets, token counts,
  repetitions, output directory).
* ``BenchGroup``: the world process group, a gloo side group for metadata, and this
  rank's EP group (strided layout, built identically on every rank).
* ``device_stats``: device time of a callable from CUDA events on the launching stream,
  either back to back (throughput) or with a synchronisation after every call (what a
  step waiting on each op sees); the per-repetition value is the max over ranks, the
  record keeps the median, min and max over repetitions. CPU ranks fall back to the
  host clock.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import torch
import torch.distributed as dist

from deepep_trn_b200.utils.benchutil import env_record  # noqa: F401  (re-exported for the scripts)
from deepep_trn_b200.utils.testing import make_routing, strided_ep_groups  # noqa: F401

PRESETS = {
    'qwen3-30b-a3b': (2048, 128, 8),
    'qwen3-235b-a22b': (4096, 128, 8),
    'deepseek-v3': (7168, 256, 8),
}
ROUTINGS = ('random', 'balanced', 'zipf', 'hot_rank0')  # routing kinds with a fixed token count


def ints(s: str) -> list[int]:
    return [int(v) for v in s.split(',') if v]


def words(s: str) -> list[str]:
    return [v for v in s.split(',') if v]


def cli(doc: str) -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=doc, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument('--backend', choices=['nvlink', 'nccl', 'gloo'], default='nvlink')
    p.add_argument('--ep', type=int, default=0, help='ranks per EP group (0: all)')
    p.add_argument('--presets', type=words, default=['deepseek-v3'])
    p.add_argument('--tokens', type=ints, default=[128, 512, 4096], help='tokens per rank')
    p.add_argument('--rounds', type=int, default=5, help='timed repetitions')
    p.add_argument('--iters', type=int, default=20, help='calls per repetition')
    p.add_argument('--out-dir', type=Path, default=ROOT / 'results' / 'adhoc')
    return p


class BenchGroup:
    def __init__(self, backend: str, ep: int = 0):
        self.backend = backend
        wait = timedelta(seconds=int(os.environ.get('B200EP_PG_TIMEOUT', '300')))
        if backend == 'gloo':
            dist.init_process_group('gloo', timeout=wait)
            self.device = torch.device('cpu')
        else:
            self.device = torch.device('cuda', int(os.environ.get('LOCAL_RANK', 0)))
            torch.cuda.set_device(self.device)
            dist.init_process_group('nccl', timeout=wait, device_id=self.device)
        self.rank, self.world = dist.get_rank(), dist.get_world_size()
        self.meta = dist.new_group(backend='gloo')
        self.ep = ep or self.world
        self.layout = strided_ep_groups(self.world, self.ep)
        for ranks in self.layout:
            g = dist.new_group(ranks=ranks, backend='gloo' if backend == 'gloo' else 'nccl')
            if self.rank in ranks:
                self.group, self.members = g, list(ranks)
        self.ep_rank = self.members.index(self.rank)

    def new_buffer(self, tokens: int, **kw):
        from deepep_trn_b200 import Buffer
        return Buffer(self.group, backend=self.backend, num_max_tokens_per_rank=tokens, **kw)

    def gather(self, obj) -> list:
        got = [None] * self.world
        dist.all_gather_object(got, obj, group=self.meta)
        return got

    def over_group(self, obj) -> list:
        """``obj`` of every member of this rank's EP group, in group order."""
        mine = dict(self.gather((self.rank, obj)))
        return [mine[r] for r in self.members]

    def sync(self) -> None:
        if self.device.type == 'cuda':
            torch.cuda.synchronize()

    def close(self) -> None:
        dist.barrier(group=self.meta)
        dist.destroy_process_group()


def device_stats(bg: BenchGroup, fn, rounds: int, iters: int, each: bool = False, warm: int = 2) -> dict:
    for _ in range(warm):
        fn()
    bg.sync()
    per = []
    for _ in range(rounds):
        dist.barrier(group=bg.meta)
        if bg.device.type == 'cuda':
            start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            for _ in range(iters):
                fn()
                if each:
                    torch.cuda.synchronize()
            stop.record()
            stop.synchronize()
            us = start.elapsed_time(stop) * 1e3 / iters
        else:
            t0 = time.perf_counter()
            for _ in range(iters):
                fn()
            us = (time.perf_counter() - t0) * 1e6 / iters
        per.append(max(bg.gather(us)))
    return {'median_us': round(statistics.median(per), 2), 'min_us': round(min(per), 2),
            'max_us': round(max(per), 2), 'iters': iters, 'rounds': rounds}


def wall_once(bg: BenchGroup, fn):
    """Host time of one call including its device work (max over ranks) and its result."""
    t0 = time.perf_counter()
    out = fn()
    bg.sync()
    return out, max(bg.gather(time.perf_counter() - t0))


def gbps(num_bytes: float, us: float) -> float:
    return round(num_bytes / us / 1e3, 3) if us > 0 else 0.0


def write_jsonl(path: Path, record: dict) -> None:
    path.parent.mkdir(parents=True, exist_ok=True)
    with path.open('a') as f:
        f.write(json.dumps(record) + '\n')
