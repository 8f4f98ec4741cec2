"""Benchmark plumbing shared by ``bench.py`` and ``bench/*.py``.

* ``DeviceTimer``: time each step with CUDA events on the launching stream, with an
  L2 flush (a write larger than the 126 MB L2) outside the timed events; totals are
  reduced as the max over ranks.
* ``ClockSampler``: ``nvidia-smi`` clocks / throttle reasons sampled every 200 ms
  during the timed region, summarised as median SM MHz under load.
* ``env_record``: versions and hardware for the JSONL records (reference
  bench/common.py:147-177 captures the same kind of metadata).
"""
from __future__ import annotations

import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch
import torch.distributed as dist

L2_FLUSH_BYTES = 256 << 20


def log(*a) -> None:
    print(*a, file=sys.stderr, flush=True)


class DeviceTimer:
    def __init__(self, flush_l2: bool = True):
        self.flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device='cuda') if flush_l2 else None
        self.events: list[tuple[torch.cuda.Event, torch.cuda.Event]] = []

    def run(self, fn):
        if self.flush is not None:
            self.flush.fill_(1)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        out = fn()
        e.record()
        self.events.append((s, e))
        return out

    def total_ms(self) -> float:
        torch.cuda.synchronize()
        return sum(s.elapsed_time(e) for s, e in self.events)


def max_over_ranks(value: float, group=None) -> float:
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device='cuda' if torch.cuda.is_available() else 'cpu')
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def sum_over_ranks(value: float, group=None) -> float:
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device='cuda' if torch.cuda.is_available() else 'cpu')
    dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return float(t.item())


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi while active."""

    FIELDS = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
              'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
              'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, gpus: list[int]):
        self.gpus = gpus
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix='.csv')
            os.close(fd)
            self.proc = subprocess.Popen(['nvidia-smi', f'--query-gpu={self.FIELDS}', '--format=csv,noheader,nounits',
                                          '-lms', '200', '-f', self.path],
                                         stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except Exception as exc:  # nvidia-smi missing
            log(f'clock sampling unavailable: {exc}')
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if self.path is None or not Path(self.path).exists():
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': ['unavailable']}
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(',')]
            if len(parts) < 9:
                continue
            try:
                idx = int(parts[0])
            except ValueError:
                continue
            if idx not in self.gpus:
                continue
            rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': ['no samples']}
        sm = [float(r[1]) for r in rows if r[1].replace('.', '').isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace('.', '').isdigit()]
        # "under load": samples above half of max (idle samples drop to ~100s of MHz)
        top = max(mx) if mx else 0
        loaded = [v for v in sm if v > 0.5 * top] or sm
        reasons = set()
        names = ('hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap')
        for r in rows:
            for n, v in zip(names, r[5:9]):
                if v.strip().lower() == 'active':
                    reasons.add(n)
        return {'sm_mhz': statistics.median(loaded) if loaded else None, 'sm_max_mhz': top or None,
                'reasons': sorted(reasons), 'samples': len(rows)}


def env_record() -> dict:
    rec = dict(torch=torch.__version__, cuda=torch.version.cuda, python=sys.version.split()[0])
    if torch.cuda.is_available():
        rec['gpu'] = torch.cuda.get_device_name()
        rec['sms'] = torch.cuda.get_device_properties(0).multi_processor_count
    try:
        rec['driver'] = subprocess.run(['nvidia-smi', '--query-gpu=driver_version', '--format=csv,noheader'],
                                       capture_output=True, text=True, timeout=20).stdout.split('\n')[0].strip()
    except Exception:
        rec['driver'] = None
    try:
        rec['nccl'] = '.'.join(map(str, torch.cuda.nccl.version()))
    except Exception:
        rec['nccl'] = None
    return rec


def append_jsonl(path: Path, record: dict) -> None:
    path.parent.mkdir(parents=True, exist_ok=True)
    with open(path, 'a') as f:
        f.write(json.dumps(record) + '\n')
