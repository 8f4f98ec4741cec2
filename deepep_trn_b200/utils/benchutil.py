"""Benchmark plumbing shared by ``bench.py`` and ``bench/*.py``.

* ``DeviceTimer``: time each step with CUDA events on the launching stream, with an
  L2 flush (a write larger than the 126 MB L2) outside the timed events; totals are
  reduced as the max over ranks.
* ``ClockSampler``: SM clocks / clock-event reasons sampled through NVML every 5 ms
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
    """Samples this process's GPU (SM clock, its maximum, power, clock-event reasons) through
    NVML while active: one sample on entry, one every ``period_s`` from a background thread,
    one on exit, so even a timed region of a few milliseconds is covered. Read-only queries;
    nothing about the GPU is changed. ``merge`` combines the ranks' summaries.
    """

    REASONS = (('hw_slowdown', 'nvmlClocksEventReasonHwSlowdown', 0x8),
               ('hw_thermal_slowdown', 'nvmlClocksEventReasonHwThermalSlowdown', 0x40),
               ('sw_thermal_slowdown', 'nvmlClocksEventReasonSwThermalSlowdown', 0x20),
               ('hw_power_brake', 'nvmlClocksEventReasonHwPowerBrakeSlowdown', 0x80),
               ('sw_power_cap', 'nvmlClocksEventReasonSwPowerCap', 0x4))

    def __init__(self, device: int | None = None, period_s: float = 0.005):
        self.period_s = period_s
        self.samples: list[tuple[float, float, int]] = []   # (sm MHz, max MHz, reason bits)
        self.nvml = None
        self.handle = None
        self._stop = None
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            dev = torch.cuda.current_device() if device is None else device
            props = torch.cuda.get_device_properties(dev)
            bus = f'{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0'
            try:
                self.handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:  # noqa: BLE001 - fall back to the enumeration index
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(dev)
            self.nvml = pynvml
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM))
        except Exception as exc:  # noqa: BLE001 - no NVML: report unavailable
            log(f'clock sampling unavailable: {exc}')

    def _sample(self) -> None:
        p = self.nvml
        try:
            sm = float(p.nvmlDeviceGetClockInfo(self.handle, p.NVML_CLOCK_SM))
            bits = int(p.nvmlDeviceGetCurrentClocksEventReasons(self.handle))
            self.samples.append((sm, self.max_mhz, bits))
        except Exception:  # noqa: BLE001 - a failed read is a missing sample
            pass

    def _loop(self) -> None:
        while not self._stop.wait(self.period_s):
            self._sample()

    def __enter__(self):
        if self.nvml is not None:
            import threading
            self._sample()
            self._stop = threading.Event()
            self._thread = threading.Thread(target=self._loop, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)
            self._sample()

    def summary(self) -> dict:
        if self.nvml is None:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': ['unavailable']}
        if not self.samples:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': ['no samples']}
        top = max(m for _, m, _ in self.samples)
        sm = [s for s, _, _ in self.samples]
        loaded = [v for v in sm if v > 0.5 * top] or sm   # under load (idle drops far below)
        reasons = set()
        for _, _, bits in self.samples:
            for name, attr, default in self.REASONS:
                if bits & int(getattr(self.nvml, attr, default)):
                    reasons.add(name)
        return {'sm_mhz': statistics.median(loaded), 'sm_max_mhz': top, 'reasons': sorted(reasons),
                'samples': len(self.samples)}

    @staticmethod
    def merge(summaries: list[dict]) -> dict:
        """All ranks' summaries -> one: median of the per-GPU medians, the lowest maximum, all reasons."""
        have = [s for s in summaries if s.get('sm_mhz') is not None]
        if not have:
            return summaries[0] if summaries else {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': ['no samples']}
        reasons = sorted({r for s in have for r in s['reasons']})
        return {'sm_mhz': statistics.median(s['sm_mhz'] for s in have),
                'sm_min_gpu_mhz': min(s['sm_mhz'] for s in have),
                'sm_max_mhz': min(s['sm_max_mhz'] for s in have), 'reasons': reasons,
                'samples': sum(s.get('samples', 0) for s in have), 'gpus': len(have)}


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
    try:  # GPU interconnect matrix (NVLink / NVSwitch paths between the GPUs of the node)
        topo = subprocess.run(['nvidia-smi', 'topo', '-m'], capture_output=True, text=True, timeout=20).stdout
        rec['topo'] = topo.strip().splitlines()[:12] if topo else None
    except Exception:
        rec['topo'] = None
    try:
        rec['nccl'] = '.'.join(map(str, torch.cuda.nccl.version()))
    except Exception:
        rec['nccl'] = None
    return rec


def append_jsonl(path: Path, record: dict) -> None:
    path.parent.mkdir(parents=True, exist_ok=True)
    with open(path, 'a') as f:
        f.write(json.dumps(record) + '\n')
