"""Opt-in per-stage timers for Buffer ops.

Same interface as the reference's ``StageTimer`` (deep_ep_trn/profiling.py:18-46):
``enabled``, ``sync``, ``stage(name)``, ``reset()``, ``per_call_us(n)`` and a module
singleton ``timer``. Two additions for the GPU:

* ``use_cuda_events = True`` times each stage with CUDA events recorded on the
  current stream instead of host wall-clock around a sync, so a stage is charged
  its device time without serialising the pipeline. Events are resolved lazily in
  ``per_call_us``.
* every stage is also an NVTX range (``torch.cuda.nvtx``) when CUDA is present, so
  the stages line up with kernels in a profiler timeline.

Stage names used by the Buffer: ``layout, dispatch, notify_wait, combine,
ll_send, ll_recv`` for the NVLink engine and the reference's ``in_d2h, plan, pack,
h2d, kernel, d2h, unpack, out_h2d`` for the transport engines.
"""
from __future__ import annotations

import time
from collections import defaultdict
from contextlib import contextmanager
from typing import Callable, Optional


class _NullStage:
    __slots__ = ()

    def __enter__(self):
        return None

    def __exit__(self, *exc):
        return False


_NULL_STAGE = _NullStage()


class StageTimer:
    def __init__(self):
        self.enabled = False
        self.sync: Optional[Callable[[], None]] = None
        self.use_cuda_events = False
        self.totals: dict[str, float] = defaultdict(float)
        self._pending: list[tuple[str, object, object]] = []

    def reset(self) -> None:
        self.totals.clear()
        self._pending.clear()

    def stage(self, name: str):
        # disabled (the default): a shared no-op context, no generator per call on the hot path
        return self._stage(name) if self.enabled else _NULL_STAGE

    @contextmanager
    def _stage(self, name: str):
        nvtx = _nvtx()
        if nvtx:
            nvtx.range_push(name)
        if self.use_cuda_events:
            import torch
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            try:
                yield
            finally:
                end.record()
                self._pending.append((name, start, end))
                if nvtx:
                    nvtx.range_pop()
            return
        if self.sync:
            self.sync()
        t0 = time.perf_counter()
        try:
            yield
        finally:
            if self.sync:
                self.sync()
            self.totals[name] += time.perf_counter() - t0
            if nvtx:
                nvtx.range_pop()

    def _resolve(self) -> None:
        for name, start, end in self._pending:
            end.synchronize()
            self.totals[name] += start.elapsed_time(end) * 1e-3
        self._pending.clear()

    def per_call_us(self, calls: int) -> dict[str, float]:
        self._resolve()
        return {k: v * 1e6 / max(calls, 1) for k, v in self.totals.items()}


def _nvtx():
    try:
        import torch
        if torch.cuda.is_available():
            return torch.cuda.nvtx
    except Exception:  # pragma: no cover - torch without CUDA bits
        pass
    return None


timer = StageTimer()
