"""deep_ep-compatible ``Buffer`` for one B200 node (expert parallelism over NVLink).

API surface and semantics follow deep_ep_trn/buffer.py:78-364 (itself deep_ep's
Python API): ``get_dispatch_layout``, ``dispatch`` / ``combine`` with reusable
handles and cached dispatch, ``low_latency_dispatch`` / ``low_latency_combine``
with receive hooks, the deep_ep static shims and the same error behaviour
(``ValueError`` for capacity, missing layout inputs, bad backend or group,
``RuntimeError`` for count mismatches).

Backends:
  ``'nvlink'`` (default on CUDA) - hand-written sm_100a kernels reading and writing
      peer GPUs' memory through an IPC-mapped symmetric heap; no NCCL on the data path.
  ``'gloo'``  - reference semantics on CPU processes; the oracle for tests.
  ``'nccl'``  - reference semantics as torch ops + NCCL all_to_all_single on the
      device; the baseline the NVLink kernels are measured against.

Beyond the reference (which raises ``NotImplementedError`` for these): fp8
``(x, scales)`` dispatch input, in-kernel fp8 quantisation (``use_fp8=True`` on
dispatch), fp8 low-latency dispatch (the deep_ep default), real ``EventOverlap``
and ``async_finish`` on a communication stream, real receive hooks,
``num_worst_tokens`` (sync-free, graph-capturable normal dispatch) and combine
``bias``. LogFMT combine is still unimplemented.
"""
from __future__ import annotations

import os
from typing import Optional

import torch
import torch.distributed as dist

from .handles import Config, DispatchHandle, EventOverlap, LowLatencyHandle
from .parallel.transport import GlooTransport, NcclTransport, Transport

__all__ = ['Buffer', 'Config', 'DispatchHandle', 'EventOverlap', 'LowLatencyHandle']


def check_agreement(group, config: dict) -> None:
    """Raise ``ValueError`` on every rank if the ranks of ``group`` were given different ``config``.

    One all-gather at construction; a mismatch (say, ranks sized for different token
    capacities) would otherwise surface later as a capacity error or a timed-out wait
    on one rank only.
    """
    world = dist.get_world_size(group)
    seen = [None] * world
    dist.all_gather_object(seen, config, group=group)
    diff = {k: {r: c.get(k) for r, c in enumerate(seen)} for k in config
            if len({repr(c.get(k)) for c in seen}) > 1}
    if diff:
        raise ValueError(f'Buffer configuration differs across the ranks of the group: {diff}')


def _default_timeout() -> float:
    return float(os.environ.get('B200EP_TIMEOUT_S', '10'))


class Buffer:
    """Expert-parallel communication buffer.

    Args:
        group: EP process group (any subgroup of the world; peers are its ranks).
        num_nvl_bytes, num_rdma_bytes, low_latency_mode: accepted for deep_ep source
            compatibility. Buffers are sized from ``num_max_tokens_per_rank`` and the
            shapes of the first op instead (pass ``hidden``/``num_experts``/``topk``
            to allocate at construction).
        num_max_tokens_per_rank: normal-mode token capacity per rank (same on every rank).
        backend: ``'nvlink'``, ``'gloo'``, ``'nccl'`` or ``'auto'`` (nvlink when CUDA is
            available, else gloo).
        replica_groups: every EP group of the world, e.g. ``[[0, 2], [1, 3]]``; only
            validated (peers are taken from ``group``).
        transport: use this transport (torch engine) instead of building one.
    """

    num_sms: int = 0  # CTAs per communication kernel, 0 = all SMs (deep_ep set_num_sms)

    def __init__(self, group, num_nvl_bytes: int = 0, num_rdma_bytes: int = 0, low_latency_mode: bool = False,
                 *, num_max_tokens_per_rank: int = 128, backend: str = 'auto', replica_groups=None,
                 transport: Optional[Transport] = None, hidden: Optional[int] = None,
                 num_experts: Optional[int] = None, topk: Optional[int] = None,
                 num_max_dispatch_tokens_per_rank: Optional[int] = None, timeout_s: Optional[float] = None,
                 **deepep_kwargs):
        self.group = group
        self.num_max_tokens_per_rank = int(num_max_tokens_per_rank)
        self.low_latency_mode = low_latency_mode
        world = dist.get_world_size(group)
        if replica_groups is not None:
            ranks = dist.get_process_group_ranks(group)
            me = dist.get_rank()
            mine = [list(g) for g in replica_groups if me in g]
            if len(mine) != 1:
                raise ValueError(f'rank {me} must be in exactly one of {replica_groups}')
            if sorted(mine[0]) != sorted(ranks):
                raise ValueError(f'replica group {mine[0]} does not match the EP group {ranks}')
        if backend == 'auto':
            backend = 'nvlink' if (transport is None and torch.cuda.is_available()) else 'gloo'
        if backend not in ('nvlink', 'gloo', 'nccl'):
            raise ValueError(f'unknown backend {backend!r}')
        self.backend = backend
        if world > 1:
            check_agreement(group, dict(backend=backend, num_max_tokens_per_rank=self.num_max_tokens_per_rank,
                                        num_max_dispatch_tokens_per_rank=num_max_dispatch_tokens_per_rank,
                                        hidden=hidden, num_experts=num_experts, topk=topk))
        self.timeout_s = timeout_s if timeout_s is not None else _default_timeout()
        self.comm_stream = torch.cuda.Stream() if torch.cuda.is_available() and backend != 'gloo' else None
        self._last_event = None
        if transport is not None or backend in ('gloo', 'nccl'):
            from .parallel.engine_torch import TorchEngine
            if transport is None:
                transport = GlooTransport(group) if backend == 'gloo' else NcclTransport(group)
            if transport.num_ranks != world:
                raise ValueError(f'transport has {transport.num_ranks} ranks, group has {world}')
            self.transport = transport
            self._engine = TorchEngine(transport, self.num_max_tokens_per_rank)
        elif backend == 'nvlink':
            from .parallel.engine_nvlink import NvlinkEngine
            from .parallel.symm import HeapSpec
            hint = None
            if hidden and num_experts and topk:
                hint = HeapSpec(self.num_max_tokens_per_rank, int(num_max_dispatch_tokens_per_rank or 1),
                                int(hidden), int(topk), int(num_experts))
            self.transport = None
            self._engine = NvlinkEngine(group, self.num_max_tokens_per_rank, self.timeout_s, hint)
        else:
            raise ValueError(f'unknown backend {backend!r}')
        self.rank = dist.get_rank(group)
        self.group_size = world

    @property
    def last_exchange(self):
        """Shape of the most recent exchange (lets benchmarks replay the bare op)."""
        return self._engine.last_exchange

    # ------------------------------------------------------------------ deep_ep statics
    @staticmethod
    def set_num_sms(new_num_sms: int) -> None:
        Buffer.num_sms = int(new_num_sms)

    @staticmethod
    def get_dispatch_config(num_ranks: int) -> Config:
        return Config(num_sms=Buffer.num_sms)

    @staticmethod
    def get_combine_config(num_ranks: int) -> Config:
        return Config(num_sms=Buffer.num_sms)

    @staticmethod
    def get_low_latency_rdma_size_hint(num_max_dispatch_tokens_per_rank: int, hidden: int, num_ranks: int,
                                       num_experts: int) -> int:
        return 0  # single node: no RDMA buffer

    @staticmethod
    def get_low_latency_nvl_size_hint(num_max_dispatch_tokens_per_rank: int, hidden: int, num_ranks: int,
                                      num_experts: int, topk: int = 8) -> int:
        from .parallel.symm import HeapSpec, heap_bytes
        return heap_bytes(num_ranks, HeapSpec(1, num_max_dispatch_tokens_per_rank, hidden, topk, num_experts))

    def destroy(self) -> None:
        if hasattr(self._engine, 'destroy'):
            self._engine.destroy()

    def clean_low_latency_buffer(self, *args, **kwargs) -> None:
        """No-op: flags are epoch-tagged, so low-latency buffers never need cleaning."""

    def device_trace(self) -> dict:
        """Per-phase device time (us) of the last normal-mode dispatch and combine (NVLink backend)."""
        return self._engine.device_trace() if hasattr(self._engine, 'device_trace') else {}

    def check_canaries(self) -> None:
        """Raise if any kernel wrote past the end of a region of this rank's symmetric heap
        (guard zones filled with a known byte at construction; NVLink backend, a debugging aid
        that synchronises the device)."""
        if hasattr(self._engine, 'check_canaries'):
            self._engine.check_canaries()

    def check(self) -> None:
        """Raise if a kernel of this buffer reported a device-side error (timeouts, capacity)."""
        if hasattr(self._engine, 'check'):
            self._engine.check()

    # ------------------------------------------------------------------ stream plumbing
    def _run(self, fn, previous_event, async_finish, allocate_on_comm_stream):
        if self.comm_stream is None or not (async_finish or previous_event is not None or allocate_on_comm_stream):
            if self._last_event is not None:
                torch.cuda.current_stream().wait_event(self._last_event)
                self._last_event = None
            return fn(), None
        compute, comm = torch.cuda.current_stream(), self.comm_stream
        if previous_event is not None and previous_event.event is not None:
            comm.wait_event(previous_event.event)
        else:
            comm.wait_stream(compute)
        with torch.cuda.stream(comm):
            result = fn()
        ev = torch.cuda.Event()
        ev.record(comm)
        _record(result, compute)
        if async_finish:
            self._last_event = ev
        else:
            compute.wait_event(ev)
        return result, ev

    def _check_tokens(self, num_tokens: int, limit: int) -> None:
        if num_tokens > limit:
            raise ValueError(f'{num_tokens} tokens exceed the per-rank capacity {limit}')

    # ------------------------------------------------------------------ normal mode
    def get_dispatch_layout(self, topk_idx: torch.Tensor, num_experts: int, previous_event=None,
                            async_finish: bool = False, allocate_on_comm_stream: bool = False):
        """Returns ``(num_tokens_per_rank [R] int32, None, num_tokens_per_expert [E] int32,
        is_token_in_rank [T, R] bool, event)``; the None is deep_ep's RDMA slot."""
        (ntr, nte, itr), ev = self._run(lambda: self._engine.get_dispatch_layout(topk_idx, num_experts),
                                        previous_event, async_finish, allocate_on_comm_stream)
        return ntr, None, nte, itr, EventOverlap(ev)

    def dispatch(self, x, handle: Optional[DispatchHandle] = None, num_tokens_per_rank=None,
                 num_tokens_per_rdma_rank=None, is_token_in_rank=None, num_tokens_per_expert=None,
                 topk_idx=None, topk_weights=None, expert_alignment: int = 1, num_worst_tokens: int = 0,
                 config=None, previous_event=None, async_finish: bool = False,
                 allocate_on_comm_stream: bool = False, use_fp8: bool = False, round_scale: bool = False):
        """Send each token once to every rank that owns one of its experts.

        ``x`` is ``[T, H]`` bf16/fp16 or an fp8 tuple ``(x_e4m3 [T, H], scales [T, H/128] fp32)``.
        ``use_fp8=True`` quantises a bf16 ``x`` to e4m3 1x128 inside the dispatch kernel.
        Received rows are ordered by source rank, then source token. Returns
        ``(recv_x, recv_topk_idx, recv_topk_weights, num_recv_tokens_per_expert_list, handle,
        event)``; the top-k outputs and the list are None for a cached dispatch.
        """
        xt = x[0] if isinstance(x, tuple) else x
        cached = handle is not None
        if not cached and (topk_idx is None or num_tokens_per_expert is None):
            raise ValueError('dispatch needs topk_idx and num_tokens_per_expert (see get_dispatch_layout)')
        self._check_tokens(xt.shape[0], self.num_max_tokens_per_rank)
        if isinstance(x, tuple) and self.backend == 'gloo' and not xt.shape[1] % 128 == 0:
            raise ValueError('fp8 dispatch needs hidden % 128 == 0')
        if use_fp8 and self.backend != 'nvlink':
            from .utils.codec import quantize_fp8_1x128
            x = quantize_fp8_1x128(xt, round_scale)
        num_experts = handle.num_experts if cached else num_tokens_per_expert.numel()
        if self.backend == 'nvlink':
            fn = lambda: self._engine.dispatch(x, handle, topk_idx, topk_weights, is_token_in_rank, num_experts,
                                               expert_alignment, num_worst_tokens, config, use_fp8, round_scale,
                                               num_tokens_per_expert)
        else:
            if num_worst_tokens:
                raise NotImplementedError('num_worst_tokens needs the nvlink backend')
            fn = lambda: self._engine.dispatch(x, handle, topk_idx, topk_weights, is_token_in_rank, num_experts,
                                               expert_alignment)
        out, ev = self._run(fn, previous_event, async_finish, allocate_on_comm_stream)
        return (*out[:5], EventOverlap(ev))

    def combine(self, x, handle: DispatchHandle, topk_weights=None, bias=None, config=None,
                previous_event=None, async_finish: bool = False, allocate_on_comm_stream: bool = False,
                pair_pos=None, pair_weights=None):
        """Return every received row to its source and sum per token (fp32, one cast).

        ``bias`` (a tensor or a pair of tensors ``[T, H]``) is added before the cast.
        With ``pair_pos`` / ``pair_weights`` (``[N, K]``), ``x`` holds the expert outputs in
        permuted order (``[P, H]``) and received row n is ``sum_k pair_weights[n, k] *
        x[pair_pos[n, k]]`` (fp32, one cast; -1 = no pair): the weighted un-permute runs
        inside the combine kernel instead of as a separate pass.
        Returns ``(combined_x, combined_topk_weights, event)``.
        """
        biases = () if bias is None else (tuple(bias) if isinstance(bias, (tuple, list)) else (bias,))
        pairs = None
        if pair_pos is not None:
            if pair_weights is None:
                raise ValueError('pair_pos needs pair_weights')
            pairs = (pair_pos, pair_weights)
        if self.backend == 'nvlink':
            fn = lambda: self._engine.combine(x, handle, topk_weights, biases, config, pairs)
        else:
            if pairs is not None:
                from .ops.moe_ops import unpermute
                x = unpermute(x, pair_pos, pair_weights)
            fn = lambda: self._engine.combine(x, handle, topk_weights, biases)
        out, ev = self._run(fn, previous_event, async_finish, allocate_on_comm_stream)
        return out[0], out[1], EventOverlap(ev)

    # ------------------------------------------------------------------ low-latency mode
    def low_latency_dispatch(self, x, topk_idx, num_max_dispatch_tokens_per_rank: int, num_experts: int,
                             cumulative_local_expert_recv_stats=None, dispatch_wait_recv_cost_stats=None,
                             use_fp8: bool = True, round_scale: bool = False, use_ue8m0: bool = False,
                             async_finish: bool = False, return_recv_hook: bool = False):
        """Dispatch into the expert-major layout ``[EL, R*M, H]`` (fp8 e4m3 + 1x128 scales by default).

        Returns ``(recv_x | (recv_x_fp8, scales), recv_count [EL] int32, handle, event, hook)``.
        Rows past ``recv_count[e]`` are unspecified. With ``return_recv_hook`` only the
        send kernel runs now; calling ``hook()`` launches the receive kernel.
        """
        M = int(num_max_dispatch_tokens_per_rank)
        self._check_tokens(x.shape[0], M)
        if self.backend == 'nvlink':
            fn = lambda: self._engine.low_latency_dispatch(
                x, topk_idx, M, num_experts, use_fp8, round_scale, use_ue8m0, cumulative_local_expert_recv_stats,
                dispatch_wait_recv_cost_stats, return_recv_hook)
            (recv_x, count, handle, _, hook), ev = self._run(fn, None, async_finish, False)
        else:
            (recv_x, count, handle), ev = self._run(
                lambda: self._engine.low_latency_dispatch(x, topk_idx, M, num_experts, use_fp8, round_scale,
                                                          use_ue8m0, cumulative_local_expert_recv_stats),
                None, async_finish, False)
            hook = _noop if return_recv_hook else None
        return recv_x, count, handle, EventOverlap(ev), hook

    def low_latency_combine(self, x, topk_idx, topk_weights, handle: LowLatencyHandle, use_logfmt: bool = False,
                            zero_copy: bool = False, async_finish: bool = False, return_recv_hook: bool = False,
                            out: Optional[torch.Tensor] = None):
        """Return one row per (token, expert); the source applies the top-k weights in fp32.

        Returns ``(combined_x [T, H], event, hook)``.
        """
        if use_logfmt:
            raise NotImplementedError('LogFMT combine is not implemented')
        if self.backend == 'nvlink':
            fn = lambda: self._engine.low_latency_combine(x, topk_idx, topk_weights, handle, zero_copy,
                                                          return_recv_hook, out)
            (combined, _, hook), ev = self._run(fn, None, async_finish, False)
        else:
            combined, ev = self._run(lambda: self._engine.low_latency_combine(x, topk_idx, topk_weights, handle, out),
                                     None, async_finish, False)
            hook = _noop if return_recv_hook else None
        return combined, EventOverlap(ev), hook


def _noop() -> None:
    pass


def _record(obj, stream) -> None:
    if isinstance(obj, torch.Tensor):
        if obj.is_cuda:
            obj.record_stream(stream)
    elif isinstance(obj, (tuple, list)):
        for o in obj:
            _record(o, stream)
