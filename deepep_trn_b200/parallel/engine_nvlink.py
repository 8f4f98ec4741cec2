"""NVLink engine: drives the sm_100a kernels over the IPC-mapped symmetric heap.

One op = one or two kernel launches on the caller's stream:

  get_dispatch_layout  -> layout kernel (N1), no host round trip
  dispatch             -> nd_dispatch (one cooperative kernel: scan, count exchange, push
                          rows into the peers' inboxes, copy received rows out); the host
                          waits on a host-mapped ticket for the receive size while the
                          kernel is still moving rows (skipped for a cached dispatch or
                          with num_worst_tokens)
  combine              -> nc_combine (one cooperative kernel: push rows home, fp32 reduce)
  low_latency_dispatch -> ll_dispatch_send [+ ll_dispatch_recv, or via the hook]
  low_latency_combine  -> ll_combine_send  [+ ll_combine_recv, or via the hook]

Low-latency ops never touch the host and are CUDA-graph capturable once the
heap exists (call them once before capture).
"""
from __future__ import annotations


import torch
import torch.distributed as dist

from ..handles import DispatchHandle, EventOverlap, LowLatencyHandle
from ..ops._ext import load
from ..utils.layout import experts_per_rank
from ..utils.profiling import timer
from .symm import HeapSpec, create_heap

ERRORS = {1: 'timeout waiting for a peer to stage dispatch data', 2: 'timeout waiting for combine rows',
          3: 'low-latency: timeout waiting for a source header', 4: 'low-latency: timeout waiting for a row',
          5: 'low-latency combine: timeout waiting for a (token, k) row', 6: 'capacity exceeded',
          7: 'timeout in device barrier', 8: 'bad input'}


class DeviceError(RuntimeError):
    pass


class NvlinkEngine:
    def __init__(self, group, num_max_tokens_per_rank: int, timeout_s: float, spec_hint: HeapSpec | None = None):
        self.C = load()
        self.group = group
        self.rank = dist.get_rank(group)
        self.R = dist.get_world_size(group)
        self.M = num_max_tokens_per_rank
        self.timeout_s = timeout_s
        self.host_timeout_s = max(4 * timeout_s, 60.0)
        self.heap = None
        self.spec: HeapSpec | None = None
        self.ticket = 0
        self._scratch = None
        self._ll_pending = False
        self._lc_pending = False
        self.last_exchange = None
        self._last_spec = None
        self._spec_cache: dict = {}
        self._covered: set = set()   # _spec keys the current heap is known to fit
        self.max_grid = int(self.C.heap_layout(1, 1, 1, 8, 1, 1)['max_grid'])
        if spec_hint is not None:
            self._ensure(spec_hint)

    # ------------------------------------------------------------------ heap
    def _ensure(self, spec: HeapSpec) -> None:
        if self.heap is not None and (spec is self._last_spec or self.spec.covers(spec)):
            return
        new = spec if self.spec is None else self.spec.merge(spec)
        if self.heap is not None:
            torch.cuda.synchronize()
            if self.R > 1:
                dist.barrier(group=self.group)
            self.heap.close()
        self.heap = create_heap(self.group, new, self.timeout_s)
        self.spec = new
        self._last_spec = None
        self._covered = set()

    def check(self) -> None:
        """Raise if any kernel of this buffer reported a device-side error."""
        if self.heap is None:
            return
        code, op, rank, peer, expected, seen, aux = self.heap.status()
        if code:
            self.heap.clear_status()
            # a kernel that gave up part-way leaves its grid counters behind: zero them so
            # the buffer stays usable for the next op
            self.heap.reset_counters()
            raise DeviceError(f'{ERRORS.get(code, "device error")} (code={code} op={op} rank={rank} '
                              f'peer={peer} expected={expected} seen={seen} aux={aux})')

    def check_canaries(self) -> None:
        """Raise if a guard zone between heap regions was overwritten (synchronises the device)."""
        if self.heap is None:
            return
        torch.cuda.synchronize()
        bad = self.heap.check_canaries()
        if bad:
            raise DeviceError(f'heap guard zones overwritten at byte offsets {bad} (rank {self.rank})')

    def device_trace(self) -> dict:
        """Phase durations (us) of the last normal-mode dispatch / combine and low-latency round
        on this rank, from %globaltimer stamps the kernels write into the heap (synchronises the
        device); ``abs.*`` are the raw stamps in ns."""
        if self.heap is None:
            return {}
        t = self.heap.trace()

        def d(a, b):
            return round((t[b] - t[a]) / 1e3, 2) if t[a] and t[b] else None
        return {'dispatch.inbox_free': d(0, 9), 'dispatch.grid_barrier': d(0, 10), 'dispatch.scan': d(0, 1), 'dispatch.counts_in': d(0, 2), 'dispatch.notified': d(0, 3),
                'dispatch.cta0_pushed': d(0, 4), 'dispatch.cta0_received': d(0, 5), 'dispatch.total': d(0, 6),
                'dispatch.cta0_published': d(0, 7), 'combine.cta0_published': d(16, 20),
                'dispatch.cta0_recv_wait': round(t[8] / 1e3, 2), 'combine.cta0_reduce_wait': round(t[21] / 1e3, 2),
                'gap.dispatch_to_combine': d(6, 16), 'combine.cta0_pushed': d(16, 17),
                'combine.cta0_reduced': d(16, 18), 'combine.total': d(16, 19),
                'step.dispatch_to_combine_end': d(0, 19),
                'll.dispatch_send': d(24, 25), 'll.gap_send_to_recv': d(25, 26), 'll.dispatch_recv_wait': d(26, 27),
                'll.dispatch_recv_copy': d(27, 28), 'll.gap_to_combine': d(28, 32), 'll.combine_send': d(32, 33),
                'll.gap_send_to_recv2': d(33, 34), 'll.combine_recv_wait': d(34, 35),
                'll.combine_recv_reduce': d(35, 36), 'll.total': d(24, 36),
                'll.send_cta0_stored': d(24, 29), 'll.send_cta0_released': d(24, 30),
                'll.combine_send_cta0_stored': d(32, 37), 'll.combine_send_cta0_released': d(32, 38),
                # raw %globaltimer stamps (ns), to line up the ranks of one node
                'abs.dispatch_start': t[0], 'abs.dispatch_end': t[6], 'abs.combine_start': t[16],
                'abs.combine_end': t[19], 'abs.barrier_exit': t[15], 'abs.raw': list(t)}

    def barrier(self) -> None:
        """Device-side barrier over the EP group (epoch flags in peer memory, bounded wait)."""
        if self.heap is not None:
            self.C.device_barrier(self.heap)

    def probe_timeout(self, timeout_ns: int) -> list:
        """Run one bounded wait on a flag that nothing sets; returns the status it left."""
        self.C.wait_probe(self.heap, int(timeout_ns))
        torch.cuda.synchronize()
        st = self.heap.status()
        self.heap.clear_status()
        return st

    def destroy(self) -> None:
        if self.heap is not None:
            torch.cuda.synchronize()
            if self.R > 1:
                dist.barrier(group=self.group)
            self.heap.close()
            self.heap = None

    def _sms(self, config) -> int:
        n = getattr(config, 'num_sms', 0) if config is not None else 0
        return int(n or _buffer_cls().num_sms or 0)

    def _grid(self, config) -> int:
        """CTAs of the normal-mode kernels (one per SM by default); every rank must use the same."""
        n = self._sms(config)
        return max(1, min(int(n) if n else self.heap.num_sms, self.max_grid))

    def _spec(self, H, K, E, Mll=None) -> HeapSpec:
        key = (H, K, E, Mll)
        sp = self._spec_cache.get(key)
        if sp is not None and key in self._covered:   # the current heap already fits this shape
            self._last_spec = sp
            return sp
        if sp is not None and self.spec is not None and self.spec.covers(sp):
            self._covered.add(key)
            self._last_spec = sp
            return sp
        cur = self.spec
        sp = HeapSpec(self.M, Mll if Mll is not None else (cur.max_ll_tokens if cur else 1), H, K, E)
        self._spec_cache[key] = sp
        return sp

    # ------------------------------------------------------------------ layout
    def get_dispatch_layout(self, topk_idx, num_experts):
        experts_per_rank(num_experts, self.R)
        T = topk_idx.shape[0]
        dev = topk_idx.device
        need = self.R + num_experts + 1
        if self._scratch is None or self._scratch.numel() < need or self._scratch.device != dev:
            self._scratch = torch.zeros(need, dtype=torch.int32, device=dev)
        with timer.stage('layout'):
            ntr, nte, itr = self.C.layout_op(topk_idx, num_experts, self.R, self._scratch)
        return ntr, nte, itr

    # ------------------------------------------------------------------ normal mode
    def dispatch(self, x, handle, topk_idx, topk_weights, is_token_in_rank, num_experts, expert_alignment,
                 num_worst_tokens, config, use_fp8=False, round_scale=False, num_tokens_per_expert=None):
        self.check()
        fp8_in = isinstance(x, tuple)
        xt = x[0] if fp8_in else x
        T, H = xt.shape
        dev = xt.device
        cached = handle is not None
        if cached:
            K, E, itr = handle.topk, handle.num_experts, handle.is_token_in_rank
        else:
            K = topk_idx.shape[1]
            E = num_experts
            nte = num_tokens_per_expert
            if is_token_in_rank is None or nte is None:
                _, lnte, litr = self.get_dispatch_layout(topk_idx, E)
                itr = is_token_in_rank if is_token_in_rank is not None else litr
                nte = nte if nte is not None else lnte
            else:
                itr = is_token_in_rank
        EL = experts_per_rank(E, self.R)
        self._ensure(self._spec(H, K, E))
        mode = 1 if fp8_in else (2 if use_fp8 else 0)
        R = self.R
        G = self._grid(config)
        self.ticket += 1
        x_scales = x[1].float() if fp8_in else None
        # Outputs are sized for the worst case (every peer sends its full capacity) so the kernel
        # is queued before the host learns the receive size; the host then waits on the notify
        # ticket while the GPU is still moving rows, and gets the first N rows.
        if num_worst_tokens:
            cap = int(num_worst_tokens)
        elif cached:
            cap = handle.num_recv if handle.num_recv is not None else handle.capacity
        else:
            cap = R * self.M
        wait = not (num_worst_tokens or cached)
        try:
            with timer.stage('dispatch'):
                (recv_x, recv_s, recv_topk, recv_w, recv_src, token_pos, send_start, recv_info, recv_off, N,
                 notify) = self.C.dispatch_op(
                    self.heap, xt, x_scales, mode, bool(round_scale),
                    None if cached else _contig(topk_idx),
                    None if (cached or topk_weights is None) else _contig(_f32(topk_weights)),
                    None if cached else _contig(nte if nte.dtype == torch.int32 else nte.to(torch.int32)),
                    _contig(itr), E, G, cap, bool(num_worst_tokens), wait, self.ticket, self.host_timeout_s)
        except RuntimeError:
            if not wait:
                raise
            # every wait of the queued kernel is bounded: let it finish so nothing of this op
            # is in flight, then raise with the device's own record
            torch.cuda.synchronize()
            self.check()
            raise
        per_expert = recv_counts = None
        if not wait:
            recv_counts = handle.recv_counts if cached else None
        else:
            recv_counts = torch.tensor(notify[:R], dtype=torch.int64)
            per_expert = notify[R:R + EL]
            if expert_alignment > 1:
                per_expert = [(c + expert_alignment - 1) // expert_alignment * expert_alignment for c in per_expert]
        new = DispatchHandle(T, K, None, recv_counts, recv_src, itr, num_recv=None if num_worst_tokens else N,
                             token_pos=token_pos, recv_off=recv_off, hidden=H, num_experts=E)
        new.capacity = cap
        new.send_start, new.recv_info, new.grid = send_start, recv_info, G
        self.last_exchange = dict(mode='normal', rows=N, hidden=H, payload_bytes=(2 * H if mode == 0 else H + H // 32))
        out_x = recv_x if mode == 0 else (recv_x, recv_s)
        if cached:
            return out_x, None, None, None, new, EventOverlap()
        if recv_w is not None and topk_weights.dtype != torch.float32:
            recv_w = recv_w.to(topk_weights.dtype)
        return out_x, recv_topk, recv_w, per_expert, new, EventOverlap()

    def combine(self, x, handle, topk_weights, bias, config, pairs=None):
        """``pairs = (pair_pos [N, K] int32, pair_w [N, K])``: ``x`` holds expert outputs in
        permuted order and row n is formed in the kernel as sum_k pair_w[n, k] * x[pair_pos[n, k]]."""
        self.check()
        N, H = (pairs[0].shape[0], x.shape[1]) if pairs is not None else x.shape
        if handle.num_recv is not None and N != handle.num_recv:
            raise ValueError(f'combine got {N} rows, dispatch delivered {handle.num_recv}')
        if x.dtype not in (torch.bfloat16, torch.float16):
            raise ValueError(f'combine needs bf16/fp16 rows, got {x.dtype}')
        K = topk_weights.shape[1] if topk_weights is not None else handle.topk
        self._ensure(self._spec(H, K, handle.num_experts))
        b = [t.contiguous() for t in bias]
        xc = x if (x.stride(1) == 1 and x.stride(0) % 8 == 0 and x.data_ptr() % 16 == 0) else x.contiguous()
        pp = pw = None
        if pairs is not None:
            xc = x.contiguous()
            pp = pairs[0] if pairs[0].dtype == torch.int32 else pairs[0].to(torch.int32)
            pp, pw = _contig(pp), _contig(_f32(pairs[1]))
        with timer.stage('combine'):
            out, out_w = self.C.combine_op(self.heap, xc,
                                           _contig(_f32(topk_weights)) if topk_weights is not None else None,
                                           handle.recv_off, handle.recv_info, handle.token_pos, handle.send_start,
                                           b[0] if len(b) > 0 else None, b[1] if len(b) > 1 else None,
                                           handle.grid, pp, pw)
        if out_w is not None and topk_weights.dtype != torch.float32:
            out_w = out_w.to(topk_weights.dtype)
        return out, out_w, EventOverlap()

    # ------------------------------------------------------------------ low latency
    def low_latency_dispatch(self, x, topk_idx, M, num_experts, use_fp8, round_scale, use_ue8m0,
                             cumulative_stats, wait_stats, return_recv_hook):
        self.check()
        if self._ll_pending:
            raise RuntimeError('call the previous low_latency_dispatch recv hook before dispatching again')
        T, H = x.shape
        K = topk_idx.shape[1]
        R = self.R
        EL = experts_per_rank(num_experts, R)
        self._ensure(self._spec(H, K, num_experts, Mll=M))
        Mll = self.spec.max_ll_tokens
        dev = x.device
        with timer.stage('ll_send'):
            self.C.ll_dispatch_send(self.heap, x, topk_idx.contiguous(), num_experts, bool(use_fp8),
                                    bool(round_scale or use_ue8m0), self._sms(None))
        if use_fp8:
            recv_x = torch.empty(EL, R * Mll, H, dtype=torch.float8_e4m3fn, device=dev)
            recv_s = torch.empty(EL, R * Mll, H // 128, dtype=torch.uint8 if use_ue8m0 else torch.float32, device=dev)
        else:
            recv_x = torch.empty(EL, R * Mll, H, dtype=x.dtype, device=dev)
            recv_s = None
        recv_count = torch.empty(EL, dtype=torch.int32, device=dev)
        src_info = torch.empty(EL, R * Mll, dtype=torch.int32, device=dev)
        layout_range = torch.empty(EL, R, dtype=torch.int64, device=dev)
        pair_meta = torch.empty(EL, R * Mll, dtype=torch.int32, device=dev)
        cum = cumulative_stats if (cumulative_stats is not None and cumulative_stats.dtype == torch.int32) else None

        def recv():
            with timer.stage('ll_recv'):
                self.C.ll_dispatch_recv(self.heap, recv_x, recv_s, recv_count, src_info, layout_range, pair_meta,
                                        num_experts, bool(use_fp8), bool(use_ue8m0), cum, wait_stats)
            if cumulative_stats is not None and cum is None:
                cumulative_stats.add_(recv_count.to(cumulative_stats.dtype))
            self._ll_pending = False

        n = R * M
        if use_fp8:
            s = recv_s[:, :n]
            if use_ue8m0 and (H // 128) % 4 == 0:
                s = recv_s.view(torch.int32)[:, :n]
            packed = (recv_x[:, :n], s)
        else:
            packed = recv_x[:, :n]
        handle = LowLatencyHandle(T, M, H, num_experts, K, src_info[:, :n], layout_range, recv_count,
                                  pair_meta=pair_meta, use_fp8=bool(use_fp8),
                                  extra=dict(src_info_full=src_info, pair_meta_full=pair_meta))
        self.last_exchange = dict(mode='ll', tokens=T, hidden=H)
        self._ll_pending = True
        hook = None
        if return_recv_hook:
            hook = _OneShot(recv)
        else:
            recv()
        return packed, recv_count, handle, EventOverlap(), hook

    def low_latency_combine(self, x, topk_idx, topk_weights, handle, zero_copy, return_recv_hook, out):
        self.check()
        if self._lc_pending:
            raise RuntimeError('call the previous low_latency_combine recv hook before combining again')
        if self._ll_pending:
            raise RuntimeError('call the low_latency_dispatch recv hook before combining')
        T, H = handle.num_tokens, handle.hidden
        if x.dim() != 3 or x.shape[-1] != H:
            raise ValueError(f'combine x must be [EL, R*M, {H}], got {tuple(x.shape)}')
        with timer.stage('ll_send'):
            self.C.ll_combine_send(self.heap, x, handle.recv_count, handle.extra['src_info_full'],
                                   handle.extra['pair_meta_full'], handle.num_experts, self._sms(None))
        result = out if out is not None else torch.empty(T, H, dtype=x.dtype, device=x.device)
        idx = topk_idx.contiguous()
        w = topk_weights.float().contiguous()

        def recv():
            with timer.stage('ll_recv'):
                self.C.ll_combine_recv(self.heap, idx, w, result, self._sms(None))
            self._lc_pending = False

        self._lc_pending = True
        hook = None
        if return_recv_hook:
            hook = _OneShot(recv)
        else:
            recv()
        return result, EventOverlap(), hook


_BUFFER = None


def _buffer_cls():
    global _BUFFER
    if _BUFFER is None:
        from ..buffer import Buffer
        _BUFFER = Buffer
    return _BUFFER


def _contig(t):
    return t if t.is_contiguous() else t.contiguous()


def _f32(t):
    return t if t.dtype == torch.float32 else t.float()


class _OneShot:
    """A receive hook: launches the receive kernel once (later calls are no-ops)."""

    def __init__(self, fn):
        self._fn = fn

    def __call__(self) -> None:
        if self._fn is not None:
            fn, self._fn = self._fn, None
            fn()
