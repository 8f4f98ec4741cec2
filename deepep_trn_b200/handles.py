"""Config, event and handle types of the deep_ep-compatible API.

Field names of the handles follow deep_ep_trn/buffer.py:49-71 so code that
inspects them keeps working; the NVLink engine adds the device-side fields its
kernels need (``token_pos``, ``recv_off``, ``pair_meta``).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import torch


@dataclass
class Config:
    """Per-op tuning (deep_ep.Config). Used for real by the NVLink engine.

    num_sms: CTAs per communication kernel; 0 means every SM of the device.
    use_tma: receivers pull rows with TMA bulk copies (else 16-byte ld/st warps).
    timeout_s: budget of every device-side wait before it reports an error.
    """
    num_sms: int = 0
    num_max_nvl_chunked_send_tokens: int = 0
    num_max_nvl_chunked_recv_tokens: int = 0
    use_tma: bool = True
    timeout_s: float = 0.0


class EventOverlap:
    """A CUDA event marking the end of an op on the communication stream.

    ``current_stream_wait()`` makes the caller's stream wait for it; used as a
    context manager it does the same on exit. ``extra_tensors`` keeps tensors
    alive until the event is consumed. On CPU transports the event is ``None``
    and waiting is a no-op (reference: deep_ep_trn/buffer.py:26-40, a stub).
    """

    def __init__(self, event: Optional[torch.cuda.Event] = None, extra_tensors=None):
        self.event = event
        self.extra_tensors = extra_tensors

    def current_stream_wait(self) -> None:
        if self.event is not None:
            torch.cuda.current_stream().wait_event(self.event)

    def __enter__(self):
        return self

    def __exit__(self, *exc) -> None:
        self.current_stream_wait()


class DispatchHandle:
    """Normal-mode handle, reusable for a cached dispatch and for combine.

    Reference fields (deep_ep_trn/buffer.py:49-57): num_tokens, topk,
    send_token_idx [N_send] (destination-major), send_counts [R], recv_counts [R],
    recv_src_idx [N_recv], is_token_in_rank [T, R].
    """

    def __init__(self, num_tokens: int, topk: int, send_counts, recv_counts, recv_src_idx,
                 is_token_in_rank, send_token_idx=None, num_recv: Optional[int] = None,
                 token_pos=None, recv_off=None, hidden: int = 0, num_experts: int = 0):
        self.num_tokens = num_tokens
        self.topk = topk
        self._send_counts = send_counts
        self.recv_counts = recv_counts
        self.recv_src_idx = recv_src_idx
        self.is_token_in_rank = is_token_in_rank
        self._send_token_idx = send_token_idx
        self.num_recv = num_recv
        self.token_pos = token_pos      # [T, R] int32: row of token t in rank r's block (-1 if not sent)
        self.recv_off = recv_off        # [R + 1] int64: first received row of each source
        self.hidden = hidden
        self.num_experts = num_experts

    @property
    def send_counts(self) -> torch.Tensor:
        if self._send_counts is None:
            self._send_counts = self.is_token_in_rank.sum(0, dtype=torch.int64)
        return self._send_counts

    @property
    def send_token_idx(self) -> torch.Tensor:
        if self._send_token_idx is None:
            from .utils.layout import send_plan
            self._send_token_idx = send_plan(self.is_token_in_rank)[0]
        return self._send_token_idx


@dataclass
class LowLatencyHandle:
    """Low-latency handle (reference deep_ep_trn/buffer.py:60-71).

    src_info [EL, R*M] int32: source token of each packed row, -1 = empty.
    layout_range [EL, R] int64: ``(start << 32) | count`` of each source's block.
    """
    num_tokens: int
    num_max_dispatch_tokens_per_rank: int
    hidden: int
    num_experts: int
    topk: int
    src_info: torch.Tensor
    layout_range: torch.Tensor
    recv_count: Optional[torch.Tensor] = None
    pair_expert: Optional[torch.Tensor] = None
    pair_pos: Optional[torch.Tensor] = None
    pairs_per_src: Optional[torch.Tensor] = None
    pair_meta: Optional[torch.Tensor] = None   # NVLink engine: src * K + k of each packed row
    use_fp8: bool = False
    extra: dict = field(default_factory=dict)
