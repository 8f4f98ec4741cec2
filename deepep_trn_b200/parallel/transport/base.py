"""Transport contract for the collective engines (CPU gloo oracle, NCCL baseline).

The contract is the reference's one exchange primitive
(deep_ep_trn/transport/base.py:15-50):

    all_to_all_fixed_slot(send[cap, W], counts[R], slot) -> recv[R * slot, W], recv_counts[R]

kept so that code written against the reference's Transport runs unchanged. On
B200 the fixed slot is not a hardware constraint, so every transport here also
implements the compact form ``all_to_all_v(send, counts) -> (recv[sum(recv_counts), W],
recv_counts)``, which the torch engine uses. The NVLink engine does not use a
transport at all: its kernels move rows between peer-mapped buffers directly.
"""
from __future__ import annotations

from abc import ABC, abstractmethod

import torch


class Transport(ABC):
    rank: int       # position of this process inside its EP group
    num_ranks: int  # EP group size

    @abstractmethod
    def slot_rows(self, send_capacity: int, max_rows_per_peer: int) -> int:
        """Rows per source slot the backend uses for this buffer shape."""

    @abstractmethod
    def all_to_all_v(self, send: torch.Tensor, counts: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Exchange rows packed by destination; returns the received rows packed by source."""

    def all_to_all_fixed_slot(self, send: torch.Tensor, counts: torch.Tensor,
                              slot_rows: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Reference contract: rows from source ``s`` land at ``[s*slot, s*slot + recv_counts[s])``."""
        counts = counts.to(torch.int64).cpu()
        self._check(send, counts, slot_rows)
        packed, recv_counts = self.all_to_all_v(send[:int(counts.sum())], counts)
        recv = send.new_zeros((self.num_ranks * slot_rows, send.shape[1]))
        starts = torch.cumsum(recv_counts, 0) - recv_counts
        for src in range(self.num_ranks):
            n, o = int(recv_counts[src]), int(starts[src])
            recv[src * slot_rows:src * slot_rows + n] = packed[o:o + n]
        return recv, recv_counts

    def _check(self, send: torch.Tensor, counts: torch.Tensor, slot_rows: int) -> None:
        if send.dim() != 2 or send.element_size() != 2:
            raise ValueError(f'send must be a 2-D 16-bit tensor, got {send.dtype} {tuple(send.shape)}')
        if tuple(counts.shape) != (self.num_ranks,):
            raise ValueError(f'counts must be [{self.num_ranks}], got {tuple(counts.shape)}')
        if int(counts.sum()) > send.shape[0]:
            raise ValueError(f'{int(counts.sum())} packed rows exceed send capacity {send.shape[0]}')
        if counts.numel() and int(counts.max()) > slot_rows:
            # a receiver could not tell that its slot overflowed
            raise ValueError(f'{int(counts.max())} rows for one peer exceed slot_rows={slot_rows}')
