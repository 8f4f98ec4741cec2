"""CPU transport over a gloo process group: the semantics oracle.

Implements the same contract as every other transport so all Buffer semantics
can be checked on CPU processes (reference: deep_ep_trn/transport/gloo.py:15-45).
Not meant to be fast.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ...utils.profiling import timer
from .base import Transport


class GlooTransport(Transport):
    def __init__(self, group):
        self.group = group
        self.rank = dist.get_rank(group)
        self.num_ranks = dist.get_world_size(group)

    def slot_rows(self, send_capacity: int, max_rows_per_peer: int) -> int:
        return max_rows_per_peer

    def all_to_all_v(self, send, counts):
        counts = counts.to(torch.int64).cpu()
        with timer.stage('kernel'):
            recv_counts = torch.empty_like(counts)
            dist.all_to_all_single(recv_counts, counts, group=self.group)
            width, dtype = send.shape[1], send.dtype
            # gloo has no bf16 all-to-all: move raw bytes
            payload = send.contiguous().view(torch.uint8)
            out = torch.empty(int(recv_counts.sum()), width * send.element_size(), dtype=torch.uint8)
            dist.all_to_all_single(out, payload, output_split_sizes=recv_counts.tolist(),
                                   input_split_sizes=counts.tolist(), group=self.group)
            return out.view(dtype), recv_counts
