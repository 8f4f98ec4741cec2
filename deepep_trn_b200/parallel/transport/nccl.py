"""Device-resident transport over NCCL ``all_to_all_single``: the B200 baseline.

This is the reference semantics run the obvious way on GPUs: the counts go
through one ``all_to_all_single``, the host reads them to size the receive
buffer, and the payload goes through a second one with split sizes. Every
other step (layout, pack, unpack, index_add combine) runs as torch ops on the
device. It exists to be measured against; the product path is the NVLink engine.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ...utils.profiling import timer
from .base import Transport


class NcclTransport(Transport):
    def __init__(self, group):
        self.group = group
        self.rank = dist.get_rank(group)
        self.num_ranks = dist.get_world_size(group)

    def slot_rows(self, send_capacity: int, max_rows_per_peer: int) -> int:
        return max_rows_per_peer

    def all_to_all_v(self, send, counts):
        dev = send.device
        with timer.stage('kernel'):
            c = counts.to(device=dev, dtype=torch.int64)
            rc = torch.empty_like(c)
            dist.all_to_all_single(rc, c, group=self.group)
            both = torch.stack([c, rc]).cpu()
            send_sizes, recv_sizes = both[0].tolist(), both[1].tolist()
            out = send.new_empty((sum(recv_sizes), send.shape[1]))
            dist.all_to_all_single(out, send.contiguous(), output_split_sizes=recv_sizes,
                                   input_split_sizes=send_sizes, group=self.group)
            return out, both[1]
