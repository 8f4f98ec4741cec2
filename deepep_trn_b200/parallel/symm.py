"""Creation of the IPC-mapped symmetric heap over an EP process group.

Each rank allocates one heap (``_C.SymmHeap``), the CUDA IPC handles are
all-gathered over the group once, every rank maps every peer's heap, and a
barrier makes sure all heaps are zeroed and mapped before any kernel touches
peer memory. Replaces the reference's per-call staging through the Neuron
collective runtime (deep_ep_trn/transport/nki_a2av.py:47-75).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from ..ops._ext import load


@dataclass(frozen=True)
class HeapSpec:
    max_tokens: int       # normal-mode tokens per rank (M)
    max_ll_tokens: int    # low-latency tokens per rank
    hidden: int
    topk: int
    num_experts: int

    def covers(self, other: 'HeapSpec') -> bool:
        return all(getattr(self, f) >= getattr(other, f) for f in self.__dataclass_fields__)

    def merge(self, other: 'HeapSpec') -> 'HeapSpec':
        return HeapSpec(*(max(getattr(self, f), getattr(other, f)) for f in self.__dataclass_fields__))


def create_heap(group, spec: HeapSpec, timeout_s: float):
    C = load()
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    device = torch.cuda.current_device()
    heap = C.SymmHeap(rank, world, spec.max_tokens, spec.max_ll_tokens, spec.hidden, spec.topk,
                      spec.num_experts, device, float(timeout_s))
    if world > 1:
        handles = [None] * world
        dist.all_gather_object(handles, heap.ipc_handle(), group=group)
        heap.open(handles)
        dist.barrier(group=group)
    return heap


def heap_bytes(R: int, spec: HeapSpec) -> int:
    return int(load().heap_bytes(R, spec.max_tokens, spec.max_ll_tokens, spec.hidden, spec.topk, spec.num_experts))
