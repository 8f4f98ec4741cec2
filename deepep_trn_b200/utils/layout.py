"""Routing-layout math in plain torch (any device).

These functions define the routing semantics that the sm_100a layout kernel
(`csrc/layout.cu`) must reproduce bit for bit; tests compare the two.

Semantics follow deep_ep_trn/layout.py:7-63 of the reference:
experts are split into contiguous blocks of ``E // R`` per rank, a negative
expert id means "masked", and a token is sent once to every rank that owns at
least one of its experts.
"""
from __future__ import annotations

import torch


def experts_per_rank(num_experts: int, num_ranks: int) -> int:
    if num_ranks <= 0 or num_experts % num_ranks:
        raise ValueError(f'num_experts={num_experts} must be divisible by num_ranks={num_ranks}')
    return num_experts // num_ranks


def rank_of_expert(topk_idx: torch.Tensor, num_experts: int, num_ranks: int) -> torch.Tensor:
    """Owning rank of every routed expert ``[T, K]``; -1 where the entry is masked.

    Reference: deep_ep_trn/layout.py:7-12.
    """
    per = experts_per_rank(num_experts, num_ranks)
    idx = topk_idx.to(torch.int64)
    return torch.where(idx < 0, torch.full_like(idx, -1), torch.div(idx, per, rounding_mode='floor'))


def token_rank_mask(topk_idx: torch.Tensor, num_experts: int, num_ranks: int) -> torch.Tensor:
    """``is_token_in_rank[T, R]``: True where the token has an expert on that rank."""
    owner = rank_of_expert(topk_idx, num_experts, num_ranks)
    T = owner.shape[0]
    mask = torch.zeros(T, num_ranks + 1, dtype=torch.bool, device=owner.device)
    # masked entries land in the spare column R and are dropped
    mask.scatter_(1, torch.where(owner < 0, torch.full_like(owner, num_ranks), owner), True)
    return mask[:, :num_ranks].contiguous()


def get_dispatch_layout(topk_idx: torch.Tensor, num_experts: int, num_ranks: int):
    """deep_ep ``get_dispatch_layout`` for one node.

    Returns ``(num_tokens_per_rank [R] int32, num_tokens_per_expert [E] int32,
    is_token_in_rank [T, R] bool)`` (reference deep_ep_trn/layout.py:15-29).
    """
    idx = topk_idx.to(torch.int64)
    in_rank = token_rank_mask(idx, num_experts, num_ranks)
    per_rank = in_rank.sum(0, dtype=torch.int32)
    valid = idx[idx >= 0]
    per_expert = torch.bincount(valid.flatten(), minlength=num_experts).to(torch.int32)
    return per_rank, per_expert, in_rank


def send_plan(is_token_in_rank: torch.Tensor):
    """Destination-major send order.

    Returns ``(token ids [N], rows per destination [R] int64)``: all tokens bound for
    rank 0 in ascending order, then rank 1, ... (reference deep_ep_trn/layout.py:32-36).
    """
    in_rank = is_token_in_rank.to(torch.bool)
    counts = in_rank.sum(0, dtype=torch.int64)
    # column-major walk over the [T, R] mask: (dst, token) lexicographic order
    flat = in_rank.t().reshape(-1).nonzero().flatten()
    T = in_rank.shape[0]
    token = flat % T if T else flat
    return token, counts


def token_positions(is_token_in_rank: torch.Tensor) -> torch.Tensor:
    """``pos[T, R]`` int32: index of the token among those sent to each rank, -1 if not sent.

    This is the per-destination exclusive prefix sum the device layout kernel emits;
    combine uses it to find a token's row in each rank's return block.
    """
    m = is_token_in_rank.to(torch.int32)
    pos = torch.cumsum(m, 0, dtype=torch.int32) - m
    return torch.where(is_token_in_rank.to(torch.bool), pos, torch.full_like(pos, -1))


def pair_plan(owner: torch.Tensor, num_ranks: int):
    """(token, k) pairs ordered by destination rank, then token, then k.

    Returns ``(token ids [P], k ids [P], pairs per destination [R] int64)``
    (reference deep_ep_trn/layout.py:39-51). Vectorised with a stable sort instead
    of a loop over ranks.
    """
    K = owner.shape[1]
    dst = owner.reshape(-1)
    keep = (dst >= 0).nonzero().flatten()
    # flat index t*K+k is already (token, k) ordered, so a stable sort on dst suffices
    order = torch.sort(dst[keep], stable=True).indices
    flat = keep[order]
    counts = torch.bincount(dst[keep], minlength=num_ranks)[:num_ranks].to(torch.int64)
    return flat // K, flat % K, counts


def slot_index(counts: torch.Tensor, slot_rows: int) -> torch.Tensor:
    """Flat positions of the valid rows in a buffer of per-source slots, source-major.

    Reference: deep_ep_trn/layout.py:54-59.
    """
    counts = counts.to(torch.int64)
    starts = torch.arange(counts.numel(), dtype=torch.int64, device=counts.device) * slot_rows
    base = torch.repeat_interleave(starts, counts)
    within = torch.arange(int(counts.sum()), dtype=torch.int64, device=counts.device)
    within = within - torch.repeat_interleave(exclusive_cumsum(counts), counts)
    return base + within


def exclusive_cumsum(counts: torch.Tensor) -> torch.Tensor:
    return torch.cumsum(counts, 0) - counts
