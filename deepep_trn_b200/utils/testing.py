"""Synthetic routing, EP group layouts and expert emulation shared by tests and benches.

Mirrors the routing kinds of deep_ep_trn/testing.py:7-69 (same distributions and
edge cases; the random streams are this library's own) and adds the
BASELINE router configurations (randn logits -> top-k -> softmax over the
chosen k; Zipf-biased logits over a seeded expert permutation).
"""
from __future__ import annotations

import math

import torch

ROUTINGS = ('random', 'balanced', 'zipf', 'hot_rank0', 'ragged', 'masked')


def strided_ep_groups(world_size: int, ep: int) -> list[list[int]]:
    """EP groups of ``ep`` ranks taken at stride ``world_size // ep``.

    ``world=4, ep=2`` gives ``[[0, 2], [1, 3]]``: TP-adjacent ranks fall into
    different EP groups (the TP2 x EP2 layout; reference testing.py:10-19).
    """
    if ep <= 0 or world_size % ep:
        raise ValueError(f'world size {world_size} is not divisible by ep {ep}')
    stride = world_size // ep
    return [[g + i * stride for i in range(ep)] for g in range(stride)]


def make_routing(kind: str, tokens: int, experts: int, topk: int, ep: int, ep_rank: int, seed: int):
    """Synthetic router output ``(topk_idx [T, K] int64, topk_weights [T, K] fp32)``.

    random     uniform distinct top-k
    balanced   every token's experts spread evenly over the ranks
    zipf       expert popularity ~ 1/rank (Gumbel top-k), so rank 0 is overloaded
    hot_rank0  every token routes only to experts of rank 0
    ragged     random, but T shrinks with ep_rank and the last rank has T = 0
    masked     random with about 30% of the entries set to -1
    Weights are uniform random, normalised to sum to one per token.
    """
    if kind not in ROUTINGS:
        raise ValueError(f'unknown routing {kind!r}; expected one of {ROUTINGS}')
    gen = torch.Generator().manual_seed(seed)
    E, K = experts, topk
    T = tokens
    if kind == 'ragged':
        T = 0 if ep_rank == ep - 1 else max(1, tokens - ep_rank * (tokens // ep))
    if kind == 'balanced':
        stride = E // K
        idx = (4 * torch.arange(T).unsqueeze(1) + stride * torch.arange(K).unsqueeze(0)) % E
    elif kind == 'hot_rank0':
        local = E // ep
        if local < K:
            raise ValueError('hot_rank0 needs experts / ep >= topk')
        idx = (torch.arange(T).unsqueeze(1) + torch.arange(K).unsqueeze(0)) % local
    elif kind == 'zipf':
        bias = -torch.log(torch.arange(1, E + 1, dtype=torch.float32))
        u = torch.rand(T, E, generator=gen).clamp(1e-9, 1 - 1e-9)
        idx = torch.topk(bias - torch.log(-torch.log(u)), K, dim=-1).indices
    else:
        idx = torch.topk(torch.rand(T, E, generator=gen), K, dim=-1).indices
    if kind == 'masked':
        drop = torch.rand(T, K, generator=gen) < 0.3
        idx = idx.masked_fill(drop, -1)
    w = torch.rand(T, K, generator=gen)
    w = w / w.sum(-1, keepdim=True).clamp_min(1e-6)
    return idx.to(torch.int64), w.to(torch.float32)


def router_topk_reference(logits: torch.Tensor, topk: int):
    """Top-k of router logits with softmax over the chosen k (fp32), ties to lower index.

    The torch definition of the router kernel: ``(topk_idx int64, topk_weights fp32)``.
    """
    lf = logits.float()
    vals, idx = torch.topk(lf, topk, dim=-1, sorted=True)
    w = torch.softmax(vals, dim=-1)
    return idx.to(torch.int64), w


def randn_router(tokens: int, experts: int, topk: int, seed: int, device='cpu'):
    """randn logits [T, E] -> top-k with softmax over the chosen k."""
    gen = torch.Generator().manual_seed(seed)
    logits = torch.randn(tokens, experts, generator=gen)
    idx, w = router_topk_reference(logits, topk)
    return idx.to(device), w.to(device)


def zipf_router(tokens: int, experts: int, topk: int, seed: int, device='cpu'):
    """logits ~ N(0,1) + log(1/r) bias over a seeded expert permutation."""
    gen = torch.Generator().manual_seed(seed)
    perm = torch.randperm(experts, generator=torch.Generator().manual_seed(12345))
    bias = torch.empty(experts)
    bias[perm] = -torch.log(torch.arange(1, experts + 1, dtype=torch.float32))
    logits = torch.randn(tokens, experts, generator=gen) + bias
    idx, w = router_topk_reference(logits, topk)
    return idx.to(device), w.to(device)


def expert_scale(global_expert: torch.Tensor) -> torch.Tensor:
    """Deterministic per-expert 'compute' ``1 + (e % 8) / 8``, exact in bf16."""
    return 1.0 + (global_expert % 8).to(torch.float32) / 8.0


def bitwise_equal(a: torch.Tensor, b: torch.Tensor) -> bool:
    if a.shape != b.shape or a.dtype != b.dtype:
        return False
    if a.numel() == 0:
        return True
    if a.element_size() in (1, 2, 4, 8) and a.dtype.is_floating_point:
        view = {1: torch.uint8, 2: torch.int16, 4: torch.int32, 8: torch.int64}[a.element_size()]
        return torch.equal(a.contiguous().view(view), b.contiguous().view(view))
    return torch.equal(a, b)


def expected_distinct_ranks(experts: int, topk: int, ranks: int) -> float:
    """E[#distinct destination ranks per token] for uniform distinct top-k."""
    local = experts // ranks
    miss = math.comb(experts - local, topk) / math.comb(experts, topk)
    return ranks * (1 - miss)
