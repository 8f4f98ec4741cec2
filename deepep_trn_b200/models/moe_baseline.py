"""The same MoE layer built the conventional way: the baseline the fused path is measured against.

Communication: ``Buffer(backend='nccl')`` (reference semantics with NCCL
``all_to_all_single``, host-synchronised split sizes). Compute: cuBLAS through
``torch._grouped_mm`` for the expert GEMMs, torch ops for routing, SwiGLU and the
permutation, and torch autograd for the backward. Weights and routing are the
same as ``MoELayer`` (``w1`` interleaved gate/up blocks, ``w2``, ``router``,
``router_bias``), so both layers can be fed identical parameters.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from ..ops.gemm import deinterleave


class _Dispatch(torch.autograd.Function):
    """dispatch forward; its backward is a combine that also returns the weight gradients."""

    @staticmethod
    def forward(ctx, x, idx, w, buf, num_experts, state):
        ntr, _, nte, itr, _ = buf.get_dispatch_layout(idx, num_experts)
        rx, ridx, rw, per_expert, handle, _ = buf.dispatch(x, topk_idx=idx, topk_weights=w, num_tokens_per_rank=ntr,
                                                           is_token_in_rank=itr, num_tokens_per_expert=nte)
        state['handle'] = handle
        ctx.buf, ctx.handle = buf, handle
        ctx.mark_non_differentiable(ridx)
        return rx, ridx, rw

    @staticmethod
    def backward(ctx, d_rx, d_ridx, d_rw):
        dx, dw, _ = ctx.buf.combine(d_rx.contiguous(), ctx.handle, topk_weights=d_rw.float().contiguous())
        return dx, None, dw, None, None, None


class _Combine(torch.autograd.Function):
    """combine forward; its backward is a cached dispatch."""

    @staticmethod
    def forward(ctx, y, buf, state):
        ctx.buf, ctx.handle = buf, state['handle']
        out, _, _ = buf.combine(y, state['handle'])
        return out

    @staticmethod
    def backward(ctx, dout):
        dy, *_ = ctx.buf.dispatch(dout.contiguous(), handle=ctx.handle)
        return dy, None, None


class BaselineMoELayer(nn.Module):
    def __init__(self, buffer, hidden, intermediate, num_experts, topk, dtype=torch.bfloat16, device=None):
        super().__init__()
        self.buffer = buffer
        self.num_experts, self.topk = num_experts, topk
        EL = num_experts // buffer.group_size
        self.router = nn.Parameter(torch.zeros(num_experts, hidden, dtype=dtype, device=device))
        self.w1 = nn.Parameter(torch.zeros(EL, 2 * intermediate, hidden, dtype=dtype, device=device))
        self.w2 = nn.Parameter(torch.zeros(EL, hidden, intermediate, dtype=dtype, device=device))
        self.register_buffer('router_bias', torch.zeros(num_experts, dtype=torch.float32, device=device))

    def forward(self, x):
        EL = self.w1.shape[0]
        logits = (x.float() @ self.router.float().t()) + self.router_bias
        vals, idx = torch.topk(logits, self.topk, dim=-1)
        w = torch.softmax(vals, -1)
        state = {}
        rx, ridx, rw = _Dispatch.apply(x, idx, w, self.buffer, self.num_experts, state)
        # expert-major permutation of the (row, local expert) pairs
        rows, ks = (ridx >= 0).nonzero(as_tuple=True)
        experts = ridx[rows, ks]
        order = torch.argsort(experts, stable=True)
        rows, ks, experts = rows[order], ks[order], experts[order]
        counts = torch.bincount(experts, minlength=EL)
        offs = torch.cumsum(counts, 0).to(torch.int32)
        a = rx[rows]
        gu = torch._grouped_mm(a, self.w1.transpose(1, 2), offs=offs)
        g, u = deinterleave(gu)
        h = torch.nn.functional.silu(g) * u
        o = torch._grouped_mm(h, self.w2.transpose(1, 2), offs=offs)
        o = o * rw[rows, ks].unsqueeze(1).to(o.dtype)
        y = torch.zeros_like(rx).index_add(0, rows, o)
        return _Combine.apply(y, self.buffer, state)
