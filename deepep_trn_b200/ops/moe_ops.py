"""Wrappers of the MoE-layer kernels (router top-k, permute/unpermute, SwiGLU backward,
transpose). CUDA tensors run the sm_100a kernels; CPU tensors run the torch definitions
below, which double as the numerics oracle in the tests."""
from __future__ import annotations

import torch

from ..utils.testing import router_topk_reference
from ._ext import load

ALIGN = 128  # expert segments of the permuted layout start at multiples of this


def padded_offsets(counts: list[int], align: int = ALIGN) -> list[int]:
    offs = [0]
    for c in counts:
        offs.append(offs[-1] + (c + align - 1) // align * align)
    return offs


def router_topk(logits: torch.Tensor, k: int):
    """Top-k over router logits (ties to the lower id) with softmax over the chosen k."""
    if not logits.is_cuda:
        return router_topk_reference(logits, k)
    logits = logits.float().contiguous()
    T = logits.shape[0]
    idx = torch.empty(T, k, dtype=torch.int64, device=logits.device)
    w = torch.empty(T, k, dtype=torch.float32, device=logits.device)
    load().router_topk(logits, k, idx, w)
    return idx, w


def router_topk_bwd(idx: torch.Tensor, w: torch.Tensor, dw: torch.Tensor, num_experts: int) -> torch.Tensor:
    """d_logits of softmax-over-chosen-k: w_k * (dw_k - sum_j w_j dw_j) at the chosen ids."""
    if not w.is_cuda:
        dot = (w * dw).sum(-1, keepdim=True)
        d = torch.zeros(w.shape[0], num_experts, dtype=torch.float32)
        return d.scatter_(1, idx, w * (dw - dot))
    out = torch.empty(w.shape[0], num_experts, dtype=torch.float32, device=w.device)
    load().router_topk_bwd(idx.contiguous(), w.float().contiguous(), dw.float().contiguous(), out)
    return out


def permute(x, local_ids: torch.Tensor, num_local_experts: int, counts: list[int] | None = None,
            keep_fp8: bool = False):
    """Rows of ``x`` [N, H] grouped by local expert, each segment padded to a multiple of 128.

    ``x`` may also be an fp8 pair ``(x_e4m3 [N, H], scales [N, H/128] fp32)`` (what an fp8
    dispatch delivers); the rows are then dequantised to bf16 on the way, or, with
    ``keep_fp8``, stay e4m3 and ``rows`` is the pair ``(rows_e4m3 [P, H], scales [P, H/128])``
    (padding rows: zeros with scale 1), the operand of ``grouped_gemm_fp8``.
    Returns ``(rows [P, H], pos [N, K] int32, offsets [EL+1] int64, counts [EL] int32)``;
    ``pos[n, k]`` is the row of pair (n, k) or -1. ``counts`` (host list), when known,
    sizes ``rows`` exactly without a device synchronisation.
    """
    scales = None
    if isinstance(x, tuple):
        x, scales = x
        if not x.is_cuda and keep_fp8:
            raise NotImplementedError('keep_fp8 permute runs on CUDA tensors')
        if not x.is_cuda:
            from ..utils.codec import dequantize_fp8_1x128
            x, scales = dequantize_fp8_1x128(x, scales).to(torch.bfloat16), None
    N, H = x.shape
    K = local_ids.shape[1]
    EL = num_local_experts
    if counts is None:
        valid = local_ids[local_ids >= 0]
        counts = torch.bincount(valid.flatten(), minlength=EL).tolist()
    offs = padded_offsets(counts)
    if not x.is_cuda:
        rows = x.new_zeros(offs[-1], H)
        pos = torch.full((N, K), -1, dtype=torch.int32)
        fill = list(offs[:-1])
        for n in range(N):
            for k in range(K):
                e = int(local_ids[n, k])
                if e >= 0:
                    rows[fill[e]] = x[n]
                    pos[n, k] = fill[e]
                    fill[e] += 1
        return rows, pos, torch.tensor(offs, dtype=torch.int64), torch.tensor(counts, dtype=torch.int32)
    dev = x.device
    keep = keep_fp8 and scales is not None
    rows = torch.empty(offs[-1], H, dtype=torch.uint8 if keep else (torch.bfloat16 if scales is not None else x.dtype),
                       device=dev)
    rows_s = torch.empty(offs[-1], H // 128, dtype=torch.float32, device=dev) if keep else None
    pos = torch.empty(N, K, dtype=torch.int32, device=dev)
    offsets = torch.empty(EL + 1, dtype=torch.int64, device=dev)
    cnt = torch.empty(EL, dtype=torch.int32, device=dev)
    nblocks = max(1, (N + 31) // 32)
    scratch = torch.empty(nblocks * EL, dtype=torch.int32, device=dev)
    from .gemm import _err  # the kernels' shared device error word (timed-out copies)
    xq = x.view(torch.uint8) if scales is not None else x
    load().permute(xq, local_ids.contiguous(), EL, rows, pos, offsets, cnt, scratch, _err(dev),
                   scales.float().contiguous() if scales is not None else None, rows_s)
    if keep:
        return (rows.view(torch.float8_e4m3fn), rows_s), pos, offsets, cnt
    return rows, pos, offsets, cnt


def unpermute(rows: torch.Tensor, pos: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """y[n] = sum_k w[n, k] * rows[pos[n, k]] (fp32 accumulation, one cast)."""
    N, K = pos.shape
    if not rows.is_cuda:
        acc = torch.zeros(N, rows.shape[1])
        for k in range(K):
            m = pos[:, k] >= 0
            acc[m] += w[m, k:k + 1].float() * rows[pos[m, k].long()].float()
        return acc.to(rows.dtype)
    y = torch.empty(N, rows.shape[1], dtype=rows.dtype, device=rows.device)
    load().unpermute(rows.contiguous(), pos, w.float().contiguous(), y)
    return y


def unpermute_bwd(dy, rows, pos, w, offsets, counts):
    """(d_rows [P, H] with zero padding rows, d_w [N, K])."""
    if not dy.is_cuda:
        drows = torch.zeros_like(rows)
        dw = torch.zeros(pos.shape, dtype=torch.float32)
        for k in range(pos.shape[1]):
            m = pos[:, k] >= 0
            p = pos[m, k].long()
            drows[p] = (dy[m].float() * w[m, k:k + 1].float()).to(rows.dtype)
            dw[m, k] = (dy[m].float() * rows[p].float()).sum(-1)
        return drows, dw
    drows = torch.empty_like(rows)
    dw = torch.empty(pos.shape, dtype=torch.float32, device=dy.device)
    load().unpermute_bwd(dy.contiguous(), rows.contiguous(), pos, w.float().contiguous(), drows, dw, offsets, counts)
    return drows, dw


def permute_bwd(drows: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
    """dx[n] = sum_k d_rows[pos[n, k]]."""
    N, K = pos.shape
    if not drows.is_cuda:
        acc = torch.zeros(N, drows.shape[1])
        for k in range(K):
            m = pos[:, k] >= 0
            acc[m] += drows[pos[m, k].long()].float()
        return acc.to(drows.dtype)
    dx = torch.empty(N, drows.shape[1], dtype=drows.dtype, device=drows.device)
    load().permute_bwd(drows.contiguous(), pos, dx)
    return dx


def swiglu_bwd(dh: torch.Tensor, pre: torch.Tensor) -> torch.Tensor:
    """Gradient w.r.t. the interleaved [gate | up] pre-activation of h = silu(gate) * up."""
    if not dh.is_cuda:
        from .gemm import deinterleave
        g, u = deinterleave(pre.float())
        s = torch.sigmoid(g)
        dg = dh.float() * u * s * (1 + g * (1 - s))
        du = dh.float() * g * s
        R, I = dh.shape
        out = torch.stack([dg.reshape(R, I // 128, 128), du.reshape(R, I // 128, 128)], 2)
        return out.reshape(R, 2 * I).to(dh.dtype)
    out = torch.empty_like(pre)
    load().swiglu_bwd(dh.contiguous(), pre.contiguous(), out)
    return out


def transpose(x: torch.Tensor) -> torch.Tensor:
    """Materialised transpose of the last two dims of a 2-D or 3-D bf16 tensor."""
    if not x.is_cuda:
        return x.transpose(-1, -2).contiguous()
    out = torch.empty(*x.shape[:-2], x.shape[-1], x.shape[-2], dtype=x.dtype, device=x.device)
    load().transpose(x.contiguous(), out)
    return out
