"""fp8 e4m3 1x128 quantisation (N6). CUDA tensors run the kernel; CPU tensors run
the torch definition in ``utils.codec`` (the CPU path is the oracle, not a fallback)."""
from __future__ import annotations

import torch

from ..utils.codec import dequantize_fp8_1x128, quantize_fp8_1x128
from ._ext import load


def quantize_fp8(x: torch.Tensor, round_scale: bool = False):
    if not x.is_cuda:
        return quantize_fp8_1x128(x, round_scale)
    x = x.contiguous()
    H = x.shape[-1]
    q = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=x.device)
    s = torch.empty(*x.shape[:-1], H // 128, dtype=torch.float32, device=x.device)
    load().quant_fp8(x, q.view(torch.uint8), s, round_scale)
    return q, s


def dequantize_fp8(q: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """bf16 of e4m3 ``q`` [.., H] times its 1x128 fp32 ``scales`` [.., H/128] (one rounding)."""
    if not q.is_cuda:
        return dequantize_fp8_1x128(q, scales).to(torch.bfloat16)
    q = q.contiguous()
    out = torch.empty(q.shape, dtype=torch.bfloat16, device=q.device)
    load().dequant_fp8(q.view(torch.uint8), scales.float().contiguous(), out)
    return out
