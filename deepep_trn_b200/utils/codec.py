"""Row formats: the 16-bit packed metadata row and the fp8 1x128 block codec.

``RowCodec`` keeps the reference wire format (deep_ep_trn/codec.py:7-14) so rows
produced by either library decode identically. In 16-bit columns:

    [0, H)          payload (bf16 / fp16)
    [H, H+2K)       top-k weights, fp32 split into two 16-bit halves
    [H+2K, H+4K)    top-k global expert ids, int32 (-1 = masked)
    [H+4K, H+4K+2)  source-local token index, int32
    [.., W)         zero padding up to a multiple of ``META_ALIGN`` columns

The CPU / NCCL engines use it to move one row per (token, rank) in a single
collective. The NVLink engine does not pack rows at all: its kernels read the
payload and the metadata from separate arrays in peer memory.

The fp8 helpers are the torch definition of the per-token, per-128-channel
e4m3 quantisation that the dispatch kernels fuse into their send path
(``scale = max(amax, 1e-4) / 448``; ``q = rn_satfinite(x * (448 / max(amax, 1e-4)))``).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

META_ALIGN = 32
SUPPORTED_DTYPES = (torch.bfloat16, torch.float16)
FP8_BLOCK = 128
FP8_MAX = 448.0
FP8_AMAX_FLOOR = 1e-4


def _as16(t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Reinterpret a 32-bit tensor [n, c] as [n, 2c] 16-bit columns (no value change)."""
    return t.contiguous().view(dtype)


@dataclass(frozen=True)
class RowCodec:
    hidden: int
    topk: int
    dtype: torch.dtype = torch.bfloat16

    def __post_init__(self):
        if self.dtype not in SUPPORTED_DTYPES:
            raise ValueError(f'payload dtype must be one of {SUPPORTED_DTYPES}, got {self.dtype}')

    @property
    def meta_cols(self) -> int:
        used = 4 * self.topk + 2
        return -(-used // META_ALIGN) * META_ALIGN

    @property
    def width(self) -> int:
        return self.hidden + self.meta_cols

    def encode(self, x: torch.Tensor, topk_idx, topk_weights, token_index: torch.Tensor) -> torch.Tensor:
        n, H, K = x.shape[0], self.hidden, self.topk
        rows = x.new_zeros((n, self.width), dtype=self.dtype)
        rows[:, :H] = x
        if topk_weights is not None:
            rows[:, H:H + 2 * K] = _as16(topk_weights.to(torch.float32), self.dtype)
        if topk_idx is None:
            ids = torch.full((n, K), -1, dtype=torch.int32, device=x.device)
        else:
            ids = topk_idx.to(torch.int32)
        rows[:, H + 2 * K:H + 4 * K] = _as16(ids, self.dtype)
        rows[:, H + 4 * K:H + 4 * K + 2] = _as16(token_index.to(torch.int32).reshape(n, 1), self.dtype)
        return rows

    def decode(self, rows: torch.Tensor):
        """Returns ``(x, topk_idx int64, topk_weights fp32, token_index int64)``, bit-exact."""
        H, K = self.hidden, self.topk
        x = rows[:, :H]
        w = rows[:, H:H + 2 * K].contiguous().view(torch.float32)
        ids = rows[:, H + 2 * K:H + 4 * K].contiguous().view(torch.int32).to(torch.int64)
        tok = rows[:, H + 4 * K:H + 4 * K + 2].contiguous().view(torch.int32).reshape(-1).to(torch.int64)
        return x, ids, w, tok


# ----------------------------------------------------------------------------- fp8 1x128
def _pow2_ceil(s: torch.Tensor) -> torch.Tensor:
    """Smallest power of two >= s for positive normal fp32 s, by exponent arithmetic."""
    bits = s.contiguous().view(torch.int32)
    mant = bits & 0x7FFFFF
    exp = (bits >> 23) & 0xFF
    exp = torch.where(mant != 0, exp + 1, exp)
    return (exp << 23).view(torch.float32)


def quantize_fp8_1x128(x: torch.Tensor, round_scale: bool = False):
    """Per-token, per-128-channel e4m3 quantisation (torch definition of the kernel).

    Returns ``(q [.., H] float8_e4m3fn, scales [.., H/128] fp32)`` with
    ``x ~= q * scale`` per block. With ``round_scale`` the scale is rounded up to
    a power of two (UE8M0-representable).
    """
    H = x.shape[-1]
    if H % FP8_BLOCK:
        raise ValueError(f'hidden={H} must be a multiple of {FP8_BLOCK} for fp8 block scales')
    xf = x.float().reshape(*x.shape[:-1], H // FP8_BLOCK, FP8_BLOCK)
    amax = xf.abs().amax(-1).clamp_min(FP8_AMAX_FLOOR)
    # IEEE divisions tensor by tensor (a python scalar on the left would become
    # reciprocal-then-multiply in torch and round differently from the kernel)
    c448 = torch.full_like(amax, FP8_MAX)
    if round_scale:
        scale = _pow2_ceil(torch.div(amax, c448))
        inv = torch.div(torch.ones_like(scale), scale)
    else:
        scale = torch.div(amax, c448)
        inv = torch.div(c448, amax)
    q = (xf * inv.unsqueeze(-1)).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return q.reshape(x.shape), scale


def dequantize_fp8_1x128(q: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    H = q.shape[-1]
    s = scales
    if s.dtype in (torch.int32, torch.uint8):
        s = ue8m0_to_float(s, H)
    qf = q.float().reshape(*q.shape[:-1], H // FP8_BLOCK, FP8_BLOCK)
    return (qf * s.unsqueeze(-1)).reshape(q.shape)


def float_to_ue8m0(scales: torch.Tensor) -> torch.Tensor:
    """Power-of-two fp32 scales -> packed UE8M0 bytes (4 blocks per int32 when H % 512 == 0)."""
    exp = ((scales.contiguous().view(torch.int32) >> 23) & 0xFF).to(torch.uint8)
    if exp.shape[-1] % 4 == 0:
        return exp.contiguous().view(torch.int32)
    return exp


def ue8m0_to_float(packed: torch.Tensor, hidden: int) -> torch.Tensor:
    b = packed.contiguous().view(torch.uint8)[..., :hidden // FP8_BLOCK].to(torch.int32)
    return (b << 23).view(torch.float32)


def fp8_error_bound(x: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """Elementwise bound on |x - deq(q(x))|: half an e4m3 ulp at |x|, in scaled units.

    e4m3 has 3 mantissa bits, so for a scaled value v the spacing is 2^(floor(log2|v|)-3)
    (subnormal spacing 2^-9 below 2^-6). Half of that, times the block scale, bounds
    round-to-nearest error; a small relative slack covers the fp32 scaling and dequantisation products.
    """
    H = x.shape[-1]
    s = scales
    if s.dtype in (torch.int32, torch.uint8):
        s = ue8m0_to_float(s, H)
    s = s.repeat_interleave(FP8_BLOCK, dim=-1)
    v = (x.float() / s).abs().clamp_max(FP8_MAX)
    e = torch.floor(torch.log2(v.clamp_min(2.0 ** -6)))
    spacing = torch.pow(2.0, e - 3)
    return (0.5 * spacing * (1 + 1e-5) + 1e-7) * s
