"""Grouped expert GEMMs on tcgen05 tensor cores (N7) with fused SwiGLU (N8).

``grouped_gemm``       C[seg_e] = A[seg_e] @ B[e]^T      A [rows, K], B [G, N, K]   (forward)
                       C[seg_e] = A[seg_e] @ B[e]        A [rows, K], B [G, K, N]   (``b_layout='kn'``: dX)
``grouped_gemm_wgrad`` C[e] = A[seg_e]^T @ B[seg_e]      A [tok, M], B [tok, N]     (dW)
``grouped_gemm_fp8``   C[seg_e] = A[seg_e] @ B[e]^T      e4m3 A, B with 1x128 power-of-two scales
                       C[e] = A[:, seg_e] @ B[:, seg_e]^T A [M, tok], B [N, tok]    (``layout='mk'``)

Transposed operands are read in place by the tensor cores (MN-major shared-memory
descriptors), never materialised.

Segments are given by ``offsets`` [G + 1] int64 on the device, multiples of 128
(``permute`` pads every expert's rows to that). The kernels read the offsets on
the device, so the calls are CUDA-graph capturable. A device error word records
a timed-out wait inside a kernel; ``check()`` raises on it.
"""
from __future__ import annotations

import torch

from ._ext import load

_errors: dict = {}
EPILOGUES = {'bf16': 0, 'f32': 1, 'swiglu': 2}


def _err(dev) -> torch.Tensor:
    key = (dev.type, dev.index)
    if key not in _errors:
        _errors[key] = torch.zeros(1, dtype=torch.int32, device=dev)
    return _errors[key]


def check(device=None) -> None:
    dev = device or torch.device('cuda', torch.cuda.current_device())
    e = _err(dev)
    if int(e.item()):
        e.zero_()
        raise RuntimeError("a grouped GEMM or permute kernel gave up on a timed-out wait on the device")


def grouped_gemm(A: torch.Tensor, B: torch.Tensor, offsets: torch.Tensor, out: torch.Tensor | None = None,
                 epilogue: str = 'bf16', h_out: torch.Tensor | None = None, save_preact: bool = True,
                 num_sms: int = 0, timeout_s: float = 10.0, b_layout: str = 'nk',
                 residual: torch.Tensor | None = None):
    """Returns C (or ``(h, pre_activation)`` for ``epilogue='swiglu'``). ``b_layout='kn'``
    takes B as [G, K, N] (e.g. a forward weight, for the input gradient). ``residual``
    (bf16 [rows, N], bf16 epilogue only) is added to the fp32 accumulator before rounding."""
    kn = b_layout == 'kn'
    rows, N = A.shape[0], B.shape[2 if kn else 1]
    if epilogue == 'swiglu':
        h = h_out if h_out is not None else torch.empty(rows, N // 2, dtype=torch.bfloat16, device=A.device)
        c = (out if out is not None else torch.empty(rows, N, dtype=torch.bfloat16, device=A.device)) \
            if save_preact else None
        load().grouped_gemm_m(A, B, offsets, c, h, 2, _err(A.device), num_sms, timeout_s, kn, None)
        return h, c
    dtype = torch.float32 if epilogue == 'f32' else torch.bfloat16
    c = out if out is not None else torch.empty(rows, N, dtype=dtype, device=A.device)
    load().grouped_gemm_m(A, B, offsets, c, None, EPILOGUES[epilogue], _err(A.device), num_sms, timeout_s, kn,
                          residual)
    return c


def grouped_gemm_wgrad(A: torch.Tensor, B: torch.Tensor, offsets: torch.Tensor, out_dtype=torch.float32,
                       out: torch.Tensor | None = None, num_sms: int = 0, timeout_s: float = 10.0,
                       layout: str = 'tok'):
    """Per-expert A_e^T B_e over each token segment: ``[G, M, N]``. ``layout='tok'`` takes the
    activations as they are (A [tok, M], B [tok, N]); ``'mk'`` takes them transposed."""
    G = offsets.numel() - 1
    tok = layout == 'tok'
    M, N = (A.shape[1], B.shape[1]) if tok else (A.shape[0], B.shape[0])
    c = out if out is not None else torch.empty(G, M, N, dtype=out_dtype, device=A.device)
    load().grouped_gemm_k(A, B, offsets, c, _err(A.device), num_sms, timeout_s, tok)
    return c


def quantize_fp8_blocks(w: torch.Tensor):
    """e4m3 copy of ``w`` [.., K] with one power-of-two fp32 scale per (row, 128-channel block):
    the operand format of ``grouped_gemm_fp8`` (the tensor cores apply the scales as UE8M0
    exponents, so they must be powers of two)."""
    from ..utils.codec import quantize_fp8_1x128
    q, sc = quantize_fp8_1x128(w, round_scale=True)
    return q.contiguous(), sc.contiguous()


def fp8_scale_tiles(scales: torch.Tensor, groups: int = 1) -> torch.Tensor:
    """Power-of-two fp32 scales [groups * rows, K/128] -> the 512-byte tiles ``grouped_gemm_fp8``
    streams into tensor memory (one per 128 rows and 128-channel block). Build them once for
    weights and pass the tiles instead of the fp32 scales to skip the per-call conversion."""
    sc = scales.reshape(-1, scales.shape[-1]).float().contiguous()
    return load().sf_tiles(sc, groups, sc.shape[0] // groups)


def grouped_gemm_fp8(A, sa, B, sb, offsets, out=None, epilogue: str = 'bf16', h_out=None, save_preact: bool = True,
                     num_sms: int = 0, timeout_s: float = 10.0):
    """Block-scaled fp8 grouped GEMM on the tensor cores (``tcgen05.mma ... kind::mxf8f6f4.block_scale``):
    ``C[seg_e] = (A * sa)[seg_e] @ (B[e] * sb[e])^T`` with A [rows, K] and B [G, N, K] e4m3, and
    power-of-two fp32 scales sa [rows, K/128], sb [G, N, K/128] (``quantize_fp8_blocks``), or
    their ``fp8_scale_tiles``.
    fp32 accumulation; epilogues as ``grouped_gemm``. The SwiGLU epilogue reads each 128-wide
    output tile as [64 gate | 64 up] (``interleave_gate_up(..., block=64)``)."""
    rows, N = A.shape[0], B.shape[1]
    a8, b8 = A.view(torch.uint8), B.view(torch.uint8)
    if sa.dtype != torch.uint8:
        sa = sa.float()
    if sb.dtype != torch.uint8:
        sb = sb.float().contiguous()
    if epilogue == 'swiglu':
        h = h_out if h_out is not None else torch.empty(rows, N // 2, dtype=torch.bfloat16, device=A.device)
        c = (out if out is not None else torch.empty(rows, N, dtype=torch.bfloat16, device=A.device)) \
            if save_preact else None
        load().grouped_gemm_fp8_m(a8, sa, b8, sb, offsets, c, h, 2, _err(A.device), num_sms, timeout_s)
        return h, c
    dtype = torch.float32 if epilogue == 'f32' else torch.bfloat16
    c = out if out is not None else torch.empty(rows, N, dtype=dtype, device=A.device)
    load().grouped_gemm_fp8_m(a8, sa, b8, sb, offsets, c, None, EPILOGUES[epilogue], _err(A.device), num_sms,
                              timeout_s)
    return c


def interleave_gate_up(w_gate: torch.Tensor, w_up: torch.Tensor, block: int = 128) -> torch.Tensor:
    """[G, I, K] gate and up weights -> [G, 2I, K] with 128-row blocks alternating gate / up,
    the layout the SwiGLU epilogue expects (each 256-wide output tile = 128 gate + 128 up)."""
    G, I, K = w_gate.shape
    assert I % block == 0
    g = w_gate.reshape(G, I // block, block, K)
    u = w_up.reshape(G, I // block, block, K)
    return torch.stack([g, u], 2).reshape(G, 2 * I, K)


def deinterleave(x: torch.Tensor, block: int = 128):
    """Inverse of the interleaving along the last dim: [.., 2I] -> (gate [.., I], up [.., I])."""
    *lead, n2 = x.shape
    v = x.reshape(*lead, n2 // (2 * block), 2, block)
    return v[..., 0, :].reshape(*lead, n2 // 2), v[..., 1, :].reshape(*lead, n2 // 2)
