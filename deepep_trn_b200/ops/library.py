"""The MoE-layer kernels as PyTorch custom operators (``torch.ops.b200ep.*``).

Registering them through ``torch.library.custom_op`` with fake (meta) implementations
lets ``torch.compile``, ``torch.export`` and FX tracing treat each kernel as one opaque
node of known output shape instead of breaking the graph at a foreign call. The
implementations are the functions of ``moe_ops`` / ``gemm`` / ``quant``: the sm_100a
kernels for CUDA tensors, the torch definitions for CPU tensors (grouped GEMMs are
CUDA-only). ``permute``'s output length depends on the routing, so its fake
implementation declares it as a data-dependent size.

    import deepep_trn_b200.ops.library  # registers the operators
    idx, w = torch.ops.b200ep.router_topk(logits, 8)
"""
from __future__ import annotations

import torch

from . import gemm as _G
from . import moe_ops as _MO
from . import quant as _Q

_LIB = 'b200ep'


@torch.library.custom_op(f'{_LIB}::router_topk', mutates_args=())
def router_topk(logits: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Top-k expert ids (int64, ties to the lower id) and softmax weights over the chosen k."""
    return _MO.router_topk(logits, k)


@router_topk.register_fake
def _(logits, k):
    T = logits.shape[0]
    return logits.new_empty(T, k, dtype=torch.int64), logits.new_empty(T, k, dtype=torch.float32)


@torch.library.custom_op(f'{_LIB}::router_topk_bwd', mutates_args=())
def router_topk_bwd(idx: torch.Tensor, w: torch.Tensor, dw: torch.Tensor, num_experts: int) -> torch.Tensor:
    """Gradient of the chosen-k softmax w.r.t. the logits [T, num_experts] (fp32)."""
    return _MO.router_topk_bwd(idx, w, dw, num_experts)


@router_topk_bwd.register_fake
def _(idx, w, dw, num_experts):
    return w.new_empty(w.shape[0], num_experts, dtype=torch.float32)


@torch.library.custom_op(f'{_LIB}::permute', mutates_args=())
def permute(x: torch.Tensor, local_ids: torch.Tensor, num_local_experts: int) -> tuple[
        torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Rows grouped by local expert in 128-row padded segments: (rows, pos, offsets, counts)."""
    return _MO.permute(x, local_ids, num_local_experts)


@permute.register_fake
def _(x, local_ids, num_local_experts):
    ctx = torch.library.get_ctx()
    P = ctx.new_dynamic_size()   # sum of the padded segment sizes: known only after routing
    N, K = local_ids.shape
    return (x.new_empty(P, x.shape[1]), x.new_empty(N, K, dtype=torch.int32),
            x.new_empty(num_local_experts + 1, dtype=torch.int64), x.new_empty(num_local_experts, dtype=torch.int32))


@torch.library.custom_op(f'{_LIB}::unpermute', mutates_args=())
def unpermute(rows: torch.Tensor, pos: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """y[n] = sum_k w[n, k] * rows[pos[n, k]] (fp32 accumulation, one rounding)."""
    return _MO.unpermute(rows, pos, w)


@unpermute.register_fake
def _(rows, pos, w):
    return rows.new_empty(pos.shape[0], rows.shape[1])


@torch.library.custom_op(f'{_LIB}::permute_bwd', mutates_args=())
def permute_bwd(drows: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
    """dx[n] = sum_k drows[pos[n, k]]."""
    return _MO.permute_bwd(drows, pos)


@permute_bwd.register_fake
def _(drows, pos):
    return drows.new_empty(pos.shape[0], drows.shape[1])


@torch.library.custom_op(f'{_LIB}::swiglu_bwd', mutates_args=())
def swiglu_bwd(dh: torch.Tensor, pre: torch.Tensor) -> torch.Tensor:
    """Gradient w.r.t. the 128-block interleaved [gate | up] pre-activation of silu(gate) * up."""
    return _MO.swiglu_bwd(dh, pre)


@swiglu_bwd.register_fake
def _(dh, pre):
    return torch.empty_like(pre)


@torch.library.custom_op(f'{_LIB}::quantize_fp8', mutates_args=())
def quantize_fp8(x: torch.Tensor, round_scale: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
    """e4m3 with one fp32 scale per 128 channels (power-of-two scales with ``round_scale``)."""
    return _Q.quantize_fp8(x, round_scale)


@quantize_fp8.register_fake
def _(x, round_scale=False):
    H = x.shape[-1]
    return (x.new_empty(x.shape, dtype=torch.float8_e4m3fn),
            x.new_empty(*x.shape[:-1], H // 128, dtype=torch.float32))


@torch.library.custom_op(f'{_LIB}::grouped_gemm', mutates_args=())
def grouped_gemm(A: torch.Tensor, B: torch.Tensor, offsets: torch.Tensor, epilogue: str = 'bf16',
                 b_layout: str = 'nk') -> torch.Tensor:
    """C[seg_e] = A[seg_e] @ B[e]^T (``b_layout='nk'``, B [G, N, K]) or @ B[e] (``'kn'``, B [G, K, N]),
    bf16 or fp32 output (tcgen05 tensor cores; CUDA only)."""
    return _G.grouped_gemm(A, B, offsets, epilogue=epilogue, b_layout=b_layout)


@grouped_gemm.register_fake
def _(A, B, offsets, epilogue='bf16', b_layout='nk'):
    N = B.shape[2] if b_layout == 'kn' else B.shape[1]
    return A.new_empty(A.shape[0], N, dtype=torch.float32 if epilogue == 'f32' else torch.bfloat16)


@torch.library.custom_op(f'{_LIB}::grouped_gemm_wgrad', mutates_args=())
def grouped_gemm_wgrad(A: torch.Tensor, B: torch.Tensor, offsets: torch.Tensor,
                       out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """Per-expert A_e^T B_e over token segments of token-major A [tok, M], B [tok, N] -> [G, M, N]."""
    return _G.grouped_gemm_wgrad(A, B, offsets, out_dtype=out_dtype)


@grouped_gemm_wgrad.register_fake
def _(A, B, offsets, out_dtype=torch.bfloat16):
    return A.new_empty(offsets.shape[0] - 1, A.shape[1], B.shape[1], dtype=out_dtype)


__all__ = ['router_topk', 'router_topk_bwd', 'permute', 'unpermute', 'permute_bwd', 'swiglu_bwd', 'quantize_fp8',
           'grouped_gemm', 'grouped_gemm_wgrad']
