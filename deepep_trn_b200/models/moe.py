"""Expert-parallel MoE layer: router top-k -> dispatch -> grouped SwiGLU experts -> combine.

Forward (per rank, EP group of the Buffer):
    logits = x @ Wr^T ; (idx, w) = router_topk(logits)               # N9
    recv = dispatch(x)  (normal mode, NVLink kernels)                 # N1 + N2
    rows = permute(recv) into 128-row padded expert segments          # N10
    h, pre = grouped_gemm(rows, W1, swiglu epilogue)                  # N7 + N8 (tcgen05)
    o = grouped_gemm(h, W2)                                           # N7
    y = combine(o, pairs=(pos, weights))  (weighted un-permute fused)  # N10 + N3
Backward reuses the dispatch handle: the gradient of combine is a cached dispatch
and the gradient of dispatch is a combine (whose weight channel carries the
routing-weight gradients home). Expert weight gradients come from the variable-K
grouped GEMM over the permuted activations.

Weights: W1 [EL, 2I, H] with gate and up rows interleaved in 128-row blocks
(``ops.gemm.interleave_gate_up``), W2 [EL, H, I], router Wr [E, H]; all bf16.
Router logits come out of the same tensor-core GEMM with an fp32 epilogue, so
expert selection matches an fp32 router up to summation order.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from ..ops import gemm as G
from ..ops import moe_ops as MO
from ..ops.quant import quantize_fp8
from ..utils.profiling import timer


_OFFS: dict = {}


def _single_segment(T: int, device) -> torch.Tensor:
    """Offsets [0, T rounded up to 128] for one-group GEMMs (cached per size and device)."""
    key = (T, str(device))
    if key not in _OFFS:
        _OFFS[key] = torch.tensor([0, (T + 127) // 128 * 128], dtype=torch.int64, device=device)
    return _OFFS[key]


def router_logits(x, Wr):
    """fp32 logits [T, E] = x @ Wr^T on the tensor cores (bf16 inputs, fp32 accumulate and output)."""
    return G.grouped_gemm(x.contiguous(), Wr.unsqueeze(0).contiguous(), _single_segment(x.shape[0], x.device),
                          epilogue='f32')


def _expert_forward(rows, offsets, W1, W2):
    h, pre = G.grouped_gemm(rows, W1, offsets, epilogue='swiglu')
    o = G.grouped_gemm(h, W2, offsets)
    return h, pre, o


class _MoEFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, Wr, W1, W2, buf, num_experts, topk, router_bias=None, fp8_dispatch=False):
        EL = num_experts // buf.group_size
        with timer.stage('moe.router'):
            logits = router_logits(x, Wr)
            if router_bias is not None:
                logits = logits + router_bias
            idx, w = MO.router_topk(logits, topk)
        with timer.stage('moe.dispatch'):
            ntr, _, nte, itr, _ = buf.get_dispatch_layout(idx, num_experts)
            # fp8_dispatch: tokens travel as e4m3 with 1x128 scales (quantised inside the
            # dispatch kernel) and are dequantised to bf16 by the permute
            recv_x, recv_idx, recv_w, per_expert, handle, _ = buf.dispatch(
                x, topk_idx=idx, topk_weights=w, num_tokens_per_rank=ntr, is_token_in_rank=itr,
                num_tokens_per_expert=nte, use_fp8=fp8_dispatch)
        with timer.stage('moe.permute'):
            rows, pos, offsets, counts = MO.permute(recv_x, recv_idx, EL, per_expert)
        with timer.stage('moe.experts'):
            h, pre, o = _expert_forward(rows, offsets, W1, W2)
        with timer.stage('moe.combine'):
            # the weighted un-permute (sum_k w * o[pos]) is formed inside the combine kernel
            y, _, _ = buf.combine(o, handle, pair_pos=pos, pair_weights=recv_w)
        ctx.save_for_backward(x, Wr, W1, W2, idx, w, recv_w, pos, offsets, counts, rows, pre, h, o)
        ctx.buf, ctx.handle, ctx.num_experts = buf, handle, num_experts
        return y

    @staticmethod
    def backward(ctx, dy):
        x, Wr, W1, W2, idx, w, recv_w, pos, offsets, counts, rows, pre, h, o = ctx.saved_tensors
        buf, handle = ctx.buf, ctx.handle
        dy = dy.contiguous().to(x.dtype)
        with timer.stage('moe.bwd.dispatch'):
            dy_recv, *_ = buf.dispatch(dy, handle=handle)                 # combine backward
        with timer.stage('moe.bwd.unpermute'):
            d_o, d_recv_w = MO.unpermute_bwd(dy_recv, o, pos, recv_w, offsets, counts)
        # transposed operands are read in place by the GEMM (MN-major tiles); fp32 accumulation,
        # one rounding to the weight dtype
        with timer.stage('moe.bwd.dgrad'):
            dh = G.grouped_gemm(d_o, W2, offsets, b_layout='kn')           # [P, I] = d_o @ W2[e]
            dpre = MO.swiglu_bwd(dh, pre)                                  # [P, 2I]
            drows = G.grouped_gemm(dpre, W1, offsets, b_layout='kn')       # [P, H] = dpre @ W1[e]
        with timer.stage('moe.bwd.wgrad'):
            dW2 = G.grouped_gemm_wgrad(d_o, h, offsets, out_dtype=W2.dtype)      # [EL, H, I]
            dW1 = G.grouped_gemm_wgrad(dpre, rows, offsets, out_dtype=W1.dtype)  # [EL, 2I, H]
        with timer.stage('moe.bwd.permute'):
            d_recv_x = MO.permute_bwd(drows, pos)
        with timer.stage('moe.bwd.combine'):
            dx, dw, _ = buf.combine(d_recv_x, handle, topk_weights=d_recv_w)   # dispatch backward
        with timer.stage('moe.bwd.router'):
            dlogits = MO.router_topk_bwd(idx, w, dw.float(), ctx.num_experts).to(x.dtype)
            seg = _single_segment(x.shape[0], x.device)
            # dx = combine's dx + dlogits @ Wr, summed in fp32 in the GEMM epilogue, one rounding
            dx = G.grouped_gemm(dlogits, Wr.unsqueeze(0), seg, b_layout='kn', residual=dx.contiguous())
            if ctx.num_experts % 64 == 0:
                dWr = G.grouped_gemm_wgrad(dlogits, x, seg, out_dtype=Wr.dtype)[0]            # [E, H]
            else:  # the token-major operand path tiles M in 64-wide atoms
                dWr = G.grouped_gemm_wgrad(MO.transpose(dlogits), MO.transpose(x), seg, out_dtype=Wr.dtype,
                                           layout='mk')[0]
        return dx, dWr, dW1, dW2, None, None, None, None, None


class MoELayer(nn.Module):
    """SwiGLU mixture-of-experts layer with expert parallelism over ``buffer``'s EP group."""

    def __init__(self, buffer, hidden: int, intermediate: int, num_experts: int, topk: int,
                 dtype=torch.bfloat16, device=None, init_std: float = 0.02, seed: int = 0,
                 fp8_dispatch: bool = False, fp8_experts: bool = False):
        super().__init__()
        R = buffer.group_size
        if num_experts % R:
            raise ValueError(f'num_experts={num_experts} must be divisible by the EP size {R}')
        if intermediate % 128 or hidden % 128:
            raise ValueError('hidden and intermediate must be multiples of 128')
        self.buffer = buffer
        self.fp8_dispatch = fp8_dispatch   # forward tokens cross NVLink as fp8 e4m3 + 1x128 scales
        # inference (no autograd): fp8 dispatch and block-scaled fp8 expert GEMMs on e4m3 weights
        self.fp8_experts = fp8_experts
        self._fp8_cache = None
        self.hidden, self.intermediate = hidden, intermediate
        self.num_experts, self.topk = num_experts, topk
        EL = num_experts // R
        # seeded on the target device (the router is shared by all ranks, the experts are per rank)
        gdev = torch.device(device) if device is not None else torch.device('cpu')
        g = torch.Generator(device=gdev).manual_seed(seed)
        g_local = torch.Generator(device=gdev).manual_seed(seed * 1000 + buffer.rank + 1)
        std = init_std

        def randn(*shape, gen):
            return (torch.randn(*shape, generator=gen, device=gdev) * std).to(dtype)
        self.router = nn.Parameter(randn(num_experts, hidden, gen=g))
        wg = randn(EL, intermediate, hidden, gen=g_local)
        wu = randn(EL, intermediate, hidden, gen=g_local)
        self.w1 = nn.Parameter(G.interleave_gate_up(wg, wu))
        del wg, wu
        self.w2 = nn.Parameter(randn(EL, hidden, intermediate, gen=g_local))
        # fp32 bias added to the router logits before top-k (not trained here; it steers load,
        # e.g. a Zipf skew for benchmarks or a balancing bias)
        self.register_buffer('router_bias', torch.zeros(num_experts, dtype=torch.float32, device=device))

    def _fp8_weights(self):
        """e4m3 copies of the expert weights with power-of-two 1x128 scales (as scale tiles),
        rebuilt when the weights change. W1 is re-interleaved in 64-row gate / up blocks, the
        layout of the fp8 GEMM's 128-wide SwiGLU tiles."""
        key = (self.w1._version, self.w2._version, self.w1.data_ptr(), self.w2.data_ptr())
        if self._fp8_cache is None or self._fp8_cache[0] != key:
            with torch.no_grad():
                EL, I2, H = self.w1.shape
                v = self.w1.reshape(EL, I2 // 256, 2, 128, H)
                gate, up = v[:, :, 0].reshape(EL, I2 // 2, H), v[:, :, 1].reshape(EL, I2 // 2, H)
                w1 = G.interleave_gate_up(gate, up, block=64)
                q1, s1 = G.quantize_fp8_blocks(w1)
                q2, s2 = G.quantize_fp8_blocks(self.w2)
                self._fp8_cache = (key, q1, G.fp8_scale_tiles(s1, EL), q2, G.fp8_scale_tiles(s2, EL))
        return self._fp8_cache[1:]

    def _forward_fp8(self, x: torch.Tensor) -> torch.Tensor:
        buf, E = self.buffer, self.num_experts
        EL = E // buf.group_size
        with timer.stage('moe.router'):
            logits = router_logits(x, self.router) + self.router_bias
            idx, w = MO.router_topk(logits, self.topk)
        with timer.stage('moe.dispatch'):
            ntr, _, nte, itr, _ = buf.get_dispatch_layout(idx, E)
            recv_x, recv_idx, recv_w, per_expert, handle, _ = buf.dispatch(
                x, topk_idx=idx, topk_weights=w, num_tokens_per_rank=ntr, is_token_in_rank=itr,
                num_tokens_per_expert=nte, use_fp8=True, round_scale=True)
        with timer.stage('moe.permute'):
            (rq, rs), pos, offsets, _ = MO.permute(recv_x, recv_idx, EL, per_expert, keep_fp8=True)
        q1, t1, q2, t2 = self._fp8_weights()
        with timer.stage('moe.experts'):
            h, _ = G.grouped_gemm_fp8(rq, rs, q1, t1, offsets, epilogue='swiglu', save_preact=False)
            hq, hs = quantize_fp8(h, round_scale=True)
            o = G.grouped_gemm_fp8(hq, hs, q2, t2, offsets)
        with timer.stage('moe.combine'):
            # the weighted un-permute (sum_k w * o[pos]) is formed inside the combine kernel
            y, _, _ = buf.combine(o, handle, pair_pos=pos, pair_weights=recv_w)
        return y

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.fp8_experts and not torch.is_grad_enabled():
            return self._forward_fp8(x)
        return _MoEFunction.apply(x, self.router, self.w1, self.w2, self.buffer, self.num_experts, self.topk,
                                  self.router_bias, self.fp8_dispatch)


def reference_moe(x, Wr, W1, W2, topk, router_bias=None):
    """fp32 torch definition of the layer on one rank holding all experts (W1 interleaved)."""
    logits = x.float() @ Wr.float().t()
    if router_bias is not None:
        logits = logits + router_bias
    idx, w = MO.router_topk(logits.cpu(), topk)
    idx, w = idx.to(x.device), w.to(x.device)
    out = torch.zeros(x.shape, dtype=torch.float32, device=x.device)
    for e in range(W1.shape[0]):
        hit = (idx == e)
        tok = hit.any(1).nonzero().flatten()
        if tok.numel() == 0:
            continue
        a = x[tok].float()
        gu = a @ W1[e].float().t()
        gate, up = G.deinterleave(gu)
        hh = torch.nn.functional.silu(gate) * up
        oo = hh @ W2[e].float().t()
        we = (w[tok] * hit[tok]).sum(1, keepdim=True)
        out[tok] += we * oo
    return out


def smoke_step(buf, dev):
    """One tiny forward + backward of the layer (used by the build/smoke entry point)."""
    torch.manual_seed(0)
    layer = MoELayer(buf, hidden=256, intermediate=256, num_experts=8 * buf.group_size, topk=2, device=dev)
    x = (torch.randn(64, 256, device=dev) * 0.5).to(torch.bfloat16).requires_grad_()
    y = layer(x)
    y.float().square().mean().backward()
    torch.cuda.synchronize()
    assert torch.isfinite(y.float()).all() and torch.isfinite(x.grad.float()).all()
    assert layer.w1.grad is not None and torch.isfinite(layer.w1.grad.float()).all()
