"""Reference-semantics engine over a ``Transport`` (gloo CPU oracle or NCCL baseline).

Every op is plan -> encode -> exchange -> decode, the control flow of
deep_ep_trn/buffer.py:143-364, written as vectorised torch on the transport's
device: CPU tensors for gloo, CUDA tensors for NCCL. This engine exists to
check the NVLink kernels against (gloo) and to be benchmarked against (NCCL);
it is not the product path.
"""
from __future__ import annotations

import math

import torch

from ..handles import DispatchHandle, EventOverlap, LowLatencyHandle
from ..utils.codec import RowCodec, quantize_fp8_1x128
from ..utils.layout import (experts_per_rank, get_dispatch_layout, pair_plan, rank_of_expert, send_plan,
                            token_rank_mask)
from ..utils.profiling import timer


def _to16(t: torch.Tensor) -> torch.Tensor:
    """Reinterpret any contiguous [n, c] tensor as 16-bit columns (bf16 view)."""
    t = t.contiguous()
    n = t.shape[0]
    cols = math.prod(t.shape[1:]) * t.element_size()
    return t.view(torch.uint8).reshape(n, cols).view(torch.bfloat16)


class TorchEngine:
    def __init__(self, transport, num_max_tokens_per_rank: int):
        self.transport = transport
        self.rank = transport.rank
        self.R = transport.num_ranks
        self.M = num_max_tokens_per_rank
        self.device = 'cpu' if type(transport).__name__ == 'GlooTransport' else None
        self.last_exchange = None

    def _dev(self, t):
        if t is None:
            return None
        return t.detach().to('cpu') if self.device == 'cpu' else t.detach()

    def _exchange(self, rows, counts):
        self.last_exchange = dict(width=rows.shape[1], counts=counts.clone().cpu(), dtype=rows.dtype)
        return self.transport.all_to_all_v(rows, counts)

    # ------------------------------------------------------------------ normal
    def get_dispatch_layout(self, topk_idx, num_experts):
        dev = topk_idx.device
        with timer.stage('plan'):
            ntr, nte, itr = get_dispatch_layout(self._dev(topk_idx), num_experts, self.R)
        return ntr.to(dev), nte.to(dev), itr.to(dev)

    def dispatch(self, x, handle, topk_idx, topk_weights, is_token_in_rank, num_experts, expert_alignment):
        fp8 = isinstance(x, tuple)
        out_dev = (x[0] if fp8 else x).device
        cached = handle is not None
        with timer.stage('in_d2h'):
            if fp8:
                xq, xs = self._dev(x[0]), self._dev(x[1]).to(torch.float32)
                T, H = xq.shape
                payload = torch.cat([_to16(xq.view(torch.uint8)), _to16(xs)], 1)
            else:
                payload = self._dev(x)
                T, H = payload.shape
            if cached:
                K, in_rank, idx, w = handle.topk, self._dev(handle.is_token_in_rank), None, None
            else:
                idx = self._dev(topk_idx).to(torch.int64)
                w = self._dev(topk_weights) if topk_weights is not None else None
                K = idx.shape[1]
                in_rank = (self._dev(is_token_in_rank) if is_token_in_rank is not None
                           else token_rank_mask(idx, num_experts, self.R))
        with timer.stage('plan'):
            token, counts = send_plan(in_rank)
        dt16 = payload.dtype if payload.dtype in (torch.bfloat16, torch.float16) else torch.bfloat16
        codec = RowCodec(payload.shape[1], K, dt16)
        with timer.stage('pack'):
            rows = codec.encode(payload.view(dt16), idx, w, torch.arange(T, device=payload.device))[token]
        recv, recv_counts = self._exchange(rows, counts)
        with timer.stage('unpack'):
            rx, ridx, rw, rtok = codec.decode(recv)
            new = DispatchHandle(T, K, counts, recv_counts, rtok, in_rank, send_token_idx=token,
                                 num_recv=int(recv_counts.sum()), hidden=H, num_experts=num_experts or 0)
            if fp8:
                qbytes = rx.contiguous().view(torch.uint8)
                recv_x = (qbytes[:, :H].contiguous().view(torch.float8_e4m3fn),
                          qbytes[:, H:].contiguous().view(torch.float32))
            else:
                recv_x = rx.contiguous()
            if cached:
                return _out(recv_x, out_dev), None, None, None, new, EventOverlap()
            EL = experts_per_rank(num_experts, self.R)
            lo = self.rank * EL
            local = (ridx >= lo) & (ridx < lo + EL)
            recv_idx = torch.where(local, ridx - lo, torch.full_like(ridx, -1))
            recv_w = torch.where(local, rw, torch.zeros_like(rw))
            per_expert = torch.bincount(recv_idx[local], minlength=EL)
            if expert_alignment > 1:
                per_expert = (per_expert + expert_alignment - 1) // expert_alignment * expert_alignment
        with timer.stage('out_h2d'):
            out_w = recv_w.to(topk_weights.dtype).to(out_dev) if topk_weights is not None else None
            return (_out(recv_x, out_dev), recv_idx.to(topk_idx.dtype).to(out_dev), out_w, per_expert.tolist(),
                    new, EventOverlap())

    def combine(self, x, handle, topk_weights, bias):
        out_dev = x.device
        with timer.stage('in_d2h'):
            xh = self._dev(x)
            wh = self._dev(topk_weights) if topk_weights is not None else None
        N, H = xh.shape
        expect = int(handle.recv_counts.sum())
        if N != expect:
            raise ValueError(f'combine got {N} rows, dispatch delivered {expect}')
        K = wh.shape[1] if wh is not None else 0
        with timer.stage('pack'):
            rows = xh if not K else torch.cat([xh, _to16(wh.to(torch.float32)).view(xh.dtype)], 1)
        back, back_counts = self._exchange(rows.contiguous(), handle.recv_counts.to(torch.int64).cpu())
        if not torch.equal(back_counts.cpu(), handle.send_counts.to(torch.int64).cpu()):
            raise RuntimeError(f'combine returned {back_counts.tolist()} rows, expected '
                               f'{handle.send_counts.tolist()}')
        with timer.stage('unpack'):
            T = handle.num_tokens
            idx = handle.send_token_idx.to(back.device)
            acc = torch.zeros(T, H, dtype=torch.float32, device=back.device).index_add_(0, idx, back[:, :H].float())
            for b in bias:
                acc += self._dev(b).float()
            combined = acc.to(xh.dtype)
            cw = None
            if K:
                wb = back[:, H:H + 2 * K].contiguous().view(torch.float32)
                cw = torch.zeros(T, K, device=back.device).index_add_(0, idx, wb).to(topk_weights.dtype)
        with timer.stage('out_h2d'):
            return combined.to(out_dev), (cw.to(out_dev) if cw is not None else None), EventOverlap()

    # ------------------------------------------------------------------ low latency
    def low_latency_dispatch(self, x, topk_idx, M, num_experts, use_fp8, round_scale, use_ue8m0,
                             cumulative_stats):
        out_dev = x.device
        with timer.stage('in_d2h'):
            xh, idx = self._dev(x), self._dev(topk_idx).to(torch.int64)
        T, H = xh.shape
        R = self.R
        EL = experts_per_rank(num_experts, R)
        lo, K = self.rank * EL, idx.shape[1]
        with timer.stage('plan'):
            in_rank = token_rank_mask(idx, num_experts, R)
            token, counts = send_plan(in_rank)
        with timer.stage('pack'):
            if use_fp8:
                q, s = quantize_fp8_1x128(xh, round_scale or use_ue8m0)
                payload = torch.cat([_to16(q.view(torch.uint8)), _to16(s)], 1)
            else:
                payload = xh
            codec = RowCodec(payload.shape[1], K, payload.dtype)
            rows = codec.encode(payload, idx, None, torch.arange(T, device=xh.device))[token]
        recv, recv_counts = self._exchange(rows, counts)
        with timer.stage('unpack'):
            rx, ridx, _, rtok = codec.decode(recv)
            src = torch.repeat_interleave(torch.arange(R, device=recv.device), recv_counts.to(recv.device))
            hit = (ridx >= lo) & (ridx < lo + EL)
            row, kk = hit.nonzero(as_tuple=True)          # (src, token, k) order
            expert = ridx[row, kk] - lo
            order = torch.sort(expert, stable=True).indices
            per_expert = torch.bincount(expert, minlength=EL)
            starts = torch.cumsum(per_expert, 0) - per_expert
            pos = torch.empty_like(expert)
            pos[order] = torch.arange(expert.numel(), device=expert.device) - starts[expert[order]]
            if use_fp8:
                qb = rx.contiguous().view(torch.uint8)
                xq = qb[:, :H].contiguous().view(torch.float8_e4m3fn)
                xs = qb[:, H:].contiguous().view(torch.float32)
                recv_x = torch.zeros(EL, R * M, H, dtype=torch.float8_e4m3fn, device=recv.device)
                recv_s = torch.zeros(EL, R * M, H // 128, dtype=torch.float32, device=recv.device)
                recv_x[expert, pos] = xq[row]
                recv_s[expert, pos] = xs[row]
                if use_ue8m0:
                    from ..utils.codec import float_to_ue8m0
                    recv_s = float_to_ue8m0(recv_s)
            else:
                recv_x = torch.zeros(EL, R * M, H, dtype=xh.dtype, device=recv.device)
                recv_x[expert, pos] = rx[row]
            src_info = torch.full((EL, R * M), -1, dtype=torch.int32, device=recv.device)
            src_info[expert, pos] = rtok[row].to(torch.int32)
            block = torch.bincount(expert * R + src[row], minlength=EL * R).reshape(EL, R)
            bstart = torch.cumsum(block, 1) - block
            handle = LowLatencyHandle(T, M, H, num_experts, K, src_info.to(out_dev),
                                      ((bstart << 32) | block).to(out_dev), per_expert.to(torch.int32).to(out_dev),
                                      expert, pos, torch.bincount(src[row], minlength=R), use_fp8=use_fp8)
            if cumulative_stats is not None:
                cumulative_stats += per_expert.to(cumulative_stats.dtype).to(cumulative_stats.device)
        with timer.stage('out_h2d'):
            packed = (recv_x.to(out_dev), recv_s.to(out_dev)) if use_fp8 else recv_x.to(out_dev)
            return packed, per_expert.to(torch.int32).to(out_dev), handle

    def low_latency_combine(self, x, topk_idx, topk_weights, handle, out):
        out_dev = x.device
        with timer.stage('in_d2h'):
            xh = self._dev(x)
            idx = self._dev(topk_idx).to(torch.int64)
            w = self._dev(topk_weights).to(torch.float32)
        R = self.R
        with timer.stage('pack'):
            y = xh[handle.pair_expert, handle.pair_pos]
        back, back_counts = self._exchange(y.contiguous(), handle.pairs_per_src.to(torch.int64).cpu())
        with timer.stage('plan'):
            owner = rank_of_expert(idx, handle.num_experts, R)
            tok, kk, expected = pair_plan(owner, R)
        if not torch.equal(back_counts.cpu(), expected.cpu()):
            raise RuntimeError(f'combine returned {back_counts.tolist()} pairs, expected {expected.tolist()}')
        with timer.stage('unpack'):
            acc = torch.zeros(handle.num_tokens, handle.hidden, dtype=torch.float32, device=back.device)
            acc.index_add_(0, tok, back.float() * w[tok, kk].unsqueeze(1))
            combined = acc.to(xh.dtype)
        with timer.stage('out_h2d'):
            combined = combined.to(out_dev)
            if out is not None:
                out.copy_(combined)
                combined = out
            return combined


def _out(recv_x, dev):
    if isinstance(recv_x, tuple):
        return tuple(t.to(dev) for t in recv_x)
    return recv_x.to(dev)
