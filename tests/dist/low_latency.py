"""Low-latency dispatch / combine against an all-gather oracle (bf16 and fp8, hooks, CUDA graphs).

torchrun --nnodes 1 --nproc-per-node 4 --master-addr 127.0.0.1 tests/dist/low_latency.py --backend gloo
(reference scenario: tests/dist/test_low_latency.py of deep_ep_trn)
"""
from harness import Scenario

import torch

from deepep_trn_b200.utils.codec import dequantize_fp8_1x128, quantize_fp8_1x128
from deepep_trn_b200.utils.testing import bitwise_equal, expert_scale, make_routing


def check_layout(kind, recv_x, recv_count, handle, peer_data, lo, EL, R, fp8):
    for e in range(EL):
        rows, toks, blocks = [], [], []
        for px, pidx in peer_data:
            t = (pidx == lo + e).any(1).nonzero().flatten()
            rows.append(px[t])
            toks.append(t)
            blocks.append(t.numel())
        rows, toks = torch.cat(rows), torch.cat(toks)
        n = int(recv_count[e])
        assert n == rows.shape[0], (kind, e, n, rows.shape[0])
        if fp8:
            q, s = quantize_fp8_1x128(rows)
            assert bitwise_equal(recv_x[0][e, :n], q) and torch.equal(recv_x[1][e, :n], s), (kind, 'fp8 rows', e)
        else:
            assert bitwise_equal(recv_x[e, :n], rows), (kind, 'recv_x', e)
        assert torch.equal(handle.src_info[e, :n].long().cpu(), toks), (kind, 'src_info', e)
        lr = handle.layout_range[e].cpu()
        counts, starts = (lr & 0xFFFFFFFF).tolist(), (lr >> 32).tolist()
        assert counts == blocks and starts == [sum(blocks[:s]) for s in range(R)], (kind, 'layout_range', e)


def main():
    sc = Scenario(__doc__)
    args, rank = sc.args, sc.rank
    buf = sc.buffer()
    dev = sc.device
    R, E, K, H, M = buf.group_size, args.experts, args.topk, args.hidden, args.max_tokens
    EL, me = E // R, buf.rank
    lo = me * EL
    for i, kind in enumerate(args.kinds.split(',')):
        idx, w = make_routing(kind, args.tokens, E, K, R, me, seed=2000 + rank)
        T = idx.shape[0]
        x = torch.randn(T, H, generator=torch.Generator().manual_seed(rank)).to(torch.bfloat16)
        peer_data = sc.share((x, idx))
        for fp8 in ((False, True) if (args.fp8 and H % 128 == 0) else (False,)):
            hook_mode = bool(i % 2)
            recv_x, recv_count, handle, _, hook = buf.low_latency_dispatch(
                x.to(dev), idx.to(dev), M, E, use_fp8=fp8, return_recv_hook=hook_mode)
            if hook_mode:
                hook()
            rx = (recv_x[0].cpu(), recv_x[1].cpu()) if fp8 else recv_x.cpu()
            rc = recv_count.cpu()
            assert rc.dtype == torch.int32
            check_layout(kind, rx, rc, handle, peer_data, lo, EL, R, fp8)
            scale = expert_scale(torch.arange(EL) + lo)[:, None, None]
            xin = dequantize_fp8_1x128(rx[0].float().to(torch.float8_e4m3fn), rx[1]) if fp8 else rx.float()
            y = (xin * scale).to(torch.bfloat16)
            combined, _, hook = buf.low_latency_combine(y.to(dev), idx.to(dev), w.to(dev), handle,
                                                        return_recv_hook=hook_mode)
            if hook_mode:
                hook()
            xs = dequantize_fp8_1x128(*quantize_fp8_1x128(x)) if fp8 else x.float()
            expert_out = (xs[:, None, :] * expert_scale(idx)[:, :, None]).to(torch.bfloat16).float()
            ref = (expert_out * (w * (idx >= 0))[:, :, None]).sum(1)
            got = combined.cpu().float()
            rel = float((got - ref).abs().mean() / ref.abs().mean().clamp_min(1e-9)) if T else 0.0
            assert torch.allclose(got, ref, rtol=1e-2, atol=1e-3) and rel < 5e-3, (kind, fp8, rel)
            if not fp8 and K <= 2 and args.backend == 'gloo':
                # identity experts on the CPU path: out == sum_k w_k * x exactly (two fp32 products, one
                # sum, one cast; the GPU kernels may fuse the multiply-add, so they keep the tolerance above)
                ident, _, _ = buf.low_latency_combine(recv_x, idx.to(dev), w.to(dev), handle)
                wk = w * (idx >= 0)
                exact = sum(x.float() * wk[:, k:k + 1] for k in range(K)).to(torch.bfloat16)
                assert torch.equal(ident.cpu(), exact), (kind, 'identity combine exact')
        if args.graph and args.backend == 'nvlink':
            # capture dispatch -> expert -> combine once, replay, and compare to the eager result
            d_x, d_idx, d_w = x.to(dev), idx.to(dev), w.to(dev)
            eager, *_ = buf.low_latency_combine(
                (buf.low_latency_dispatch(d_x, d_idx, M, E, use_fp8=False)[0].float() * 2).to(torch.bfloat16),
                d_idx, d_w, buf.low_latency_dispatch(d_x, d_idx, M, E, use_fp8=False)[2])
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                with torch.cuda.graph(g, stream=s):
                    rx_g, _, h_g, _, _ = buf.low_latency_dispatch(d_x, d_idx, M, E, use_fp8=False)
                    out_g, _, _ = buf.low_latency_combine((rx_g.float() * 2).to(torch.bfloat16), d_idx, d_w, h_g)
            torch.cuda.current_stream().wait_stream(s)
            for _ in range(3):
                out_g.zero_()
                g.replay()
                torch.cuda.synchronize()
                assert torch.equal(out_g, eager), (kind, 'cuda graph replay')
            del g
        buf.check()
        buf.check_canaries()
        print(f'RANK={rank} low_latency {kind}: T={T} recv_count_sum={int(rc.sum())} combine_rel={rel:.2e} PASS',
              flush=True)
    sc.done('LOW_LATENCY')


if __name__ == '__main__':
    main()
