"""Normal-mode dispatch / combine against an all-gather oracle.

torchrun --nnodes 1 --nproc-per-node 4 --master-addr 127.0.0.1 tests/dist/intranode.py --backend gloo --ep 2
(reference scenario: tests/dist/test_intranode.py of deep_ep_trn)
"""
from common import (bitwise_equal, device, expert_scale, finish, gather_peers, init, make_buffer, make_routing,
                    parse_args)

import torch

from deepep_trn_b200.utils.codec import quantize_fp8_1x128
from deepep_trn_b200.utils.layout import rank_of_expert


def naive_layout(idx, experts, ep):
    local = experts // ep
    in_rank = torch.zeros(idx.shape[0], ep, dtype=torch.bool)
    per_expert = torch.zeros(experts, dtype=torch.int64)
    for t in range(idx.shape[0]):
        for e in idx[t].tolist():
            if e >= 0:
                in_rank[t, e // local] = True
                per_expert[e] += 1
    return in_rank.sum(0), per_expert, in_rank


def main():
    args = parse_args(__doc__)
    rank, world, control = init(args.backend)
    buf, peers = make_buffer(args.backend, args.ep, args.max_tokens)
    dev = device(args.backend)
    R, E, K, H = buf.group_size, args.experts, args.topk, args.hidden
    EL, me = E // R, buf.rank
    lo = me * EL
    for kind in args.kinds.split(','):
        idx, w = make_routing(kind, args.tokens, E, K, R, me, seed=1000 + rank)
        T = idx.shape[0]
        x = torch.randn(T, H, generator=torch.Generator().manual_seed(rank)).to(torch.bfloat16)
        d_x, d_idx, d_w = x.to(dev), idx.to(dev), w.to(dev)

        ntr, _, nte, itr, _ = buf.get_dispatch_layout(d_idx, E)
        ref_ntr, ref_nte, ref_itr = naive_layout(idx, E, R)
        assert torch.equal(ntr.cpu().long(), ref_ntr) and torch.equal(nte.cpu().long(), ref_nte), (kind, 'layout')
        assert torch.equal(itr.cpu(), ref_itr), (kind, 'is_token_in_rank')

        recv_x, recv_idx, recv_w, per_expert, handle, _ = buf.dispatch(
            d_x, topk_idx=d_idx, topk_weights=d_w, num_tokens_per_rank=ntr, is_token_in_rank=itr,
            num_tokens_per_expert=nte)
        recv_x, recv_idx, recv_w = recv_x.cpu(), recv_idx.cpu(), recv_w.cpu()

        exp_x, exp_idx, exp_w, exp_src = [], [], [], []
        for px, pidx, pw in gather_peers((x, idx, w), peers, control):
            owner = rank_of_expert(pidx, E, R)
            rows = (owner == me).any(1).nonzero().flatten()
            local = owner[rows] == me
            exp_x.append(px[rows])
            exp_src.append(rows)
            exp_idx.append(torch.where(local, pidx[rows] - lo, torch.full_like(pidx[rows], -1)))
            exp_w.append(torch.where(local, pw[rows], torch.zeros_like(pw[rows])))
        exp_x, exp_idx, exp_w, exp_src = (torch.cat(v) for v in (exp_x, exp_idx, exp_w, exp_src))
        assert bitwise_equal(recv_x, exp_x), (kind, 'recv_x')
        assert torch.equal(recv_idx, exp_idx), (kind, 'recv_topk_idx')
        assert torch.equal(recv_w, exp_w), (kind, 'recv_topk_weights')
        assert torch.equal(handle.recv_src_idx.cpu().long(), exp_src), (kind, 'recv_src_idx')
        assert per_expert == torch.bincount(exp_idx[exp_idx >= 0], minlength=EL).tolist(), (kind, 'per_expert')

        cached_x, *_ = buf.dispatch(d_x, handle=handle)
        assert bitwise_equal(cached_x.cpu(), recv_x), (kind, 'cached dispatch')

        # identity combine: each token comes back once per rank it visited
        combined, combined_w, _ = buf.combine(recv_x.to(dev), handle, topk_weights=recv_w.to(dev))
        ref = (x.float() * ref_itr.sum(1, keepdim=True)).to(torch.bfloat16)
        assert torch.equal(combined.cpu(), ref), (kind, 'identity combine')
        assert torch.equal(combined_w.cpu(), torch.where(idx >= 0, w, torch.zeros_like(w))), (kind, 'weights')

        # emulated experts: the receiver reduces its local experts per row, combine sums ranks
        coef = (expert_scale(recv_idx + lo) * recv_w * (recv_idx >= 0)).sum(-1, keepdim=True)
        y = (recv_x.float() * coef).to(torch.bfloat16)
        combined, _, _ = buf.combine(y.to(dev), handle)
        ref = x.float() * (expert_scale(idx) * w * (idx >= 0)).sum(-1, keepdim=True)
        diff = (combined.cpu().float() - ref).abs()
        rel = float(diff.mean() / ref.abs().mean().clamp_min(1e-9)) if T else 0.0
        assert torch.allclose(combined.cpu().float(), ref, rtol=2e-2, atol=2e-3) and rel < 1e-2, (kind, rel)

        # combine with bias: added in fp32 before the single cast
        bias = torch.randn(T, H, generator=torch.Generator().manual_seed(7 + rank)).to(torch.bfloat16)
        combined, _, _ = buf.combine(recv_x.to(dev), handle, bias=bias.to(dev))
        ref = (x.float() * ref_itr.sum(1, keepdim=True) + bias.float()).to(torch.bfloat16)
        assert torch.equal(combined.cpu(), ref), (kind, 'bias combine')

        if args.fp8 and H % 128 == 0:
            # fp8 in the dispatch kernel: receiver gets q/scales of exactly the oracle rows
            (rq, rs), *_ = buf.dispatch(d_x, topk_idx=d_idx, topk_weights=d_w, num_tokens_per_rank=ntr,
                                        is_token_in_rank=itr, num_tokens_per_expert=nte, use_fp8=True)
            eq, es = quantize_fp8_1x128(exp_x)
            assert bitwise_equal(rq.cpu(), eq) and torch.equal(rs.cpu(), es), (kind, 'fp8 dispatch')
            # pre-quantised tuple input passes through bit-exactly
            q, s = quantize_fp8_1x128(x, round_scale=True)
            (rq, rs), *_ = buf.dispatch((q.to(dev), s.to(dev)), handle=handle)
            eq, es = quantize_fp8_1x128(exp_x, round_scale=True)
            assert bitwise_equal(rq.cpu(), eq) and torch.equal(rs.cpu(), es), (kind, 'fp8 tuple dispatch')
        if args.backend == 'nvlink' and kind == args.kinds.split(',')[0]:
            # repeat-and-compare: the same dispatch / combine on 1..all SMs must give the same bits
            # (an ordering race would show up as a difference between grid sizes)
            from deepep_trn_b200 import Buffer
            ident = (x.float() * ref_itr.sum(1, keepdim=True)).to(torch.bfloat16)
            for n in (1, 3, 7, 16, 61, 0):
                Buffer.set_num_sms(n)
                rx2, _, _, _, h2, _ = buf.dispatch(d_x, topk_idx=d_idx, topk_weights=d_w, num_tokens_per_rank=ntr,
                                                   is_token_in_rank=itr, num_tokens_per_expert=nte)
                c2, _, _ = buf.combine(rx2, h2)
                assert bitwise_equal(rx2.cpu(), recv_x), (kind, 'repeat dispatch', n)
                assert torch.equal(c2.cpu(), ident), (kind, 'repeat combine', n)
            Buffer.set_num_sms(0)
        buf.check()
        buf.check_canaries()
        print(f'RANK={rank} intranode {kind}: T={T} sent={handle.send_counts.tolist()} '
              f'recv={handle.recv_counts.tolist()} expert_combine_rel={rel:.2e} PASS', flush=True)
    finish(control, buf)
    if rank == 0:
        print(f'INTRANODE_PASS backend={args.backend} ep={R}', flush=True)


if __name__ == '__main__':
    main()
