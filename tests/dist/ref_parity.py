"""The reference (unmodified, from baseline/_ref) and this library on identical inputs.

Both Buffers run on the same gloo EP group; every output must match exactly:
layout, normal dispatch (rows, ids, weights, per-expert counts, cached dispatch),
combine (identity and with weights), low-latency bf16 dispatch (rows, counts,
src_info, layout_range) and low-latency combine.

torchrun --nnodes 1 --nproc-per-node 4 --master-addr 127.0.0.1 tests/dist/ref_parity.py
"""
import sys
from pathlib import Path

from harness import ROUTING_KINDS, Scenario

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / 'baseline' / '_ref'))

import torch
import torch.distributed as dist

from deepep_trn_b200.utils.testing import bitwise_equal, make_routing


def main():
    from deep_ep_trn import Buffer as RefBuffer
    from deepep_trn_b200 import Buffer
    sc = Scenario(__doc__)
    rank, world = sc.rank, sc.world
    group = dist.new_group(backend='gloo')
    M, H, E, K = 32, 256, 32, 4
    ref = RefBuffer(group, backend='gloo', num_max_tokens_per_rank=M)
    ours = Buffer(group, backend='gloo', num_max_tokens_per_rank=M)
    for kind in ROUTING_KINDS.split(','):
        idx, w = make_routing(kind, 24, E, K, world, rank, seed=3000 + rank)
        T = idx.shape[0]
        x = torch.randn(T, H, generator=torch.Generator().manual_seed(rank)).to(torch.bfloat16)
        a = ref.get_dispatch_layout(idx, E)
        b = ours.get_dispatch_layout(idx, E)
        for i in (0, 2, 3):
            assert torch.equal(a[i], b[i]), (kind, 'layout', i)
        ra = ref.dispatch(x, topk_idx=idx, topk_weights=w, num_tokens_per_rank=a[0], is_token_in_rank=a[3],
                          num_tokens_per_expert=a[2])
        rb = ours.dispatch(x, topk_idx=idx, topk_weights=w, num_tokens_per_rank=b[0], is_token_in_rank=b[3],
                           num_tokens_per_expert=b[2])
        assert bitwise_equal(ra[0], rb[0]), (kind, 'recv_x')
        assert torch.equal(ra[1], rb[1]) and torch.equal(ra[2], rb[2]), (kind, 'recv topk')
        assert ra[3] == rb[3], (kind, 'per expert')
        assert torch.equal(ra[4].recv_src_idx, rb[4].recv_src_idx), (kind, 'recv_src_idx')
        assert bitwise_equal(ref.dispatch(x, handle=ra[4])[0], ours.dispatch(x, handle=rb[4])[0]), (kind, 'cached')
        ca = ref.combine(ra[0], ra[4], topk_weights=ra[2])
        cb = ours.combine(rb[0], rb[4], topk_weights=rb[2])
        assert bitwise_equal(ca[0], cb[0]) and torch.equal(ca[1], cb[1]), (kind, 'combine')
        la = ref.low_latency_dispatch(x, idx, M, E, use_fp8=False)
        lb = ours.low_latency_dispatch(x, idx, M, E, use_fp8=False)
        assert torch.equal(la[1], lb[1]), (kind, 'll count')
        for e in range(E // world):
            n = int(la[1][e])
            assert bitwise_equal(la[0][e, :n], lb[0][e, :n]), (kind, 'll recv_x', e)
        assert torch.equal(la[2].src_info, lb[2].src_info), (kind, 'src_info')
        assert torch.equal(la[2].layout_range, lb[2].layout_range), (kind, 'layout_range')
        y = (la[0].float() * 1.5).to(torch.bfloat16)
        oa = ref.low_latency_combine(y, idx, w, la[2])[0]
        ob = ours.low_latency_combine(y, idx, w, lb[2])[0]
        assert bitwise_equal(oa, ob), (kind, 'll combine')
        print(f'RANK={rank} parity {kind}: T={T} PASS', flush=True)
    sc.done('REF_PARITY')


if __name__ == '__main__':
    main()
