"""CPU unit tests: codec, layout math, fp8 codec, routing helpers, transports contract.

Scenarios follow deep_ep_trn tests/unit/test_codec_layout.py.
"""
import pytest
import torch

from deepep_trn_b200 import RowCodec, get_dispatch_layout
from deepep_trn_b200.utils.codec import (dequantize_fp8_1x128, float_to_ue8m0, fp8_error_bound, quantize_fp8_1x128,
                                         ue8m0_to_float)
from deepep_trn_b200.utils.layout import pair_plan, rank_of_expert, send_plan, slot_index, token_positions
from deepep_trn_b200.utils.testing import (ROUTINGS, expected_distinct_ranks, make_routing, randn_router,
                                           router_topk_reference, strided_ep_groups, zipf_router)


def test_codec_roundtrip_is_bit_exact():
    g = torch.Generator().manual_seed(0)
    T, H, K = 37, 256, 8
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    idx = torch.randint(-1, 128, (T, K), generator=g)
    w = torch.randn(T, K, generator=g)
    w[0, 0], w[1, 1] = float('inf'), -0.0
    token = torch.arange(T) * 1_000_003
    codec = RowCodec(H, K)
    assert codec.width % 32 == 0 and codec.width >= H + 4 * K + 2
    rx, ridx, rw, rtok = codec.decode(codec.encode(x, idx, w, token))
    assert torch.equal(rx.view(torch.int16), x.view(torch.int16))
    assert torch.equal(ridx, idx) and torch.equal(rtok, token)
    assert torch.equal(rw.view(torch.int32), w.view(torch.int32))
    with pytest.raises(ValueError):
        RowCodec(H, K, torch.float32)


def test_layout_matches_naive():
    g = torch.Generator().manual_seed(1)
    T, E, K, R = 50, 64, 6, 4
    idx = torch.rand(T, E, generator=g).topk(K, dim=-1).indices
    idx[::7, 2] = -1
    per_rank, per_expert, in_rank = get_dispatch_layout(idx, E, R)
    naive = torch.zeros(T, R, dtype=torch.bool)
    for t in range(T):
        for e in idx[t].tolist():
            if e >= 0:
                naive[t, e // (E // R)] = True
    assert torch.equal(in_rank, naive)
    assert per_rank.dtype == torch.int32 and per_expert.dtype == torch.int32
    assert torch.equal(per_rank.long(), naive.sum(0))
    assert torch.equal(per_expert.long(), torch.bincount(idx[idx >= 0], minlength=E))
    token, counts = send_plan(in_rank)
    expected = torch.cat([naive[:, r].nonzero().flatten() for r in range(R)])
    assert torch.equal(token, expected) and torch.equal(counts, naive.sum(0))
    pos = token_positions(in_rank)
    for r in range(R):
        rows = naive[:, r].nonzero().flatten()
        assert torch.equal(pos[rows, r].long(), torch.arange(rows.numel()))
        assert (pos[~naive[:, r], r] == -1).all()
    tok, kk, pcounts = pair_plan(rank_of_expert(idx, E, R), R)
    assert int(pcounts.sum()) == int((idx >= 0).sum())
    assert torch.equal(rank_of_expert(idx[tok, kk], E, R), torch.repeat_interleave(torch.arange(R), pcounts))
    # (dst, token, k) order
    keys = rank_of_expert(idx[tok, kk], E, R) * (T * K) + tok * K + kk
    assert torch.equal(keys, keys.sort().values)
    with pytest.raises(ValueError):
        rank_of_expert(idx, 63, 4)


def test_slot_index():
    assert slot_index(torch.tensor([2, 0, 3]), 4).tolist() == [0, 1, 8, 9, 10]
    assert slot_index(torch.tensor([0, 0]), 4).tolist() == []


def test_fp8_codec_bounds_and_ue8m0():
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(33, 512, generator=g) * torch.logspace(-3, 2, 512)).to(torch.bfloat16)
    x[0] = 0
    for rs in (False, True):
        q, s = quantize_fp8_1x128(x, round_scale=rs)
        assert q.dtype == torch.float8_e4m3fn and s.shape == (33, 4)
        err = (dequantize_fp8_1x128(q, s) - x.float()).abs()
        assert (err <= fp8_error_bound(x, s)).all()
        if rs:
            packed = float_to_ue8m0(s)
            assert packed.dtype == torch.int32 and packed.shape == (33, 1)
            assert torch.equal(ue8m0_to_float(packed, 512), s)
            m = s.view(torch.int32) & 0x7FFFFF
            assert (m == 0).all()
    # amax floor keeps all-zero blocks finite
    assert torch.isfinite(quantize_fp8_1x128(torch.zeros(2, 128))[1]).all()


def test_testing_helpers():
    assert strided_ep_groups(4, 2) == [[0, 2], [1, 3]] and strided_ep_groups(4, 4) == [[0, 1, 2, 3]]
    assert strided_ep_groups(8, 2) == [[0, 4], [1, 5], [2, 6], [3, 7]]
    with pytest.raises(ValueError):
        strided_ep_groups(6, 4)
    T, E, K, R = 24, 128, 8, 4
    for kind in ROUTINGS:
        for ep_rank in range(R):
            idx, w = make_routing(kind, T, E, K, R, ep_rank, seed=ep_rank)
            n = idx.shape[0]
            assert idx.shape == (n, K) and w.shape == (n, K) and n <= T
            assert not n or (int(idx.max()) < E and int(idx.min()) >= -1)
            if kind not in ('masked', 'ragged'):
                assert n == T and (idx >= 0).all()
            if kind == 'hot_rank0':
                assert (idx < E // R).all()
            if n:
                assert torch.allclose(w.sum(-1), torch.ones(n), atol=1e-5)
    assert make_routing('ragged', T, E, K, R, R - 1, 0)[0].shape[0] == 0
    assert abs(expected_distinct_ranks(256, 8, 8) - 5.295) < 1e-3


def test_routers():
    idx, w = randn_router(64, 256, 8, seed=0)
    assert idx.shape == (64, 8) and torch.allclose(w.sum(-1), torch.ones(64))
    assert all(len(set(r)) == 8 for r in idx.tolist())
    zi, _ = zipf_router(4096, 256, 8, seed=1)
    counts = torch.bincount(zi.flatten(), minlength=256)
    assert counts.max() > 4 * counts.float().mean()  # skewed
    logits = torch.tensor([[1.0, 3.0, 2.0, 3.0]])
    i, ww = router_topk_reference(logits, 2)
    assert sorted(i[0].tolist()) == [1, 3]


def test_custom_ops_trace_without_graph_breaks():
    """The kernels are registered as torch.ops.b200ep.* with fake implementations: they pass
    torch.library.opcheck and compile with fullgraph=True (CPU definitions run here)."""
    import torch._dynamo
    import deepep_trn_b200.ops.library  # noqa: F401 - registers the operators
    from deepep_trn_b200.ops import moe_ops as MO
    ops = torch.ops.b200ep
    g = torch.Generator().manual_seed(3)
    logits = torch.randn(40, 16, generator=g)
    torch.library.opcheck(ops.router_topk, (logits, 4))
    idx, w = ops.router_topk(logits, 4)
    torch.library.opcheck(ops.router_topk_bwd, (idx, w, torch.randn(40, 4, generator=g), 16))
    x = torch.randn(40, 256, generator=g).to(torch.bfloat16)
    torch.library.opcheck(ops.quantize_fp8, (x, True))
    local = torch.where(idx < 8, idx, torch.full_like(idx, -1))   # experts 0..7 are local
    rows, pos, offs, cnt = ops.permute(x, local, 8)
    torch.library.opcheck(ops.unpermute, (rows, pos, w))
    torch.library.opcheck(ops.permute_bwd, (rows, pos))

    def layer(logits, x):
        i, ww = ops.router_topk(logits, 4)
        q, s = ops.quantize_fp8(x, True)
        y = ops.unpermute(x.repeat_interleave(4, 0), torch.arange(160, dtype=torch.int32).reshape(40, 4), ww)
        return i, y, s

    torch._dynamo.reset()
    compiled = torch.compile(layer, fullgraph=True, backend='aot_eager')
    ref = layer(logits, x)
    got = compiled(logits, x)
    assert all(torch.equal(a, b) for a, b in zip(ref, got))
    eg, _ = MO.router_topk(logits, 4)
    assert torch.equal(eg, ref[0])


def test_report_summarises_moe_and_gemm_records(tmp_path):
    import json
    import subprocess
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    moe = dict(bench='moe', ep=8, tokens=4096, hidden=7168, inter=2048, experts=256, topk=8, routing='zipf',
               ours=dict(ms_per_step=18.8, tokens_per_s=1.74e6, expert_tflops_per_rank=460.9),
               nccl=dict(ms_per_step=33.1, tokens_per_s=0.99e6, expert_tflops_per_rank=261.8))
    (tmp_path / 'moe_ep8.jsonl').write_text(json.dumps(moe) + '\n')
    (tmp_path / 'gemm.jsonl').write_text('log line\n' + json.dumps(
        dict(experts=32, gemm1_swiglu=dict(ms=1.5, tflops=1279.2), fp8_gemm2=dict(ms=0.63, tflops=1521.7))) + '\n')
    p = subprocess.run([sys.executable, str(root / 'bench' / 'report.py'), str(tmp_path)], capture_output=True,
                       text=True)
    assert p.returncode == 0, p.stderr
    text = (tmp_path / 'summary.md').read_text()
    assert '## MoE layer' in text and '18.8' in text and '33.1' in text
    assert 'fp8_gemm2' in text and '1521.7' in text


@pytest.mark.parametrize('R,M,Mll,H,K,E', [(1, 4, 1, 128, 1, 8), (8, 4096, 128, 7168, 8, 256), (3, 100, 7, 384, 6, 30)])
def test_heap_layout_regions_fit_and_guards_separate_them(R, M, Mll, H, K, E):
    """The symmetric heap's layout (computed by the C++ runtime, no GPU needed): every region has
    room for what the kernels put there, starts 256-byte aligned, and is followed by its own
    guard zone before the next region begins."""
    from deepep_trn_b200.ops._ext import available, load
    if not available():
        pytest.skip('extension not built')
    L = load().heap_layout(R, M, Mll, H, K, E)
    rs = L['row_stride']
    assert rs >= 2 * H and rs % 16 == 0
    ins = L['inbox_stride']
    assert ins % 128 == 0 and ins >= 2 * H + 8 * K + 4                 # 16-bit dispatch row + metadata
    cins = L['cinbox_stride']
    assert cins % 128 == 0 and cins >= 2 * H + 4 * K                    # 16-bit combine row + weights
    G = L['max_grid']
    single = {'inbox': R * M * ins, 'cinbox': R * M * cins, 'nd_nte': E * 8, 'nd_rcnt': G * R * 4,
              'info': R * G * 8, 'prog': R * G * 8, 'cprog': R * G * 8}
    need = {'ll_rows': R * Mll * rs, 'll_ids': R * Mll * K * 4, 'lc_rows': Mll * K * 2 * H}
    regions = [(L['sig'], L['signals_bytes']), (L['local'], L['local_state_bytes'])]
    regions += [(off, need[name]) for name in need for off in L[name]]
    regions += [(L[name], size) for name, size in single.items()]
    regions.sort()
    guards = sorted(L['guards'])
    gb = L['guard_bytes']
    assert len(guards) == len(regions)
    for (off, size), g in zip(regions, guards):
        assert off % 256 == 0 and off + size <= g, (off, size, g)     # the region fits before its guard
    for (g, (nxt, _)) in zip(guards, regions[1:]):
        assert g + gb <= nxt                                          # the guard ends before the next region
    assert guards[-1] + gb <= L['total']


def test_heap_fits_the_headline_config_in_a_fixed_budget():
    """EP8, 4096 tokens per rank, H=7168, top-8 of 256 experts, 128 low-latency tokens: the
    symmetric heap (a dispatch inbox and a combine inbox of 0.47 GB each, no double
    buffering) stays under 1.1 GB per GPU."""
    from deepep_trn_b200.ops._ext import available
    if not available():
        pytest.skip('extension not built')
    from deepep_trn_b200.parallel.symm import HeapSpec, heap_bytes
    assert heap_bytes(8, HeapSpec(4096, 128, 7168, 8, 256)) < 1.1e9


class _FakeNative:
    """Stands in for the extension's host ops: records the arguments and returns tensors
    shaped like the real ones (CPU tensors; nothing runs on a device)."""

    def __init__(self, T, H, K, E, R, N, per_expert):
        self.T, self.H, self.K, self.E, self.R, self.N, self.per_expert = T, H, K, E, R, N, per_expert
        self.calls = []

    def layout_op(self, idx, E, R, scratch):
        self.calls.append(('layout', E, R))
        return (torch.zeros(R, dtype=torch.int32), torch.zeros(E, dtype=torch.int32),
                torch.zeros(idx.shape[0], R, dtype=torch.bool))

    def dispatch_op(self, heap, x, xs, mode, round_scale, topk, topk_w, nte, itr, E, G, cap, pad, wait, ticket, tmo):
        self.calls.append(('dispatch', mode, cap, pad, wait, ticket, G))
        R, K, H = self.R, self.K, x.shape[1]
        n = self.N if wait else cap
        rx = torch.zeros(cap, H, dtype=x.dtype if mode == 0 else torch.float8_e4m3fn)[:n]
        rs = None if mode == 0 else torch.zeros(cap, H // 128)[:n]
        rt = None if topk is None else torch.full((cap, K), -1, dtype=topk.dtype)[:n]
        rw = None if topk_w is None else torch.zeros(cap, K)[:n]
        notify = ([self.N // R] * R + self.per_expert) if wait else []
        return (rx, rs, rt, rw, torch.zeros(cap, dtype=torch.int64)[:n], torch.zeros(x.shape[0], R, dtype=torch.int32),
                torch.zeros(G, R, dtype=torch.int32), torch.zeros(R, 256, 2, dtype=torch.int32),
                torch.zeros(R + 1, dtype=torch.int64), n, notify)

    def combine_op(self, heap, x, w, recv_off, recv_info, token_pos, send_start, b0, b1, G, pp, pw):
        self.calls.append(('combine', G, pp is not None))
        out_w = None if w is None else torch.zeros(token_pos.shape[0], w.shape[1])
        return torch.zeros(token_pos.shape[0], x.shape[1], dtype=x.dtype), out_w


class _FakeHeap:
    num_sms = 148

    def status(self):
        return (0, 0, 0, 0, 0, 0, 0)


def _fake_engine(T=64, H=256, K=4, E=16, R=2, N=96, per_expert=None):
    from deepep_trn_b200.parallel import engine_nvlink as EN
    from deepep_trn_b200.parallel.symm import HeapSpec
    eng = EN.NvlinkEngine.__new__(EN.NvlinkEngine)
    eng.C = _FakeNative(T, H, K, E, R, N, per_expert or [3, 5, 0, 7, 1, 2, 4, 6][:E // R])
    eng.heap, eng.R, eng.M, eng.rank, eng.ticket = _FakeHeap(), R, T, 0, 0
    eng.spec, eng._last_spec, eng._spec_cache, eng._covered = HeapSpec(T, 8, H, K, E), None, {}, set()
    eng.max_grid, eng.host_timeout_s, eng._scratch, eng.last_exchange = 256, 60.0, None, None
    return eng


def test_nvlink_engine_host_path_with_a_fake_extension():
    """The NVLink engine's host side (one native call per op): outputs cut to the notified
    receive size, handle fields, per-expert counts rounded up by expert_alignment, fp8 tuple
    output, num_worst_tokens (no wait, padded capacity), cached dispatch and combine with pair
    mode. A fake extension stands in for the kernels, so this runs without a GPU."""
    T, H, K, E, R, N = 64, 256, 4, 16, 2, 96
    eng = _fake_engine(T, H, K, E, R, N)
    x = torch.randn(T, H).to(torch.bfloat16)
    idx = torch.randint(0, E, (T, K))
    w = torch.rand(T, K)
    ntr, nte, itr = eng.get_dispatch_layout(idx, E)
    assert ntr.shape == (R,) and nte.shape == (E,) and itr.shape == (T, R)
    rx, rt, rw, per_expert, h, _ = eng.dispatch(x, None, idx, w, itr, E, 4, 0, None, num_tokens_per_expert=nte)
    assert rx.shape == (N, H) and rt.shape == (N, K) and rw.shape == (N, K)
    assert per_expert == [4, 8, 0, 8, 4, 4, 4, 8]                         # [3,5,0,7,1,2,4,6] rounded to 4
    assert h.num_recv == N and h.recv_counts.tolist() == [N // R] * R and h.grid == 148
    assert eng.C.calls[-1][:5] == ('dispatch', 0, R * T, False, True)    # worst-case outputs, waits
    # fp8 in-kernel quantisation returns (e4m3, scales)
    (q, s), *_ = eng.dispatch(x, None, idx, w, itr, E, 1, 0, None, use_fp8=True, num_tokens_per_expert=nte)
    assert q.dtype == torch.float8_e4m3fn and s.shape == (N, H // 128)
    # num_worst_tokens: no wait, every output keeps the padded capacity
    wx, wt, _, pe, wh, _ = eng.dispatch(x, None, idx, w, itr, E, 1, 160, None, num_tokens_per_expert=nte)
    assert wx.shape[0] == 160 and wt.shape[0] == 160 and wh.num_recv is None and pe is None
    assert eng.C.calls[-1][2:5] == (160, True, False)
    # cached dispatch: no top-k outputs, capacity from the handle
    cx, ct, cw, cpe, ch, _ = eng.dispatch(x, h, None, None, None, E, 1, 0, None)
    assert cx.shape[0] == N and ct is None and cw is None and cpe is None and ch.num_recv == N
    # combine: shape check against the handle, weights channel, pair mode
    out, out_w, _ = eng.combine(torch.zeros(N, H, dtype=torch.bfloat16), h, torch.rand(N, K), (), None)
    assert out.shape == (T, H) and out_w.shape == (T, K)
    with pytest.raises(ValueError):
        eng.combine(torch.zeros(N + 1, H, dtype=torch.bfloat16), h, None, (), None)
    pp = torch.zeros(N, K, dtype=torch.int64)
    eng.combine(torch.zeros(N * K, H, dtype=torch.bfloat16), h, None, (), None, pairs=(pp, torch.rand(N, K)))
    assert eng.C.calls[-1] == ('combine', 148, True)
    tickets = [c[5] for c in eng.C.calls if c[0] == 'dispatch']
    assert tickets == sorted(set(tickets))                               # a fresh ticket per dispatch
