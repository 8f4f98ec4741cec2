"""Multi-process CPU tests over gloo: the full Buffer semantics without a GPU."""
import pytest
import torch
import torch.distributed as dist


@pytest.fixture(scope='module')
def single_rank_group(tmp_path_factory):
    path = tmp_path_factory.mktemp('pg') / 'store'
    dist.init_process_group('gloo', init_method=f'file://{path}', rank=0, world_size=1)
    yield dist.group.WORLD
    dist.destroy_process_group()


def test_single_rank_roundtrip(single_rank_group):
    from deepep_trn_b200 import Buffer
    g = torch.Generator().manual_seed(2)
    T, H, E, K, M = 20, 128, 16, 4, 32
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    idx = torch.rand(T, E, generator=g).topk(K, dim=-1).indices
    w = torch.rand(T, K, generator=g)
    buf = Buffer(single_rank_group, backend='gloo', num_max_tokens_per_rank=M)
    ntr, _, nte, itr, _ = buf.get_dispatch_layout(idx, E)
    rx, ridx, rw, per_expert, handle, _ = buf.dispatch(
        x, topk_idx=idx, topk_weights=w, num_tokens_per_rank=ntr, is_token_in_rank=itr, num_tokens_per_expert=nte)
    assert torch.equal(rx, x) and torch.equal(ridx, idx) and torch.equal(rw, w)
    assert per_expert == nte.tolist()
    combined, cw, _ = buf.combine(rx, handle, topk_weights=rw)
    assert torch.equal(combined, x) and torch.equal(cw, w)

    recv_x, count, ll_handle, _, hook = buf.low_latency_dispatch(x, idx, M, E, use_fp8=False, return_recv_hook=True)
    hook()
    assert recv_x.shape == (E, M, H) and int(count.sum()) == T * K
    out, _, _ = buf.low_latency_combine(recv_x, idx, w, ll_handle)
    ref = (x.float() * w.sum(-1, keepdim=True)).to(torch.bfloat16)
    assert torch.allclose(out.float(), ref.float(), rtol=1e-2, atol=1e-3)

    (q, s), count, ll_handle, _, _ = buf.low_latency_dispatch(x, idx, M, E)  # fp8 by default
    assert q.dtype == torch.float8_e4m3fn and s.shape == (E, M, H // 128)

    with pytest.raises(ValueError):
        buf.dispatch(torch.zeros(M + 1, H, dtype=torch.bfloat16), topk_idx=idx.repeat(2, 1)[:M + 1],
                     num_tokens_per_expert=nte)
    with pytest.raises(ValueError):
        buf.dispatch(x, topk_idx=idx)  # missing num_tokens_per_expert
    with pytest.raises(ValueError):
        buf.combine(rx[:-1], handle)
    with pytest.raises(NotImplementedError):
        buf.low_latency_combine(recv_x, idx, w, ll_handle, use_logfmt=True)
    with pytest.raises(ValueError):
        Buffer(single_rank_group, backend='bogus')


@pytest.mark.parametrize('ep', [4, 2])
def test_intranode_gloo(run_dist, ep):
    rc, out = run_dist('intranode.py', 4, '--backend', 'gloo', '--ep', ep, '--hidden', 256, '--experts', 32,
                       '--topk', 4, timeout=600)
    assert rc == 0 and 'INTRANODE_PASS' in out, out[-4000:]


@pytest.mark.parametrize('ep', [4, 2])
def test_low_latency_gloo(run_dist, ep):
    rc, out = run_dist('low_latency.py', 4, '--backend', 'gloo', '--ep', ep, '--hidden', 256, '--experts', 32,
                       '--topk', 4, timeout=600)
    assert rc == 0 and 'LOW_LATENCY_PASS' in out, out[-4000:]


def test_low_latency_roundtrip_exact_gloo(run_dist):
    # world 2, T=64, H=256, E=8, K=2: identity experts give out == sum_k w_k * x exactly
    rc, out = run_dist('low_latency.py', 2, '--backend', 'gloo', '--hidden', 256, '--experts', 8, '--topk', 2,
                       '--tokens', 64, '--max-tokens', 64, timeout=600)
    assert rc == 0 and 'LOW_LATENCY_PASS' in out, out[-4000:]


REF = __import__('pathlib').Path(__file__).resolve().parents[1] / 'baseline' / '_ref' / 'deep_ep_trn'


@pytest.mark.skipif(not REF.exists(), reason='reference not installed under baseline/_ref')
@pytest.mark.parametrize('nproc', [4, 2])
def test_reference_parity_gloo(run_dist, nproc):
    rc, out = run_dist('ref_parity.py', nproc, timeout=600)
    assert rc == 0 and 'REF_PARITY_PASS' in out, out[-4000:]


@pytest.mark.parametrize('case', ['config', 'exit', 'counts'])
def test_host_made_failures_raise(run_dist, case):
    """Failures made on the host end in exceptions on the ranks that can see them, not in hangs."""
    import re
    rc, out = run_dist('failures.py', 3, '--case', case, timeout=240, env={'B200EP_PG_TIMEOUT': '20'})
    lines = re.findall(r'RANK=(\d+) (DETECTED=\w+?|UNDETECTED);', out)
    status = {int(r): s for r, s in lines}
    if case == 'config':
        assert rc == 0 and all(status.get(r) == 'DETECTED=ValueError' for r in range(3)), out[-3000:]
    elif case == 'exit':
        assert 'RANK=2 LEAVING' in out, out[-3000:]
        assert all(status.get(r, '').startswith('DETECTED=') for r in (0, 1)), out[-3000:]
    else:
        assert rc == 0 and len(status) == 3, out[-3000:]
        assert any(s == 'DETECTED=RuntimeError' for s in status.values()), out[-3000:]


def test_transport_probe_gloo(tmp_path):
    """bench/probe_transport.py: an empty peer and a full-capacity peer, reported as PROBE json."""
    import json
    import subprocess
    import sys
    from pathlib import Path
    from conftest import free_port
    root = Path(__file__).resolve().parents[1]
    cmd = [sys.executable, '-m', 'torch.distributed.run', '--nnodes', '1', '--nproc-per-node', '2',
           '--master-addr', '127.0.0.1', '--master-port', str(free_port()), str(root / 'bench' / 'probe_transport.py'),
           '--backend', 'gloo']
    p = subprocess.run(['timeout', '-k', '30', '300', *cmd], capture_output=True, text=True, cwd=str(root))
    recs = [json.loads(line[len('PROBE '):]) for line in p.stdout.splitlines() if line.startswith('PROBE ')]
    assert p.returncode == 0 and len(recs) == 2, p.stdout[-2000:] + p.stderr[-2000:]
    assert all(r['status'] == 'pass' for r in recs) and sorted(r['tokens'] for r in recs) == [0, 64]


def test_baseline_moe_layer_cpu(single_rank_group):
    """The NCCL + grouped-matmul baseline layer (here over gloo on CPU) against the fp32 definition."""
    from deepep_trn_b200 import Buffer
    from deepep_trn_b200.models.moe import reference_moe
    from deepep_trn_b200.models.moe_baseline import BaselineMoELayer
    buf = Buffer(single_rank_group, backend='gloo', num_max_tokens_per_rank=64)
    T, H, I, E, K = 48, 256, 128, 8, 2
    layer = BaselineMoELayer(buf, H, I, E, K)
    torch.manual_seed(0)
    with torch.no_grad():
        for p in layer.parameters():
            p.normal_(0, 0.05)
    x = (torch.randn(T, H) * 0.5).to(torch.bfloat16).requires_grad_()
    y = layer(x)
    yr = reference_moe(x.detach().float(), layer.router.detach().float(), layer.w1.detach().float(),
                       layer.w2.detach().float(), K)
    assert ((y.float() - yr).norm() / yr.norm()).item() < 2e-2
    y.float().square().sum().backward()
    assert x.grad is not None and torch.isfinite(x.grad.float()).all() and layer.w1.grad.abs().sum() > 0
