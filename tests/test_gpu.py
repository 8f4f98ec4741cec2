"""GPU tests of the sm_100a kernels (need a B200).

Kernel numerics are compared against the torch definitions in ``utils``; the
Buffer scenarios run the same torchrun scripts as the gloo tests with
``--backend nvlink`` (1 GPU here; every visible GPU when there are several).
"""
import os
import subprocess
import sys

import pytest
import torch

from deepep_trn_b200.utils.testing import ROUTINGS, make_routing

pytestmark = pytest.mark.gpu

needs_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason='needs CUDA')


def _ext():
    from deepep_trn_b200.ops import load
    return load()


@needs_cuda
@pytest.mark.parametrize('R', [1, 2, 4, 8])
@pytest.mark.parametrize('T', [0, 1, 3, 128, 4096])
def test_layout_kernel_matches_torch(R, T):
    from deepep_trn_b200.utils.layout import get_dispatch_layout
    C = _ext()
    E, K = 256, 8
    dev = torch.device('cuda')
    scratch = torch.zeros(R + E + 1, dtype=torch.int32, device=dev)
    for kind in ('random', 'masked', 'hot_rank0', 'zipf'):
        idx, _ = make_routing(kind, T, E, K, R, 0, seed=T + R)
        for dtype in (torch.int64, torch.int32):
            d = idx.to(dtype).to(dev)
            ntr = torch.empty(R, dtype=torch.int32, device=dev)
            nte = torch.empty(E, dtype=torch.int32, device=dev)
            itr = torch.empty(idx.shape[0], R, dtype=torch.bool, device=dev)
            C.layout(d, E, R, ntr, nte, itr, scratch)
            r_ntr, r_nte, r_itr = get_dispatch_layout(idx, E, R)
            assert torch.equal(ntr.cpu(), r_ntr) and torch.equal(nte.cpu(), r_nte), (kind, dtype)
            assert torch.equal(itr.cpu(), r_itr), (kind, dtype)
    assert int(scratch.abs().sum()) == 0  # scratch is left zeroed for the next call


@needs_cuda
@pytest.mark.parametrize('H', [128, 512, 7168])
@pytest.mark.parametrize('round_scale', [False, True])
def test_quant_kernel_bitwise(H, round_scale):
    from deepep_trn_b200.ops import quantize_fp8
    from deepep_trn_b200.utils.codec import quantize_fp8_1x128
    g = torch.Generator().manual_seed(H)
    x = (torch.randn(67, H, generator=g) * torch.logspace(-4, 3, H)).to(torch.bfloat16)
    x[3] = 0
    q, s = quantize_fp8(x.cuda(), round_scale)
    rq, rs = quantize_fp8_1x128(x, round_scale)
    assert torch.equal(q.cpu().view(torch.uint8), rq.view(torch.uint8))
    assert torch.equal(s.cpu(), rs)
    from deepep_trn_b200.ops.quant import dequantize_fp8
    assert torch.equal(dequantize_fp8(q, s).cpu().view(torch.int16), dequantize_fp8(rq, rs).view(torch.int16))


@needs_cuda
def test_bounded_wait_reports_timeout(run_dist):
    # a wait on a flag nothing sets must come back as an error status, not a hang or a fault
    code = r'''
import os, torch, torch.distributed as dist
from deepep_trn_b200 import Buffer
os.environ.setdefault("MASTER_ADDR", "127.0.0.1"); os.environ.setdefault("MASTER_PORT", "29591")
torch.cuda.set_device(0)
dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device("cuda", 0))
buf = Buffer(dist.group.WORLD, backend="nvlink", num_max_tokens_per_rank=8, hidden=256, num_experts=8, topk=2)
st = buf._engine.probe_timeout(20_000_000)
assert st[0] == 7 and st[1] == 99, st
buf.check()  # cleared by the probe
x = torch.randn(8, 256, device="cuda").to(torch.bfloat16)
idx = torch.randint(0, 8, (8, 2), device="cuda")
ntr, _, nte, itr, _ = buf.get_dispatch_layout(idx, 8)
rx, *_ , h, _ = buf.dispatch(x, topk_idx=idx, num_tokens_per_rank=ntr, is_token_in_rank=itr, num_tokens_per_expert=nte)
out, _, _ = buf.combine(rx, h)
torch.cuda.synchronize()
assert torch.equal(out, (x.float() * itr.sum(1, keepdim=True)).to(torch.bfloat16))
buf._engine.barrier(); torch.cuda.synchronize(); buf.check()
buf.destroy(); dist.destroy_process_group(); print("PROBE_OK")
'''
    env = dict(os.environ, MASTER_PORT=str(__import__('conftest').free_port()))
    p = subprocess.run([sys.executable, '-c', code], capture_output=True, text=True, timeout=300, env=env)
    assert p.returncode == 0 and 'PROBE_OK' in p.stdout, p.stdout + p.stderr


def _ngpus():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@needs_cuda
@pytest.mark.parametrize('hidden,experts,topk,tokens,maxt', [(256, 32, 4, 24, 32), (7168, 256, 8, 96, 128),
                                                           (128, 8, 1, 1, 4), (256, 16, 2, 3, 8)])
def test_intranode_nvlink(run_dist, hidden, experts, topk, tokens, maxt):
    n = _ngpus()
    nproc = n if n in (1, 2, 4, 8) else 1
    rc, out = run_dist('intranode.py', nproc, '--backend', 'nvlink', '--hidden', hidden, '--experts', experts,
                       '--topk', topk, '--tokens', tokens, '--max-tokens', maxt, '--graph', 1, timeout=900)
    assert rc == 0 and 'INTRANODE_PASS' in out, out[-6000:]


@needs_cuda
@pytest.mark.parametrize('hidden,experts,topk,tokens,maxt', [(256, 32, 4, 24, 32), (7168, 256, 8, 96, 128),
                                                           (128, 8, 1, 1, 4), (256, 16, 2, 3, 8)])
def test_low_latency_nvlink(run_dist, hidden, experts, topk, tokens, maxt):
    n = _ngpus()
    nproc = n if n in (1, 2, 4, 8) else 1
    rc, out = run_dist('low_latency.py', nproc, '--backend', 'nvlink', '--hidden', hidden, '--experts', experts,
                       '--topk', topk, '--tokens', tokens, '--max-tokens', maxt, '--graph', 1, timeout=900)
    assert rc == 0 and 'LOW_LATENCY_PASS' in out, out[-6000:]


@needs_cuda
@pytest.mark.skipif(_ngpus() < 4, reason='needs 4 GPUs for strided EP groups')
def test_intranode_nvlink_strided_groups(run_dist):
    rc, out = run_dist('intranode.py', 4, '--backend', 'nvlink', '--ep', 2, timeout=900)
    assert rc == 0 and 'INTRANODE_PASS' in out, out[-6000:]


@needs_cuda
def test_smoke_entry():
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    p = subprocess.run([sys.executable, os.path.join(root, '__graft_entry__.py')], capture_output=True, text=True,
                       timeout=600, cwd=root)
    assert p.returncode == 0 and 'smoke OK' in p.stdout, p.stdout + p.stderr


@needs_cuda
@pytest.mark.skipif(_ngpus() < 2, reason='needs 2 GPUs')
@pytest.mark.parametrize('case', ['normal', 'll'])
def test_absent_peer_times_out_cleanly(run_dist, case):
    # rank 1 skips the op; rank 0's bounded waits must turn into a DeviceError within seconds
    rc, out = run_dist('peer_absent.py', 2, '--case', case, timeout=300, env={'NCCL_NVLS_ENABLE': '0'})
    assert rc == 0 and 'PEER_ABSENT_PASS' in out, out[-6000:]


@needs_cuda
def test_transport_probe_nvlink():
    # an empty peer and a full-capacity peer through the NVLink kernels (one rank per GPU, up to 2)
    import json
    n = min(2, _ngpus())
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    cmd = [sys.executable, '-m', 'torch.distributed.run', '--nnodes', '1', '--nproc-per-node', str(n),
           '--master-addr', '127.0.0.1', '--master-port', str(__import__('conftest').free_port()),
           os.path.join(root, 'bench', 'probe_transport.py'), '--backend', 'nvlink']
    p = subprocess.run(['timeout', '-k', '30', '300', *cmd], capture_output=True, text=True, cwd=root)
    recs = [json.loads(line[len('PROBE '):]) for line in p.stdout.splitlines() if line.startswith('PROBE ')]
    assert p.returncode == 0 and len(recs) == n and all(r['status'] == 'pass' for r in recs), p.stdout[-3000:]
