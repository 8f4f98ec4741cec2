"""MoE-layer kernels and the full layer forward + backward on one B200 (EP group of one),
against plain fp32 torch definitions."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu
needs_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason='needs CUDA')


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


@needs_cuda
@pytest.mark.parametrize('E,K', [(8, 2), (256, 8), (64, 6)])
def test_router_topk(E, K):
    from deepep_trn_b200.ops.moe_ops import router_topk, router_topk_bwd
    from deepep_trn_b200.utils.testing import router_topk_reference
    g = torch.Generator().manual_seed(E)
    logits = torch.randn(300, E, generator=g)
    idx, w = router_topk(logits.cuda(), K)
    ridx, rw = router_topk_reference(logits, K)
    assert torch.equal(idx.cpu(), ridx)
    assert torch.allclose(w.cpu(), rw, atol=1e-6, rtol=1e-5)
    dw = torch.randn(300, K, generator=g)
    d = router_topk_bwd(idx, w, dw.cuda(), E)
    lr = logits.clone().requires_grad_()
    vals = torch.topk(lr, K, dim=-1).values
    torch.softmax(vals, -1).mul(dw).sum().backward()
    assert torch.allclose(d.cpu(), lr.grad, atol=1e-5, rtol=1e-4)


@needs_cuda
def test_permute_family_matches_cpu():
    from deepep_trn_b200.ops import moe_ops as MO
    g = torch.Generator().manual_seed(0)
    N, H, K, EL = 700, 256, 4, 6
    x = torch.randn(N, H, generator=g).to(torch.bfloat16)
    ids = torch.randint(-1, EL, (N, K), generator=g)
    for n in range(N):  # distinct local ids per row (as dispatch delivers them)
        seen = set()
        for k in range(K):
            if int(ids[n, k]) in seen:
                ids[n, k] = -1
            seen.add(int(ids[n, k]))
    w = torch.rand(N, K, generator=g)
    rows_c, pos_c, offs_c, cnt_c = MO.permute(x, ids, EL)
    rows, pos, offs, cnt = MO.permute(x.cuda(), ids.cuda(), EL, cnt_c.tolist())
    torch.cuda.synchronize()
    assert torch.equal(pos.cpu(), pos_c) and torch.equal(offs.cpu(), offs_c) and torch.equal(cnt.cpu(), cnt_c)
    assert torch.equal(rows.cpu().view(torch.int16), rows_c.view(torch.int16))
    y = MO.unpermute(rows, pos, w.cuda())
    assert _rel(y.cpu(), MO.unpermute(rows_c, pos_c, w)) < 1e-2
    dy = torch.randn(N, H, generator=g).to(torch.bfloat16)
    drows, dw = MO.unpermute_bwd(dy.cuda(), rows, pos, w.cuda(), offs, cnt)
    drows_c, dw_c = MO.unpermute_bwd(dy, rows_c, pos_c, w, offs_c, cnt_c)
    assert _rel(drows.cpu(), drows_c) < 1e-2 and _rel(dw.cpu(), dw_c) < 1e-3
    assert torch.equal(drows.cpu()[rows_c.float().abs().sum(1) == 0].float().abs().sum(), torch.tensor(0.0))
    dx = MO.permute_bwd(rows, pos)
    assert _rel(dx.cpu(), MO.permute_bwd(rows_c, pos_c)) < 1e-2


@needs_cuda
def test_swiglu_bwd_and_transpose():
    from deepep_trn_b200.ops import moe_ops as MO
    g = torch.Generator().manual_seed(1)
    pre = torch.randn(300, 512, generator=g).to(torch.bfloat16)
    dh = torch.randn(300, 256, generator=g).to(torch.bfloat16)
    assert _rel(MO.swiglu_bwd(dh.cuda(), pre.cuda()).cpu(), MO.swiglu_bwd(dh, pre)) < 2e-2
    a = torch.randn(3, 130, 70, generator=g).to(torch.bfloat16)
    assert torch.equal(MO.transpose(a.cuda()).cpu(), a.transpose(1, 2).contiguous())


def _init_single():
    import torch.distributed as dist
    if dist.is_initialized():
        return
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        os.environ['MASTER_PORT'] = str(s.getsockname()[1])
    torch.cuda.set_device(0)
    dist.init_process_group('nccl', rank=0, world_size=1, device_id=torch.device('cuda', 0))


@needs_cuda
def test_permute_fp8_input_dequantises():
    from deepep_trn_b200.ops import moe_ops as MO
    from deepep_trn_b200.utils.codec import quantize_fp8_1x128
    g = torch.Generator().manual_seed(5)
    N, H, K, EL = 300, 512, 4, 5
    x = torch.randn(N, H, generator=g).to(torch.bfloat16)
    ids = torch.stack([torch.randperm(EL + 2, generator=g)[:K] - 2 for _ in range(N)]).clamp_min(-1)
    q, sc = quantize_fp8_1x128(x)
    rows_c, pos_c, offs_c, cnt_c = MO.permute((q, sc), ids, EL)
    rows, pos, offs, cnt = MO.permute((q.cuda(), sc.cuda()), ids.cuda(), EL, cnt_c.tolist())
    torch.cuda.synchronize()
    assert rows.dtype == torch.bfloat16 and torch.equal(pos.cpu(), pos_c) and torch.equal(offs.cpu(), offs_c)
    assert torch.equal(rows.cpu().view(torch.int16), rows_c.view(torch.int16))


@needs_cuda
@pytest.mark.parametrize('fp8_dispatch', [False, True])
def test_moe_layer_forward_backward_matches_fp32(fp8_dispatch):
    import torch.distributed as dist
    from deepep_trn_b200 import Buffer
    from deepep_trn_b200.models.moe import MoELayer, reference_moe
    _init_single()
    buf = Buffer(dist.group.WORLD, backend='nvlink', num_max_tokens_per_rank=512)
    T, H, I, E, K = 384, 512, 256, 16, 4
    layer = MoELayer(buf, H, I, E, K, device='cuda', init_std=0.05, fp8_dispatch=fp8_dispatch)
    x = (torch.randn(T, H, device='cuda') * 0.5).to(torch.bfloat16).requires_grad_()
    y = layer(x)
    dy = torch.randn(T, H, device='cuda').to(torch.bfloat16)
    y.backward(dy)
    torch.cuda.synchronize()
    # fp32 reference with autograd through the chosen-k softmax and the experts
    xr = x.detach().float().requires_grad_()
    Wr = layer.router.detach().float().requires_grad_()
    W1 = layer.w1.detach().float().requires_grad_()
    W2 = layer.w2.detach().float().requires_grad_()
    yr = reference_moe(xr, Wr, W1, W2, K)
    yr.backward(dy.float())
    # fp8 dispatch: the experts see e4m3 inputs (about 3 % relative error per row)
    tol = 1.0 if not fp8_dispatch else 2.0
    assert _rel(y, yr) < 3e-2 * tol, _rel(y, yr)
    assert _rel(x.grad, xr.grad) < 5e-2 * tol, _rel(x.grad, xr.grad)
    assert _rel(layer.w1.grad, W1.grad) < 5e-2 * tol, _rel(layer.w1.grad, W1.grad)
    assert _rel(layer.w2.grad, W2.grad) < 5e-2 * tol, _rel(layer.w2.grad, W2.grad)
    assert _rel(layer.router.grad, Wr.grad) < 8e-2 * tol, _rel(layer.router.grad, Wr.grad)
    buf.check()
    buf.destroy()


@needs_cuda
def test_moe_layer_fp8_experts_inference_matches_fp32():
    # fp8 dispatch + block-scaled fp8 expert GEMMs (inference forward) against the fp32 layer
    import torch.distributed as dist
    from deepep_trn_b200 import Buffer
    from deepep_trn_b200.models.moe import MoELayer, reference_moe
    _init_single()
    buf = Buffer(dist.group.WORLD, backend='nvlink', num_max_tokens_per_rank=512)
    T, H, I, E, K = 384, 512, 256, 16, 4
    layer = MoELayer(buf, H, I, E, K, device='cuda', init_std=0.05, fp8_experts=True)
    x = (torch.randn(T, H, device='cuda') * 0.5).to(torch.bfloat16)
    with torch.no_grad():
        y = layer(x)
        y2 = layer(x)   # weights cached in fp8 after the first call
    torch.cuda.synchronize()
    yr = reference_moe(x.float(), layer.router.float(), layer.w1.float(), layer.w2.float(), K)
    assert _rel(y, yr) < 8e-2, _rel(y, yr)
    assert torch.equal(y, y2)
    buf.check()
    buf.destroy()
