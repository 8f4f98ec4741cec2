"""tcgen05 grouped GEMM numerics against a plain fp32 torch reference (needs a B200)."""
import pytest
import torch

pytestmark = pytest.mark.gpu
needs_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason='needs CUDA')


def _segments(counts, align=128):
    padded = [((c + align - 1) // align) * align for c in counts]
    offs = [0]
    for p in padded:
        offs.append(offs[-1] + p)
    return offs


def _close(got, ref, tol=2e-2):
    if ref.numel() == 0:
        return
    err = (got.float() - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err <= tol * scale, (err, scale)


@needs_cuda
@pytest.mark.parametrize('G,counts,N,K', [
    (3, [128, 0, 256], 256, 256),
    (2, [100, 300], 512, 192),
    (4, [1024, 896, 128, 1280], 4096, 7168),
])
def test_grouped_gemm_forward(G, counts, N, K):
    from deepep_trn_b200.ops.gemm import check, grouped_gemm
    torch.manual_seed(0)
    offs = _segments(counts)
    rows = offs[-1]
    A = (torch.randn(rows, K, device='cuda') * 0.5).to(torch.bfloat16)
    B = (torch.randn(G, N, K, device='cuda') * 0.05).to(torch.bfloat16)
    o = torch.tensor(offs, dtype=torch.int64, device='cuda')
    C = grouped_gemm(A, B, o)
    Cf = grouped_gemm(A, B, o, epilogue='f32')
    torch.cuda.synchronize()
    check()
    for e in range(G):
        s, t = offs[e], offs[e] + counts[e]
        ref = A[s:t].float() @ B[e].float().t()
        _close(C[s:t], ref)
        _close(Cf[s:t], ref, tol=1e-3)


@needs_cuda
def test_grouped_gemm_swiglu():
    from deepep_trn_b200.ops.gemm import check, deinterleave, grouped_gemm, interleave_gate_up
    torch.manual_seed(1)
    G, counts, I, K = 2, [256, 384], 512, 1024
    offs = _segments(counts)
    A = (torch.randn(offs[-1], K, device='cuda') * 0.5).to(torch.bfloat16)
    wg = (torch.randn(G, I, K, device='cuda') * 0.05).to(torch.bfloat16)
    wu = (torch.randn(G, I, K, device='cuda') * 0.05).to(torch.bfloat16)
    W = interleave_gate_up(wg, wu)
    h, pre = grouped_gemm(A, W, torch.tensor(offs, device='cuda'), epilogue='swiglu')
    torch.cuda.synchronize()
    check()
    for e in range(G):
        s, t = offs[e], offs[e] + counts[e]
        g = A[s:t].float() @ wg[e].float().t()
        u = A[s:t].float() @ wu[e].float().t()
        _close(h[s:t], torch.nn.functional.silu(g) * u, tol=3e-2)
        pg, pu = deinterleave(pre[s:t])
        _close(pg, g)
        _close(pu, u)


@needs_cuda
def test_grouped_gemm_wgrad():
    from deepep_trn_b200.ops.gemm import check, grouped_gemm_wgrad
    torch.manual_seed(2)
    G, counts, M, N = 3, [256, 0, 384], 384, 512
    offs = _segments(counts)
    tok = offs[-1]
    At = (torch.randn(M, tok, device='cuda') * 0.5).to(torch.bfloat16)
    Bt = (torch.randn(N, tok, device='cuda') * 0.5).to(torch.bfloat16)
    for e in range(G):  # padding columns are zero, as permute leaves them
        At[:, offs[e] + counts[e]:offs[e + 1]] = 0
        Bt[:, offs[e] + counts[e]:offs[e + 1]] = 0
    o = torch.tensor(offs, device='cuda')
    C = grouped_gemm_wgrad(At, Bt, o, layout='mk')
    # the same product from the untransposed activations (MN-major operands), bf16 out
    Ct = grouped_gemm_wgrad(At.t().contiguous(), Bt.t().contiguous(), o, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    check()
    for e in range(G):
        s, t = offs[e], offs[e + 1]
        ref = At[:, s:t].float() @ Bt[:, s:t].float().t()
        _close(C[e], ref, tol=1e-3)
        _close(Ct[e], ref, tol=1e-2)


@needs_cuda
@pytest.mark.parametrize('G,counts,N,K', [
    (3, [128, 0, 256], 256, 256),
    (2, [100, 300], 192, 200),       # N tail inside a 256 tile, K tail inside a 64 block
    (4, [1024, 896, 128, 1280], 7168, 2048),
])
def test_grouped_gemm_b_kn(G, counts, N, K):
    # B given as [G, K, N] (the forward weight for the input gradient), read MN-major in place
    from deepep_trn_b200.ops.gemm import check, grouped_gemm
    torch.manual_seed(3)
    offs = _segments(counts)
    A = (torch.randn(offs[-1], K, device='cuda') * 0.5).to(torch.bfloat16)
    B = (torch.randn(G, K, N, device='cuda') * 0.05).to(torch.bfloat16)
    o = torch.tensor(offs, dtype=torch.int64, device='cuda')
    C = grouped_gemm(A, B, o, b_layout='kn')
    torch.cuda.synchronize()
    check()
    for e in range(G):
        s, t = offs[e], offs[e] + counts[e]
        _close(C[s:t], A[s:t].float() @ B[e].float())


@needs_cuda
def test_grouped_gemm_residual_epilogue():
    # C = A @ B + R with the sum taken in fp32 before the one bf16 rounding
    from deepep_trn_b200.ops.gemm import check, grouped_gemm
    torch.manual_seed(4)
    T, K, N = 300, 256, 7168
    A = (torch.randn(T, K, device='cuda') * 0.5).to(torch.bfloat16)
    B = (torch.randn(1, K, N, device='cuda') * 0.05).to(torch.bfloat16)
    R = torch.randn(T, N, device='cuda').to(torch.bfloat16)
    o = torch.tensor([0, (T + 127) // 128 * 128], dtype=torch.int64, device='cuda')
    C = grouped_gemm(A, B, o, b_layout='kn', residual=R)
    torch.cuda.synchronize()
    check()
    _close(C, A.float() @ B[0].float() + R.float(), tol=1e-2)


def _fp8_operand(shape, g, row_spread=True):
    """Random data whose rows and 128-channel blocks differ in magnitude (so that every
    scale differs), quantised to e4m3 with power-of-two 1x128 scales."""
    from deepep_trn_b200.ops.gemm import quantize_fp8_blocks
    x = torch.randn(*shape, generator=g)
    K = shape[-1]
    blk = torch.pow(2.0, torch.randint(-3, 4, (*shape[:-1], K // 128), generator=g).float())
    x = x * blk.repeat_interleave(128, -1)
    q, sc = quantize_fp8_blocks(x.cuda())
    deq = (q.float().reshape(*shape[:-1], K // 128, 128) * sc.unsqueeze(-1)).reshape(shape)
    return q, sc, deq


@needs_cuda
@pytest.mark.parametrize('counts,N,K', [([128, 0, 256], 128, 256), ([100, 300], 384, 640),
                                        ([1024, 896, 128, 1280], 2048, 7168)])
def test_grouped_gemm_fp8_block_scaled(counts, N, K):
    from deepep_trn_b200.ops.gemm import check, grouped_gemm_fp8
    g = torch.Generator().manual_seed(11)
    G = len(counts)
    offs = _segments(counts)
    qa, sa, A = _fp8_operand((offs[-1], K), g)
    qb, sb, B = _fp8_operand((G, N, K), g)
    o = torch.tensor(offs, dtype=torch.int64, device='cuda')
    C = grouped_gemm_fp8(qa, sa, qb, sb, o)
    from deepep_trn_b200.ops.gemm import fp8_scale_tiles
    Cf = grouped_gemm_fp8(qa, sa, qb, fp8_scale_tiles(sb, G), o, epilogue='f32')   # prebuilt weight tiles
    torch.cuda.synchronize()
    check()
    for e in range(G):
        s, t = offs[e], offs[e] + counts[e]
        ref = A[s:t] @ B[e].t()      # fp32 product of the same quantised operands
        _close(Cf[s:t], ref, tol=1e-3)
        _close(C[s:t], ref)


@needs_cuda
def test_grouped_gemm_fp8_swiglu():
    from deepep_trn_b200.ops.gemm import check, deinterleave, grouped_gemm_fp8, interleave_gate_up
    g = torch.Generator().manual_seed(12)
    counts, I, K = [256, 384], 256, 1024
    G = len(counts)
    offs = _segments(counts)
    qa, sa, A = _fp8_operand((offs[-1], K), g)
    qg, sg, Wg = _fp8_operand((G, I, K), g)
    qu, su, Wu = _fp8_operand((G, I, K), g)
    qw = interleave_gate_up(qg.view(torch.uint8), qu.view(torch.uint8), block=64).view(torch.float8_e4m3fn)
    sw = interleave_gate_up(sg, su, block=64)
    h, pre = grouped_gemm_fp8(qa, sa, qw.contiguous(), sw.contiguous(), torch.tensor(offs, device='cuda'),
                              epilogue='swiglu')
    torch.cuda.synchronize()
    check()
    for e in range(G):
        s, t = offs[e], offs[e] + counts[e]
        gt = A[s:t] @ Wg[e].t()
        ut = A[s:t] @ Wu[e].t()
        _close(h[s:t], torch.nn.functional.silu(gt) * ut, tol=3e-2)
        pg, pu = deinterleave(pre[s:t], block=64)
        _close(pg, gt)
        _close(pu, ut)


@needs_cuda
def test_custom_ops_on_cuda():
    # the registered operators run the sm_100a kernels and trace into one graph
    import torch._dynamo
    import deepep_trn_b200.ops.library  # noqa: F401
    ops = torch.ops.b200ep
    torch.manual_seed(6)
    A = (torch.randn(256, 512, device='cuda') * 0.5).to(torch.bfloat16)
    B = (torch.randn(2, 256, 512, device='cuda') * 0.05).to(torch.bfloat16)
    o = torch.tensor([0, 128, 256], dtype=torch.int64, device='cuda')
    torch.library.opcheck(ops.grouped_gemm, (A, B, o, 'bf16', 'nk'))
    torch.library.opcheck(ops.grouped_gemm_wgrad, (A, A, o, torch.bfloat16))

    def f(A, B, o):
        c = ops.grouped_gemm(A, B, o, 'f32', 'nk')
        return ops.router_topk(c, 4)

    torch._dynamo.reset()
    got = torch.compile(f, fullgraph=True, backend='aot_eager')(A, B, o)
    ref = f(A, B, o)
    assert torch.equal(got[0], ref[0]) and torch.equal(got[1], ref[1])
