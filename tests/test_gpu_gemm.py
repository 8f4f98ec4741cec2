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
