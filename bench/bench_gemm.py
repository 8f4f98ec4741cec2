"""Grouped expert GEMM throughput (tcgen05 kernel) on one GPU, against cuBLAS.

Shapes follow the MoE layer of BASELINE config 5 per rank at EP=8: 32 local experts,
``--rows`` rows per expert, H=7168, I=2048 (GEMM1: [rows, H] x [2I, H]^T with the
SwiGLU epilogue; GEMM2: [rows, I] x [H, I]^T). Reports TFLOP/s from CUDA events
(after warm-up, L2 flushed between timed calls) and the same work as one cuBLAS
bf16 matmul per expert for comparison.

python bench/bench_gemm.py --experts 8 --rows 1024
"""
import argparse
import json
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import torch

from deepep_trn_b200.ops import gemm as G


def timed(fn, iters, flush):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(iters):
        flush.fill_(1)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        total += s.elapsed_time(e)
    return total / iters


def main():
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument('--experts', type=int, default=32)
    p.add_argument('--rows', type=int, default=1024)
    p.add_argument('--hidden', type=int, default=7168)
    p.add_argument('--inter', type=int, default=2048)
    p.add_argument('--iters', type=int, default=10)
    p.add_argument('--no-cublas', action='store_true')
    args = p.parse_args()
    E, m, H, I = args.experts, args.rows, args.hidden, args.inter
    dev = torch.device('cuda')
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    rows = E * m
    offs = torch.arange(E + 1, device=dev, dtype=torch.int64) * m
    A = (torch.randn(rows, H, device=dev) * 0.5).to(torch.bfloat16)
    W1 = (torch.randn(E, 2 * I, H, device=dev) * 0.02).to(torch.bfloat16)
    W2 = (torch.randn(E, H, I, device=dev) * 0.02).to(torch.bfloat16)
    h = torch.empty(rows, I, device=dev, dtype=torch.bfloat16)
    pre = torch.empty(rows, 2 * I, device=dev, dtype=torch.bfloat16)
    out = torch.empty(rows, H, device=dev, dtype=torch.bfloat16)
    res = {}
    f1 = 2.0 * rows * H * 2 * I
    f2 = 2.0 * rows * I * H
    ms = timed(lambda: G.grouped_gemm(A, W1, offs, out=pre, epilogue='swiglu', h_out=h), args.iters, flush)
    res['gemm1_swiglu'] = dict(ms=round(ms, 4), tflops=round(f1 / ms / 1e9, 1))
    ms = timed(lambda: G.grouped_gemm(h, W2, offs, out=out), args.iters, flush)
    res['gemm2'] = dict(ms=round(ms, 4), tflops=round(f2 / ms / 1e9, 1))
    dO = (torch.randn(rows, H, device=dev) * 0.1).to(torch.bfloat16)
    # backward shapes, operands read in place (MN-major): dX = dO @ W2, dW2 = dO^T @ h
    dh = torch.empty(rows, I, device=dev, dtype=torch.bfloat16)
    ms = timed(lambda: G.grouped_gemm(dO, W2, offs, out=dh, b_layout='kn'), args.iters, flush)
    res['dgrad2_kn'] = dict(ms=round(ms, 4), tflops=round(f2 / ms / 1e9, 1))
    dpre = (torch.randn(rows, 2 * I, device=dev) * 0.1).to(torch.bfloat16)
    dA = torch.empty(rows, H, device=dev, dtype=torch.bfloat16)
    ms = timed(lambda: G.grouped_gemm(dpre, W1, offs, out=dA, b_layout='kn'), args.iters, flush)
    res['dgrad1_kn'] = dict(ms=round(ms, 4), tflops=round(f1 / ms / 1e9, 1))
    dW2 = torch.empty(E, H, I, device=dev, dtype=torch.bfloat16)
    ms = timed(lambda: G.grouped_gemm_wgrad(dO, h, offs, out=dW2), args.iters, flush)
    res['wgrad2_tok'] = dict(ms=round(ms, 4), tflops=round(f2 / ms / 1e9, 1))
    dW1 = torch.empty(E, 2 * I, H, device=dev, dtype=torch.bfloat16)
    ms = timed(lambda: G.grouped_gemm_wgrad(dpre, A, offs, out=dW1), args.iters, flush)
    res['wgrad1_tok'] = dict(ms=round(ms, 4), tflops=round(f1 / ms / 1e9, 1))
    dOt, ht = dO.t().contiguous(), h.t().contiguous()
    dW2f = torch.empty(E, H, I, device=dev, dtype=torch.float32)
    ms = timed(lambda: G.grouped_gemm_wgrad(dOt, ht, offs, out=dW2f, layout='mk'), args.iters, flush)
    res['wgrad2_mk_f32'] = dict(ms=round(ms, 4), tflops=round(f2 / ms / 1e9, 1))
    # fp8 block-scaled (e4m3, power-of-two 1x128 scales), same shapes
    qa, sa = G.quantize_fp8_blocks(A)
    qw1, sw1 = G.quantize_fp8_blocks(W1)
    qh, shh = G.quantize_fp8_blocks(h)
    qw2, sw2 = G.quantize_fp8_blocks(W2)
    sw1, sw2 = G.fp8_scale_tiles(sw1, E), G.fp8_scale_tiles(sw2, E)   # weights: once, outside the timing
    ms = timed(lambda: G.grouped_gemm_fp8(qa, sa, qw1, sw1, offs, out=pre, epilogue='swiglu', h_out=h), args.iters,
               flush)
    res['fp8_gemm1_swiglu'] = dict(ms=round(ms, 4), tflops=round(f1 / ms / 1e9, 1))
    ms = timed(lambda: G.grouped_gemm_fp8(qh, shh, qw2, sw2, offs, out=out), args.iters, flush)
    res['fp8_gemm2'] = dict(ms=round(ms, 4), tflops=round(f2 / ms / 1e9, 1))
    G.check()
    if not args.no_cublas:
        def cublas1():
            for e in range(E):
                torch.matmul(A[e * m:(e + 1) * m], W1[e].t())
        ms = timed(cublas1, args.iters, flush)
        res['cublas_gemm1_loop'] = dict(ms=round(ms, 4), tflops=round(f1 / ms / 1e9, 1))
        ms = timed(lambda: torch._grouped_mm(A, W1.transpose(1, 2), offs=offs[1:].to(torch.int32)), args.iters, flush) \
            if hasattr(torch, '_grouped_mm') else None
        if ms:
            res['torch_grouped_mm_gemm1'] = dict(ms=round(ms, 4), tflops=round(f1 / ms / 1e9, 1))
    print(json.dumps(dict(experts=E, rows_per_expert=m, hidden=H, inter=I, **res)), flush=True)


if __name__ == '__main__':
    main()
