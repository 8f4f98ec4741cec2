"""Raw NVLink engine curve: every rank moves the same number of bytes to (push) or from
(pull) every other rank at once, with the engines of ``csrc/nvlbench.cu``.

Engines: pull_tma (one thread per CTA drives bulk copies from the peer), pull_lsu and
push_lsu (16-byte loads / stores from every warp), push_tma (bulk stores into the peer).
The dispatch and combine kernels push with 16-byte stores (the fastest engine on this
fabric in these measurements). Reports off-rank GB/s per GPU. Counterpart of the
reference's bench/bench_transport.py (its NKI all-to-all-v row-width x rows sweep).

torchrun --nnodes 1 --nproc-per-node 8 --master-addr 127.0.0.1 bench/bench_transport.py
"""
from __future__ import annotations

from harness import BenchGroup, cli, device_stats, ints, words, write_jsonl

ENGINES = {'pull_tma': 0, 'pull_lsu': 1, 'push_tma': 2, 'push_lsu': 3}


def main():
    p = cli(__doc__)
    p.add_argument('--engines', type=words, default=list(ENGINES))
    p.add_argument('--mib', type=ints, default=[8, 64, 256], help='MiB per (rank, peer) pair')
    p.add_argument('--chunk', type=int, default=14336, help='bytes per transfer (one 7168-wide bf16 row)')
    args = p.parse_args()
    bg = BenchGroup('nccl', args.ep)
    from deepep_trn_b200.ops import load
    from deepep_trn_b200.parallel.symm import HeapSpec, create_heap
    C = load()
    H = 7168
    biggest = max(args.mib) << 20
    heap = create_heap(bg.group, HeapSpec(-(-2 * biggest // (2 * H)) + 64, 1, H, 8, max(bg.ep, 8)), 10.0)
    for mib in args.mib:
        bpp = (mib << 20) // args.chunk * args.chunk
        for name in args.engines:
            mode = ENGINES[name]
            res = device_stats(bg, lambda: C.nvl_bw(heap, mode, bpp, args.chunk, 4, 0, 256), args.rounds, args.iters)
            moved = (bg.ep - 1) * bpp if bg.ep > 1 else bpp
            rec = dict(bench='transport', ep=bg.ep, engine=name, chunk=args.chunk, mib_per_peer=mib, device_us=res,
                       gbps_per_gpu=round(moved / res['median_us'] / 1e3, 1), status=list(heap.status()))
            if bg.rank == 0:
                write_jsonl(args.out_dir / f'transport_ep{bg.ep}.jsonl', rec)
                print(f"[transport] ep={bg.ep} {name} {mib} MiB/peer: {res['median_us']} us, "
                      f"{rec['gbps_per_gpu']} GB/s per GPU", flush=True)
    bg.sync()
    heap.close()
    bg.close()


if __name__ == '__main__':
    main()
