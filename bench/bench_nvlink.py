"""Raw NVLink engine sweep: which way of moving bytes between B200s is fastest.

Every rank reads (pull) or writes (push) ``--mib`` MiB to or from every other rank at
the same time, with each engine of ``csrc/nvlbench.cu`` (TMA bulk copies driven by one
thread per CTA or per warp, or 16-byte loads/stores from all warps), over a sweep of
transfer sizes, ring depths and CTA counts. Prints one JSON line per configuration:
device time (CUDA events, max over ranks) and off-rank GB/s per GPU.

    torchrun --nnodes 1 --nproc-per-node 8 --master-addr 127.0.0.1 bench/bench_nvlink.py
"""
from __future__ import annotations

import argparse
import itertools
import json
import os
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import torch
import torch.distributed as dist

MODES = {0: 'pull_tma', 1: 'pull_lsu', 2: 'push_tma', 3: 'push_lsu', 4: 'pull_tma_nostore', 5: 'pull_tma_warp'}


def main():
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument('--mib', type=int, default=32, help='MiB moved per (rank, peer) pair')
    p.add_argument('--modes', default='0,1,2,3,4,5')
    p.add_argument('--chunks', default='14336,32768,65536')
    p.add_argument('--stages', default='4,8,12')
    p.add_argument('--grids', default='148,296')
    p.add_argument('--threads', default='256')
    p.add_argument('--iters', type=int, default=10)
    args = p.parse_args()
    local = int(os.environ.get('LOCAL_RANK', 0))
    torch.cuda.set_device(local)
    dist.init_process_group('nccl', timeout=timedelta(seconds=120), device_id=torch.device('cuda', local))
    rank, world = dist.get_rank(), dist.get_world_size()
    from deepep_trn_b200.ops import load
    from deepep_trn_b200.parallel.symm import HeapSpec, create_heap
    C = load()
    bpp_target = args.mib << 20
    # each half of the inbox (R*M rows of about 2H bytes) holds R blocks of bpp bytes
    H = 7168
    M = max(1, -(-2 * bpp_target // (2 * H)) + 64)
    heap = create_heap(dist.group.WORLD, HeapSpec(M, 1, H, 8, max(world, 8)), 10.0)
    ints = lambda s: [int(v) for v in s.split(',') if v]
    for mode, chunk, ns, grid, thr in itertools.product(ints(args.modes), ints(args.chunks), ints(args.stages),
                                                       ints(args.grids), ints(args.threads)):
        if mode in (1, 3) and ns != ints(args.stages)[0]:
            continue  # stages do not apply to the LSU engines
        rings = thr // 32 if mode == 5 else 1
        if mode not in (1, 3) and rings * ns * chunk > 200 * 1024:
            continue
        bpp = bpp_target // chunk * chunk
        run = lambda: C.nvl_bw(heap, mode, bpp, chunk, ns, grid, thr)
        run()
        torch.cuda.synchronize()
        dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(args.iters):
            run()
        e.record()
        torch.cuda.synchronize()
        us = s.elapsed_time(e) * 1e3 / args.iters
        t = torch.tensor([us], device='cuda', dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        us = float(t.item())
        st = heap.status()
        ok = st[0] == 0
        moved = (world - 1) * bpp if world > 1 else bpp
        if rank == 0:
            print(json.dumps(dict(bench='nvlink_engine', mode=MODES[mode], ep=world, chunk=chunk, stages=ns, grid=grid,
                                  threads=thr, bytes_per_peer=bpp, us=round(us, 1),
                                  gbps_per_gpu=round(moved / us / 1e3, 1), ok=ok)), flush=True)
        if not ok:
            heap.clear_status()
    torch.cuda.synchronize()
    dist.barrier()
    heap.close()
    dist.destroy_process_group()


if __name__ == '__main__':
    main()
