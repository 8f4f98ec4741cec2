"""Raw NVLink transfer curve of the dispatch pull path: rows per peer x row width x fill.

Each rank stages ``rows`` rows per peer and every peer pulls them (the same
``nd_prepare`` + ``nd_pull`` kernels the Buffer uses), with ``fill`` < 1 sending
fewer rows than the capacity. Reports payload and off-rank GB/s per rank, so the
kernel's bandwidth can be read without routing or host work. Counterpart of the
reference's bench/bench_transport.py (which sweeps its NKI all-to-all-v).

torchrun --nnodes 1 --nproc-per-node 8 --master-addr 127.0.0.1 bench/bench_transport.py
"""
from common import PRESETS, Ctx, append_jsonl, base_parser, csv_list, gbps

import torch


def main():
    p = base_parser(__doc__)
    p.add_argument('--rows', type=csv_list(int), default=[8, 32, 128, 512, 2048])
    p.add_argument('--fills', type=csv_list(float), default=[1.0, 0.25])
    p.add_argument('--tma', type=csv_list(int), default=[1, 0])
    args = p.parse_args()
    ctx = Ctx('nvlink', args.ep)
    R = ctx.ep
    widths = sorted({PRESETS[n][0] for n in args.presets})
    from deepep_trn_b200 import Config
    for H in widths:
        for rows in args.rows:
            T = rows * R
            buf = ctx.buffer(T, hidden=H, num_experts=R, topk=1)
            for fill in args.fills:
                n = max(1, round(rows * fill))
                # token t of this rank goes to rank (t // rows); only the first n of each block
                dest = torch.arange(T) // rows
                keep = (torch.arange(T) % rows) < n
                idx = torch.where(keep, dest, torch.full_like(dest, -1)).unsqueeze(1).to(ctx.device)
                x = torch.randn(T, H, device=ctx.device).to(torch.bfloat16)
                ntr, _, nte, itr, _ = buf.get_dispatch_layout(idx, R)
                for tma in args.tma:
                    cfg = Config(use_tma=bool(tma))
                    call = lambda: buf.dispatch(x, topk_idx=idx, num_tokens_per_rank=ntr, is_token_in_rank=itr,
                                                num_tokens_per_expert=nte, config=cfg)
                    res = ctx.measure(call, args.rounds, args.iters)
                    payload = R * n * H * 2
                    rec = dict(bench='transport', ep=R, hidden=H, rows_per_peer=rows, fill=fill, tma=tma,
                               device_us=res, payload_bytes=payload, off_rank_bytes=(R - 1) * n * H * 2,
                               payload_gbps=gbps(payload, res['median_us']),
                               off_rank_gbps=gbps((R - 1) * n * H * 2, res['median_us']))
                    if ctx.rank == 0:
                        append_jsonl(args.out_dir / f'transport_ep{R}.jsonl', rec)
                        print(f"[transport] ep={R} H={H} rows/peer={rows} fill={fill} tma={tma}: "
                              f"{res['median_us']}us payload={rec['payload_gbps']}GB/s "
                              f"off-rank={rec['off_rank_gbps']}GB/s", flush=True)
            buf.destroy()
    ctx.finish()


if __name__ == '__main__':
    main()
