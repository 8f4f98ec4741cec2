#!/usr/bin/env bash
# Benchmark suite on one B200 node: bash bench/run_suite.sh [quick|default] [num_gpus]
# Results: results/<RUN_ID>/{env.json,*.jsonl,summary.md,ops.csv}.
set -uo pipefail
cd "$(dirname "$0")/.."
SUITE=${1:-quick}
NGPU=${2:-$(python -c 'import torch; print(torch.cuda.device_count())')}
RUN_ID=${RUN_ID:-$(date +%Y%m%d-%H%M%S)-$SUITE}
OUT=results/$RUN_ID
TIMEOUT=${BENCH_TIMEOUT:-1800}
mkdir -p "$OUT"
run() {
  timeout -k 60 "$TIMEOUT" python -m torch.distributed.run --nnodes 1 --nproc-per-node "$NGPU" \
    --master-addr 127.0.0.1 --master-port $((29500 + RANDOM % 1000)) "$@" --out-dir "$OUT" 2>&1 | tee -a "$OUT/suite.log"
}
if [ "$SUITE" = quick ]; then
  run bench/bench_ops.py --tokens 128,4096 --routings random --rounds 3 --iters 10
  run bench/bench_baselines.py --tokens 128,4096 --rounds 3 --iters 10
else
  run bench/bench_ops.py --tokens 128,512,4096 --routings random,balanced,zipf,hot_rank0 --fp8 0,1
  run bench/bench_transport.py
  run bench/bench_baselines.py --tokens 128,512,4096
  run bench/bench_moe.py --steps 5
  run bench/bench_moe.py --steps 5 --forward-only --fp8 --impls ours
  timeout -k 60 "$TIMEOUT" python bench/bench_gemm.py 2>&1 | tee -a "$OUT/gemm.jsonl"
fi
python bench/report.py "$OUT"
