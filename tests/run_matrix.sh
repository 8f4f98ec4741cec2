#!/usr/bin/env bash
# GPU test matrix on one B200 node: the multi-GPU scenarios at every EP size the node allows.
#
#   bash tests/run_matrix.sh [max_gpus]
#
# For N in 1 2 4 8 (up to max_gpus, default: every visible GPU) the GPU tests run with the
# first N GPUs visible, so the torchrun scenarios of tests/test_gpu.py (normal mode,
# low-latency mode, strided EP groups at N >= 4, absent peer at N >= 2) run with N ranks.
# The kernel-level tests (layout, fp8, GEMM, MoE, allocation-free entry point) run once, at
# N = 1. Stops at the first failing N and prints one PASS/FAIL line per N.
set -uo pipefail
cd "$(dirname "$0")/.."
MAX=${1:-$(python -c 'import torch; print(torch.cuda.device_count())')}
export NCCL_NVLS_ENABLE=${NCCL_NVLS_ENABLE:-0}
status=0
for N in 1 2 4 8; do
  [ "$N" -gt "$MAX" ] && break
  DEVS=$(seq -s, 0 $((N - 1)))
  if [ "$N" -eq 1 ]; then
    SEL=(tests -m gpu)
  else
    SEL=(tests/test_gpu.py -m gpu -k "intranode or low_latency or absent or probe")
  fi
  if CUDA_VISIBLE_DEVICES=$DEVS timeout -k 60 3600 python -m pytest "${SEL[@]}" -x -q > "/tmp/b200ep_matrix_$N.log" 2>&1; then
    echo "EP$N PASS ($(tail -n 1 /tmp/b200ep_matrix_$N.log))"
  else
    echo "EP$N FAIL (log: /tmp/b200ep_matrix_$N.log)"
    tail -n 30 "/tmp/b200ep_matrix_$N.log"
    status=1
    break
  fi
done
exit $status
