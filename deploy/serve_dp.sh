#!/bin/bash
# Independent server replicas, one per GPU group, on consecutive ports (the
# out-of-engine data parallelism an external load balancer spreads over).
#   deploy/serve_dp.sh REPLICAS [GPUS_PER_REPLICA] [BASE_PORT]
# Logs go to ${B200MOE_LOG_DIR:-/tmp}/b200moe-replica-<i>.log; PIDs to .pid files.
set -euo pipefail
ROOT=$(cd "$(dirname "$0")/.." && pwd)
N=${1:?replica count}
G=${2:-1}
PORT0=${3:-${B200MOE_PORT:-8000}}
LOG=${B200MOE_LOG_DIR:-/tmp}
for ((i = 0; i < N; i++)); do
  first=$((i * G))
  devs=$(seq -s, "$first" $((first + G - 1)))
  port=$((PORT0 + i))
  CUDA_VISIBLE_DEVICES=$devs B200MOE_PORT=$port B200MOE_TENSOR_PARALLEL_SIZE=$G \
    nohup "$ROOT/deploy/serve.sh" >"$LOG/b200moe-replica-$i.log" 2>&1 &
  echo $! >"$LOG/b200moe-replica-$i.pid"
  echo "replica $i: GPUs $devs port $port pid $!"
done
