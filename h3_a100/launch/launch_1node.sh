#!/usr/bin/env bash
# One-node launcher: torchrun standalone over NPROC GPUs (1, 2, 4 or 8).
#   CONFIG=configs/h3_dmd_b200_world8.yaml NPROC=8 h3_a100/launch/launch_1node.sh
set -euo pipefail
REPO_ROOT=$(cd "$(dirname "${BASH_SOURCE[0]}")/../.." && pwd)
CONFIG=${CONFIG:-"${REPO_ROOT}/configs/h3_dmd_b200_world8.yaml"}
NPROC=${NPROC:-8}
MASTER_PORT=${MASTER_PORT:-29511}
export PYTHONPATH="${REPO_ROOT}:${PYTHONPATH:-}"
export OMP_NUM_THREADS=${OMP_NUM_THREADS:-4}
export TORCH_NCCL_ASYNC_ERROR_HANDLING=${TORCH_NCCL_ASYNC_ERROR_HANDLING:-1}
export NCCL_DEBUG=${NCCL_DEBUG:-WARN}
export H3_EXPECTED_WORLD_SIZE=${H3_EXPECTED_WORLD_SIZE:-${NPROC}}
export H3_BENCHMARK_SEED=${H3_BENCHMARK_SEED:-20260817}
[[ -f "${CONFIG}" ]] || { echo "Missing config: ${CONFIG}" >&2; exit 1; }
if [[ ${H3_SKIP_PREFLIGHT:-0} != 1 ]]; then
  python -m h3_a100.preflight --config "${CONFIG}" > /dev/null || { echo "preflight failed" >&2; exit 1; }
fi
exec timeout -k 60 "${H3_LAUNCH_TIMEOUT:-21600}" python -m torch.distributed.run \
  --nnodes=1 --nproc-per-node="${NPROC}" --master-addr 127.0.0.1 --master-port "${MASTER_PORT}" \
  -m h3_a100.entrypoint --config "${CONFIG}"
