#!/usr/bin/env bash
# Tiny matched DMD cycle on one GPU with the native kernels.
set -euo pipefail
REPO_ROOT=$(cd "$(dirname "${BASH_SOURCE[0]}")/../.." && pwd)
export PYTHONPATH="${REPO_ROOT}:${PYTHONPATH:-}"
export H3_EXPECTED_WORLD_SIZE=1
exec python -m h3_a100.entrypoint --config "${REPO_ROOT}/configs/h3_dmd_smoke_gpu.yaml"
