#!/usr/bin/env bash
# One small ncu capture of one kernel of the per-kernel microbenchmark, after a
# plain run of the same command exited 0.  Clocks are never locked.
# The default shape is a small case (16,384 tokens) so that the capture ends by itself.
#   KERNEL=attn_fwd_kernel OP=attention_fwd OUT=ncu_reports/prof h3_a100/launch/ncu_kernel.sh
set -euo pipefail
REPO_ROOT=$(cd "$(dirname "${BASH_SOURCE[0]}")/../.." && pwd)
cd "${REPO_ROOT}"
KERNEL=${KERNEL:?kernel name regex}
OP=${OP:?microbenchmark op label}
OUT=${OUT:-ncu_reports/prof_${OP}}
mkdir -p "$(dirname "${OUT}")"
SHAPE=${SHAPE:-"--tokens 16384 --hidden 5376 --heads 42 --ffn 25088"}
CMD="python -m h3_a100.bench_kernels --which native --iters 1 --only ${OP} ${SHAPE}"
${CMD} > "${OUT}.plain.log" 2>&1
exec ncu --set full --clock-control none -k "regex:${KERNEL}" -s "${SKIP:-0}" -c 1 -o "${OUT}" ${CMD}
