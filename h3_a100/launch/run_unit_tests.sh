#!/usr/bin/env bash
# CPU test suite (the GPU suite is `python -m pytest tests -m gpu`).
set -euo pipefail
REPO_ROOT=$(cd "$(dirname "${BASH_SOURCE[0]}")/../.." && pwd)
cd "${REPO_ROOT}"
python -m pytest tests -m "not gpu" -q
