#!/usr/bin/env bash
# Entry point of the five-arm experiment: preview by default, --execute to run.
set -euo pipefail
repo=$(cd -- "$(dirname -- "${BASH_SOURCE[0]}")/../.." && pwd)
python_bin=${TDB_PYTHON:-python3}
export PYTHONDONTWRITEBYTECODE=1
cd -- "$repo"
exec "$python_bin" -m tempname_dcu_b200.experiment.controller "$@"
