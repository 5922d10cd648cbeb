#!/usr/bin/env bash
# Build everything, then run the native self-test and the test suites.
#   tests/run_tests.sh          CPU tiers (no GPU needed)
#   tests/run_tests.sh --gpu    also the GPU tier (needs a B200)
set -euo pipefail
cd "$(dirname "$0")/.."
python -c "from statespectre_b200 import _build; _build.build()"
statespectre_b200/bin/ofld_selftest
python -m pytest tests -x -q -m "not gpu"
if [[ "${1:-}" == "--gpu" ]]; then
  python -m pytest tests -x -q -m gpu
fi
