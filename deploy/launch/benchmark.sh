#!/usr/bin/env bash
# Benchmark report of a checkpoint. Arguments are passed through, e.g. deploy/launch/benchmark.sh --help
set -euo pipefail
source "$(dirname "${BASH_SOURCE[0]}")/_common.sh"
exec "$PYTHON" -m quantaweave_b200.tools.benchmark "$@"
