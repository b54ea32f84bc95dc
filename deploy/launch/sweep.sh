#!/usr/bin/env bash
# Hyperparameter sweep. Arguments are passed through, e.g. deploy/launch/sweep.sh --help
set -euo pipefail
source "$(dirname "${BASH_SOURCE[0]}")/_common.sh"
exec "$PYTHON" -m quantaweave_b200.tools.sweep "$@"
