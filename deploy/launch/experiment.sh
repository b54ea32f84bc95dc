#!/usr/bin/env bash
# Tracked experiment runs. Arguments are passed through, e.g. deploy/launch/experiment.sh --help
set -euo pipefail
source "$(dirname "${BASH_SOURCE[0]}")/_common.sh"
exec "$PYTHON" -m quantaweave_b200.tools.experiment_manager "$@"
