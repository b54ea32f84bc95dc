#!/usr/bin/env bash
# Distil into a student checkpoint. Arguments are passed through, e.g. deploy/launch/distill.sh --help
set -euo pipefail
source "$(dirname "${BASH_SOURCE[0]}")/_common.sh"
exec "$PYTHON" -m quantaweave_b200.tools.distill "$@"
