#!/usr/bin/env bash
# Export an inference bundle. Arguments are passed through, e.g. deploy/launch/export.sh --help
set -euo pipefail
source "$(dirname "${BASH_SOURCE[0]}")/_common.sh"
exec "$PYTHON" -m quantaweave_b200.tools.export "$@"
