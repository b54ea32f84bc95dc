#!/usr/bin/env bash
# HTTP inference server (any tools.serve option). Arguments are passed through, e.g. deploy/launch/serve.sh --help
set -euo pipefail
source "$(dirname "${BASH_SOURCE[0]}")/_common.sh"
exec "$PYTHON" -m quantaweave_b200.tools.serve "$@"
