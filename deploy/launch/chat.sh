#!/usr/bin/env bash
# Interactive or batch chat (any tools.chat option). Arguments are passed through, e.g. deploy/launch/chat.sh --help
set -euo pipefail
source "$(dirname "${BASH_SOURCE[0]}")/_common.sh"
exec "$PYTHON" -m quantaweave_b200.tools.chat "$@"
