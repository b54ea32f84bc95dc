#!/usr/bin/env bash
# QLoRA fine-tune of a checkpoint. Arguments are passed through, e.g. deploy/launch/finetune.sh --help
set -euo pipefail
source "$(dirname "${BASH_SOURCE[0]}")/_common.sh"
exec "$PYTHON" -m quantaweave_b200.tools.finetune "$@"
