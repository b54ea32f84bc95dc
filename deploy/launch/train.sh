#!/usr/bin/env bash
# Single-GPU (or CPU) training.  QW_DATA=data.jsonl QW_STEPS=1000 QW_EXTRA_ARGS="--preset moe-1b-e64" deploy/launch/train.sh
set -euo pipefail
source "$(dirname "${BASH_SOURCE[0]}")/_common.sh"
"$PYTHON" -m quantaweave_b200.train \
  --data "${QW_DATA:-data/smoke/tinystories.jsonl}" --output "${QW_OUTPUT:-artifacts/outputs/quantweave-moe-out}" \
  --steps "${QW_STEPS:-10}" --examples "${QW_EXAMPLES:-10000}" --sequence-length "${QW_SEQUENCE_LENGTH:-128}" \
  --batch-size "${QW_BATCH_SIZE:-2}" --total-experts "${QW_TOTAL_EXPERTS:-16}" --active-experts "${QW_ACTIVE_EXPERTS:-2}" \
  --device "${QW_DEVICE:-auto}" ${QW_EXTRA_ARGS:-}
