#!/usr/bin/env bash
# Train -> benchmark -> export (int8) -> chat checks, on one data file.
#   QW_DATA=data.jsonl QW_STEPS=200 deploy/launch/eval_pipeline.sh
set -euo pipefail
source "$(dirname "${BASH_SOURCE[0]}")/_common.sh"
DATA=${QW_DATA:-data/smoke/tinystories.jsonl}
OUT=${QW_OUTPUT:-artifacts/outputs/quantweave-eval}
"$PYTHON" -m quantaweave_b200.train --data "$DATA" --output "$OUT" --checkpoint-dir "$OUT-ckpt" --steps "${QW_STEPS:-50}" \
  --no-archive --device "${QW_DEVICE:-auto}" ${QW_EXTRA_ARGS:-}
"$PYTHON" -m quantaweave_b200.tools.benchmark --checkpoint "$OUT" --data "$DATA" --output "$OUT/benchmark.json"
"$PYTHON" -m quantaweave_b200.tools.export --checkpoint "$OUT" --output "$OUT-export" --quantize 8
"$PYTHON" -m quantaweave_b200.tools.chat --checkpoint "$OUT" -m "Once upon a time" --temperature 0 --tokens 40
