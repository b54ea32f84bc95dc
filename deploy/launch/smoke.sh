#!/usr/bin/env bash
# End-to-end smoke: synthetic data, a few steps, then chat and benchmark the result.
set -euo pipefail
source "$(dirname "${BASH_SOURCE[0]}")/_common.sh"
OUT=${QW_OUTPUT:-artifacts/outputs/quantweave-smoke}
"$PYTHON" -m quantaweave_b200.train --preset tiny-cpu --synthetic-data zipf --vocab-size 512 --steps "${QW_STEPS:-20}" \
  --batch-size 4 --sequence-length 64 --output "$OUT" --checkpoint-dir "$OUT-ckpt" --no-archive --no-power-tracking \
  --device "${QW_DEVICE:-auto}"
"$PYTHON" -c "import quantaweave_b200; print('package ok:', quantaweave_b200.__name__)"
