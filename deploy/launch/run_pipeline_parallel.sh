#!/usr/bin/env bash
# Pipeline-parallel training (optionally x data parallel), one rank per GPU.
#   QW_GPUS=4 QW_MICROBATCHES=8 QW_SCHEDULE=1f1b deploy/launch/run_pipeline_parallel.sh
set -euo pipefail
source "$(dirname "${BASH_SOURCE[0]}")/_common.sh"
timeout -k 60 "${QW_TIMEOUT:-86400}" "${TORCHRUN[@]}" --nproc-per-node "${QW_GPUS:-2}" -m quantaweave_b200.train \
  --pipeline-parallel --microbatches "${QW_MICROBATCHES:-4}" --pipeline-schedule "${QW_SCHEDULE:-1f1b}" \
  --pipeline-data-parallel "${QW_PIPELINE_DATA_PARALLEL:-1}" \
  --data "${QW_DATA:-data/smoke/tinystories.jsonl}" --output "${QW_OUTPUT:-artifacts/outputs/quantweave-moe-pp-out}" \
  --steps "${QW_STEPS:-10}" --examples "${QW_EXAMPLES:-10000}" --sequence-length "${QW_SEQUENCE_LENGTH:-128}" \
  --batch-size "${QW_BATCH_SIZE:-4}" --layers "${QW_LAYERS:-4}" --total-experts "${QW_TOTAL_EXPERTS:-8}" \
  --device "${QW_DEVICE:-auto}" ${QW_EXTRA_ARGS:-}
