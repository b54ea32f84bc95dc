#!/usr/bin/env bash
# Expert (x tensor) parallel training, one rank per GPU.
#   QW_GPUS=8 QW_TENSOR_PARALLEL=1 QW_EXTRA_ARGS="--shard-optimizer --straggler-routing" deploy/launch/run_expert_parallel.sh
# QW_GPUS is the total number of ranks (= expert-parallel size x QW_TENSOR_PARALLEL). QW_EP_TRANSPORT=p2p selects the
# NVLink peer-memory exchange instead of NCCL all-to-all.
set -euo pipefail
source "$(dirname "${BASH_SOURCE[0]}")/_common.sh"
timeout -k 60 "${QW_TIMEOUT:-86400}" "${TORCHRUN[@]}" --nproc-per-node "${QW_GPUS:-2}" -m quantaweave_b200.train \
  --expert-parallel --tensor-parallel "${QW_TENSOR_PARALLEL:-1}" \
  --data "${QW_DATA:-data/smoke/tinystories.jsonl}" --output "${QW_OUTPUT:-artifacts/outputs/quantweave-moe-ep-out}" \
  --steps "${QW_STEPS:-10}" --examples "${QW_EXAMPLES:-10000}" --sequence-length "${QW_SEQUENCE_LENGTH:-128}" \
  --batch-size "${QW_BATCH_SIZE:-2}" --total-experts "${QW_TOTAL_EXPERTS:-16}" --active-experts "${QW_ACTIVE_EXPERTS:-2}" \
  --device "${QW_DEVICE:-auto}" --checkpoint-dir "${QW_CHECKPOINT_DIR:-artifacts/checkpoints/quantweave-moe-ep-checkpoint}" \
  --checkpoint-interval "${QW_CHECKPOINT_INTERVAL:-1000}" ${QW_EXTRA_ARGS:-}
