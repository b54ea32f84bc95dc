#!/usr/bin/env bash
# Multi-node expert-parallel training: one task per node, each running torchrun over its 8 B200s (c10d rendezvous).
#SBATCH --job-name=quantaweave-b200
#SBATCH --nodes=2
#SBATCH --ntasks-per-node=1
#SBATCH --gpus-per-node=8
#SBATCH --exclusive
#SBATCH --time=24:00:00
set -euo pipefail
HEAD=$(scontrol show hostnames "$SLURM_JOB_NODELIST" | head -n 1)
export QW_PG_TIMEOUT_S=${QW_PG_TIMEOUT_S:-900}
srun timeout -k 60 86400 python -m torch.distributed.run --nnodes "$SLURM_NNODES" --nproc-per-node 8 \
  --rdzv-backend c10d --rdzv-endpoint "$HEAD:29500" --rdzv-id "$SLURM_JOB_ID" -m quantaweave_b200.train \
  --expert-parallel --preset "${QW_PRESET:-moe-1b-e64}" --token-data "${QW_TOKEN_DATA:-data/tokens}" \
  --sequence-length "${QW_SEQUENCE_LENGTH:-2048}" --batch-size "${QW_BATCH_SIZE:-8}" --steps "${QW_STEPS:-100000}" \
  --output "${QW_OUTPUT:-artifacts/outputs/multinode}" --checkpoint-dir "${QW_CHECKPOINT_DIR:-artifacts/checkpoints/multinode}" \
  --checkpoint-interval 1000 ${QW_EXTRA_ARGS:-}
