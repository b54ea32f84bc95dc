# Shared settings for the launch wrappers (sourced, not run).
ROOT_DIR=$(cd "$(dirname "${BASH_SOURCE[0]}")/../.." && pwd)
cd "$ROOT_DIR"
PYTHON=${QW_PYTHON:-python}
# one process per GPU over NCCL; NVLink/NVSwitch is picked up by NCCL itself (NVLS when the fabric offers it)
TORCHRUN=("$PYTHON" -m torch.distributed.run --nnodes=1 --master-addr "${QW_MASTER_ADDR:-127.0.0.1}" --master-port "${QW_MASTER_PORT:-29500}")
