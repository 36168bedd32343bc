#!/usr/bin/env bash
# Launch train.py on GPUS local ranks (default 2) with configs/train.json; extra arguments are passed on.
set -euo pipefail
cd "$(dirname "$0")"
if [[ -z "${CUDA_HOME:-}" ]] && command -v nvcc >/dev/null; then
  export CUDA_HOME="$(dirname "$(dirname "$(command -v nvcc)")")"
fi
export TORCH_NCCL_ASYNC_ERROR_HANDLING="${TORCH_NCCL_ASYNC_ERROR_HANDLING:-1}"
export OMP_NUM_THREADS="${OMP_NUM_THREADS:-1}"
exec python -m torch.distributed.run --nnodes=1 --nproc-per-node="${GPUS:-2}" \
  --master-addr="${MASTER_ADDR:-127.0.0.1}" --master-port="${MASTER_PORT:-29500}" \
  train.py --config configs/train.json "$@"
