#!/usr/bin/env bash
# Conditional-LoRA diffusion training of Uno Qwen3-8B.  On one node: torchrun
# over the node's GPUs (FSDP base weights, ZeRO-2 LoRA state) with the released
# run's curriculum (block sizes 2 -> 16 over three epochs, 128 rows per step)
# unless CURRICULUM names a YAML.  On Slurm: NODES=N uno_b200/train/run_slurm.sh.
set -euo pipefail
cd "$(dirname "${BASH_SOURCE[0]}")/../.."
MODEL="${MODEL:-preset:qwen3-8b}"
DATA="${DATA:-synthetic}"        # or a directory written by `python -m uno_b200.train.prepare`
GPUS="${GPUS:-8}"
exec python -m torch.distributed.run --standalone --nproc-per-node "${GPUS}" -m uno_b200.train \
  --model "${MODEL}" --data "${DATA}" --output-dir "${OUTPUT_DIR:-runs/uno-qwen3-8b}" --fsdp \
  --seq-len "${SEQ_LEN:-4096}" --micro-batch "${MICRO_BATCH:-1}" --curriculum "${CURRICULUM:-released}" \
  --lora-rank "${LORA_RANK:-64}" --lora-alpha "${LORA_ALPHA:-128}" --lr "${LR:-1e-4}" --max-grad-norm 1.0 \
  --checkpoint-layers "$@"
