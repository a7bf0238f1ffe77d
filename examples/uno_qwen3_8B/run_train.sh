#!/usr/bin/env bash
# Conditional-LoRA diffusion training of Uno Qwen3-8B with the released recipe:
# the six-stage curriculum (block sizes 2 -> 16 over three epochs), 128 rows of
# 4,096 tokens per step, LoRA rank 128 / alpha 2048 on every projection,
# learning rate 1e-5 with 562 warm-up steps, TV loss only.
#
# Inside or for a Slurm allocation (SLURM_JOB_ID set, or NODES > 1) it hands over
# to uno_b200/train/run_slurm.sh, like the reference recipe; otherwise it runs
# torchrun over this node's GPUs.  CURRICULUM (or CURRICULUM_PATH) names another
# curriculum YAML; DRY_RUN=1 prints the command.
set -euo pipefail
cd "$(dirname "${BASH_SOURCE[0]}")/../.."
export RUN_NAME="${RUN_NAME:-uno-qwen3-8b-3epoch-$(date -u +%Y%m%dT%H%M%SZ)}"
export CURRICULUM="${CURRICULUM:-${CURRICULUM_PATH:-released}}"
if [[ -n "${SLURM_JOB_ID:-}" || "${NODES:-1}" -gt 1 ]]; then
  exec bash uno_b200/train/run_slurm.sh
fi
GPUS="${GPUS:-8}"
GLOBAL_BATCH="${GLOBAL_BATCH:-128}"
cmd=(python -m torch.distributed.run --standalone --nproc-per-node "${GPUS}" -m uno_b200.train
     --model "${MODEL:-preset:qwen3-8b}" --data "${DATA:-synthetic}"
     --output-dir "${OUTPUT_DIR:-runs/${RUN_NAME}}" --run-name "${RUN_NAME}" --fsdp
     --seq-len "${SEQ_LEN:-4096}" --global-batch "${GLOBAL_BATCH}" --micro-batch "${MICRO_BATCH:-1}"
     --curriculum "${CURRICULUM}" --lora-target all --lora-rank "${LORA_RANK:-128}"
     --lora-alpha "${LORA_ALPHA:-2048}" --lr "${LR:-1e-5}" --warmup-steps "${WARMUP_STEPS:-562}"
     --tv-weight 1 --kl-weight 0 --ce-weight 0 --max-grad-norm 1.0 --checkpoint-layers
     --wandb-mode "${WANDB_MODE:-disabled}" "$@")
if [[ "${DRY_RUN:-0}" == "1" ]]; then
  printf '%q ' "${cmd[@]}"; printf '\n'
  exit 0
fi
exec "${cmd[@]}"
