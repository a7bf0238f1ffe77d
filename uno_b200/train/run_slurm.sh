#!/usr/bin/env bash
# Multi-node conditional-LoRA training under Slurm: one torchrun per node, one
# process per GPU, NCCL over NVLink within a node and the cluster fabric across
# nodes.  Run it with sbatch-style settings in the environment; it submits
# itself (one task per node) and each task execs torchrun with this
# framework's trainer (`python -m uno_b200.train`, FSDP base weights + ZeRO-2
# LoRA optimizer state).
#
# CURRICULUM defaults to the released run's schedule (block sizes 2-16 over
# three epochs); FIXED_BLOCK_SIZE=B (with EPOCHS, default 1) instead trains at
# one block size through a generated one-stage curriculum.
#
# Required: MODEL (checkpoint dir or preset:NAME), DATA (prepared rows.jsonl
# directory or "synthetic"), OUTPUT_ROOT (shared storage).  Optional knobs
# below; GLOBAL_BATCH must divide by NODES * GPUS_PER_NODE * MICRO_BATCH
# (the quotient is the gradient-accumulation count).
#
# DRY_RUN=1 prints the sbatch / srun / torchrun command it would run and exits.
set -euo pipefail

launch() {
  if [[ "${DRY_RUN:-0}" == "1" ]]; then
    printf '%q ' "$@"; printf '\n'
    exit 0
  fi
  exec "$@"
}

REPO_ROOT="${UNO_REPO_ROOT:-$(cd "$(dirname "${BASH_SOURCE[0]}")/../.." && pwd)}"
PYTHON_BIN="${PYTHON_BIN:-python}"
NODES="${NODES:-2}"
GPUS_PER_NODE="${GPUS_PER_NODE:-8}"
CPUS_PER_TASK="${CPUS_PER_TASK:-64}"
TIME_LIMIT="${TIME_LIMIT:-7-00:00:00}"
MICRO_BATCH="${MICRO_BATCH:-1}"
GLOBAL_BATCH="${GLOBAL_BATCH:-128}"
SEQ_LEN="${SEQ_LEN:-4096}"
LORA_RANK="${LORA_RANK:-128}"
LORA_TARGET="${LORA_TARGET:-all}"
LR="${LR:-1e-5}"
WARMUP_STEPS="${WARMUP_STEPS:-562}"
TV_WEIGHT="${TV_WEIGHT:-1.0}"
KL_WEIGHT="${KL_WEIGHT:-0.0}"
CE_WEIGHT="${CE_WEIGHT:-0.0}"
CE_TARGET="${CE_TARGET:-teacher}"
CURRICULUM="${CURRICULUM:-released}"   # the released run's six-stage schedule, or a YAML path
RUN_NAME="${RUN_NAME:-uno-$(date -u +%Y%m%dT%H%M%SZ)}"
WANDB_MODE="${WANDB_MODE:-online}"       # online needs `wandb login` or WANDB_API_KEY; offline or disabled otherwise
WANDB_PROJECT="${WANDB_PROJECT:-uno-training}"
: "${MODEL:?set MODEL to a checkpoint directory or preset:NAME}"
: "${DATA:?set DATA to a prepared corpus directory or synthetic}"
: "${OUTPUT_ROOT:?set OUTPUT_ROOT to shared storage}"

per_step=$((NODES * GPUS_PER_NODE * MICRO_BATCH))
if (( GLOBAL_BATCH % per_step != 0 )); then
  echo "GLOBAL_BATCH=${GLOBAL_BATCH} is not a multiple of nodes*gpus*micro-batch=${per_step}" >&2
  exit 2
fi
OUTPUT_DIR="${OUTPUT_DIR:-${OUTPUT_ROOT}/runs/${RUN_NAME}}"
LOG_DIR="${LOG_DIR:-${OUTPUT_ROOT}/logs/${RUN_NAME}}"
if [[ -n "${FIXED_BLOCK_SIZE:-}" && "${UNO_NODE_WORKER:-0}" != "1" ]]; then
  # one block size for EPOCHS passes (python -m uno_b200.train.make_curriculum)
  CURRICULUM="${OUTPUT_DIR}/curriculum-b${FIXED_BLOCK_SIZE}.yaml"
  (cd "${REPO_ROOT}" && "${PYTHON_BIN}" -m uno_b200.train.make_curriculum fixed --output "${CURRICULUM}" \
    --epochs "${EPOCHS:-1}" --block-size "${FIXED_BLOCK_SIZE}" --sequence-length "${SEQ_LEN}" \
    --global-batch-size "${GLOBAL_BATCH}")
fi
export REPO_ROOT PYTHON_BIN NODES GPUS_PER_NODE MICRO_BATCH GLOBAL_BATCH SEQ_LEN LORA_RANK LORA_TARGET LR \
  WARMUP_STEPS TV_WEIGHT KL_WEIGHT CE_WEIGHT CE_TARGET CURRICULUM RUN_NAME MODEL DATA OUTPUT_DIR LOG_DIR \
  WANDB_MODE WANDB_PROJECT

if [[ "${UNO_NODE_WORKER:-0}" == "1" ]]; then
  # one task per node: exec torchrun for this node's GPUs
  export TMPDIR="${SLURM_TMPDIR:-/tmp}/uno-${SLURM_JOB_ID:-0}-${SLURM_PROCID:-0}"
  mkdir -p "${TMPDIR}"
  cmd=("${PYTHON_BIN}" -m torch.distributed.run --nnodes="${SLURM_NNODES}" --nproc-per-node="${GPUS_PER_NODE}"
       --node-rank="${SLURM_PROCID}" --master-addr="${MASTER_ADDR}" --master-port="${MASTER_PORT}"
       -m uno_b200.train --model "${MODEL}" --data "${DATA}" --output-dir "${OUTPUT_DIR}" --fsdp
       --seq-len "${SEQ_LEN}" --global-batch "${GLOBAL_BATCH}" --micro-batch "${MICRO_BATCH}"
       --lora-rank "${LORA_RANK}" --lora-target "${LORA_TARGET}" --lr "${LR}" --warmup-steps "${WARMUP_STEPS}"
       --tv-weight "${TV_WEIGHT}" --kl-weight "${KL_WEIGHT}" --ce-weight "${CE_WEIGHT}" --ce-target "${CE_TARGET}"
       --checkpoint-layers --run-name "${RUN_NAME}" --wandb-mode "${WANDB_MODE}" --wandb-project "${WANDB_PROJECT}")
  [[ -n "${CURRICULUM}" ]] && cmd+=(--curriculum "${CURRICULUM}")
  [[ -n "${LORA_ALPHA:-}" ]] && cmd+=(--lora-alpha "${LORA_ALPHA}")
  [[ -n "${RESUME:-}" ]] && cmd+=(--resume "${RESUME}")
  printf 'node %s:' "${SLURM_PROCID}"; printf ' %q' "${cmd[@]}"; printf '\n'
  cd "${REPO_ROOT}"
  launch "${cmd[@]}"
fi

mkdir -p "${LOG_DIR}" "${OUTPUT_DIR}"
if [[ -n "${SLURM_JOB_ID:-}" ]]; then
  # already inside an allocation: start one worker task per node
  export MASTER_ADDR="${MASTER_ADDR:-$(scontrol show hostnames "${SLURM_JOB_NODELIST}" | head -n 1)}"
  export MASTER_PORT="${MASTER_PORT:-$((20000 + SLURM_JOB_ID % 20000))}"
  UNO_NODE_WORKER=1 launch srun --nodes="${NODES}" --ntasks-per-node=1 --cpus-per-task="${CPUS_PER_TASK}" \
    --kill-on-bad-exit=1 bash "${BASH_SOURCE[0]}"
fi
launch sbatch --job-name="${RUN_NAME}" --nodes="${NODES}" --ntasks-per-node=1 --gpus-per-node="${GPUS_PER_NODE}" \
  --cpus-per-task="${CPUS_PER_TASK}" --time="${TIME_LIMIT}" --output="${LOG_DIR}/%x-%j.out" \
  --export=ALL "${BASH_SOURCE[0]}"
