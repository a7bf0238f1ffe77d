#!/usr/bin/env bash
#SBATCH --exclusive
# Pull-based evaluation inside one Slurm allocation (normally submitted by
# submit_pull_suite.sh, one benchmark per allocation because the canonical
# samples, temperature and budgets differ per benchmark):
#   1. jobs:        expand BENCHMARKS into RUN_DIR/jobs.jsonl + manifest.json;
#   2. coordinator: on this (the first) node, serving the jobs on PORT;
#   3. workers:     one engine per GPU on every node (srun), pulling jobs;
#   4. score:       split the results per benchmark and grade them.
# Required: MODEL.  Optional: BENCHMARKS, DATA_ROOT, NUM_SAMPLES, LIMIT,
# DIFFUSION_BLOCK_SIZE, TEMPERATURE, TOP_P, TOP_K, PROTOCOL_ARM (required for
# any departure from the benchmark's canonical settings), RESULTS_ROOT, RUN_NAME,
# SKIP_GRADING=1, DRY_RUN=1 (print the four commands, run nothing).  The
# reference launcher's NANO_* variables are read as defaults by every role.
set -euo pipefail
REPO_ROOT="${UNO_REPO_ROOT:-${SLURM_SUBMIT_DIR:-$(pwd)}}"
PYTHON_BIN="${PYTHON_BIN:-python}"
: "${MODEL:?set MODEL to a checkpoint directory, hub id or preset}"
JOB="${SLURM_JOB_ID:-0}"
NODES="${SLURM_NNODES:-1}"
WORKERS="${SLURM_NTASKS:-$((NODES * ${GPUS_PER_NODE:-8}))}"
RUN_NAME="${RUN_NAME:-pull-${JOB}}"
RUN_DIR="${RESULTS_ROOT:-${REPO_ROOT}/results/pull}/${RUN_NAME}"
HOST="$(scontrol show hostnames "${SLURM_JOB_NODELIST:-}" 2>/dev/null | head -n 1 || true)"
HOST="${HOST:-$(hostname)}"
PORT="${UNO_SUITE_PORT:-$((20000 + JOB % 20000))}"
export UNO_SUITE_AUTHKEY="${UNO_SUITE_AUTHKEY:-uno-${JOB}-${RANDOM}}"
common=(--manifest "${RUN_DIR}/manifest.json")
jobs_cmd=("${PYTHON_BIN}" -m uno_b200.eval.pull_suite jobs "${common[@]}" --jobs "${RUN_DIR}/jobs.jsonl"
          --model "${MODEL}" --diffusion-block-size "${DIFFUSION_BLOCK_SIZE:-16}")
for b in ${BENCHMARKS:-gsm8k}; do jobs_cmd+=(--benchmark "${b}"); done
[[ -n "${DATA_ROOT:-}" ]] && jobs_cmd+=(--data-root "${DATA_ROOT}")
[[ -n "${NUM_SAMPLES:-}" ]] && jobs_cmd+=(--num-samples "${NUM_SAMPLES}")
[[ -n "${LIMIT:-}" ]] && jobs_cmd+=(--limit "${LIMIT}")
[[ -n "${TEMPERATURE:-}" ]] && jobs_cmd+=(--temperature "${TEMPERATURE}")
[[ -n "${TOP_P:-}" ]] && jobs_cmd+=(--top-p "${TOP_P}")
[[ -n "${TOP_K:-}" ]] && jobs_cmd+=(--top-k "${TOP_K}")
[[ -n "${PROTOCOL_ARM:-}" ]] && jobs_cmd+=(--protocol-arm "${PROTOCOL_ARM}")
coord_cmd=("${PYTHON_BIN}" -m uno_b200.eval.pull_suite coordinator "${common[@]}" --jobs "${RUN_DIR}/jobs.jsonl"
           --output "${RUN_DIR}/results.jsonl" --address "0.0.0.0:${PORT}" --num-workers "${WORKERS}")
worker_cmd=(srun --nodes="${NODES}" --ntasks="${WORKERS}" --ntasks-per-node="$((WORKERS / NODES))"
            --gpus-per-task=1 --kill-on-bad-exit=1 --output="${RUN_DIR}/logs/worker-%t.out"
            "${PYTHON_BIN}" -m uno_b200.eval.pull_suite worker "${common[@]}" --address "${HOST}:${PORT}")
score_cmd=("${PYTHON_BIN}" -m uno_b200.eval.pull_suite score "${common[@]}" --output "${RUN_DIR}/results.jsonl"
           --out-dir "${RUN_DIR}")
for name in jobs_cmd coord_cmd worker_cmd score_cmd; do
  declare -n ref="${name}"
  printf '%s:' "${name%_cmd}"; printf ' %q' "${ref[@]}"; printf '\n'
done
[[ "${DRY_RUN:-0}" == "1" ]] && exit 0
cd "${REPO_ROOT}"
mkdir -p "${RUN_DIR}/logs"
"${jobs_cmd[@]}"
"${coord_cmd[@]}" > "${RUN_DIR}/logs/coordinator.out" 2>&1 &
coord=$!
"${worker_cmd[@]}"
wait "${coord}"
[[ "${SKIP_GRADING:-0}" == "1" ]] && { echo "generation done; grading skipped"; exit 0; }
"${score_cmd[@]}"
