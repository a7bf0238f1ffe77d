#!/usr/bin/env bash
# Submits pull-based evaluation allocations (run_pull_suite_slurm.sh), one per
# benchmark.  Environment: MODEL (required), BENCHMARKS, NODES, GPUS_PER_NODE,
# CPUS_PER_TASK, SLURM_TIME, RESULTS_ROOT, RUN_NAME, SBATCH_ARGS, DRY_RUN=1.
set -euo pipefail
REPO_ROOT="${UNO_REPO_ROOT:-$(cd "$(dirname "${BASH_SOURCE[0]}")/../.." && pwd)}"
PYTHON_BIN="${PYTHON_BIN:-python}"
: "${MODEL:?set MODEL to a checkpoint directory, hub id or preset}"
NODES="${NODES:-1}"
GPUS_PER_NODE="${GPUS_PER_NODE:-8}"
RUN_NAME="${RUN_NAME:-pull}"
RESULTS_ROOT="${RESULTS_ROOT:-${REPO_ROOT}/results/pull}"
read -r -a extra <<< "${SBATCH_ARGS:-}"
if [[ -n "${BENCHMARKS:-}" ]]; then
  read -r -a suite <<< "${BENCHMARKS}"
else
  read -r -a suite <<< "$(cd "${REPO_ROOT}" && "${PYTHON_BIN}" -c \
    'from uno_b200.eval.benchmarks import list_benchmarks; print(" ".join(list_benchmarks()))')"
fi
LOG_DIR="${RESULTS_ROOT}/${RUN_NAME}/slurm-submit"
[[ "${DRY_RUN:-0}" == "1" ]] || mkdir -p "${LOG_DIR}"
for bench in "${suite[@]}"; do
  cmd=(sbatch --parsable --nodes="${NODES}" --ntasks="$((NODES * GPUS_PER_NODE))"
       --ntasks-per-node="${GPUS_PER_NODE}" --gres="gpu:${GPUS_PER_NODE}" --cpus-per-task="${CPUS_PER_TASK:-8}"
       --time="${SLURM_TIME:-2-00:00:00}" --job-name="uno-pull-${bench}" --output="${LOG_DIR}/%x-%j.out"
       --export="ALL,BENCHMARKS=${bench},RUN_NAME=${RUN_NAME}/${bench},RESULTS_ROOT=${RESULTS_ROOT},UNO_REPO_ROOT=${REPO_ROOT}"
       ${extra[@]+"${extra[@]}"} "${REPO_ROOT}/uno_b200/eval/run_pull_suite_slurm.sh")
  printf 'submit:'; printf ' %q' "${cmd[@]}"; printf '\n'
  [[ "${DRY_RUN:-0}" == "1" ]] && continue
  echo "${bench}: $("${cmd[@]}")"
done
