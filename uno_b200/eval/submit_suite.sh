#!/usr/bin/env bash
# Submits the evaluation suite to Slurm, one single-node job per benchmark
# (uno_b200/eval/run_slurm.sh).  Environment: BENCHMARKS, MODEL_EXAMPLE,
# RESULTS_ROOT, RUN_NAME, LOG_DIR, SLURM_TIME, SLURM_CPUS_PER_JOB,
# SBATCH_ARGS (extra sbatch flags), DRY_RUN=1 (print the sbatch commands only).
set -euo pipefail
REPO_ROOT="${UNO_REPO_ROOT:-$(cd "$(dirname "${BASH_SOURCE[0]}")/../.." && pwd)}"
PYTHON_BIN="${PYTHON_BIN:-python}"
MODEL_EXAMPLE="${MODEL_EXAMPLE:-uno_qwen3_8B}"
RUN_NAME="${RUN_NAME:-suite}"
RESULTS_ROOT="${RESULTS_ROOT:-${REPO_ROOT}/results/${MODEL_EXAMPLE}}"
LOG_DIR="${LOG_DIR:-${RESULTS_ROOT}/${RUN_NAME}/slurm}"
read -r -a extra <<< "${SBATCH_ARGS:-}"
if [[ -n "${BENCHMARKS:-}" ]]; then
  read -r -a suite <<< "${BENCHMARKS}"
else
  read -r -a suite <<< "$(cd "${REPO_ROOT}" && "${PYTHON_BIN}" -c \
    'from uno_b200.eval.benchmarks import list_benchmarks; print(" ".join(list_benchmarks()))')"
fi
[[ "${DRY_RUN:-0}" == "1" ]] || mkdir -p "${LOG_DIR}"
export MODEL_EXAMPLE RUN_NAME RESULTS_ROOT UNO_REPO_ROOT="${REPO_ROOT}"
for bench in "${suite[@]}"; do
  cmd=(sbatch --parsable --job-name="uno-eval-${bench}" --time="${SLURM_TIME:-2-00:00:00}"
       --cpus-per-task="${SLURM_CPUS_PER_JOB:-64}" --output="${LOG_DIR}/%x-%j.out" --error="${LOG_DIR}/%x-%j.err"
       ${extra[@]+"${extra[@]}"} "${REPO_ROOT}/uno_b200/eval/run_slurm.sh" "${bench}")
  printf 'submit:'; printf ' %q' "${cmd[@]}"; printf '\n'
  [[ "${DRY_RUN:-0}" == "1" ]] && continue
  echo "${bench}: $("${cmd[@]}")"
done
