#!/usr/bin/env bash
#SBATCH --nodes=1
#SBATCH --ntasks=1
#SBATCH --gres=gpu:8
#SBATCH --exclusive
# One benchmark of the evaluation suite inside a Slurm allocation: the model
# recipe with data-parallel replicas on the node's GPUs.  Usage (normally via
# submit_suite.sh): sbatch uno_b200/eval/run_slurm.sh BENCHMARK
set -euo pipefail
if [[ $# -ne 1 ]]; then
  echo "usage: $0 BENCHMARK" >&2
  exit 2
fi
REPO_ROOT="${UNO_REPO_ROOT:-${SLURM_SUBMIT_DIR:-$(pwd)}}"
RECIPE="${REPO_ROOT}/examples/${MODEL_EXAMPLE:-uno_qwen3_8B}/run_eval.sh"
[[ -f "${RECIPE}" ]] || { echo "no evaluation recipe at ${RECIPE}" >&2; exit 127; }
export DP="${DP:-${SLURM_GPUS_ON_NODE:-8}}"
BENCHMARKS="$1" exec bash "${RECIPE}"
