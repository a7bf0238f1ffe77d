#!/usr/bin/env bash
# Evaluation suite on this machine: each benchmark in turn through a model
# recipe (examples/$MODEL_EXAMPLE/run_eval.sh), collecting the ones that fail.
#   BENCHMARKS="gsm8k math500"  subset (default: every registered benchmark)
#   MODEL_EXAMPLE=uno_qwen3_8B  recipe directory under examples/
#   DRY_RUN=1                   print the commands, run nothing
set -uo pipefail
REPO_ROOT="${UNO_REPO_ROOT:-$(cd "$(dirname "${BASH_SOURCE[0]}")/../.." && pwd)}"
PYTHON_BIN="${PYTHON_BIN:-python}"
MODEL_EXAMPLE="${MODEL_EXAMPLE:-uno_qwen3_8B}"
RECIPE="${REPO_ROOT}/examples/${MODEL_EXAMPLE}/run_eval.sh"
if [[ ! -f "${RECIPE}" ]]; then
  echo "no evaluation recipe at ${RECIPE} (MODEL_EXAMPLE is one of: $(ls "${REPO_ROOT}/examples" | tr '\n' ' '))" >&2
  exit 127
fi
if [[ -n "${BENCHMARKS:-}" ]]; then
  read -r -a suite <<< "${BENCHMARKS}"
else
  read -r -a suite <<< "$(cd "${REPO_ROOT}" && "${PYTHON_BIN}" -c \
    'from uno_b200.eval.benchmarks import list_benchmarks; print(" ".join(list_benchmarks()))')"
fi
failed=()
for bench in "${suite[@]}"; do
  cmd=(env "BENCHMARKS=${bench}" bash "${RECIPE}")
  printf 'run:'; printf ' %q' "${cmd[@]}"; printf '\n'
  [[ "${DRY_RUN:-0}" == "1" ]] && continue
  "${cmd[@]}" || failed+=("${bench}")
done
if (( ${#failed[@]} )); then
  echo "failed: ${failed[*]}" >&2
  exit 1
fi
