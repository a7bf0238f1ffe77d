#!/usr/bin/env bash
# Uno Qwen3-8B on the evaluation protocol: prepare the pinned data once
# (SOURCE_DIR = a protocol bundle), then generate and grade each benchmark
# with DP replicas (one per GPU).
#
#   bash examples/uno_qwen3_8B/run_eval.sh gsm8k [run.py flags...]   one benchmark
#   BENCHMARKS="gsm8k math500" bash examples/uno_qwen3_8B/run_eval.sh   several
# RESULTS_ROOT, DATA_PARALLEL_SIZE (or DP) and UNO_EVAL_DATA_DIR as in the reference recipes.
set -euo pipefail
cd "$(dirname "${BASH_SOURCE[0]}")/../.."
if [[ $# -gt 0 && "$1" != -* ]]; then BENCHMARKS="$1"; shift; fi
# Default: the published bundle s-sahoo/uno-qwen3-8B (pinned revision, adapter in its
# "adapter" subfolder).  With MODEL set, pass the adapter options yourself.
pinned=()
if [[ -z "${MODEL:-}" ]]; then
  MODEL="s-sahoo/uno-qwen3-8B"
  pinned=(--model-revision "${MODEL_REVISION:-b8a7577b3223bdcf2b3af0f2fc6e95258b3bbc29}"
          --gated-lora-subfolder "${GATED_LORA_SUBFOLDER:-adapter}")
fi
OUT="${OUT:-${RESULTS_ROOT:-eval_runs}/${RUN_NAME:-$(date -u +%Y%m%dT%H%M%SZ)}}"
BENCHMARKS=(${BENCHMARKS:-gsm8k math500 aime25 gpqa_diamond humaneval mbpp ifeval})
run() {  # DRY_RUN=1 prints each command instead of running it
  if [[ "${DRY_RUN:-0}" == "1" ]]; then printf '%q ' "$@"; printf '\n'; else "$@"; fi
}
[[ "${DRY_RUN:-0}" == "1" ]] || mkdir -p "${OUT}"
run python -m uno_b200.eval.prepare "${BENCHMARKS[@]}" ${SOURCE_DIR:+--source-dir "${SOURCE_DIR}"}
for b in "${BENCHMARKS[@]}"; do
  run python -m uno_b200.eval.run --benchmark "${b}" --model "${MODEL}" \
    --data-parallel-size "${DATA_PARALLEL_SIZE:-${DP:-8}}" --diffusion-block-size "${BLOCK:-8}" \
    --output "${OUT}/${b}.jsonl" --summary-output "${OUT}/${b}.summary.json" ${pinned[@]+"${pinned[@]}"} "$@"
done
