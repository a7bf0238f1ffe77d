#!/usr/bin/env bash
# Uno Qwen3-8B on the evaluation protocol: prepare the pinned data once
# (SOURCE_DIR = a protocol bundle), then generate and grade each benchmark
# with DP replicas (one per GPU).
set -euo pipefail
cd "$(dirname "${BASH_SOURCE[0]}")/../.."
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
mkdir -p "${OUT}"
python -m uno_b200.eval.prepare "${BENCHMARKS[@]}" ${SOURCE_DIR:+--source-dir "${SOURCE_DIR}"}
for b in "${BENCHMARKS[@]}"; do
  python -m uno_b200.eval.run --benchmark "${b}" --model "${MODEL}" \
    --data-parallel-size "${DP:-8}" --diffusion-block-size "${BLOCK:-8}" \
    --output "${OUT}/${b}.jsonl" --summary-output "${OUT}/${b}.summary.json" ${pinned[@]+"${pinned[@]}"} "$@"
done
