#!/usr/bin/env bash
# Uno Qwen3-8B on the evaluation protocol: prepare the pinned data once
# (SOURCE_DIR = a protocol bundle), then generate and grade each benchmark
# with DP replicas (one per GPU).
set -euo pipefail
cd "$(dirname "${BASH_SOURCE[0]}")/../.."
MODEL="${MODEL:?set MODEL to the Uno Qwen3-8B checkpoint directory or hub id}"
OUT="${OUT:-${RESULTS_ROOT:-eval_runs}/${RUN_NAME:-$(date -u +%Y%m%dT%H%M%SZ)}}"
BENCHMARKS=(${BENCHMARKS:-gsm8k math500 aime25 gpqa_diamond humaneval mbpp ifeval})
mkdir -p "${OUT}"
python -m uno_b200.eval.prepare "${BENCHMARKS[@]}" ${SOURCE_DIR:+--source-dir "${SOURCE_DIR}"}
for b in "${BENCHMARKS[@]}"; do
  python -m uno_b200.eval.run --benchmark "${b}" --model "${MODEL}" \
    --data-parallel-size "${DP:-8}" --diffusion-block-size "${BLOCK:-8}" \
    --output "${OUT}/${b}.jsonl" --summary-output "${OUT}/${b}.summary.json" "$@"
done
