#!/usr/bin/env bash
# K2-Horizon-7B + Uno adapter on the evaluation protocol, through the generic
# recipe (DP replicas, pinned data).  Judge-graded benchmarks (hle, lcr,
# omniscience) read the judge endpoint from UNO_JUDGE_BASE_URL / UNO_JUDGE_API_KEY.
set -euo pipefail
cd "$(dirname "${BASH_SOURCE[0]}")/../.."
if [[ $# -gt 0 && "$1" != -* ]]; then export BENCHMARKS="$1"; shift; fi  # run_eval.sh BENCHMARK [flags]
MODEL="${MODEL:-IFM/K2-Horizon-7B}" exec bash examples/uno_qwen3_8B/run_eval.sh \
  --model-revision "${MODEL_REVISION:-586b03f0fd1fbbf2f13eeafc33749e95ae34dd10}" \
  --gated-lora-path "${GATED_LORA_PATH:-IFM/K2-Horizon-7B-Uno}" \
  --gated-lora-revision "${GATED_LORA_REVISION:-ec92bbd768f4a404319625204544782e3377bcd7}" \
  --mask-token-id "${MASK_TOKEN_ID:-250624}" --stop-token-ids "${STOP_TOKEN_IDS:-250019,1}" "$@"
