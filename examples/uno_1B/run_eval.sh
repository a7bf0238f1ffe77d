#!/usr/bin/env bash
# 0.9B-class Uno model (K2-Horizon-0.9B + Uno adapter by default) on the
# evaluation protocol, through the generic recipe with DP replicas, block 16.
set -euo pipefail
cd "$(dirname "${BASH_SOURCE[0]}")/../.."
if [[ $# -gt 0 && "$1" != -* ]]; then export BENCHMARKS="$1"; shift; fi  # run_eval.sh BENCHMARK [flags]
MODEL="${MODEL:-IFM/K2-Horizon-0.9B}" BLOCK="${BLOCK:-16}" exec bash examples/uno_qwen3_8B/run_eval.sh \
  --model-revision "${MODEL_REVISION:-ee770e713760cf6350e4322cdbbff91a163b7d70}" \
  --gated-lora-path "${GATED_LORA_PATH:-IFM/K2-Horizon-0.9B-Uno}" \
  --gated-lora-revision "${GATED_LORA_REVISION:-b0d8896a301a2f4bc755538b1234a35100da50d0}" \
  --mask-token-id "${MASK_TOKEN_ID:-64256}" --stop-token-ids "${STOP_TOKEN_IDS:-64019,1}" "$@"
