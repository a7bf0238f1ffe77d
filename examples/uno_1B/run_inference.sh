#!/usr/bin/env bash
# 0.9B-class Uno model (K2-Horizon-0.9B with its published Uno adapter by
# default; any 16-layer, hidden-2048 Llama-style checkpoint via MODEL):
# high-concurrency serving with one data-parallel replica per GPU, block 16.
# The published model's mask token is 64256 and it stops on 64019 or 1.
set -euo pipefail
cd "$(dirname "${BASH_SOURCE[0]}")/../.."
args=(--model "${MODEL:-IFM/K2-Horizon-0.9B}" --model-revision "${MODEL_REVISION:-ee770e713760cf6350e4322cdbbff91a163b7d70}"
      --gated-lora-path "${GATED_LORA_PATH:-IFM/K2-Horizon-0.9B-Uno}"
      --gated-lora-revision "${GATED_LORA_REVISION:-b0d8896a301a2f4bc755538b1234a35100da50d0}"
      --mask-token-id "${MASK_TOKEN_ID:-64256}" --stop-token-ids "${STOP_TOKEN_IDS:-64019,1}"
      --max-model-len "${MAX_MODEL_LEN:-131072}" --max-num-batched-tokens "${MAX_NUM_BATCHED_TOKENS:-131072}"
      --data-parallel-size "${DP:-8}" --diffusion-block-size "${BLOCK:-16}" --max-num-seqs "${MAX_NUM_SEQS:-256}"
      --max-tokens "${MAX_TOKENS:-1024}" --prompt "${PROMPT:-Write a haiku about GPUs.}")
exec python -m uno_b200.inference "${args[@]}" "$@"
