#!/usr/bin/env bash
# 0.9B-class Uno model (16 layers, hidden 2048): high-concurrency serving with
# one data-parallel replica per GPU, block size 16.
set -euo pipefail
cd "$(dirname "${BASH_SOURCE[0]}")/../.."
MODEL="${MODEL:?set MODEL to the checkpoint directory or hub id}"
exec python -m uno_b200.inference --model "${MODEL}" --data-parallel-size "${DP:-8}" \
  --diffusion-block-size "${BLOCK:-16}" --max-num-seqs "${MAX_NUM_SEQS:-256}" --max-tokens "${MAX_TOKENS:-1024}" \
  --prompt "${PROMPT:-Write a haiku about GPUs.}" "$@"
