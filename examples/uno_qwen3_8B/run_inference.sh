#!/usr/bin/env bash
# Uno Qwen3-8B: one Psi-Spec generation on one node.  TP shards the model over
# TP GPUs (one process per GPU, fused NVLink collectives); DP starts that many
# independent replicas.  SAMPLER=tree verifies a 64-node draft tree per cycle.
set -euo pipefail
cd "$(dirname "${BASH_SOURCE[0]}")/../.."
args=()
if [[ -z "${MODEL:-}" ]]; then  # the published bundle, adapter in its "adapter" subfolder
  MODEL="s-sahoo/uno-qwen3-8B"
  args+=(--model-revision "${MODEL_REVISION:-b8a7577b3223bdcf2b3af0f2fc6e95258b3bbc29}"
         --gated-lora-subfolder "${GATED_LORA_SUBFOLDER:-adapter}")
fi
args+=(--model "${MODEL}" --tensor-parallel-size "${TP:-1}" --data-parallel-size "${DP:-1}"
      --diffusion-block-size "${BLOCK:-8}" --temperature "${TEMPERATURE:-1.0}" --max-tokens "${MAX_TOKENS:-2048}"
      --prompt "${PROMPT:-Explain speculative decoding in one paragraph.}")
[[ -n "${LORA:-}" ]] && args+=(--gated-lora-path "${LORA}")
[[ "${SAMPLER:-linear}" == "tree" ]] && args+=(--tree-verify-size 64 --tree-candidate-top-k 4)
exec python -m uno_b200.inference "${args[@]}" "$@"
