#!/usr/bin/env bash
# K2-Horizon-7B with its published Uno conditional-LoRA adapter: one Psi-Spec
# generation.  The model's mask token is 250624 and it stops on 250019 or 1.
# No training recipe is published for this model, so there is no run_train.sh.
set -euo pipefail
cd "$(dirname "${BASH_SOURCE[0]}")/../.."
args=(--model "${MODEL:-IFM/K2-Horizon-7B}" --model-revision "${MODEL_REVISION:-586b03f0fd1fbbf2f13eeafc33749e95ae34dd10}"
      --gated-lora-path "${GATED_LORA_PATH:-IFM/K2-Horizon-7B-Uno}"
      --gated-lora-revision "${GATED_LORA_REVISION:-ec92bbd768f4a404319625204544782e3377bcd7}"
      --mask-token-id "${MASK_TOKEN_ID:-250624}" --stop-token-ids "${STOP_TOKEN_IDS:-250019,1}"
      --max-model-len "${MAX_MODEL_LEN:-262144}" --max-num-batched-tokens "${MAX_NUM_BATCHED_TOKENS:-262144}"
      --tensor-parallel-size "${TP:-1}" --diffusion-block-size "${BLOCK:-8}")
exec python -m uno_b200.inference "${args[@]}" "$@"
