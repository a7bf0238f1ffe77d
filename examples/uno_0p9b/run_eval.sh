#!/usr/bin/env bash
# 0.9B-class Uno model on the evaluation protocol with DP replicas.
set -euo pipefail
cd "$(dirname "${BASH_SOURCE[0]}")/../.."
MODEL="${MODEL:?set MODEL}" BLOCK="${BLOCK:-16}" exec bash examples/uno_qwen3_8b/run_eval.sh "$@"
