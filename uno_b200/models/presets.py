"""Named model architectures used by the benchmarks and tests.

* ``qwen3-8b``: Uno-Qwen3-8B (36 layers, hidden 4096, 32/8 heads, head_dim 128,
  QK-norm, SwiGLU 12288, vocab 151936, RoPE theta 1e6, untied).
* ``uno-0.9b``: the Llama-style 0.9B-class model (16 layers, hidden 2048,
  16/16 heads, head_dim 128, SwiGLU 5632, vocab 151936).
* ``tiny-qwen3``: the 2-layer CPU oracle model (hidden 256, 4/2 heads,
  head_dim 64, SwiGLU 768, vocab 4096).
"""

from __future__ import annotations

import copy

from uno_b200.utils.hf_compat import ModelConfig

_PRESETS = {
    "qwen3-8b": ModelConfig(
        model_type="qwen3",
        vocab_size=151936,
        hidden_size=4096,
        intermediate_size=12288,
        num_hidden_layers=36,
        num_attention_heads=32,
        num_key_value_heads=8,
        head_dim=128,
        rms_norm_eps=1e-6,
        rope_theta=1_000_000.0,
        max_position_embeddings=40960,
        tie_word_embeddings=False,
        eos_token_id=151645,
        pad_token_id=151643,
        mask_token_id=151669,
    ),
    "uno-0.9b": ModelConfig(
        model_type="llama",
        vocab_size=151936,
        hidden_size=2048,
        intermediate_size=5632,
        num_hidden_layers=16,
        num_attention_heads=16,
        num_key_value_heads=16,
        head_dim=128,
        rms_norm_eps=1e-6,
        rope_theta=1_000_000.0,
        max_position_embeddings=32768,
        tie_word_embeddings=False,
        query_key_norm=False,
        eos_token_id=151645,
        pad_token_id=151643,
        mask_token_id=151669,
    ),
    "tiny-qwen3": ModelConfig(
        model_type="qwen3",
        vocab_size=4096,
        hidden_size=256,
        intermediate_size=768,
        num_hidden_layers=2,
        num_attention_heads=4,
        num_key_value_heads=2,
        head_dim=64,
        rms_norm_eps=1e-6,
        rope_theta=1_000_000.0,
        max_position_embeddings=4096,
        tie_word_embeddings=False,
        torch_dtype="float32",
        eos_token_id=None,
        mask_token_id=4095,
    ),
}


def preset_names() -> list[str]:
    return sorted(_PRESETS)


def resolve_preset(name: str) -> ModelConfig:
    try:
        return copy.deepcopy(_PRESETS[name])
    except KeyError:
        raise ValueError(f"unknown preset {name!r}; choose from {preset_names()}") from None
