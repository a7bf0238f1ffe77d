"""Model-config and tokenizer loading without remote code.

The reference resolves configs through ``transformers.AutoConfig`` with
``trust_remote_code`` and special-cases K2/XLLM checkpoints whose modelling code
is not importable (``nano_vllm_uno/utils/hf_compat.py:17-86``).  Here every
checkpoint's ``config.json`` is parsed into one plain ``ModelConfig`` object that
carries exactly the fields the two supported architectures read, so no remote
code ever runs and the synthetic (random-init) presets use the same type.
"""

from __future__ import annotations

import json
import os
from dataclasses import asdict, dataclass, field
from typing import Any

QWEN3_TYPES = {"qwen3", "sdar"}
LLAMA_TYPES = {"xllm", "k2_aurora", "k2_horizon", "llama"}
NATIVE_K2_MODEL_TYPES = {"xllm", "k2_aurora", "k2_horizon"}


@dataclass
class ModelConfig:
    model_type: str = "qwen3"
    vocab_size: int = 151936
    hidden_size: int = 4096
    intermediate_size: int = 12288
    num_hidden_layers: int = 36
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    head_dim: int | None = None
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    rope_scaling: dict | None = None
    max_position_embeddings: int = 40960
    tie_word_embeddings: bool = False
    attention_bias: bool = False
    # Qwen3 applies per-head RMSNorm to q and k whenever attention_bias is off;
    # Llama-style checkpoints opt in through ``query_key_norm``.
    query_key_norm: bool | None = None
    layernorm_num_groups: int = 1
    hidden_act: str = "silu"
    torch_dtype: str = "bfloat16"
    eos_token_id: int | list[int] | None = None
    pad_token_id: int | None = None
    bos_token_id: int | None = None
    mask_token_id: int | None = None
    num_experts: int = 0
    extra: dict[str, Any] = field(default_factory=dict)

    def __post_init__(self) -> None:
        self.model_type = str(self.model_type).lower()
        if self.head_dim is None:
            self.head_dim = self.hidden_size // self.num_attention_heads
        if self.query_key_norm is None:
            self.query_key_norm = (
                not self.attention_bias if self.model_type in QWEN3_TYPES else False
            )

    @property
    def family(self) -> str:
        if self.model_type in QWEN3_TYPES:
            return "qwen3"
        if self.model_type in LLAMA_TYPES:
            return "llama"
        raise ValueError(
            f"Unsupported model_type={self.model_type!r}. Supported: "
            f"{sorted(QWEN3_TYPES | LLAMA_TYPES)}"
        )

    @property
    def dtype_name(self) -> str:
        return str(self.torch_dtype).removeprefix("torch.")

    def to_dict(self) -> dict[str, Any]:
        data = asdict(self)
        extra = data.pop("extra")
        data.update(extra)
        return data

    def num_params(self) -> int:
        h, i, v = self.hidden_size, self.intermediate_size, self.vocab_size
        q = self.num_attention_heads * self.head_dim
        kv = self.num_key_value_heads * self.head_dim
        per_layer = h * (q + 2 * kv) + q * h + 3 * h * i + 2 * h
        emb = v * h * (1 if self.tie_word_embeddings else 2)
        return self.num_hidden_layers * per_layer + emb + h


_KNOWN = set(ModelConfig.__dataclass_fields__) - {"extra"}


def model_config_from_dict(data: dict[str, Any]) -> ModelConfig:
    data = dict(data)
    # Newer transformers store RoPE parameters in ``rope_parameters``.
    rope_parameters = data.get("rope_parameters")
    if isinstance(rope_parameters, dict):
        if data.get("rope_theta") is None and "rope_theta" in rope_parameters:
            data["rope_theta"] = rope_parameters["rope_theta"]
        if data.get("rope_scaling") is None and rope_parameters.get(
            "rope_type", rope_parameters.get("type", "default")
        ) not in (None, "default"):
            data["rope_scaling"] = rope_parameters
    if "dtype" in data and "torch_dtype" not in data:
        data["torch_dtype"] = data["dtype"]
    known = {k: v for k, v in data.items() if k in _KNOWN and v is not None}
    extra = {k: v for k, v in data.items() if k not in _KNOWN}
    cfg = ModelConfig(**known)
    cfg.extra = extra
    return cfg


def load_model_config(path: str) -> ModelConfig:
    with open(os.path.join(path, "config.json"), "r", encoding="utf-8") as fh:
        return model_config_from_dict(json.load(fh))


def save_model_config(cfg: ModelConfig, path: str) -> None:
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w", encoding="utf-8") as fh:
        json.dump(cfg.to_dict(), fh, indent=2, sort_keys=True)


def is_native_k2_model(path: str) -> bool:
    try:
        return load_model_config(path).model_type in NATIVE_K2_MODEL_TYPES
    except (OSError, ValueError, TypeError):
        return False


class TokenIdTokenizer:
    """Stand-in tokenizer for checkpoints that ship none (synthetic models).

    Prompts must be token-id lists; ``decode`` renders ids as text so that
    ``generate(..., detokenize=True)`` still returns a string.
    """

    chat_template = None

    def __init__(self, vocab_size: int, eos_token_id: int | None = None, pad_token_id: int | None = None):
        self.vocab_size = int(vocab_size)
        self.eos_token_id = eos_token_id
        self.pad_token_id = pad_token_id
        self.mask_token_id = None
        self.unk_token_id = None

    def encode(self, text: str) -> list[int]:
        raise ValueError(
            "This model has no tokenizer; pass prompts as lists of token ids"
        )

    def decode(self, token_ids, skip_special_tokens: bool = False) -> str:
        return " ".join(str(int(t)) for t in token_ids)

    def convert_tokens_to_ids(self, token: str):
        return None


def load_tokenizer(path: str | None, cfg: ModelConfig, **kwargs):
    """HF tokenizer when the directory has one, else :class:`TokenIdTokenizer`."""
    eos = cfg.eos_token_id[0] if isinstance(cfg.eos_token_id, list) else cfg.eos_token_id
    if path and os.path.isdir(path) and any(
        os.path.exists(os.path.join(path, name))
        for name in ("tokenizer.json", "tokenizer_config.json", "tokenizer.model")
    ):
        from transformers import AutoTokenizer

        return AutoTokenizer.from_pretrained(path, **kwargs)
    return TokenIdTokenizer(cfg.vocab_size, eos, cfg.pad_token_id)
