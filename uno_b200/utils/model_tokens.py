"""Resolve the diffusion mask id and the stop ids of a model.

Rules of ``nano_vllm_uno/utils/model_tokens.py:61-160``:

* mask id: explicit argument, else ``mask_token_id`` of the model config, else
  the tokenizer's ``mask_token_id``, else the ``<|MASK|>`` token; for K2/XLLM
  checkpoints with uniform noise the id one past the vocabulary is allowed;
* stop ids: explicit list, else the union (in order, de-duplicated) of
  ``generation_config.json``'s ``eos_token_id``, the config's and the
  tokenizer's EOS;
* every id is checked against the vocabulary (uniform noise may use
  ``vocab_size`` itself as the mask id).
"""

from __future__ import annotations

import json
import os
from collections.abc import Iterable
from typing import Any

from uno_b200.utils.hf_compat import NATIVE_K2_MODEL_TYPES, ModelConfig, load_model_config


def _ids(value: Any) -> list[int]:
    if value is None:
        return []
    if isinstance(value, int):
        return [value]
    if isinstance(value, Iterable) and not isinstance(value, (str, bytes, dict)):
        return [int(v) for v in value if v is not None]
    return [int(value)]


def _unique(values: Iterable[int]) -> list[int]:
    out: list[int] = []
    for v in values:
        if int(v) not in out:
            out.append(int(v))
    return out


def _generation_config(path: str | None) -> dict[str, Any]:
    if not path:
        return {}
    f = os.path.join(path, "generation_config.json")
    if not os.path.isfile(f):
        return {}
    with open(f, encoding="utf-8") as fh:
        data = json.load(fh)
    return data if isinstance(data, dict) else {}


def resolve_model_token_ids(model: str | ModelConfig, tokenizer: Any, *, mask_token_id: int | None = None,
                            stop_token_ids: list[int] | None = None,
                            noise_mode: str = "mask") -> tuple[int, list[int], int]:
    """Return ``(mask_id, stop_ids, vocab_size)``."""
    path = None
    if isinstance(model, ModelConfig):
        cfg = model
    elif isinstance(model, str) and model.startswith("preset:"):
        from uno_b200.models.presets import resolve_preset

        cfg = resolve_preset(model[len("preset:"):])
    else:
        path = os.path.abspath(os.path.expanduser(str(model)))
        cfg = load_model_config(path)
    vocab = int(cfg.vocab_size)

    mask = mask_token_id
    if mask is None:
        mask = cfg.mask_token_id
    if mask is None:
        mask = getattr(tokenizer, "mask_token_id", None)
    if mask is None and hasattr(tokenizer, "convert_tokens_to_ids"):
        cand = tokenizer.convert_tokens_to_ids("<|MASK|>")
        if cand is not None and cand != getattr(tokenizer, "unk_token_id", None):
            mask = cand
    uniform = noise_mode in {"random_uniform", "deterministic_uniform"}
    if mask is None and uniform and cfg.model_type in NATIVE_K2_MODEL_TYPES:
        mask = vocab
    if mask is None:
        raise ValueError("Could not resolve the diffusion mask token. Set --mask-token-id or add "
                         "mask_token_id to the model config.")
    mask = int(mask)

    if stop_token_ids is None:
        stops = _unique([*_ids(_generation_config(path).get("eos_token_id")), *_ids(cfg.eos_token_id),
                         *_ids(getattr(tokenizer, "eos_token_id", None))])
    else:
        stops = _unique(stop_token_ids)

    bad = [] if 0 <= mask < (vocab + 1 if uniform else vocab) else [mask]
    bad += [t for t in stops if not 0 <= t < vocab]
    if bad:
        raise ValueError(f"Token IDs {bad} are outside model vocabulary [0, {vocab}). "
                         "Do not reuse token IDs from a different checkpoint family.")
    return mask, stops, vocab
