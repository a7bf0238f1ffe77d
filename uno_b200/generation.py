"""Prompt formatting and timed generation shared by inference and evaluation.

Equivalent of the reference's top-level ``generation.py:13-124``:

* :func:`resolve_model_sources` -- a model bundle whose gated-LoRA adapter
  lives in a subfolder resolves to ``(model_dir, adapter_dir)``;
* :func:`format_chat_prompt` -- renders chat messages with the tokenizer's
  chat template (as text and as token ids), merging an optional instruction
  into the system message;
* :func:`generate` -- builds an :class:`~uno_b200.LLM`, generates, and returns
  the outputs with the throughput metrics: output tokens per second of wall
  time (TPS) and tokens per sequence forward (TPF = accepts / forwards).
"""

from __future__ import annotations

from pathlib import Path
from time import perf_counter
from typing import Any

from uno_b200.sampling_params import SamplingParams
from uno_b200.utils.hub import resolve_hf_snapshot


def resolve_model_sources(model: str, gated_lora_path: str | None, *, model_revision: str | None = None,
                          gated_lora_subfolder: str | None = None, hf_cache_dir: str | None = None,
                          hf_local_files_only: bool = False) -> tuple[str, str | None]:
    """Resolve a model bundle when its adapter lives in a subfolder."""
    if gated_lora_subfolder is None:
        return model, gated_lora_path
    if gated_lora_path is not None:
        raise ValueError("Use either --gated-lora-path or --gated-lora-subfolder, not both")
    model_dir = resolve_hf_snapshot(model, revision=model_revision, cache_dir=hf_cache_dir,
                                    local_files_only=hf_local_files_only, artifact_name="model bundle")
    adapter_dir = Path(model_dir) / gated_lora_subfolder
    if not (adapter_dir / "adapter_config.json").is_file():
        raise ValueError(f"Adapter subfolder is invalid: {adapter_dir}")
    return model_dir, str(adapter_dir)


def format_chat_prompt(tokenizer: Any, messages: list[dict[str, Any]], instruction: str = "",
                       chat_template_kwargs: dict[str, Any] | None = None
                       ) -> tuple[list[int], str, list[dict[str, Any]]]:
    """Render messages once as text and once as token ids."""
    messages = [dict(m) for m in messages]
    instruction = instruction.strip()
    if instruction:
        system = next((m for m in messages if m["role"] == "system"), None)
        if system is None:
            messages.insert(0, {"role": "system", "content": instruction})
        elif instruction not in system["content"]:
            old = system["content"].strip()
            system["content"] = f"{instruction}\n\n{old}" if old else instruction
    if getattr(tokenizer, "chat_template", None) is None:
        raise ValueError("The tokenizer needs a chat_template to render messages")
    kw = dict(chat_template_kwargs or {})
    text = tokenizer.apply_chat_template(messages, tokenize=False, add_generation_prompt=True, **kw)
    ids = tokenizer.apply_chat_template(messages, tokenize=True, add_generation_prompt=True, return_dict=False,
                                        **kw)
    return list(ids), text, messages


def generation_metrics(outputs: list[dict[str, Any]], stats: dict[str, Any], elapsed: float) -> dict[str, Any]:
    total = sum(len(o["token_ids"]) for o in outputs)
    forwards = int(stats.get("forwards", 0))
    return {
        "total_output_tokens": total,
        "elapsed_seconds": elapsed,
        "output_tokens_per_second": total / elapsed if elapsed else 0.0,
        "decoder_stats": dict(stats),
        "decoder_tokens_per_sequence_forward": int(stats.get("accepts", 0)) / forwards if forwards else 0.0,
    }


def generate(prompts: list[list[int]], sampling_params: SamplingParams, *, model: Any,
             tokenizer_path: str | None = None, request_max_tokens: list[int] | None = None,
             use_tqdm: bool = True, **engine_kwargs: Any) -> tuple[list[dict[str, Any]], dict[str, Any]]:
    """Generate tokenized prompts; return the outputs and throughput metrics."""
    from uno_b200.llm import LLM

    llm = LLM(model, tokenizer_path=tokenizer_path, **engine_kwargs)
    start = perf_counter()
    try:
        outputs = llm.generate(prompts, sampling_params, request_max_tokens=request_max_tokens, use_tqdm=use_tqdm)
        elapsed = perf_counter() - start
        stats = dict(getattr(llm, "last_generate_stats", {}))
    finally:
        llm.exit()
    return outputs, generation_metrics(outputs, stats, elapsed)
