"""Prompt rendering and timed generation shared by the inference and evaluation CLIs.

Interface of the reference's top-level ``generation.py:13-124`` (same function
names, arguments and metric keys):

* :func:`resolve_model_sources` -- a model bundle whose gated-LoRA adapter
  lives in a subfolder resolves to ``(model_dir, adapter_dir)``;
* :func:`format_chat_prompt` -- chat messages rendered with the tokenizer's
  chat template, as text and as token ids, with an optional instruction
  merged into the system message;
* :func:`generate` -- builds an :class:`~uno_b200.LLM`, generates, and reports
  TPS (output tokens per wall-clock second) and TPF (accepted tokens per
  sequence forward).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from pathlib import Path
from time import perf_counter
from typing import Any

from uno_b200.sampling_params import SamplingParams
from uno_b200.utils.hub import resolve_hf_snapshot


def resolve_model_sources(model: str, gated_lora_path: str | None, *, model_revision: str | None = None,
                          gated_lora_subfolder: str | None = None, hf_cache_dir: str | None = None,
                          hf_local_files_only: bool = False) -> tuple[str, str | None]:
    """``(model, adapter)`` to load: unchanged, or the bundle snapshot and its adapter subfolder."""
    if gated_lora_subfolder is not None and gated_lora_path is not None:
        raise ValueError("An adapter can come from --gated-lora-path or from --gated-lora-subfolder; "
                         "pass only one of them (got both)")
    if gated_lora_subfolder is None:
        return model, gated_lora_path
    bundle = Path(resolve_hf_snapshot(model, revision=model_revision, cache_dir=hf_cache_dir,
                                      local_files_only=hf_local_files_only, artifact_name="model bundle"))
    adapter = bundle / gated_lora_subfolder
    if not adapter.joinpath("adapter_config.json").is_file():
        raise ValueError(f"Adapter subfolder {adapter} is invalid: it has no adapter_config.json")
    return str(bundle), str(adapter)


def _with_instruction(messages: list[dict[str, Any]], instruction: str) -> list[dict[str, Any]]:
    """Copy of ``messages`` whose system message starts with ``instruction``.

    No system message: one is prepended.  A system message that already
    contains the instruction is left alone; otherwise the instruction goes
    first, separated from the existing text by a blank line."""
    out = [dict(m) for m in messages]
    if not instruction:
        return out
    for msg in out:
        if msg["role"] != "system":
            continue
        body = msg["content"]
        if instruction not in body:
            rest = body.strip()
            msg["content"] = instruction if not rest else instruction + "\n\n" + rest
        return out
    return [{"role": "system", "content": instruction}] + out


def format_chat_prompt(tokenizer: Any, messages: list[dict[str, Any]], instruction: str = "",
                       chat_template_kwargs: dict[str, Any] | None = None
                       ) -> tuple[list[int], str, list[dict[str, Any]]]:
    """``(token_ids, text, messages)`` of the rendered conversation, ready for generation."""
    if getattr(tokenizer, "chat_template", None) is None:
        raise ValueError("Cannot render chat messages: the tokenizer has no chat_template")
    final = _with_instruction(messages, instruction.strip())
    render = dict(add_generation_prompt=True, **(chat_template_kwargs or {}))
    text = tokenizer.apply_chat_template(final, tokenize=False, **render)
    token_ids = tokenizer.apply_chat_template(final, tokenize=True, return_dict=False, **render)
    return list(token_ids), text, final


@dataclass
class GenerationReport:
    """Throughput of one ``generate`` call."""

    output_tokens: int
    seconds: float
    decoder_stats: dict[str, int] = field(default_factory=dict)

    @property
    def tps(self) -> float:
        return self.output_tokens / self.seconds if self.seconds else 0.0

    @property
    def tpf(self) -> float:
        forwards = int(self.decoder_stats.get("forwards", 0))
        return int(self.decoder_stats.get("accepts", 0)) / forwards if forwards else 0.0

    def as_metrics(self) -> dict[str, Any]:
        return {"total_output_tokens": self.output_tokens, "elapsed_seconds": self.seconds,
                "output_tokens_per_second": self.tps, "decoder_stats": dict(self.decoder_stats),
                "decoder_tokens_per_sequence_forward": self.tpf}


def generation_metrics(outputs: list[dict[str, Any]], stats: dict[str, Any], elapsed: float) -> dict[str, Any]:
    return GenerationReport(sum(len(o["token_ids"]) for o in outputs), elapsed, dict(stats)).as_metrics()


def generate(prompts: list[list[int]], sampling_params: SamplingParams, *, model: Any,
             tokenizer_path: str | None = None, request_max_tokens: list[int] | None = None,
             use_tqdm: bool = True, **engine_kwargs: Any) -> tuple[list[dict[str, Any]], dict[str, Any]]:
    """Generate tokenized prompts on a fresh engine; return the outputs and throughput metrics.

    The clock covers ``LLM.generate`` only (engine construction and shutdown excluded)."""
    from uno_b200.llm import LLM

    llm = LLM(model, tokenizer_path=tokenizer_path, **engine_kwargs)
    try:
        t0 = perf_counter()
        outputs = llm.generate(prompts, sampling_params, request_max_tokens=request_max_tokens, use_tqdm=use_tqdm)
        seconds = perf_counter() - t0
        stats = dict(getattr(llm, "last_generate_stats", {}) or {})
    finally:
        llm.exit()
    return outputs, generation_metrics(outputs, stats, seconds)
