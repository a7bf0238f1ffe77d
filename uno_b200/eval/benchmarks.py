"""Canonical evaluation protocol: the 13 benchmarks and their pinned settings.

The table restates ``evaluation/benchmarks.py:23-198`` of the reference (the
"K2V3 Eval Protocol"): rows, samples per question, completion budget,
context length, answer parser, grader timeout, the pinned dataset file and
its sha256, and the LLM judge where one is used.  Sampling is top-p 0.95 at
temperature 1.0 (0.6 for GPQA-diamond), chat templates render with
``reasoning_effort="high"``.  Datasets are read from ``UNO_EVAL_DATA_DIR``
(default ``~/.cache/uno-b200/benchmarks``) as ``{name}.jsonl``.
"""

from __future__ import annotations

import os
from dataclasses import dataclass, field
from pathlib import Path

DEFAULT_DATA_ROOT = Path(os.environ.get(
    "UNO_EVAL_DATA_DIR", Path(os.environ.get("XDG_CACHE_HOME", Path.home() / ".cache")) / "uno-b200" / "benchmarks"))
PROTOCOL_NAME = "K2V3 Eval Protocol"
PROTOCOL_DATE = "2026-09-01"


@dataclass(frozen=True)
class BenchmarkConfig:
    name: str
    task: str
    expected_rows: int
    data_path: Path
    num_samples: int = 1
    temperature: float = 1.0
    top_p: float = 0.95
    max_tokens: int = 131_072
    max_model_len: int = 262_144
    top_k: int | None = None
    max_num_seqs: int = 4
    instruction: str = ""
    parser: str = "passthrough"
    chat_template_kwargs: dict = field(default_factory=lambda: {"reasoning_effort": "high"})
    grader_timeout: float = 10.0
    source_filename: str | None = None
    data_sha256: str | None = None
    judge: str | None = None


def _b(name, *, rows, samples, max_tokens, context, task=None, temperature=1.0, parser="passthrough",
       max_num_seqs=4, source, sha256, judge=None) -> BenchmarkConfig:
    return BenchmarkConfig(name=name, task=task or name, expected_rows=rows, data_path=DEFAULT_DATA_ROOT / f"{name}.jsonl",
                           num_samples=samples, temperature=temperature, max_tokens=max_tokens,
                           max_model_len=context, max_num_seqs=max_num_seqs, parser=parser, source_filename=source,
                           data_sha256=sha256, judge=judge)


BENCHMARKS: dict[str, BenchmarkConfig] = {b.name: b for b in (
    _b("aime24", rows=30, samples=10, max_tokens=500_000, context=500_000, source="aime-2024/aime-2024.jsonl",
       sha256="266dcb058c1983ff3c7520a74c32962a7cb5ee2386c9f274aa9406e9909af9e5"),
    _b("aime25", rows=30, samples=32, max_tokens=500_000, context=500_000, source="aime-2025/aime-2025.jsonl",
       sha256="25673735af85a06ec49de6c74a412819ad1e4f6b2deef2e50004dc78d15a09aa"),
    _b("aime26", rows=30, samples=32, max_tokens=500_000, context=500_000, source="aime-2026/aime-2026.jsonl",
       sha256="476869564d174db87072caad1bcf4bb3b2d3baf811c1352a4887d5e1b0f1709c"),
    _b("arc_challenge", rows=1172, samples=1, max_tokens=131_072, context=262_144, parser="mc_answer",
       source="arc-challenge/arc_challenge.jsonl",
       sha256="11199fe212915b7bfd3fc166c9452f2006d974300d2432c141f63a99b4f9fec1"),
    _b("gpqa_diamond", rows=198, samples=5, temperature=0.6, max_tokens=262_144, context=262_144,
       parser="mc_answer", source="gpqa-diamond/gpqa_diamond.jsonl",
       sha256="66f387c172aabe10089de0d97dbe1d120fff4b55ab371746a633ca37ef088f59"),
    _b("gsm8k", rows=1319, samples=2, max_tokens=131_072, context=262_144,
       source="gsm8k_cot_zeroshot/gsm8k_cot_zeroshot.jsonl",
       sha256="94d4be9a732880b5518d1c1ab5385cf2e9f1375653ce2561ba02d539c1065c51"),
    _b("hle", rows=2158, samples=1, max_tokens=262_144, context=262_144, source="hle/hle.jsonl",
       sha256="58b8356aff4324d808a9001dfa6e89f2c93b70d3c949ee1be55bafbd7aabd2ec", judge="gpt-5.5-no-tools-medium"),
    _b("humaneval", rows=164, samples=2, max_tokens=131_072, context=262_144, parser="code_completion",
       source="humaneval/humaneval.jsonl",
       sha256="2910cac0699d8179df4e357ce017b6cd7a6c6653f22e55c5da7512f49f4fd595"),
    _b("ifeval", rows=541, samples=1, max_tokens=500_000, context=500_000, max_num_seqs=64,
       source="ifeval/ifeval.jsonl", sha256="b58c072afb150ba249ccb36577001d52f8f872ce06c4b3877e01d35e730db03f"),
    _b("lcr", task="aa_lcr", rows=100, samples=1, max_tokens=32_768, context=262_144, source="lcr/lcr.jsonl",
       sha256="3a7271a1dc30cd65c06b6bb2bde18172f15f72f45d15ce7d173fbd47f121ef2d", judge="GLM-5.2-FP8"),
    _b("math500", rows=500, samples=2, max_tokens=131_072, context=262_144, source="math500/math500.jsonl",
       sha256="e9db693a52216152e9a18ca70110d393fcaa5dd04178693008dbfd20f1a233c8"),
    _b("mbpp", rows=500, samples=2, max_tokens=131_072, context=262_144, source="mbpp_zeroshot/mbpp_zeroshot.jsonl",
       sha256="3b14ca75991841aba4b9276333e2303c6edb28fe2447c6597682044fb392671e"),
    _b("omniscience", task="aa_omniscience", rows=600, samples=1, max_tokens=131_072, context=262_144,
       source="omniscience/omniscience.jsonl",
       sha256="e654f02c2981e3f0e0ba1290fb00f1ba4cd2a0d086bb1213307d3a2f5ef6b5ac", judge="GLM-5.2-FP8"),
)}

ALIASES = {"aime-24": "aime24", "aime-25": "aime25", "aime-26": "aime26", "arc": "arc_challenge",
           "arc-c": "arc_challenge", "arc-challenge": "arc_challenge", "gpqa-diamond": "gpqa_diamond",
           "human-eval": "humaneval", "aa-lcr": "lcr", "aa_lcr": "lcr", "aa-omniscience": "omniscience",
           "aa_omniscience": "omniscience"}


def normalize_benchmark_name(name: str) -> str:
    n = name.strip().lower().replace(" ", "_")
    return ALIASES.get(n, n)


def get_benchmark(name: str) -> BenchmarkConfig:
    n = normalize_benchmark_name(name)
    if n not in BENCHMARKS:
        raise KeyError(f"Unknown benchmark {name!r}. Available: {', '.join(BENCHMARKS)}")
    return BENCHMARKS[n]


def list_benchmarks() -> tuple[str, ...]:
    return tuple(BENCHMARKS)
