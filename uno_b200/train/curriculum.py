"""Block-size curriculum: YAML stages -> optimizer-step ranges.

Format and rules of ``training/curriculum.py:21-171``: a YAML mapping with
``tokens_per_step`` (= ``sequence_length * global_batch_size``), ``seed``,
optional ``total_tokens`` and ``stages`` (strictly increasing ``block_size``
with a ``tokens`` budget each).  A stage ends at step
``floor(cumulative_tokens / tokens_per_step)``; every stage end is a
checkpoint boundary (``completed_block_size_{B}``); the plan's sha256 (of its
canonical manifest) pins a resume to the same curriculum.
"""

from __future__ import annotations

import bisect
import hashlib
import json
from dataclasses import dataclass
from pathlib import Path
from typing import Any


@dataclass(frozen=True)
class CurriculumStage:
    block_size: int
    token_budget: int
    start_step: int
    end_step: int


def _int(m: dict[str, Any], key: str, positive: bool = True) -> int:
    v = m.get(key)
    if not isinstance(v, int) or isinstance(v, bool):
        raise ValueError(f"{key} must be an integer.")
    if positive and v <= 0:
        raise ValueError(f"{key} must be positive.")
    return v


class BlockCurriculumPlan:
    def __init__(self, *, tokens_per_step: int, sequence_length: int, global_batch_size: int, seed: int,
                 stages: list[CurriculumStage], source_path: Path | None = None) -> None:
        if not stages:
            raise ValueError("Curriculum stages must be a non-empty list.")
        self.source_path = source_path
        self.tokens_per_step = tokens_per_step
        self.sequence_length = sequence_length
        self.global_batch_size = global_batch_size
        self.seed = seed
        self.stages = tuple(stages)
        self._ends = tuple(s.end_step for s in stages)
        self.checkpoint_reasons = {s.end_step: f"completed_block_size_{s.block_size}" for s in stages}

    @classmethod
    def from_mapping(cls, raw: dict[str, Any], source_path: Path | None = None) -> "BlockCurriculumPlan":
        if not isinstance(raw, dict):
            raise ValueError("Curriculum YAML must contain a mapping.")
        if raw.get("replay") not in (None, {}, False):
            raise ValueError("Smaller-block replay is not supported.")
        tps = _int(raw, "tokens_per_step")
        seq = _int(raw, "sequence_length")
        gbs = _int(raw, "global_batch_size")
        seed = _int(raw, "seed", positive=False)
        if tps != seq * gbs:
            raise ValueError("tokens_per_step must equal sequence_length * global_batch_size.")
        items = raw.get("stages")
        if not isinstance(items, list) or not items:
            raise ValueError("Curriculum stages must be a non-empty list.")
        stages, total, prev_end, prev_block = [], 0, 0, 0
        for i, item in enumerate(items):
            if not isinstance(item, dict):
                raise ValueError(f"Curriculum stage {i} must be a mapping.")
            block = _int(item, "block_size")
            budget = _int(item, "tokens")
            if block <= prev_block:
                raise ValueError("Curriculum block sizes must be strictly increasing.")
            total += budget
            end = total // tps
            if end <= prev_end:
                raise ValueError(f"Curriculum stage B={block} is shorter than one step.")
            stages.append(CurriculumStage(block, budget, prev_end, end))
            prev_end, prev_block = end, block
        if raw.get("total_tokens") is not None and raw["total_tokens"] != total:
            raise ValueError("total_tokens does not match the sum of stage token budgets.")
        return cls(tokens_per_step=tps, sequence_length=seq, global_batch_size=gbs, seed=seed, stages=stages,
                   source_path=source_path)

    @classmethod
    def from_yaml(cls, path: str | Path) -> "BlockCurriculumPlan":
        import yaml

        p = Path(path).expanduser().resolve()
        if not p.is_file():
            raise FileNotFoundError(f"Curriculum file not found: {p}")
        return cls.from_mapping(yaml.safe_load(p.read_text()), p)

    @classmethod
    def fixed(cls, block_sizes: list[int], steps_per_stage: int, sequence_length: int, global_batch_size: int,
              seed: int = 0) -> "BlockCurriculumPlan":
        tps = sequence_length * global_batch_size
        return cls.from_mapping({"tokens_per_step": tps, "sequence_length": sequence_length,
                                 "global_batch_size": global_batch_size, "seed": seed,
                                 "stages": [{"block_size": b, "tokens": steps_per_stage * tps} for b in block_sizes]})

    @property
    def max_steps(self) -> int:
        return self.stages[-1].end_step

    @property
    def total_tokens(self) -> int:
        return sum(s.token_budget for s in self.stages)

    def stage_for_step(self, step: int) -> CurriculumStage:
        if not 0 <= step < self.max_steps:
            raise ValueError(f"Optimizer step {step} is outside [0, {self.max_steps}).")
        return self.stages[bisect.bisect_right(self._ends, step)]

    def validate_runtime(self, *, world_size: int, per_device_batch: int, accumulation: int) -> None:
        got = world_size * per_device_batch * accumulation
        if got != self.global_batch_size:
            raise ValueError(f"Curriculum global batch mismatch: runtime={got}, expected={self.global_batch_size}.")

    def manifest(self) -> dict[str, Any]:
        return {"version": 1, "tokens_per_step": self.tokens_per_step, "sequence_length": self.sequence_length,
                "global_batch_size": self.global_batch_size, "seed": self.seed, "total_tokens": self.total_tokens,
                "max_steps": self.max_steps, "replay_smaller_blocks": False,
                "stages": [{"block_size": s.block_size, "token_budget": s.token_budget, "start_step": s.start_step,
                            "end_step": s.end_step} for s in self.stages]}

    def sha256(self) -> str:
        return hashlib.sha256(json.dumps(self.manifest(), sort_keys=True, separators=(",", ":")).encode()).hexdigest()


# The released recipe's data definition: 4,096-token rows, 128 rows per optimizer
# step and 9,375 steps per pass over the corpus (``training/constants.py:14-18``).
RECIPE_SEQUENCE_LENGTH = 4096
RECIPE_GLOBAL_BATCH = 128
RECIPE_STEPS_PER_EPOCH = 9375
RECIPE_SEED = 20260813


def fixed_curriculum(epochs, *, block_size: int = 8, sequence_length: int = RECIPE_SEQUENCE_LENGTH,
                     global_batch_size: int = RECIPE_GLOBAL_BATCH, steps_per_epoch: int = RECIPE_STEPS_PER_EPOCH,
                     seed: int = RECIPE_SEED) -> dict[str, Any]:
    """A one-stage curriculum mapping: ``epochs`` passes at one block size.

    The step count is ``epochs * steps_per_epoch`` rounded half up (at least
    one step), so a fractional epoch count names a whole number of optimizer
    steps; the mapping records both the requested and the resolved epochs.
    Behaviour of ``training/create_fixed_curriculum.py``.
    """
    from decimal import ROUND_HALF_UP, Decimal, InvalidOperation

    try:
        e = Decimal(str(epochs))
    except InvalidOperation as exc:
        raise ValueError(f"epochs must be a number, got {epochs!r}") from exc
    if not e.is_finite() or e <= 0:
        raise ValueError("epochs must be a finite positive number")
    if min(block_size, sequence_length, global_batch_size, steps_per_epoch) <= 0:
        raise ValueError("block size, sequence length, global batch and steps per epoch must be positive")
    steps = max(1, int((e * steps_per_epoch).to_integral_value(rounding=ROUND_HALF_UP)))
    tps = sequence_length * global_batch_size
    return {"version": 1, "requested_epochs": str(e), "resolved_epochs": str(Decimal(steps) / Decimal(steps_per_epoch)),
            "steps_per_epoch": steps_per_epoch, "tokens_per_step": tps, "sequence_length": sequence_length,
            "global_batch_size": global_batch_size, "total_tokens": steps * tps, "seed": seed,
            "stages": [{"block_size": block_size, "tokens": steps * tps}]}


def write_curriculum(path: str | Path, mapping: dict[str, Any]) -> Path:
    """Writes the YAML atomically; an existing file must already hold the same plan."""
    import yaml

    path = Path(path)
    text = yaml.safe_dump(mapping, sort_keys=False)
    if path.exists():
        if path.read_text() != text:
            raise FileExistsError(f"{path} holds a different curriculum; refusing to replace it")
        return path
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_name(path.name + ".tmp")
    tmp.write_text(text)
    tmp.replace(path)
    return path


RELEASED_BLOCK_SIZES = (2, 4, 6, 8, 12, 16)


def released_curriculum(epochs: int = 3, block_sizes=RELEASED_BLOCK_SIZES) -> dict[str, Any]:
    """The block-size schedule of the released Uno Qwen3-8B run as a curriculum mapping.

    ``epochs`` passes over the recipe corpus (9,375 steps each) split into
    ``len(block_sizes)`` stages of equal length in increasing block size: with
    the defaults, six half-epoch stages that alternate 4,688 and 4,687 steps,
    so every adjacent pair is exactly one epoch (28,125 steps, 14.7456 B
    tokens in all).  Stage lengths are the cumulative split points rounded
    half up (``training/configs/uno_3epoch_curriculum.yaml``).
    """
    from decimal import ROUND_HALF_UP, Decimal

    total_steps = int(epochs) * RECIPE_STEPS_PER_EPOCH
    n = len(block_sizes)
    tps = RECIPE_SEQUENCE_LENGTH * RECIPE_GLOBAL_BATCH
    ends = [int((Decimal(total_steps) * (i + 1) / n).to_integral_value(rounding=ROUND_HALF_UP)) for i in range(n)]
    stages, prev = [], 0
    for b, end in zip(block_sizes, ends):
        stages.append({"block_size": int(b), "tokens": (end - prev) * tps})
        prev = end
    return {"version": 1, "tokens_per_step": tps, "sequence_length": RECIPE_SEQUENCE_LENGTH,
            "global_batch_size": RECIPE_GLOBAL_BATCH, "total_tokens": total_steps * tps, "seed": RECIPE_SEED,
            "stages": stages}
