"""Training objective, LoRA settings and run manifests.

Semantics of ``training/config.py:21-133`` and ``training/constants.py``:

* the public objective is ``ce_weight * CE + kl_weight * KL(student||teacher)
  + tv_weight * TV``, uniform noise, a frozen base-model teacher; CE targets
  are the clean teacher's argmax ("teacher") or the data ("ground_truth");
* a run writes ``uno_training_manifest.json`` whose ``compatibility_sha256``
  (sha256 of the canonical JSON of everything a resume must agree on) is
  checked before resuming; JSON is written atomically (temp file + rename).
"""

from __future__ import annotations

import hashlib
import json
import math
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Any, Literal

IGNORE_INDEX = -100
DEFAULT_LORA_RANK = 128
DEFAULT_LORA_ALPHA_RATIO = 16
SUPPORTED_LORA_MODULES = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")

CeTarget = Literal["teacher", "ground_truth"]


@dataclass(frozen=True)
class UnoObjectiveConfig:
    ce_target: CeTarget = "teacher"
    noise: str = "uniform"
    reverse_kl: bool = True
    teacher_base_only: bool = True
    ce_weight: float = 0.0
    kl_weight: float = 0.0
    tv_weight: float = 1.0

    def validate(self) -> None:
        if self.ce_target not in ("teacher", "ground_truth"):
            raise ValueError("ce_target must be either 'teacher' or 'ground_truth'.")
        if self.noise != "uniform":
            raise ValueError("Uno training supports uniform noise only.")
        if not self.reverse_kl:
            raise ValueError("Uno training supports reverse KL only.")
        if not self.teacher_base_only:
            raise ValueError("The Uno teacher must use the frozen base weights only.")
        w = (self.ce_weight, self.kl_weight, self.tv_weight)
        if any(not isinstance(x, (int, float)) or not math.isfinite(x) or x < 0 for x in w):
            raise ValueError("Uno loss weights must be finite and non-negative.")
        if not any(x > 0 for x in w):
            raise ValueError("At least one Uno loss weight must be positive.")

    @property
    def internal_ce_target(self) -> str:
        self.validate()
        return "clean_argmax" if self.ce_target == "teacher" else "data"


@dataclass(frozen=True)
class LoraSettings:
    target: str = "all"
    rank: int = DEFAULT_LORA_RANK
    alpha: int | None = None
    dropout: float = 0.0

    @property
    def resolved_alpha(self) -> int:
        return self.alpha if self.alpha is not None else DEFAULT_LORA_ALPHA_RATIO * self.rank

    @property
    def modules(self) -> tuple[str, ...]:
        if self.target == "all":
            return SUPPORTED_LORA_MODULES
        mods = tuple(m.strip() for m in self.target.split(",") if m.strip())
        bad = [m for m in mods if m not in SUPPORTED_LORA_MODULES]
        if bad or not mods:
            raise ValueError(f"Unsupported LoRA target modules: {bad or self.target}")
        return mods

    def validate(self) -> None:
        if self.rank <= 0:
            raise ValueError("LoRA rank must be positive.")
        if self.alpha is not None and self.alpha <= 0:
            raise ValueError("LoRA alpha must be positive.")
        if not 0.0 <= self.dropout < 1.0:
            raise ValueError("LoRA dropout must be in [0, 1).")
        _ = self.modules


def canonical_json(payload: dict[str, Any]) -> str:
    return json.dumps(payload, sort_keys=True, separators=(",", ":"))


def manifest_digest(payload: dict[str, Any]) -> str:
    return hashlib.sha256(canonical_json(payload).encode("utf-8")).hexdigest()


def write_json_atomic(path: Path, payload: dict[str, Any]) -> None:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_suffix(path.suffix + ".tmp")
    tmp.write_text(json.dumps(payload, indent=2, sort_keys=True) + "\n")
    tmp.replace(path)


def write_run_manifest(output_dir: Path, compatibility: dict[str, Any], extra: dict[str, Any] | None = None) -> None:
    write_json_atomic(Path(output_dir) / "uno_training_manifest.json",
                      {"compatibility": compatibility, "compatibility_sha256": manifest_digest(compatibility),
                       **(extra or {})})


def validate_resume_manifest(output_dir: Path, expected: dict[str, Any]) -> None:
    path = Path(output_dir) / "uno_training_manifest.json"
    if not path.is_file():
        raise FileNotFoundError(f"Cannot resume without the original run manifest: {path}")
    actual = json.loads(path.read_text())
    want = manifest_digest(expected)
    if actual.get("compatibility_sha256") != want:
        raise ValueError("Resume configuration does not match the original training run. Expected "
                         f"compatibility hash {want}, got {actual.get('compatibility_sha256')}.")


def dataclass_dict(value: Any) -> dict[str, Any]:
    return asdict(value)
