"""Training objective, LoRA settings and the run manifest.

What must agree with ``training/config.py:21-133`` and ``training/constants.py``
of the reference:

* the objective is ``ce_weight * CE + kl_weight * KL(student || teacher)
  + tv_weight * TV`` with uniform noise and the frozen base model as teacher;
  CE targets are the clean teacher's arg-max (``ce_target="teacher"``) or the
  data (``"ground_truth"``);
* a run writes ``uno_training_manifest.json`` holding ``compatibility`` (every
  setting a resume must share) and ``compatibility_sha256``, the sha256 of its
  canonical JSON (sorted keys, no whitespace); a resume recomputes the digest
  and refuses to continue on a mismatch.

The validation rules below are stated as data (predicate, message) and the
manifest file is replaced atomically (written to a temporary file in the same
directory, flushed to disk, then renamed over the old one).
"""

from __future__ import annotations

import hashlib
import json
import math
import os
import tempfile
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Any, Literal

IGNORE_INDEX = -100
DEFAULT_LORA_RANK = 128
DEFAULT_LORA_ALPHA_RATIO = 16  # alpha = 16 * rank unless given
SUPPORTED_LORA_MODULES = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
MANIFEST_NAME = "uno_training_manifest.json"

CeTarget = Literal["teacher", "ground_truth"]
_CE_TARGET_KIND = {"teacher": "clean_argmax", "ground_truth": "data"}


def _check(rules) -> None:
    """Raise ``ValueError`` with the message of the first rule whose predicate is false."""
    for ok, message in rules:
        if not ok():
            raise ValueError(message)


def _is_weight(x) -> bool:
    return isinstance(x, (int, float)) and not isinstance(x, bool) and math.isfinite(x) and x >= 0


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
        weights = (self.ce_weight, self.kl_weight, self.tv_weight)
        _check((
            (lambda: self.ce_target in _CE_TARGET_KIND,
             f"ce_target={self.ce_target!r}: CE targets are 'teacher' (clean arg-max) or 'ground_truth' (data)"),
            (lambda: self.noise == "uniform", f"noise={self.noise!r}: the objective is defined for uniform noise"),
            (lambda: self.reverse_kl, "the KL term is the reverse KL(student || teacher); forward KL is not offered"),
            (lambda: self.teacher_base_only, "the teacher is the frozen base model (no LoRA on clean rows)"),
            (lambda: all(_is_weight(w) for w in weights),
             f"loss weights (ce, kl, tv) = {weights} must be finite numbers >= 0"),
            (lambda: any(w > 0 for w in weights), "all loss weights are zero: nothing would be trained"),
        ))

    @property
    def internal_ce_target(self) -> str:
        self.validate()
        return _CE_TARGET_KIND[self.ce_target]


@dataclass(frozen=True)
class LoraSettings:
    target: str = "all"
    rank: int = DEFAULT_LORA_RANK
    alpha: int | None = None
    dropout: float = 0.0

    @property
    def resolved_alpha(self) -> int:
        return DEFAULT_LORA_ALPHA_RATIO * self.rank if self.alpha is None else self.alpha

    @property
    def modules(self) -> tuple[str, ...]:
        """Projection names that carry the adapter (``"all"`` or a comma list)."""
        if self.target == "all":
            return SUPPORTED_LORA_MODULES
        names = tuple(filter(None, (part.strip() for part in self.target.split(","))))
        unknown = sorted(set(names) - set(SUPPORTED_LORA_MODULES))
        if not names or unknown:
            raise ValueError(f"LoRA target {self.target!r}: unknown modules {unknown or '(none given)'}; "
                             f"choose from {', '.join(SUPPORTED_LORA_MODULES)}")
        return names

    def validate(self) -> None:
        _check((
            (lambda: self.rank > 0, f"LoRA rank {self.rank} must be at least 1"),
            (lambda: self.alpha is None or self.alpha > 0, f"LoRA alpha {self.alpha} must be positive"),
            (lambda: 0.0 <= self.dropout < 1.0, f"LoRA dropout {self.dropout} must lie in [0, 1)"),
        ))
        self.modules  # noqa: B018  (raises on unknown target modules)


def canonical_json(payload: dict[str, Any]) -> str:
    """The byte-stable JSON text the compatibility digest is taken over."""
    return json.dumps(payload, sort_keys=True, separators=(",", ":"))


def manifest_digest(payload: dict[str, Any]) -> str:
    return hashlib.sha256(canonical_json(payload).encode("utf-8")).hexdigest()


def write_json_atomic(path: Path, payload: dict[str, Any]) -> None:
    """Replace ``path`` with ``payload`` as indented JSON; readers see the old or the new file, never a mix."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    fd, tmp = tempfile.mkstemp(prefix=path.name + ".", suffix=".part", dir=path.parent)
    try:
        with os.fdopen(fd, "w") as fh:
            fh.write(json.dumps(payload, indent=2, sort_keys=True) + "\n")
            fh.flush()
            os.fsync(fh.fileno())
        os.replace(tmp, path)
    except BaseException:
        if os.path.exists(tmp):
            os.unlink(tmp)
        raise


def write_run_manifest(output_dir: Path, compatibility: dict[str, Any], extra: dict[str, Any] | None = None) -> None:
    record = dict(extra or {})
    record["compatibility"] = compatibility
    record["compatibility_sha256"] = manifest_digest(compatibility)
    write_json_atomic(Path(output_dir) / MANIFEST_NAME, record)


def validate_resume_manifest(output_dir: Path, expected: dict[str, Any]) -> None:
    """Refuse to resume into ``output_dir`` unless its manifest digest equals that of ``expected``."""
    path = Path(output_dir) / MANIFEST_NAME
    if not path.is_file():
        raise FileNotFoundError(f"{path} is missing: a run can only resume from its own output directory")
    found = json.loads(path.read_text()).get("compatibility_sha256")
    want = manifest_digest(expected)
    if found != want:
        raise ValueError(f"the resumed run does not match the run in {output_dir}: compatibility digest "
                         f"{found} on disk, {want} for the current settings")


def dataclass_dict(value: Any) -> dict[str, Any]:
    return asdict(value)
