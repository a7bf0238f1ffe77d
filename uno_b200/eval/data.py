"""Evaluation records: JSONL loading, field lookup, protocol fingerprints.

A record carries ``chat_input`` (list of chat messages), an id (first of
``id``, ``problem_id``, ``index``, ``row``) and a reference answer (first of
``ground_truth``, ``answer``); code tasks carry their tests.  The protocol
fingerprint of a dataset is its row count and the sha256 of the file bytes
(``evaluation/data.py:145-161``).
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path
from typing import Any, Iterable

ID_FIELDS = ("id", "problem_id", "index", "row")
ANSWER_FIELDS = ("ground_truth", "answer")


def read_jsonl(path: str | Path) -> list[dict[str, Any]]:
    out = []
    with open(path, encoding="utf-8") as fh:
        for n, line in enumerate(fh, 1):
            if line.strip():
                row = json.loads(line)
                if not isinstance(row, dict):
                    raise ValueError(f"{path}:{n}: each line must be a JSON object")
                out.append(row)
    return out


def append_jsonl(path: str | Path, rows: Iterable[dict[str, Any]]) -> None:
    with open(path, "a", encoding="utf-8") as fh:
        for row in rows:
            fh.write(json.dumps(row, ensure_ascii=False) + "\n")
        fh.flush()


def load_records(path: str | Path, limit: int | None = None) -> list[dict[str, Any]]:
    rows = read_jsonl(path)
    return rows[:limit] if limit is not None else rows


def first_field(record: dict[str, Any], names: tuple[str, ...]) -> Any | None:
    for n in names:
        if record.get(n) is not None:
            return record[n]
    return None


def protocol_artifact_fingerprint(path: str | Path) -> tuple[int, str]:
    h = hashlib.sha256()
    with open(path, "rb") as fh:
        for chunk in iter(lambda: fh.read(1 << 20), b""):
            h.update(chunk)
    with open(path, "rb") as fh:
        rows = sum(1 for line in fh if line.strip())
    return rows, h.hexdigest()
