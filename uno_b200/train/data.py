"""Training data: synthetic Zipf batches, padded or packed token rows, manifests.

* :func:`synthetic_batches` -- random token ids drawn Zipf(a) over a fixed
  permutation of the vocabulary (the benchmark configs' "Zipf(1.1) random token
  ids"), optionally with an unsupervised prompt prefix;
* :func:`pad_rows` -- one pre-tokenised ``{"input_ids", "labels"}`` row per
  sequence, right-padded with IGNORE labels (the released recipe's collator,
  ``training/data.py:209-239``); the default of ``uno_b200.train``;
* :func:`pack_rows` -- greedy packing of several rows into one sequence,
  positions restarting per row (``--pack-rows``; not the recipe);
* :func:`data_manifest` -- sha256 of the data files, pinned in the run
  manifest (``training/data.py:139-206``).
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path
from typing import Iterator

import numpy as np
import torch

from uno_b200.train.config import IGNORE_INDEX


def synthetic_batches(batch_size: int, seq_len: int, vocab_size: int, *, zipf_a: float = 1.1,
                      prompt_len: int = 0, seed: int = 0, low: int = 1) -> Iterator[dict[str, torch.Tensor]]:
    rng = np.random.default_rng(seed)
    perm = rng.permutation(np.arange(low, vocab_size))
    while True:
        ranks = np.minimum(rng.zipf(zipf_a, size=(batch_size, seq_len)) - 1, len(perm) - 1)
        ids = torch.from_numpy(perm[ranks]).long()
        labels = ids.clone()
        if prompt_len:
            labels[:, :prompt_len] = IGNORE_INDEX
        yield {"input_ids": ids, "labels": labels,
               "position_ids": torch.arange(seq_len).expand(batch_size, seq_len).clone()}


def pad_rows(rows: list[dict], seq_len: int, pad_id: int = 0) -> list[dict[str, torch.Tensor]]:
    """One prepared row per sequence, right-padded to ``seq_len`` with ignored labels -- the
    released recipe's collation (``training/data.py:209-239``).  The layout is causal, so the real
    tokens never see the padding after them.  A row longer than ``seq_len`` is an error."""
    out = []
    for i, row in enumerate(rows):
        ids = list(row["input_ids"])
        lab = list(row.get("labels", ids))
        if len(ids) != len(lab):
            raise ValueError(f"row {i}: input_ids and labels must have the same length")
        if len(ids) > seq_len:
            raise ValueError(f"row {i} has {len(ids)} tokens, more than the sequence length {seq_len} "
                             "(raise --seq-len, or pack rows with --pack-rows)")
        pad = seq_len - len(ids)
        out.append({"input_ids": torch.tensor(ids + [pad_id] * pad), "labels": torch.tensor(lab + [IGNORE_INDEX] * pad),
                    "position_ids": torch.arange(seq_len)})
    return out


def pack_rows(rows: list[dict], seq_len: int, pad_id: int = 0) -> list[dict[str, torch.Tensor]]:
    """Greedy first-fit packing of token rows into ``seq_len`` sequences (positions restart per
    row, but a later row attends to the earlier rows of its pack: an option, not the recipe)."""
    out, cur_ids, cur_lab, cur_pos = [], [], [], []

    def flush():
        if not cur_ids:
            return
        n = len(cur_ids)
        ids = cur_ids + [pad_id] * (seq_len - n)
        lab = cur_lab + [IGNORE_INDEX] * (seq_len - n)
        last = cur_pos[-1] if cur_pos else -1
        pos = cur_pos + list(range(last + 1, last + 1 + seq_len - n))
        out.append({"input_ids": torch.tensor(ids), "labels": torch.tensor(lab), "position_ids": torch.tensor(pos)})
        cur_ids.clear(), cur_lab.clear(), cur_pos.clear()

    for row in rows:
        ids = list(row["input_ids"])[:seq_len]
        lab = list(row.get("labels", ids))[:seq_len]
        if len(ids) != len(lab):
            raise ValueError("input_ids and labels must have the same length")
        if len(cur_ids) + len(ids) > seq_len:
            flush()
        cur_ids.extend(ids)
        cur_lab.extend(lab)
        cur_pos.extend(range(len(ids)))
    flush()
    return out


def load_jsonl(path: str | Path) -> list[dict]:
    """Token rows ``{"input_ids", "labels"}`` from a JSONL file or a prepared corpus directory:
    ``rows.jsonl`` (written by ``uno_b200.train.prepare``) or a Hugging Face ``datasets``
    directory saved with ``save_to_disk`` (the reference preparer's output)."""
    path = Path(path)
    if path.is_dir():
        if (path / "rows.jsonl").is_file():
            path = path / "rows.jsonl"
        elif (path / "state.json").is_file() or (path / "dataset_info.json").is_file():
            from datasets import load_from_disk

            return [{"input_ids": list(r["input_ids"]), "labels": list(r["labels"])}
                    for r in load_from_disk(str(path))]
        else:
            raise FileNotFoundError(f"{path} has neither rows.jsonl nor a saved datasets directory")
    with open(path, encoding="utf-8") as fh:
        return [json.loads(line) for line in fh if line.strip()]


def batches_from_rows(packed: list[dict[str, torch.Tensor]], batch_size: int, seed: int = 0
                      ) -> Iterator[dict[str, torch.Tensor]]:
    g = torch.Generator().manual_seed(seed)
    while True:
        order = torch.randperm(len(packed), generator=g).tolist()
        for i in range(0, len(order) - batch_size + 1, batch_size):
            items = [packed[j] for j in order[i:i + batch_size]]
            yield {k: torch.stack([it[k] for it in items]) for k in items[0]}


def data_manifest(paths: list[str | Path]) -> dict:
    """sha256 and size of every data file (a directory contributes its files, and the corpus
    hash of its ``uno_dataset_manifest.json`` when present)."""
    files, corpus = [], None
    expanded = []
    for x in paths:
        x = Path(x)
        if x.is_dir():
            manifest = x / "uno_dataset_manifest.json"
            if manifest.is_file():
                corpus = json.loads(manifest.read_text()).get("hash")
            expanded += [f for f in sorted(x.rglob("*")) if f.is_file() and not f.name.startswith(".")]
        else:
            expanded.append(x)
    for p in sorted(str(x) for x in expanded):
        h = hashlib.sha256()
        with open(p, "rb") as fh:
            for chunk in iter(lambda: fh.read(1 << 20), b""):
                h.update(chunk)
        files.append({"path": Path(p).name, "sha256": h.hexdigest(), "bytes": Path(p).stat().st_size})
    out = {"version": 1, "files": files}
    if corpus is not None:
        out["corpus_hash"] = corpus
    return out
