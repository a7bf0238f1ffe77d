"""Tokenise an OpenThoughts-style ShareGPT corpus into Uno training rows.

Behaviour of ``training/prepare_openthoughts.py`` and the encoder of
``training/data.py:25-128`` (the released preprocessing recipe, reproduced so
that a corpus prepared here hashes to the reference's manifest):

* each (human, gpt) pair renders as ``<|im_start|>user\\n{q}<|im_end|>\\n
  <|im_start|>assistant\\n`` (unsupervised) and ``{a}<|im_end|>\\n``
  (supervised); an answer without think tags gets an empty
  ``<think>\\n\\n</think>\\n\\n`` block in front;
* the cutoff (4096) is rounded down to a multiple of the token alignment (3);
  each pair is cut to the remaining budget with the recipe's split rule
  (:func:`split_budget`); pairs stop once the budget is used;
* the row is right-padded to a multiple of the alignment with the pad token,
  and those pad positions are labelled with the pad id (they are data);
* the corpus hash is sha256 over, per row, its length (u64 little-endian),
  input ids and labels (i32 little-endian), in source order, with row, token
  and supervised-token counts.

Output: ``rows.jsonl`` (one ``{"input_ids", "labels"}`` object per row, the
format :func:`uno_b200.train.data.load_jsonl` reads) and
``uno_dataset_manifest.json`` (source, tokenizer, recipe, hash).  Input is a
local JSONL / JSON file with a ``conversations`` field per row, or a dataset
id that the ``datasets`` package can load when a network is available.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import struct
from datetime import datetime, timezone
from pathlib import Path
from typing import Any, Iterable, Sequence

import numpy as np

from uno_b200.utils.hub import PINNED_MODEL_ID, PINNED_MODEL_REVISION

IGNORE = -100
CUTOFF = 4096
ALIGN = 3
THINK_OPEN, THINK_CLOSE = "<think>\n", "\n</think>\n\n"
DATASET_ID = "open-thoughts/OpenThoughts3-1.2M"
DATASET_REVISION = "61bcf9d4eb38b30295efc2021227a63cc5bb34c8"
MODEL_ID, MODEL_REVISION = PINNED_MODEL_ID, PINNED_MODEL_REVISION
HASH_ALGORITHM = "sha256-rowlen-u64le-input-i32le-label-i32le-v1"


def split_budget(src: int, tgt: int, budget: int) -> tuple[int, int]:
    """Tokens kept of a (prompt, answer) pair under ``budget``.

    The answer keeps everything when it is under half the budget; else the
    prompt keeps everything when it is under half; else the budget splits in
    proportion to the two lengths.  The prompt gets what the answer leaves.
    """
    if 2 * tgt < budget:
        cap = budget
    elif 2 * src < budget:
        cap = budget - src
    else:
        cap = int(budget * (tgt / (src + tgt)))
    keep_tgt = min(cap, tgt)
    return min(max(budget - keep_tgt, 0), src), keep_tgt


def encode_conversation(conversations: Sequence[dict], tokenizer, *, cutoff: int = CUTOFF,
                        align: int = ALIGN) -> dict[str, list[int]]:
    budget_total = cutoff - cutoff % align
    if budget_total <= 0:
        raise ValueError("cutoff rounded to the alignment must be positive")
    if not conversations or len(conversations) % 2:
        raise ValueError("a conversation needs complete (human, gpt) pairs")
    ids: list[int] = []
    labels: list[int] = []
    for q, a in zip(conversations[0::2], conversations[1::2]):
        if q.get("from") != "human" or a.get("from") != "gpt":
            raise ValueError("conversation turns must alternate 'human' and 'gpt'")
        if len(ids) >= budget_total:
            break
        answer = str(a.get("value", ""))
        if THINK_OPEN not in answer and THINK_CLOSE not in answer:
            answer = THINK_OPEN + THINK_CLOSE + answer
        src = tokenizer.encode(f"<|im_start|>user\n{q.get('value', '')}<|im_end|>\n<|im_start|>assistant\n",
                               add_special_tokens=False)
        tgt = tokenizer.encode(answer + "<|im_end|>\n", add_special_tokens=False)
        ns, nt = split_budget(len(src), len(tgt), budget_total - len(ids))
        ids += list(src[:ns]) + list(tgt[:nt])
        labels += [IGNORE] * ns + list(tgt[:nt])
    if not ids:
        raise ValueError("conversation produced no tokens")
    pad = tokenizer.pad_token_id
    if pad is None:
        raise ValueError("the tokenizer needs a pad token")
    extra = (-len(ids)) % align
    ids += [pad] * extra
    labels += [pad] * extra
    return {"input_ids": ids, "labels": labels}


def corpus_hash(rows: Iterable[dict[str, Sequence[int]]]) -> dict[str, Any]:
    h = hashlib.sha256()
    n_rows = n_tok = n_sup = 0
    for row in rows:
        ids = np.asarray(row["input_ids"], dtype="<i4")
        lab = np.asarray(row["labels"], dtype="<i4")
        if ids.shape != lab.shape:
            raise ValueError(f"row {n_rows}: input and label lengths differ")
        h.update(struct.pack("<Q", ids.size))
        h.update(ids.tobytes())
        h.update(lab.tobytes())
        n_rows += 1
        n_tok += int(ids.size)
        n_sup += int((lab != IGNORE).sum())
    return {"algorithm": HASH_ALGORITHM, "content_sha256": h.hexdigest(), "row_count": n_rows,
            "token_count": n_tok, "supervised_token_count": n_sup}


def _source_rows(source: str, max_samples: int | None, cache_dir: str | None = None) -> Iterable[dict]:
    path = Path(source)
    if path.is_file():
        if path.suffix == ".json":
            rows = json.loads(path.read_text())
        else:
            rows = (json.loads(line) for line in path.open(encoding="utf-8") if line.strip())
    else:
        from datasets import load_dataset  # network / cache path

        rows = load_dataset(source, revision=DATASET_REVISION if source == DATASET_ID else None, split="train",
                            streaming=max_samples is not None, cache_dir=cache_dir)
    for i, row in enumerate(rows):
        if max_samples is not None and i >= max_samples:
            break
        yield row


_WORKER_TOKENIZER = None


def _encode_in_worker(conversations):
    return encode_conversation(conversations, _WORKER_TOKENIZER)


def _encoded_rows(rows: Iterable[dict], tokenizer, num_proc: int) -> Iterable[dict]:
    """Encoded rows in source order; ``num_proc`` > 1 encodes in forked worker processes."""
    if num_proc <= 1:
        for row in rows:
            yield encode_conversation(row["conversations"], tokenizer)
        return
    import multiprocessing as mp

    global _WORKER_TOKENIZER
    _WORKER_TOKENIZER = tokenizer  # inherited by the forked workers
    with mp.get_context("fork").Pool(num_proc) as pool:
        yield from pool.imap(_encode_in_worker, (row["conversations"] for row in rows), chunksize=64)


def prepare(source: str, output: Path, tokenizer, *, max_samples: int | None = None,
            verify_against: Path | None = None, num_proc: int = 1, writer_batch_size: int = 1000,
            cache_dir: str | None = None) -> dict[str, Any]:
    """Encode ``source`` into ``output/rows.jsonl`` plus its manifest.

    ``num_proc`` encoding processes keep the source order (the hash depends on
    it); rows are written ``writer_batch_size`` at a time."""
    output = Path(output)
    if output.exists() and (not output.is_dir() or any(output.iterdir())):
        raise FileExistsError(f"output must be an empty directory: {output}")
    output.mkdir(parents=True, exist_ok=True)
    rows_path = output / "rows.jsonl"
    encoded = []
    pending: list[str] = []
    with rows_path.open("w", encoding="utf-8") as fh:
        for enc in _encoded_rows(_source_rows(source, max_samples, cache_dir), tokenizer, num_proc):
            pending.append(json.dumps(enc) + "\n")
            encoded.append(enc)
            if len(pending) >= max(1, writer_batch_size):
                fh.write("".join(pending))
                pending.clear()
        fh.write("".join(pending))
    digest = corpus_hash(encoded)
    if verify_against is not None:
        ref = Path(verify_against)
        ref = ref if ref.is_file() else ref / "uno_dataset_manifest.json"
        want = json.loads(ref.read_text())["hash"]
        for key in ("row_count", "content_sha256"):
            if digest[key] != want.get(key):
                raise RuntimeError(f"prepared corpus {key} {digest[key]} != reference {want.get(key)}")
    manifest = {
        "version": 1, "created_at": datetime.now(timezone.utc).isoformat(),
        "source": {"dataset_id": DATASET_ID if source == DATASET_ID else str(source),
                   "revision": DATASET_REVISION if source == DATASET_ID else None, "split": "train",
                   "source_order_preserved": True},
        "tokenizer": {"class": type(tokenizer).__name__, "pad_token_id": tokenizer.pad_token_id},
        "preprocessing": {"template": "qwen3-sharegpt-reasoning", "cutoff_length": CUTOFF, "token_alignment": ALIGN,
                          "max_preprocessed_length": CUTOFF - 1, "prompt_label_id": IGNORE, "truncate_mode": "cut"},
        "smoke_max_samples": max_samples, "rows_file": rows_path.name, "hash": digest,
    }
    (output / "uno_dataset_manifest.json").write_text(json.dumps(manifest, indent=2, sort_keys=True) + "\n")
    return manifest


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description="Tokenise a ShareGPT corpus into Uno training rows.")
    ap.add_argument("--source", default=DATASET_ID, help="local .jsonl/.json file or a dataset id")
    ap.add_argument("--output", required=True, type=Path)
    ap.add_argument("--tokenizer", default=MODEL_ID, help="tokenizer directory or hub id")
    ap.add_argument("--max-samples", type=int)
    ap.add_argument("--verify-against", type=Path)
    ap.add_argument("--cache-dir", help="Hugging Face cache for the dataset and tokenizer")
    ap.add_argument("--num-proc", type=int, default=1, help="encoding processes (source order is kept)")
    ap.add_argument("--writer-batch-size", type=int, default=1000)
    ap.add_argument("--tokenizer-local-files-only", action="store_true")
    args = ap.parse_args(argv)
    from transformers import AutoTokenizer

    tok = AutoTokenizer.from_pretrained(args.tokenizer, revision=MODEL_REVISION if args.tokenizer == MODEL_ID else None,
                                        trust_remote_code=True, cache_dir=args.cache_dir,
                                        local_files_only=args.tokenizer_local_files_only)
    if tok.pad_token_id is None:
        tok.pad_token = tok.eos_token
    print(json.dumps(prepare(args.source, args.output, tok, max_samples=args.max_samples,
                             verify_against=args.verify_against, num_proc=args.num_proc,
                             writer_batch_size=args.writer_batch_size, cache_dir=args.cache_dir),
                     indent=2, sort_keys=True))


if __name__ == "__main__":
    main()
