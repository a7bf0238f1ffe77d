"""Pinned benchmark data for the evaluation protocol: fetch, validate, build.

Behaviour of ``evaluation/data.py`` and ``evaluation/prepare_data.py``:

* a benchmark with a pinned artifact (file name + sha256 in the registry) is
  copied from a protocol source bundle -- flat (``{name}.jsonl``) or laid out
  like the source repository (``{source_filename}``) -- found in
  ``--source-dir`` / ``UNO_EVAL_PROTOCOL_SOURCE_DIR``, else downloaded from the
  pinned dataset revision when ``huggingface_hub`` and a network are present;
  the row count and sha256 must match before the file is installed (atomic
  rename), and an existing output is re-validated instead of rebuilt;
* benchmarks without a pinned artifact are built from their public rows by a
  builder that renders the protocol's prompt text and grading metadata (the
  text is part of the protocol, so it is reproduced exactly); builders take
  the raw rows as input, so they run offline from any local copy;
* LiveCodeBench private tests are JSON or base64(zlib(pickle(json string)));
  the pickle is read with an unpickler that refuses every global, so a
  payload cannot construct objects.

CLI: ``python -m uno_b200.eval.prepare [BENCHMARK ...] [--output-dir D]
[--source-dir S] [--overwrite]``.
"""

from __future__ import annotations

import argparse
import base64
import hashlib
import io
import json
import os
import pickle
import random
import zlib
from pathlib import Path
from typing import Any, Callable, Iterable, Mapping

from uno_b200.eval.benchmarks import BENCHMARKS, DEFAULT_DATA_ROOT, get_benchmark, normalize_benchmark_name
from uno_b200.eval.data import protocol_artifact_fingerprint

SOURCE_DIR_ENV = "UNO_EVAL_PROTOCOL_SOURCE_DIR"
PROTOCOL_REPO = "LLM360/eval-360-sources"
PROTOCOL_REVISION = "f1d3a57020a52de762e73faba260ed15d9a8b6d7"

# ------------------------------------------------------------ prompt texts
HUMANEVAL_INSTRUCTION = ("Read the following function signature and docstring, and fully implement the function "
                         "described. Your response should only contain the code for this function.")
MBPP_TEXT_OVERRIDES = {388: "Write a python function to find the highest power of 2 that is less than or equal to n."}
LCB_SYSTEM = ("You are an expert Python programmer. You will be given a question (problem specification) and will "
              "generate a correct Python program that matches the specification and passes all tests. You will NOT "
              "return anything except for the program.")
LCB_WITH_STARTER = ("You will use the following starter code to write the solution to the problem and enclose your "
                    "code within delimiters.")
LCB_WITHOUT_STARTER = ("Read the inputs from stdin solve the problem and write the answer to stdout (do not directly "
                       "test on the sample inputs). Enclose your code within delimiters as follows.")
GPQA_HEADER = ("Answer the following multiple choice question. The last line of your response should be of the "
               "following format: 'ANSWER: $LETTER' (without quotes) where LETTER is one of ABCD. Think step by step "
               "before answering.")


def _record(i, truth, prompt, chat=None) -> dict[str, Any]:
    return {"row": i, "ground_truth": truth, "completion_input": prompt,
            "chat_input": chat if chat is not None else [{"role": "user", "content": prompt}]}


def build_gsm8k(rows: Iterable[Mapping]) -> list[dict]:
    return [_record(i, r["answer"], f"Q: {r['question']}\nA: Let's think step by step.") for i, r in enumerate(rows)]


def build_math500(rows: Iterable[Mapping]) -> list[dict]:
    return [_record(i, r["answer"], r["problem"]) for i, r in enumerate(rows)]


def build_aime(rows: Iterable[Mapping]) -> list[dict]:
    return [_record(i, str(r.get("answer", r.get("solution"))).strip(), f"Question: {r['problem']}\nAnswer:")
            for i, r in enumerate(rows)]


def build_humaneval(rows: Iterable[Mapping]) -> list[dict]:
    out = []
    for i, r in enumerate(rows):
        prompt = str(r["prompt"])
        out.append(_record(i, {"test": r["test"], "entry_point": r["entry_point"]}, prompt,
                           [{"role": "user", "content": f"{HUMANEVAL_INSTRUCTION}\n{prompt}"}]))
    return out


def _mbpp_task(r: Mapping) -> str:
    text = MBPP_TEXT_OVERRIDES.get(int(r["task_id"]), str(r["text"]))
    tests = "\n".join(str(t) for t in r["test_list"])
    return (f"You are an expert Python programmer, and here is your task: {text} Your code should pass these tests:"
            f"\n\n{tests}\n[BEGIN]\n")


def build_mbpp(rows: Iterable[Mapping], prompt_rows: Iterable[Mapping]) -> list[dict]:
    """Three-shot prompt from the ``prompt`` split's tasks 2, 3 and 4, then the test task."""
    shots = {int(r["task_id"]): r for r in prompt_rows}
    prefix = "".join(_mbpp_task(shots[t]) + str(shots[t]["code"]) + "\n[DONE]\n\n" for t in (2, 3, 4))
    return [_record(i, "\n".join(r["test_list"]), prefix + _mbpp_task(r)) for i, r in enumerate(rows)]


class _NoGlobals(pickle.Unpickler):
    def find_class(self, module, name):
        raise pickle.UnpicklingError(f"refusing to load {module}.{name} from a LiveCodeBench payload")


def decode_lcb_tests(value: str) -> list[dict]:
    try:
        tests = json.loads(value)
    except json.JSONDecodeError:
        raw = zlib.decompress(base64.b64decode(value.encode("utf-8")))
        tests = json.loads(_NoGlobals(io.BytesIO(raw)).load())
    if not isinstance(tests, list):
        raise ValueError("LiveCodeBench tests must decode to a list")
    return tests


def build_lcb(rows: Iterable[Mapping]) -> list[dict]:
    out = []
    for i, r in enumerate(rows):
        tests = json.loads(r["public_test_cases"]) + decode_lcb_tests(r["private_test_cases"])
        fn = json.loads(r["metadata"]).get("func_name")
        if fn:
            tests = [dict(t, method_name=fn) for t in tests]
        starter = str(r.get("starter_code", "")).strip()
        fmt = (f"### Format: {LCB_WITH_STARTER}\n```python\n{starter}\n```\n\n" if starter else
               f"### Format: {LCB_WITHOUT_STARTER}\n```python\n# YOUR CODE HERE\n```\n\n")
        user = f"### Question:\n{r['question_content']}\n\n{fmt}### Answer: (use the provided format with backticks)\n\n"
        out.append(_record(str(i), json.dumps(tests), f"{LCB_SYSTEM}\n\n{user}",
                           [{"role": "system", "content": LCB_SYSTEM}, {"role": "user", "content": user}]))
    return out


def gpqa_order(question: str) -> list[int]:
    """Choice order of a GPQA question: a shuffle seeded by the first 32 bits of its md5."""
    seed = int(hashlib.md5(question.encode(), usedforsecurity=False).hexdigest()[:8], 16)
    order = list(range(4))
    random.Random(seed).shuffle(order)
    return order


def build_gpqa(rows: Iterable[Mapping]) -> list[dict]:
    out = []
    for i, r in enumerate(rows):
        q = str(r["Question"])
        choices = [str(r["Correct Answer"]), str(r["Incorrect Answer 1"]), str(r["Incorrect Answer 2"]),
                   str(r["Incorrect Answer 3"])]
        order = gpqa_order(q)
        listing = "\n".join(f"{'ABCD'[k]}) {choices[j]}" for k, j in enumerate(order))
        out.append(_record(i, "ABCD"[order.index(0)], f"{GPQA_HEADER}\n\n{q}\n\n{listing}"))
    return out


def build_ifeval(rows: Iterable[Mapping]) -> list[dict]:
    out = []
    for i, r in enumerate(rows):
        kwargs = [{k: v for k, v in kw.items() if v is not None} for kw in r["kwargs"]]
        out.append(_record(i, {"instruction_id_list": list(r["instruction_id_list"]), "kwargs": kwargs},
                           str(r["prompt"])))
    return out


# benchmark -> (builder, public dataset coordinates: (repo, config, split))
BUILDERS: dict[str, tuple[Callable, tuple]] = {
    "gsm8k": (build_gsm8k, ("openai/gsm8k", "main", "test")),
    "math500": (build_math500, ("HuggingFaceH4/MATH-500", None, "test")),
    "aime24": (build_aime, ("hypaai/Hypa_AIME2024", None, "english")),
    "aime25": (build_aime, ("math-ai/aime25", None, "test")),
    "aime26": (build_aime, ("math-ai/aime26", None, "test")),
    "humaneval": (build_humaneval, ("openai/openai_humaneval", None, "test")),
    "gpqa_diamond": (build_gpqa, ("Idavidrein/gpqa", "gpqa_diamond", "train")),
    "ifeval": (build_ifeval, ("google/IFEval", None, "train")),
}


# ------------------------------------------------------------------ install
def _atomic_write(path: Path, data: bytes) -> None:
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_suffix(path.suffix + ".tmp")
    tmp.write_bytes(data)
    tmp.replace(path)


def validate_artifact(path: Path, rows: int, sha256: str | None) -> None:
    n, digest = protocol_artifact_fingerprint(path)
    if n != rows:
        raise ValueError(f"{path} has {n} rows; the protocol pins {rows}")
    if sha256 is not None and digest != sha256:
        raise ValueError(f"{path} has sha256 {digest}; the protocol pins {sha256}")


def _find_source(source_dir: Path, name: str, source_filename: str | None) -> Path:
    candidates = [source_dir / f"{name}.jsonl"] + ([source_dir / source_filename] if source_filename else [])
    for c in candidates:
        if c.is_file():
            return c
    raise FileNotFoundError(f"no protocol artifact for {name} in {source_dir} (looked for "
                            f"{', '.join(str(c) for c in candidates)})")


def _download_pinned(source_filename: str) -> Path:
    try:
        from huggingface_hub import hf_hub_download
    except ImportError as exc:  # pragma: no cover - depends on the environment
        raise RuntimeError("huggingface_hub is not installed; pass --source-dir") from exc
    return Path(hf_hub_download(repo_id=PROTOCOL_REPO, repo_type="dataset", filename=source_filename,
                                revision=PROTOCOL_REVISION))


def _public_rows(repo: str, config: str | None, split: str) -> list[dict]:
    try:
        from datasets import load_dataset
    except ImportError as exc:
        raise RuntimeError("building from the public dataset needs the `datasets` package (or pass rows to the "
                           "builder directly)") from exc
    return [dict(r) for r in load_dataset(repo, config, split=split)]


def prepare_benchmark_data(name: str, *, output_dir: Path = DEFAULT_DATA_ROOT, source_dir: Path | None = None,
                           overwrite: bool = False, rows: list[dict] | None = None) -> Path:
    """Install the benchmark's JSONL into ``output_dir``; returns its path."""
    bench = get_benchmark(name)
    out = Path(output_dir) / bench.data_path.name
    if out.is_file() and not overwrite:
        validate_artifact(out, bench.expected_rows, bench.data_sha256)
        return out
    if source_dir is None and os.environ.get(SOURCE_DIR_ENV):
        source_dir = Path(os.environ[SOURCE_DIR_ENV])
    if bench.data_sha256 is not None and rows is None:
        if source_dir is not None:
            src = _find_source(Path(source_dir), bench.name, bench.source_filename)
        elif bench.source_filename:
            try:
                src = _download_pinned(bench.source_filename)
            except Exception as exc:
                raise RuntimeError(f"cannot obtain the pinned {bench.name} artifact: set {SOURCE_DIR_ENV} or pass "
                                   "--source-dir with a flat or repository-shaped protocol bundle") from exc
        else:  # pragma: no cover - every pinned entry names its file
            raise RuntimeError(f"{bench.name} has a pinned sha256 but no source file name")
        validate_artifact(src, bench.expected_rows, bench.data_sha256)
        _atomic_write(out, src.read_bytes())
        return out
    if bench.name not in BUILDERS:
        raise KeyError(f"no public-data builder for {bench.name}")
    builder, coords = BUILDERS[bench.name]
    records = builder(rows if rows is not None else _public_rows(*coords))
    if len(records) != bench.expected_rows:
        raise ValueError(f"{bench.name}: built {len(records)} rows, the protocol pins {bench.expected_rows}")
    _atomic_write(out, "".join(json.dumps(r, ensure_ascii=False) + "\n" for r in records).encode("utf-8"))
    return out


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("benchmarks", nargs="*", metavar="BENCHMARK")
    ap.add_argument("--output-dir", type=Path, default=DEFAULT_DATA_ROOT)
    ap.add_argument("--source-dir", type=Path)
    ap.add_argument("--overwrite", action="store_true")
    args = ap.parse_args(argv)
    names = [normalize_benchmark_name(b) for b in args.benchmarks] or list(BENCHMARKS)
    unknown = [n for n in names if n not in BENCHMARKS]
    if unknown:
        ap.error(f"unknown benchmark(s) {', '.join(unknown)}; choose from {', '.join(BENCHMARKS)}")
    for n in names:
        print(f"{n}: {prepare_benchmark_data(n, output_dir=args.output_dir, source_dir=args.source_dir, overwrite=args.overwrite)}")


if __name__ == "__main__":
    main()
