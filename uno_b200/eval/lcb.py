"""LiveCodeBench (v6) grading: run generated programs against the task's tests.

Behaviour of ``evaluation/graders/lcb.py`` and ``evaluation/lcb_utils.py``:

* the program is the last fenced code block of the completion (a short
  language label on the fence's first line is dropped), else the whole text;
* ``ground_truth`` is a JSON list of ``{"input", "output", "testtype"}``
  objects, all of one type: ``stdin`` programs read the input text and print;
  ``functional`` tests call ``method_name`` (on ``Solution()`` when the program
  defines that class) with one JSON value per input line as arguments and
  compare the return value with the JSON output (tuples count as lists);
* stdin output matches when the stripped lines agree one by one, either
  exactly or as whitespace-separated numbers compared as decimals;
* tests run in order and stop at the first failure; per-test codes are
  ``True`` (pass), ``-2`` (wrong answer), ``-3`` (time limit), ``-4``
  (compile or runtime error); a generation is correct iff every code is
  positive;
* pass@k uses the unbiased estimator 1 - C(n-c, k)/C(n, k) (Chen et al.,
  "Evaluating Large Language Models Trained on Code", 2021).

Isolation is this module's own: each generation runs in a fresh ``python -I``
subprocess in a temporary directory (stripped environment, address-space and
CPU limits, own session) that executes a small harness; the harness runs the
tests with a per-test alarm and prints one JSON line of codes.
"""

from __future__ import annotations

import json
import os
import re
import subprocess
import sys
import tempfile
from concurrent.futures import ThreadPoolExecutor
from typing import Any

_FENCE = re.compile(r"```[^\n`]*\n?(.*?)```", re.DOTALL)
_LABEL = re.compile(r"[A-Za-z0-9_.+-]+")

PASS, WRONG, TIMEOUT, ERROR = True, -2, -3, -4


def extract_python_code(completion: str | None) -> str:
    text = "" if completion is None else str(completion)
    if not text.strip():
        return ""
    blocks = _FENCE.findall(text)
    if not blocks:
        return text.strip()
    block = blocks[-1].strip()
    first, sep, rest = block.partition("\n")
    if sep and len(first.strip()) < 32 and _LABEL.fullmatch(first.strip()):
        return rest.strip()
    return block


def parse_tests(ground_truth: Any) -> dict[str, Any]:
    """Normalise a row's tests to ``{"mode", "inputs", "outputs", "fn_name"}``."""
    tests = json.loads(ground_truth) if isinstance(ground_truth, str) else ground_truth
    if not isinstance(tests, list) or not tests:
        raise ValueError("LiveCodeBench ground_truth must be a non-empty JSON list of test cases")
    kinds = {t.get("testtype", "stdin") for t in tests}
    if len(kinds) != 1:
        raise ValueError(f"mixed LiveCodeBench test types: {sorted(kinds)}")
    mode = kinds.pop()
    if mode not in ("stdin", "functional"):
        raise ValueError(f"unsupported LiveCodeBench test type {mode!r}")
    fn_name = tests[0].get("method_name") if mode == "functional" else None
    if mode == "functional" and not fn_name:
        raise ValueError("functional LiveCodeBench tests need method_name")
    return {"mode": mode, "inputs": [t["input"] for t in tests], "outputs": [t["output"] for t in tests],
            "fn_name": fn_name}


# The harness runs inside the sandboxed interpreter; it only uses the standard library.
_HARNESS = r'''
import builtins, io, json, signal, sys
from decimal import Decimal, InvalidOperation

try:
    sys.set_int_max_str_digits(0)
except AttributeError:
    pass
sys.setrecursionlimit(50000)
PRELUDE = ("from string import *\nfrom re import *\nfrom datetime import *\nfrom collections import *\n"
           "from heapq import *\nfrom bisect import *\nfrom copy import *\nfrom math import *\n"
           "from random import *\nfrom statistics import *\nfrom itertools import *\nfrom functools import *\n"
           "from operator import *\nfrom io import *\nfrom sys import *\nfrom json import *\n"
           "from builtins import *\nfrom typing import *\nimport string, re, datetime, collections, heapq, "
           "bisect, copy, math, random, statistics, itertools, functools, operator, io, sys, json\n")

class Alarm(Exception):
    pass

def on_alarm(signum, frame):
    raise Alarm()

signal.signal(signal.SIGALRM, on_alarm)
spec = json.load(open(sys.argv[1], encoding="utf-8"))
code, per_test = spec["code"], int(spec["timeout"])

def lines(text):
    return [ln.strip() for ln in str(text).strip().split("\n")]

def as_decimals(line):
    try:
        return [Decimal(x) for x in line.split()]
    except (InvalidOperation, ValueError):
        return None

def same_output(got, want):
    a, b = lines(got), lines(want)
    if len(a) != len(b):
        return False
    for x, y in zip(a, b):
        if x == y:
            continue
        dx, dy = as_decimals(x), as_decimals(y)
        if dx is None or dy is None or dx != dy:
            return False
    return True

codes = []
real_stdin, real_stdout = sys.stdin, sys.stdout
try:
    compiled = compile(PRELUDE + "\n" + code, "<solution>", "exec")
except BaseException:
    compiled = None
if compiled is None:
    codes = [-4]
elif spec["mode"] == "functional":
    env = {"__name__": "solution"}
    try:
        signal.alarm(per_test)
        exec(compiled, env)
        signal.alarm(0)
        target = env["Solution"]() if "Solution" in env else env
        fn = getattr(target, spec["fn_name"]) if "Solution" in env else env[spec["fn_name"]]
    except BaseException:
        signal.alarm(0)
        fn = None
        codes = [-4]
    if fn is not None:
        for raw_in, raw_out in zip(spec["inputs"], spec["outputs"]):
            try:
                args = [json.loads(ln) for ln in raw_in.split("\n")]
                want = json.loads(raw_out)
                signal.alarm(per_test)
                got = fn(*args)
                signal.alarm(0)
            except Alarm:
                codes.append(-3)
                break
            except BaseException:
                signal.alarm(0)
                codes.append(-4)
                break
            if isinstance(got, tuple):
                got = list(got)
            ok = got == want
            codes.append(True if ok else False)
            if not ok:
                break
else:
    for raw_in, raw_out in zip(spec["inputs"], spec["outputs"]):
        buf = io.StringIO()
        sys.stdin, sys.stdout = io.StringIO(raw_in), buf
        try:
            signal.alarm(per_test)
            exec(compiled, {"__name__": "__main__"})
            signal.alarm(0)
            status = None
        except Alarm:
            status = -3
        except SystemExit:
            signal.alarm(0)
            status = None
        except BaseException:
            signal.alarm(0)
            status = -4
        finally:
            sys.stdin, sys.stdout = real_stdin, real_stdout
        if status is not None:
            codes.append(status)
            break
        if not same_output(buf.getvalue(), raw_out):
            codes.append(-2)
            break
        codes.append(True)
real_stdout.write("\n__LCB_RESULT__" + json.dumps(codes) + "\n")
'''

_SAFE_ENV = ("PATH", "LANG", "LC_ALL")


def run_generation(code: str, tests: dict[str, Any], timeout: int = 6, memory_mb: int = 4096) -> list:
    """Codes of one generation against one task's tests (see the module docstring)."""
    if not code:
        return [ERROR]
    env = {k: os.environ[k] for k in _SAFE_ENV if k in os.environ}
    env.update(PYTHONDONTWRITEBYTECODE="1", PYTHONNOUSERSITE="1", PYTHONHASHSEED="0")
    n = max(1, len(tests["inputs"]))
    wall = timeout * n + 10

    def limits():
        try:
            import resource

            resource.setrlimit(resource.RLIMIT_AS, (memory_mb << 20, memory_mb << 20))
            resource.setrlimit(resource.RLIMIT_CPU, (wall, wall))
        except (ImportError, ValueError, OSError):
            pass
        os.setsid()

    with tempfile.TemporaryDirectory(prefix="uno_lcb_") as tmp:
        spec = os.path.join(tmp, "spec.json")
        harness = os.path.join(tmp, "harness.py")
        with open(spec, "w", encoding="utf-8") as fh:
            json.dump({"code": code, "timeout": int(timeout), **tests}, fh)
        with open(harness, "w", encoding="utf-8") as fh:
            fh.write(_HARNESS)
        try:
            proc = subprocess.run([sys.executable, "-I", harness, spec], cwd=tmp, env=env, capture_output=True,
                                  text=True, timeout=wall, preexec_fn=limits)
        except subprocess.TimeoutExpired:
            return [TIMEOUT]
    marker = proc.stdout.rfind("__LCB_RESULT__")
    if marker < 0:
        return [ERROR]
    try:
        return json.loads(proc.stdout[marker + len("__LCB_RESULT__"):].strip().splitlines()[0])
    except (ValueError, IndexError):
        return [ERROR]


def generation_passed(codes: list) -> bool:
    return bool(codes) and all(c is True or (not isinstance(c, bool) and c > 0) for c in codes)


def pass_at_k(n: int, c: int, k: int) -> float:
    """Unbiased pass@k of one task with n samples of which c pass."""
    if n - c < k:
        return 1.0
    prob_all_fail = 1.0
    for i in range(n - c + 1, n + 1):
        prob_all_fail *= 1.0 - k / i
    return 1.0 - prob_all_fail


def score_lcb(rows: list[dict[str, Any]], *, timeout: int = 6, workers: int | None = None) -> tuple[list, dict]:
    """Grade rows ``{"ground_truth", "generations" | "generation", ...}``; returns (graded rows, summary)."""
    jobs = []
    per_row = []
    for i, row in enumerate(rows):
        tests = parse_tests(row.get("ground_truth"))
        gens = row.get("generations")
        if gens is None:
            gens = [row.get("generation", "")]
        codes = [extract_python_code(g) for g in gens]
        per_row.append(len(codes))
        jobs.extend((i, j, c, tests) for j, c in enumerate(codes))
    results: dict[tuple[int, int], list] = {}
    workers = workers or min(32, os.cpu_count() or 1)
    with ThreadPoolExecutor(max_workers=workers) as pool:
        futs = {pool.submit(run_generation, c, t, timeout): (i, j) for i, j, c, t in jobs}
        for fut, key in futs.items():
            results[key] = fut.result()
    graded, all_ok, counts = [], [], []
    for i, row in enumerate(rows):
        codes = [results[(i, j)] for j in range(per_row[i])]
        ok = [generation_passed(c) for c in codes]
        all_ok.extend(ok)
        counts.append((len(ok), sum(ok)))
        graded.append({**row, "correct": ok, "test_results": codes,
                       "accuracy": sum(ok) / len(ok) if ok else float("nan"), "grader": "lcb_subprocess"})
    summary: dict[str, Any] = {"grader": "lcb_subprocess", "num_rows": len(rows), "num_generations": len(all_ok),
                               "num_correct": sum(all_ok),
                               "accuracy": sum(all_ok) / len(all_ok) if all_ok else float("nan"),
                               "timeout": timeout}
    for k in (1, 5):
        if counts and all(n >= k for n, _ in counts):
            summary[f"pass@{k}"] = sum(pass_at_k(n, c, k) for n, c in counts) / len(counts)
    return graded, summary
