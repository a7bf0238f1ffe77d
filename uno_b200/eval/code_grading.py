"""HumanEval and MBPP grading of the evaluation protocol (``evaluation/graders/code.py``).

HumanEval: the parsed completion (``code_completion``: the text after the
first reasoning block, the first fenced Python block) is taken from its own
fence when it still has one, loses a repeated prompt, and then either replaces
the prompt's signature (a complete re-emitted function, which may rename
parameters) or loses a re-emitted signature and docstring; the program is
prompt + completion + the tests + ``check(entry_point)``.

MBPP: from the raw generation, the first fenced block that defines a function
the asserts call, else the first block that looks like Python, else the rest
after an unclosed fence, else the bare text when it looks like Python; the
program is that code followed by the asserts.

A program passes when it exits 0 in the sandbox (``graders.run_code_sandboxed``).
Records are the prepared protocol rows (``ground_truth`` with the tests,
``completion_input`` with the HumanEval prompt) or the datasets' own rows
(``prompt`` / ``test`` / ``entry_point``, ``test_list``).
"""

from __future__ import annotations

import json
import re
from typing import Any

_PY_BLOCK = re.compile(r"```(?:python|py)\s*\n(.*?)\n?```", re.DOTALL | re.IGNORECASE)
_ANY_BLOCK = re.compile(r"```(?:[A-Za-z0-9_+-]*)\s*\n(.*?)\n?```", re.DOTALL)
_PY_START = re.compile(r"(?m)^\s*(?:from\s+\S+\s+import\s+|import\s+|def\s+|class\s+)")
_ASSERTED = re.compile(r"assert\s+([A-Za-z_]\w*)\s*\(")
_DEFINED = re.compile(r"(?m)^\s*def\s+([A-Za-z_]\w*)\s*\(")
_FIRST_FENCE = re.compile(r"```(?:python|py)?\s*\n(.*?)```", re.DOTALL)
_OPEN_FENCE = re.compile(r"```(?:python|py)?\s*\n")


# ------------------------------------------------------------------ MBPP
def _bare(text: str) -> str:
    """A code block without chat scaffolding: a leading 'thought' line, a closing fence,
    language / BEGIN lines on top, DONE / END lines at the bottom, prose before the code."""
    t = text.strip()
    if t.startswith("thought\n"):
        t = t[len("thought\n"):].lstrip()
    if t.endswith("```"):
        t = t[:-3].rstrip()
    lines = t.splitlines()
    while lines and lines[0].strip().lower() in {"python", "py"}:
        lines.pop(0)
    while lines and lines[0].strip() in {"[BEGIN]", "BEGIN"}:
        lines.pop(0)
    while lines and lines[-1].strip() in {"[DONE]", "DONE", "[END]", "END"}:
        lines.pop()
    t = "\n".join(lines).strip()
    start = _PY_START.search(t)
    return t[start.start():].lstrip() if start and start.start() > 0 else t


def extract_mbpp_code(text: str, tests: str | None = None) -> str:
    if not text:
        return ""
    blocks, seen = [], set()
    for raw in _PY_BLOCK.findall(text) + _ANY_BLOCK.findall(text):
        b = _bare(raw)
        if b and b not in seen:
            seen.add(b)
            blocks.append(b)
    wanted = set(_ASSERTED.findall(tests or ""))
    for b in blocks:
        if wanted & set(_DEFINED.findall(b)):
            return b
    for b in blocks:
        if _PY_START.search(b):
            return b
    open_fence = re.search(r"```(?:[A-Za-z0-9_+-]*)\s*\n", text)
    if open_fence:
        return _bare(text[open_fence.end():])
    b = _bare(text)
    return b if _PY_START.search(b) else ""


def mbpp_tests(record: dict) -> str:
    tests = record.get("ground_truth", record.get("test_list"))
    if isinstance(tests, list):
        tests = "\n".join(str(t) for t in tests)
    return str(tests or "")


def grade_mbpp(generation: str, record: dict, timeout: float = 10.0) -> dict:
    from uno_b200.eval.graders import run_code_sandboxed

    tests = mbpp_tests(record)
    code = extract_mbpp_code(generation or "", tests)
    if not code:
        return {"correct": False, "status": "no code", "picked": ""}
    res = run_code_sandboxed(code + "\n" + tests + "\n", timeout)
    return {"correct": res["passed"], "status": res["status"], "picked": code[:400]}


# ------------------------------------------------------------- HumanEval
def _fenced(text: str) -> str:
    m = _FIRST_FENCE.search(text)
    if m:
        return m.group(1)
    m = _OPEN_FENCE.search(text)
    return text[m.end():] if m else text


def _drop_signature(completion: str, entry_point: str) -> str:
    """Remove a re-emitted ``def entry_point(...):`` line (and a docstring right after it)."""
    m = re.match(rf"^\s*def\s+{re.escape(entry_point)}\s*\(.*?\)\s*(?:->.*?)?:\s*\n", completion, re.DOTALL)
    if not m:
        return completion
    body = completion[m.end():]
    doc = re.match(r'\s*""".*?"""\s*\n', body, re.DOTALL)
    return body[doc.end():] if doc else body


def humaneval_program(prompt: str, test: str, entry_point: str, completion: str) -> tuple[str, str]:
    """``(program, completion used)`` of one HumanEval completion."""
    if "```" in completion:
        completion = _fenced(completion)
    if completion.startswith(prompt):
        completion = completion[len(prompt):]
    full_def = re.match(rf"^[ \t]*(?:async[ \t]+)?def[ \t]+{re.escape(entry_point)}[ \t]*\(", completion)
    prompt_def = re.search(rf"(?m)^[ \t]*(?:async[ \t]+)?def[ \t]+{re.escape(entry_point)}[ \t]*\(", prompt)
    if full_def is not None and prompt_def is not None:
        # a whole function: it replaces the prompt's signature and docstring (keeping its own parameter names)
        prompt, completion = prompt[: prompt_def.start()], completion.lstrip()
    else:
        completion = _drop_signature(completion, entry_point)
    return f"{prompt}{completion}\n{test}\ncheck({entry_point})", completion


def humaneval_problem(record: dict) -> tuple[str, str, str]:
    gt = record.get("ground_truth")
    if isinstance(gt, str):
        gt = json.loads(gt)
    if isinstance(gt, dict) and "test" in gt:
        return str(record.get("completion_input") or record.get("prompt") or ""), str(gt["test"]), \
            str(gt["entry_point"])
    return str(record.get("prompt", "")), str(record["test"]), str(record["entry_point"])


def grade_humaneval(completion: str, record: dict, timeout: float = 10.0) -> dict:
    from uno_b200.eval.graders import run_code_sandboxed

    prompt, test, entry = humaneval_problem(record)
    program, used = humaneval_program(prompt, test, entry, completion or "")
    res = run_code_sandboxed(program, timeout)
    return {"correct": res["passed"], "status": res["status"], "picked": used[:400]}


def is_humaneval_record(record: dict) -> bool:
    gt = record.get("ground_truth")
    if isinstance(gt, str) and gt.lstrip().startswith("{"):
        try:
            gt = json.loads(gt)
        except ValueError:
            return False
    return (isinstance(gt, dict) and "entry_point" in gt) or ("entry_point" in record and "test" in record)


def grade_code_record(generation: str, parsed: str | None, record: dict, timeout: float = 10.0) -> dict:
    """HumanEval rows grade the parsed completion; MBPP rows extract from the raw generation."""
    if is_humaneval_record(record):
        return grade_humaneval(parsed if parsed is not None else generation, record, timeout)
    return grade_mbpp(generation, record, timeout)
