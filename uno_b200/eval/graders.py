"""Graders: math equivalence, multiple choice, sandboxed code execution, LLM judge.

Behaviour of ``evaluation/graders/*.py``:

* **math** -- the parsed answer (boxed, else the final line) is equivalent to
  the reference if the normalised strings match or, failing that, the two
  parse to numerically / symbolically equal expressions (LaTeX fractions,
  roots and powers are rewritten for sympy);
* **multiple choice** -- option letters compare case-insensitively;
* **code** -- the program plus the task's tests runs in a fresh Python
  subprocess in a temporary directory, with a stripped environment (no
  proxies, tokens or user site), a CPU-time/wall timeout and a memory cap;
  it passes iff the process exits 0 (``evaluation/graders/code.py:106-124``);
* **LLM judge** -- an OpenAI-compatible chat-completions endpoint grades free
  answers; the transport is injectable so the grader runs without network.
"""

from __future__ import annotations

import os
import re
import subprocess
import sys
import tempfile
from typing import Any, Callable

from uno_b200.eval.parsers import last_boxed, strip_reasoning

# --------------------------------------------------------------------- math
_TEXT = re.compile(r"\\text\{([^{}]*)\}")


def normalize_math(ans: str | None) -> str:
    if ans is None:
        return ""
    s = str(ans).strip()
    s = _TEXT.sub(r"\1", s)
    for tok in ("\\left", "\\right", "\\!", "\\,", "\\;", "\\displaystyle", "$", "\\%", "%", "^\\circ",
                "^{\\circ}", "\\dfrac", "\\tfrac"):
        s = s.replace(tok, "\\frac" if tok in ("\\dfrac", "\\tfrac") else "")
    s = s.replace(" ", "").rstrip(".")
    if s.startswith("x=") or s.startswith("y="):
        s = s[2:]
    if re.fullmatch(r"-?\d{1,3}(,\d{3})+(\.\d+)?", s):
        s = s.replace(",", "")
    return s


def _latex_to_sympy(s: str) -> str:
    prev = None
    while prev != s:  # innermost first
        prev = s
        s = re.sub(r"\\frac\{([^{}]*)\}\{([^{}]*)\}", r"((\1)/(\2))", s)
        s = re.sub(r"\\sqrt\{([^{}]*)\}", r"sqrt(\1)", s)
    s = re.sub(r"\\frac(\d)(\d)", r"((\1)/(\2))", s)
    s = s.replace("\\pi", "pi").replace("\\cdot", "*").replace("\\times", "*").replace("^", "**")
    s = s.replace("{", "(").replace("}", ")")
    return s


def math_equal(pred: str | None, truth: str | None, tol: float = 1e-6) -> bool:
    a, b = normalize_math(pred), normalize_math(truth)
    if not a or not b:
        return False
    if a == b:
        return True
    try:
        import sympy
        from sympy.parsing.sympy_parser import (implicit_multiplication_application, parse_expr,
                                                standard_transformations)

        tr = standard_transformations + (implicit_multiplication_application,)
        ea = parse_expr(_latex_to_sympy(a), transformations=tr)
        eb = parse_expr(_latex_to_sympy(b), transformations=tr)
        if sympy.simplify(ea - eb) == 0:
            return True
        return abs(complex(ea.evalf()) - complex(eb.evalf())) <= tol * max(1.0, abs(complex(eb.evalf())))
    except Exception:
        return False


def grade_math(generation: str, ground_truth: Any) -> dict:
    body = strip_reasoning(generation)
    pred = last_boxed(body)
    if pred is None:
        lines = [ln for ln in body.splitlines() if ln.strip()]
        pred = lines[-1] if lines else ""
    return {"prediction": pred, "correct": math_equal(pred, str(ground_truth))}


# ------------------------------------------------------------ multiple choice
def grade_multiple_choice(prediction: str | None, ground_truth: Any) -> dict:
    truth = str(ground_truth).strip().upper()
    return {"prediction": prediction, "correct": prediction is not None and prediction.strip().upper() == truth}


# ------------------------------------------------------------------- code
_SAFE_ENV_KEYS = ("PATH", "LANG", "LC_ALL", "SYSTEMROOT")


def run_code_sandboxed(program: str, timeout: float = 10.0, memory_mb: int = 2048) -> dict:
    env = {k: os.environ[k] for k in _SAFE_ENV_KEYS if k in os.environ}
    env.update(PYTHONDONTWRITEBYTECODE="1", PYTHONNOUSERSITE="1", PYTHONHASHSEED="0")

    def limits():  # runs in the child before exec
        try:
            import resource

            resource.setrlimit(resource.RLIMIT_AS, (memory_mb << 20, memory_mb << 20))
            cpu = int(timeout) + 1
            resource.setrlimit(resource.RLIMIT_CPU, (cpu, cpu))
        except (ImportError, ValueError, OSError):
            pass
        os.setsid()

    with tempfile.TemporaryDirectory(prefix="uno_eval_") as tmp:
        path = os.path.join(tmp, "program.py")
        with open(path, "w", encoding="utf-8") as fh:
            fh.write(program)
        try:
            proc = subprocess.run([sys.executable, "-I", path], cwd=tmp, env=env, capture_output=True, text=True,
                                  timeout=timeout, preexec_fn=limits)
        except subprocess.TimeoutExpired:
            return {"passed": False, "status": "timeout"}
        return {"passed": proc.returncode == 0, "status": "ok" if proc.returncode == 0 else "failed",
                "stderr": proc.stderr[-2000:]}


def grade_code(code: str | None, record: dict, timeout: float = 10.0) -> dict:
    """HumanEval-style (``prompt``/``test``/``entry_point``) or MBPP-style (``test_list``) tasks."""
    if not code:
        return {"correct": False, "status": "no code"}
    if "test" in record and "entry_point" in record:
        prefix = record.get("prompt", "") if f"def {record['entry_point']}" not in code else ""
        program = f"{prefix}{code}\n\n{record['test']}\n\ncheck({record['entry_point']})\n"
    elif "test_list" in record:
        setup = record.get("test_setup_code", "")
        program = "\n".join([setup, code, *record["test_list"]]) + "\n"
    elif "tests" in record:
        program = f"{code}\n\n{record['tests']}\n"
    else:
        raise ValueError("code record needs test/entry_point, test_list or tests")
    res = run_code_sandboxed(program, timeout)
    return {"correct": res["passed"], "status": res["status"]}


# -------------------------------------------------------------- LLM judge
JUDGE_TEMPLATE = ("Judge whether the response answers the question correctly, compared with the reference "
                  "answer. Reply with exactly CORRECT or INCORRECT.\n\nQuestion:\n{question}\n\nReference answer:\n"
                  "{answer}\n\nResponse:\n{response}")


def http_chat_transport(base_url: str, api_key: str | None = None, timeout: float = 300.0) -> Callable:
    """POST ``{base_url}/chat/completions`` (OpenAI-compatible) and return the message text."""
    def send(payload: dict) -> str:
        import requests

        headers = {"Authorization": f"Bearer {api_key}"} if api_key else {}
        r = requests.post(base_url.rstrip("/") + "/chat/completions", json=payload, headers=headers,
                          timeout=timeout)
        r.raise_for_status()
        return r.json()["choices"][0]["message"]["content"]

    return send


def _judge_payload(model: str, content: str, temperature: float | None, max_tokens: int | None,
                   reasoning_effort: str | None, default_max_tokens: int) -> dict:
    payload = {"model": model, "temperature": 0.0 if temperature is None else float(temperature),
               "max_tokens": default_max_tokens if max_tokens is None else int(max_tokens),
               "messages": [{"role": "user", "content": content}]}
    if reasoning_effort:
        payload["reasoning_effort"] = reasoning_effort
    return payload


def grade_with_judge(question: str, answer: Any, response: str, *, model: str, transport: Callable,
                     temperature: float | None = None, max_tokens: int | None = None,
                     reasoning_effort: str | None = None) -> dict:
    payload = _judge_payload(model, JUDGE_TEMPLATE.format(question=question, answer=answer,
                                                          response=strip_reasoning(response)),
                             temperature, max_tokens, reasoning_effort, 4096)
    verdict = transport(payload).strip().upper()
    return {"judge": verdict[:64], "correct": verdict.startswith("CORRECT")}


# ------------------------------------------------------------------ AA-LCR
# Behaviour of ``evaluation/graders/lcr.py``: a judge model sees the question,
# the candidate answer and the reference answer and must reply with a JSON
# grade; anything without a parsable ``"GRADE"`` counts as incorrect.  The
# endpoint and model come from UNO_LCR_JUDGE_URL / UNO_LCR_JUDGE_MODEL (key:
# UNO_LCR_JUDGE_API_KEY); a base URL without ``/v1`` gets it appended.
LCR_TEMPLATE = ("Decide whether the candidate answer to the question below is semantically correct, using the "
                "reference answer as ground truth. Respond with only {{\"GRADE\":\"CORRECT\"}} or "
                "{{\"GRADE\":\"INCORRECT\"}}.\n\nQuestion:\n{question}\n\nCandidate answer:\n{answer}\n\n"
                "Reference answer:\n{reference}")
_LCR_GRADE = re.compile(r'"GRADE"\s*:\s*"(CORRECT|INCORRECT)"', re.IGNORECASE)


def lcr_transport_from_env() -> Callable:
    url = os.environ.get("UNO_LCR_JUDGE_URL")
    if not url or not os.environ.get("UNO_LCR_JUDGE_MODEL"):
        raise RuntimeError("AA-LCR grading needs UNO_LCR_JUDGE_URL and UNO_LCR_JUDGE_MODEL")
    url = url.rstrip("/")
    if not url.endswith("/v1"):
        url += "/v1"
    return http_chat_transport(url, os.environ.get("UNO_LCR_JUDGE_API_KEY"))


def grade_lcr(question: str, answer: str, reference: Any, *, transport: Callable | None = None,
              model: str | None = None, temperature: float | None = None, max_tokens: int | None = None,
              reasoning_effort: str | None = None) -> dict:
    transport = transport or lcr_transport_from_env()
    model = model or os.environ.get("UNO_LCR_JUDGE_MODEL", "judge")
    payload = _judge_payload(model, LCR_TEMPLATE.format(question=question, answer=strip_reasoning(answer),
                                                        reference=reference),
                             temperature, max_tokens, reasoning_effort, 32)
    reply = transport(payload)
    m = _LCR_GRADE.search(reply or "")
    return {"judge": (reply or "")[:256], "correct": bool(m) and m.group(1).upper() == "CORRECT"}
