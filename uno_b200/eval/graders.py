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

import json
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
    """Math grading of the evaluation protocol (:mod:`uno_b200.eval.math_grading`, on
    ``math_verify``); without that package, the last boxed answer after the
    reasoning (else the last line) compared with sympy."""
    from uno_b200.eval import math_grading

    if math_grading.available():
        return math_grading.grade(generation, ground_truth)
    body = strip_reasoning(generation)
    pred = last_boxed(body)
    if pred is None:
        lines = [ln for ln in body.splitlines() if ln.strip()]
        pred = lines[-1] if lines else ""
    return {"prediction": pred, "correct": math_equal(pred, str(ground_truth))}


# ------------------------------------------------------------ multiple choice
def grade_multiple_choice(prediction: str | None, ground_truth: Any) -> dict:
    """The predicted option against the reference's first character (digits 1-5 read as A-E)."""
    from uno_b200.eval.parsers import normalise_choice

    truth = normalise_choice(str(ground_truth)[:1]) if ground_truth is not None else None
    return {"prediction": prediction,
            "correct": prediction is not None and truth is not None and prediction.strip().upper() == truth}


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


# ------------------------------------------------------- judge protocols
# The LLM-graded benchmarks (AA-LCR, HLE, AA-Omniscience) are graded by a
# judge model with fixed prompts and verdict formats; the prompt texts below
# are those benchmarks' grading protocol (as the reference evaluation sends
# them), because a different prompt changes the grades.  The judge reads only
# the visible answer, after the last reasoning block.  Verdicts: AA-LCR a JSON
# {"GRADE": ...} (or a bare CORRECT / INCORRECT); HLE a "correct: yes|no"
# line; AA-Omniscience one letter, A correct (+1), B incorrect (-1), C partial
# and D not attempted (0).  LCR endpoints come from UNO_LCR_JUDGE_URL /
# UNO_LCR_JUDGE_MODEL (key: UNO_LCR_JUDGE_API_KEY) when none is passed.
LCR_SYSTEM = "You are a teacher grading a quiz, and output JSON."
LCR_PROMPT = ("You are a teacher grading a quiz.\nYou are given a question, the student's answer, and the true "
              "answer, and are asked to score the student answer as either CORRECT or INCORRECT.\n\nExample "
              "Format:\nQUESTION: {query}\nSTUDENT ANSWER: {result}\nTRUE ANSWER: {answer}\n\nOutput:\n"
              "{{\"GRADE\": \"CORRECT\" or \"INCORRECT\"}}")
HLE_PROMPT = (
    "Judge whether the following [response] to [question] is correct or not based on the precise and "
    "unambiguous [correct_answer] below.\n\n[question]: {question}\n\n[response]: {response}\n\nYour judgement "
    "must be in the format and criteria specified below:\n\nextracted_final_answer: The final exact answer "
    "extracted from the [response]. Put the extracted answer as 'None' if there is no exact, final answer to "
    "extract from the response.\n\n[correct_answer]: {correct_answer}\n\nreasoning: Explain why the "
    "extracted_final_answer is correct or incorrect based on [correct_answer], focusing only on if there are "
    "meaningful differences between [correct_answer] and the extracted_final_answer. Do not comment on any "
    "background to the problem, do not attempt to solve the problem, do not argue for any answer different than "
    "[correct_answer], focus only on whether the answers match.\n\ncorrect: Answer 'yes' if "
    "extracted_final_answer matches the [correct_answer] given above, or is within a small margin of error for "
    "numerical problems. Answer 'no' otherwise, i.e. if there if there is any inconsistency, ambiguity, "
    "non-equivalency, or if the extracted answer is incorrect.\n\nconfidence: The extracted confidence score "
    "between 0% and 100% from [response]. Put 100 if there is no confidence score available.")
OMNISCIENCE_PROMPT = (
    "Your job is to look at a question, a gold target, and a predicted answer, and then assign a grade of either "
    "[\"CORRECT\", \"INCORRECT\", \"PARTIAL_ANSWER\", \"NOT_ATTEMPTED\"].\n\nCORRECT: The answer fully matches or "
    "is equivalent to the gold target\nINCORRECT: The answer contradicts or differs in meaning from the gold "
    "target\nPARTIAL_ANSWER: The answer is accurate and nearly complete but not at the correct level of detail\n"
    "NOT_ATTEMPTED: Used only when the model refuses, omits, or explicitly states it does not know the answer, or "
    "needs more context or tools to answer the question\n\nHere is a new example.\n\nQuestion: {question}\n"
    "Gold target: {target}\nPredicted answer: {predicted_answer}\n\nGrade the predicted answer of this new "
    "question as one of:\nA: CORRECT\nB: INCORRECT\nC: PARTIAL_ANSWER\nD: NOT_ATTEMPTED\n\nJust return the "
    "letters \"A\", \"B\", \"C\", or \"D\", with no text around it.")
JUDGED_TASKS = ("aa_lcr", "hle", "aa_omniscience")
OMNISCIENCE_DENOMINATOR = 600  # the benchmark's question count: scores are per question of the full set
_THINK_CLOSE = re.compile(r"</(?:ifm\|)?think[^>]*>", re.IGNORECASE)


def visible_answer(text: str | None) -> str:
    """The text after the last reasoning block."""
    value = text or ""
    closes = list(_THINK_CLOSE.finditer(value))
    return value[closes[-1].end():].strip() if closes else value.strip()


def judge_messages(task: str, question: str, answer: Any, response: str) -> list[dict]:
    response = response or "No answer"
    if task == "aa_lcr":
        q = question.split("\n=== QUESTION ===\n")[-1]
        if q.endswith("\n\nAnswer:"):
            q = q[: -len("\n\nAnswer:")]
        return [{"role": "system", "content": LCR_SYSTEM},
                {"role": "user", "content": LCR_PROMPT.format(query=q.strip(), result=response, answer=answer)}]
    if task == "hle":
        return [{"role": "user", "content": HLE_PROMPT.format(question=question, response=response,
                                                              correct_answer=answer)}]
    if task == "aa_omniscience":
        return [{"role": "user", "content": OMNISCIENCE_PROMPT.format(question=question, target=answer,
                                                                      predicted_answer=response)}]
    raise ValueError(f"no judge protocol for task {task!r}")


def parse_verdict(task: str, reply: str | None) -> int:
    """+1 correct, -1 incorrect (AA-Omniscience only), 0 otherwise."""
    text = visible_answer(reply)
    if task == "hle":
        m = re.search(r'"?correct"?\s*:\s*"?(yes|no)"?', text, re.IGNORECASE)
        return int(bool(m) and m.group(1).lower() == "yes")
    if task == "aa_omniscience":
        m = re.search(r"\b([ABCD])\b", text.upper())
        return {"A": 1, "B": -1}.get(m.group(1), 0) if m else 0
    braces = re.search(r"\{.*\}", text, re.DOTALL)
    if braces:
        try:
            obj = json.loads(braces.group(0))
            grade = obj.get("GRADE", obj.get("grade"))
            if isinstance(obj.get("answer"), dict):
                grade = obj["answer"].get("GRADE", obj["answer"].get("grade", grade))
            if isinstance(grade, str):
                return int(grade.upper() == "CORRECT")
        except ValueError:
            pass
    m = re.search(r"\b(CORRECT|INCORRECT)\b", text, re.IGNORECASE)
    return int(bool(m) and m.group(1).upper() == "CORRECT")


def lcr_transport_from_env() -> Callable:
    url = os.environ.get("UNO_LCR_JUDGE_URL")
    if not url or not os.environ.get("UNO_LCR_JUDGE_MODEL"):
        raise RuntimeError("AA-LCR grading needs UNO_LCR_JUDGE_URL and UNO_LCR_JUDGE_MODEL")
    url = url.rstrip("/")
    if not url.endswith("/v1"):
        url += "/v1"
    return http_chat_transport(url, os.environ.get("UNO_LCR_JUDGE_API_KEY"))


def grade_judged(task: str, question: str, response: str, answer: Any, *, transport: Callable, model: str,
                 temperature: float | None = None, max_tokens: int | None = None,
                 reasoning_effort: str | None = None) -> dict:
    """One judge call under the task's protocol: ``{"grade", "correct", "judge"}``."""
    payload = {"model": model, "messages": judge_messages(task, question, answer, response)}
    if temperature is not None:
        payload["temperature"] = float(temperature)
    if max_tokens is not None:
        payload["max_tokens"] = int(max_tokens)
    if reasoning_effort:
        payload["reasoning_effort"] = reasoning_effort
    try:
        reply = transport(payload)
    except Exception as exc:  # a failed judge call grades 0, as the protocol does
        return {"grade": 0, "correct": False, "judge_error": str(exc)[:256]}
    grade = parse_verdict(task, reply)
    return {"grade": grade, "correct": grade == 1, "judge": (reply or "")[:256]}


def grade_lcr(question: str, answer: str, reference: Any, *, transport: Callable | None = None,
              model: str | None = None, temperature: float | None = None, max_tokens: int | None = None,
              reasoning_effort: str | None = None) -> dict:
    """AA-LCR grade (``grade_judged`` with the endpoint from the environment when none is given)."""
    return grade_judged("aa_lcr", question, answer, reference, transport=transport or lcr_transport_from_env(),
                        model=model or os.environ.get("UNO_LCR_JUDGE_MODEL", "judge"), temperature=temperature,
                        max_tokens=max_tokens, reasoning_effort=reasoning_effort)