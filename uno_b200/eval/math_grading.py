"""Math answer grading of the evaluation protocol (AIME, MATH-500, GSM8K).

Behaviour of ``evaluation/graders/math.py``; the steps and their order decide
which answers count, so they are kept:

1. candidates: the content of the last ``\\boxed{}`` / ``\\fbox{}`` anywhere in
   the generation, as a parsed expression, as normalised text and as written;
   with no box, one answer read from the text (a math parse of the whole
   text, then "the answer is ..." style phrases, a trailing "= N", a
   sentence ending in a verb and a number, and finally the last number of the
   last sentence that has one);
2. a candidate matches a reference answer when the normalised texts agree
   (or as numbers, as a lettered choice, or component-wise for vectors), or
   when ``math_verify`` finds them equivalent in either direction.

``math_verify`` (Hugging Face Math-Verify) parses and compares LaTeX
expressions; this module is a thin protocol layer around it.
"""

from __future__ import annotations

import re
import threading
from typing import Any

try:  # the grader needs math_verify; the import is checked when grading
    from math_verify import parse as _mv_parse, verify as _mv_verify
except ImportError:  # pragma: no cover - the evaluation image ships it
    _mv_parse = _mv_verify = None


def _main_thread() -> bool:
    return threading.current_thread() is threading.main_thread()


# math_verify bounds each parse / comparison with a SIGALRM timer, which only the
# main thread may set; grading threads run without that bound.
def mv_parse(text: str):
    return _mv_parse(text) if _main_thread() else _mv_parse(text, parsing_timeout=None)


def mv_verify(gold, target) -> bool:
    return _mv_verify(gold, target) if _main_thread() else _mv_verify(gold, target, timeout_seconds=None)


def available() -> bool:
    return _mv_parse is not None


def last_boxed_content(text: str | None) -> str | None:
    """Content of the last ``\\boxed{...}`` or ``\\fbox{...}`` with balanced braces, ``$`` stripped."""
    if not text:
        return None
    for m in reversed(list(re.finditer(r"\\(?:boxed|fbox)\s*\{", text, flags=re.IGNORECASE))):
        depth, i = 1, m.end()
        while i < len(text) and depth:
            depth += {"{": 1, "}": -1}.get(text[i], 0)
            i += 1
        if depth == 0:
            return text[m.end(): i - 1].strip().strip("$").strip()
    return None


# Normalisation of an answer text, applied in order.
_NORMALISE = [
    (re.compile(r"\\(?:boxed|fbox)\s*\{(.+)\}\s*$"), r"\1"),
    (re.compile(r"\\[dt]frac"), r"\\frac"),
    (re.compile(r"\\(?:left|right|bigl|bigr|Bigl|Bigr|big|Big)"), ""),
    (re.compile(r"\\displaystyle"), ""),
    (re.compile(r"\\mathbf\s*\{([^{}]+)\}"), r"\1"),
    (re.compile(r"\\mathbf\s+([A-Za-z])"), r"\1"),
    (re.compile(r"\\\\\s*\[[^\]]+\]"), r"\\\\"),
    (re.compile(r"\\frac\s*\{([^{}]+)\}\s*\{([^{}]+)\}"), r"\1/\2"),
    (re.compile(r"\\frac\s*([+-]?\d+)\s*([+-]?\d+)"), r"\1/\2"),
    (re.compile(r"\{,\}"), ""),
    (re.compile(r"\\(?:,|;|!|:)"), ""),
    (re.compile(r"\\%"), "%"),
    (re.compile(r"\\?\$"), ""),
    (re.compile(r"\\(?:text|mathrm)\s*\{([^{}]*)\}"), r"\1"),
    (re.compile(r"\^\{([^{}])\}"), r"^\1"),
    (re.compile(r"_\{([^{}])\}"), r"_\1"),
    (re.compile(r"\s+"), ""),
    (re.compile(r"(?<=\d),(?=\d{3}(?:\D|$))"), ""),
    (re.compile(r"^[A-Za-z]+=(?=\\begin\{pmatrix\})"), ""),
]


def normalise_answer(text: str | None) -> str:
    if text is None:
        return ""
    t = str(text).strip().strip("$").strip()
    final = re.search(r"####\s*([^\n]+)", t)  # GSM8K-style final line
    if final:
        t = final.group(1).strip()
    for pattern, repl in _NORMALISE:
        t = pattern.sub(repl, t)
    return t


def _has_variable(text: str) -> bool:
    t = re.sub(r"\\(?:text|mathrm)\s*\{[^{}]*\}", "", text)
    t = re.sub(r"\\[A-Za-z]+", "", t)
    return bool(re.search(r"[A-Za-z]", t))


def _parse_first(*texts: str) -> Any:
    for t in texts:
        try:
            got = mv_parse(t)
        except Exception:
            continue
        if got:
            return got
    return None


def _number(num: str) -> Any:
    num = num.replace(",", "").strip().rstrip(".")
    try:
        return mv_parse(num)
    except Exception:
        return num


def parse_boxed(boxed: str) -> Any:
    b = normalise_answer(boxed)
    lead = re.match(r"\s*([-+]?[0-9][0-9,]*(?:\.[0-9]+)?)", b)
    if lead and re.fullmatch(r"[A-Za-z]+", b[lead.end():]):  # a number with a unit word
        return _number(lead.group(1))
    if _has_variable(b):
        return b
    got = _parse_first(f"${b}$", b)
    if got:
        return got
    return _number(lead.group(1)) if lead else b


_UNIT = r"(?:miles?|minutes?|hours?|dollars?|GB)"
_ANSWER_PHRASES = [re.compile(p, re.IGNORECASE) for p in (
    r"The answer is:?\s*\$?([\-0-9\.,]+)",
    r"#### ?\$?([\-0-9\.,]+)",
    r"Therefore,? the answer is:?\s*\$?([\-0-9\.,]+)",
    r"So,? the answer is:?\s*\$?([\-0-9\.,]+)",
    r"Thus,? the answer is:?\s*\$?([\-0-9\.,]+)",
    r"Hence,? the answer is:?\s*\$?([\-0-9\.,]+)",
    r"Final answer:?\s*\$?([\-0-9\.,]+)",
    r"The final answer is:?\s*\$?([\-0-9\.,]+)",
    rf"The answer is:?\s*\$?([\-0-9\.,]+)\s*{_UNIT}?",
    rf"=\s*\$?([\-0-9\.,]+)\s*{_UNIT}?\.?\s*(?:The answer|$)",
)]
_VERB_END = re.compile(r"(?:is|are|equals?|makes?|has|have|gets?|arrives?|covers?|travels?)\s+\$?([\-0-9\.,]+)"
                       rf"(?:\s*{_UNIT})?\.?\s*$", re.MULTILINE | re.IGNORECASE)


def parse_unboxed(text: str) -> Any:
    got = _parse_first(f"${text}$", text)
    if got:
        return got
    for pattern in _ANSWER_PHRASES:
        hits = pattern.findall(text)
        if hits:
            ans = hits[-1].replace(",", "").strip().rstrip(".")
            if ans:
                return _number(ans)
    m = _VERB_END.search(text)
    if m:
        ans = m.group(1).replace(",", "").strip().rstrip(".")
        if ans:
            return _number(ans)
    for sentence in reversed(text.split(".")):
        if "Human:" in sentence or "Assistant:" in sentence:
            continue
        nums = re.findall(r"[-+]?[0-9]*\.?[0-9]+", sentence)
        if nums:
            return _number(nums[-1].lstrip("0") or "0")
    return None


def parse_answer(text: str) -> Any:
    boxed = last_boxed_content(text)
    return parse_boxed(boxed) if boxed else parse_unboxed(text)


def candidates(text: str) -> list[Any]:
    boxed = last_boxed_content(text)
    raw = [parse_boxed(boxed), normalise_answer(boxed), boxed] if boxed else [parse_unboxed(text)]
    out, seen = [], set()
    for c in raw:
        if c is None or repr(c) in seen:
            continue
        seen.add(repr(c))
        out.append(c)
    return out


def _components(text: str) -> tuple[str, ...] | None:
    m = re.fullmatch(r"\\begin\{pmatrix\}(.+)\\end\{pmatrix\}", text)
    if m:
        return tuple(p for p in m.group(1).split(r"\\") if p)
    m = re.fullmatch(r"\(([^()]+)\)", text)
    if m and "," in m.group(1):
        return tuple(p for p in m.group(1).split(",") if p)
    return None


def texts_match(answer: str, gold: str) -> bool:
    a, g = normalise_answer(answer), normalise_answer(gold)
    if a == g:
        return True
    try:
        if float(a.rstrip("%")) == float(g.rstrip("%")):
            return True
    except ValueError:
        pass
    if re.fullmatch(r"\([A-Za-z]\)", g) and a == g[1:-1]:
        return True
    ca, cg = _components(a), _components(g)
    return bool(ca and ca == cg)


def answers_match(answer: Any, gold: str | None) -> bool:
    if not answer or gold is None:
        return False
    if isinstance(answer, str) and texts_match(answer, gold):
        return True
    try:
        if mv_verify(answer, gold):
            return True
        gold_parsed = parse_answer(gold)
        if gold_parsed and mv_verify(gold_parsed, answer):
            return True
    except Exception:
        pass
    return isinstance(answer, str) and texts_match(answer, gold)


def grade(generation: str, ground_truth: Any) -> dict:
    """``{"prediction", "candidates", "correct"}`` of one generation against one or more reference answers."""
    golds = ground_truth if isinstance(ground_truth, list) else [ground_truth]
    cands = candidates(generation or "")
    ok = any(answers_match(c, str(g)) for c in cands for g in golds if g is not None)
    return {"prediction": str(cands[0]) if cands else None, "candidates": [str(c) for c in cands], "correct": ok}
