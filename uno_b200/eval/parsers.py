"""Answer extraction from generations (``evaluation/parsers.py`` behaviour).

* ``boxed``: content of the last ``\\boxed{...}`` (balanced braces);
* ``mc_answer``: the chosen option letter (A-J), preferring an explicit
  "answer is X" / "Answer: X" statement, then a boxed letter, then the last
  standalone letter of the final lines;
* ``code_completion``: the last fenced code block (``python`` blocks first),
  else the text after a reasoning block;
* ``passthrough``: the generation after any ``</think>`` marker.
"""

from __future__ import annotations

import re

_THINK_END = "</think>"


def strip_reasoning(text: str | None) -> str:
    if text is None:
        return ""
    return text.rsplit(_THINK_END, 1)[-1].strip() if _THINK_END in text else text.strip()


def last_boxed(text: str | None) -> str | None:
    if not text:
        return None
    start = text.rfind("\\boxed")
    while start >= 0:
        brace = text.find("{", start)
        if brace < 0:
            return None
        depth, i = 0, brace
        while i < len(text):
            if text[i] == "{":
                depth += 1
            elif text[i] == "}":
                depth -= 1
                if depth == 0:
                    return text[brace + 1:i].strip()
            i += 1
        start = text.rfind("\\boxed", 0, start)
    return None


_MC_STRONG = [re.compile(p, re.IGNORECASE) for p in (
    r"answer\s*(?:is|:)?\s*[\(\[]?\s*\**\s*([A-J])\b",
    r"\bchoice\s*(?:is|:)\s*[\(\[]?([A-J])\b",
    r"\boption\s*(?:is|:)?\s*[\(\[]?([A-J])\b",
)]
_MC_WEAK = re.compile(r"(?:^|[\s\(\[\*])([A-J])(?:[\)\]\.\*:]|\s*$)")


def extract_mc_answer(text: str | None) -> str | None:
    body = strip_reasoning(text)
    if not body:
        return None
    boxed = last_boxed(body)
    if boxed:
        m = re.search(r"\b([A-J])\b", boxed.replace("\\text{", " ").replace("}", " "))
        if m:
            return m.group(1).upper()
    for pat in _MC_STRONG:
        hits = pat.findall(body)
        if hits:
            return hits[-1].upper()
    for line in reversed([ln.strip() for ln in body.splitlines() if ln.strip()][-3:]):
        hits = _MC_WEAK.findall(line)
        if hits:
            return hits[-1].upper()
    return None


_FENCE = re.compile(r"```([A-Za-z0-9_+-]*)\s*\n(.*?)```", re.DOTALL)


def extract_code(text: str | None) -> str | None:
    body = strip_reasoning(text)
    blocks = _FENCE.findall(body)
    if blocks:
        python = [code for lang, code in blocks if lang.lower() in ("python", "py", "python3")]
        return (python or [code for _, code in blocks])[-1].strip("\n")
    return body or None


PARSERS = {
    "passthrough": strip_reasoning,
    "boxed": last_boxed,
    "mc_answer": extract_mc_answer,
    "code_completion": extract_code,
}


def parse_generation(parser: str, text: str | None):
    if parser not in PARSERS:
        raise ValueError(f"unknown parser {parser!r}; known: {sorted(PARSERS)}")
    return PARSERS[parser](text)
