"""Answer extraction from generations (``evaluation/parsers.py`` behaviour).

* ``boxed``: content of the last ``\\boxed{...}`` (balanced braces);
* ``mc_answer``: the chosen option (A-E, digits 1-5 read as A-E) by the
  protocol's ordered line and tail rules (``extract_mc_answer``);
* ``code_completion``: the first fenced Python block after the first
  reasoning block (``extract_code``);
* ``passthrough``: the generation after any ``</think>`` marker;
* ``noop`` / ``identity``: the generation unchanged;
* ``gpqa_answer`` / ``mmlu_pro_answer``: the terminal option letter (A-D /
  A-J) of a reasoning response, ``"?"`` when it names none;
* ``lcb_code``: LiveCodeBench program extraction -- the final-channel
  message of a channelled response, special tokens removed, the last fenced
  Python block that defines something (or the last block), reduced to its
  top-level definitions and imports;
* ``humaneval`` and ``multiple_choice_answer`` are other names of
  ``code_completion`` and ``mc_answer``.
The extraction rules of the choice and LiveCodeBench parsers, and the order in
which they are tried, are those of the reference protocol: they decide what is
graded.
"""

from __future__ import annotations

import re

_THINK_END = "</think>"


_REASONING_CLOSE = re.compile(r"</(?:ifm\|)?think[^>]*>", re.IGNORECASE)  # </think>, K2's </ifm|think>


def strip_reasoning(text: str | None) -> str:
    """The text after the last reasoning block (``</think>`` or ``</ifm|think>``), stripped."""
    if text is None:
        return ""
    closes = list(_REASONING_CLOSE.finditer(text))
    return text[closes[-1].end():].strip() if closes else text.strip()


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


# Multiple-choice answers (A-E, or 1-5 read as A-E), in the protocol's order:
# the first line after the reasoning (answer tags, a boxed letter, or a whole
# line that states the answer), then the last lines from the bottom up (also
# statements inside a sentence), then a choice leading a line after the
# reasoning, then the last tag or statement in the final 4,096 characters.
_EMPH = r"(?:\*\*|__|`)?"
_CHOICE = r"([A-E1-5])"
_ANSWER_WORDS = rf"(?:final[.:]?\s*)?answer\b\s*[:：-]?\s*(?:is\s*)?{_EMPH}\s*(?:option\s*)?[\(\[]?\s*{_CHOICE}"
_CHOICE_WORDS = rf"(?:the\s+)?choice\s+is\s+{_EMPH}\s*(?:option\s*)?[\(\[]?\s*{_CHOICE}"
_LINE_END = rf"\s*[\)\]]?\s*{_EMPH}\s*(?:[.!?])?\s*$"
_MC_TAGS = [re.compile(p, re.IGNORECASE) for p in (
    rf"<(?:final\s*)?answer>\s*[\(\[]?\s*{_CHOICE}\s*[\)\]]?\s*</(?:final\s*)?answer>",
    rf"<answer>\s*[\(\[]?\s*{_CHOICE}\s*[\)\]]?\s*</answer>",
    rf"\\(?:boxed|fbox)\s*\{{\s*{_CHOICE}\s*\}}",
)]
_MC_LINE = [re.compile(p, re.IGNORECASE) for p in (
    rf"^\s*{_ANSWER_WORDS}{_LINE_END}",
    rf"^\s*{_CHOICE_WORDS}{_LINE_END}",
    rf"^\s*{_EMPH}\s*[\(\[]?\s*{_CHOICE}{_LINE_END}",
)]
_MC_INLINE = [re.compile(p, re.IGNORECASE) for p in (
    rf"\b{_ANSWER_WORDS}\s*[\)\]]?\s*{_EMPH}",
    rf"\b{_CHOICE_WORDS}\s*[\)\]]?\s*{_EMPH}",
    rf"\b(?:option|choice)\s*{_EMPH}\s*[\(\[]?\s*{_CHOICE}\s*[\)\]]?\s*{_EMPH}\s+"
    r"(?:is|would\s+be|remains?|works?|fits?|correct|best|right|compatible|consistent|larger)\b",
)]
_MC_LEADING = re.compile(rf"^\s*(?:final\s+(?:answer|choice)\s*[:=-]?\s*)?(?:option\s*)?[\(\[]?\s*{_CHOICE}"
                         r"(?=[\s\)\].,:;!\-]|$)", re.IGNORECASE)
_CHAT_END = re.compile(r"(?:<\|(?:ifm\|)?im_end\|>|<\|endoftext\|>)\s*$", re.IGNORECASE)
_REASONING_END = re.compile(r"</(?:ifm\|)?think[^>]*>", re.IGNORECASE)
_MC_LINES, _MC_TAIL = 96, 4096


def normalise_choice(value: str | None) -> str | None:
    """Upper-case letter; the digits 1-5 stand for A-E."""
    if value is None:
        return None
    v = value.strip().upper()
    return "ABCDE"[int(v) - 1] if v in {"1", "2", "3", "4", "5"} else (v or None)


def _line_choice(line: str, inline: bool) -> str | None:
    for pattern in _MC_TAGS + _MC_LINE + (_MC_INLINE if inline else []):
        m = pattern.search(line)
        if m:
            return normalise_choice(m.group(1))
    return None


def extract_mc_answer(text: str | None) -> str | None:
    if text is None:
        return None
    text = _CHAT_END.sub("", text).strip()
    if not text:
        return None
    closes = list(_REASONING_END.finditer(text))
    body = (text[closes[-1].end():].strip() or text) if closes else text
    lines = [ln.strip() for ln in body.splitlines() if ln.strip()]
    last_lines = lines[-_MC_LINES:]
    if lines:
        got = _line_choice(lines[0], inline=False)
        if got is not None:
            return got
        if closes:
            m = _MC_LEADING.match(lines[0])
            if m:
                return normalise_choice(m.group(1))
    for line in reversed(last_lines):
        got = _line_choice(line, inline=True)
        if got is not None:
            return got
    if closes:
        for line in reversed(last_lines):
            m = _MC_LEADING.match(line)
            if m:
                return normalise_choice(m.group(1))
    tail = body[-_MC_TAIL:]
    for pattern in _MC_TAGS + _MC_INLINE:
        hits = list(pattern.finditer(tail))
        if hits:
            return normalise_choice(hits[-1].group(1))
    return None


_CODE_FENCE = re.compile(r"```(?:python|py)?\s*\n(.*?)```", re.DOTALL)


def extract_code(text: str | None) -> str | None:
    """``code_completion``: the text after the first reasoning block (for a block that
    never closes, its first fenced block or last paragraph), then its first fenced
    Python block; ``None`` when nothing but whitespace is left."""
    if text is None:
        return None
    t = _CHAT_END.sub("", text)
    close = re.search(r"</(?:think|ifm\|think)>\s*", t, re.IGNORECASE)
    if close:
        t = t[close.end():]
    elif re.match(r"\s*<(?:think|ifm\|think)>", t, re.IGNORECASE):
        fence = _CODE_FENCE.search(t)
        t = fence.group(1) if fence else t.split("\n\n")[-1]
    fence = _CODE_FENCE.search(t)
    if fence:
        t = fence.group(1)
    return t if t.strip() else None


# ------------------------------------------------------- terminal choices
def _final_part(text: str) -> str:
    """The answer part of a reasoning response: after the first ``</think>``, else its last 500 characters."""
    return text.split(_THINK_END, 1)[1].lstrip() if _THINK_END in text else text[-500:]


def _choice_rules(hi: str, strict: bool) -> list[tuple[re.Pattern, int]]:
    """``(pattern, mode)`` rules for option letters A..hi, in the order they are tried; mode 0 takes
    the first match, 1 a closing mark at the very end, 2 the last letter standing alone on a line."""
    opt = f"[A-{hi}a-{hi.lower()}]"
    tail = re.compile(rf"(?:\*\*\(?({opt})\)?\*\*|\(({opt})\))\s*[.\s]*$")
    boxed = re.compile(rf"\\boxed\{{[^}}]*?({opt})[^A-{hi}a-{hi.lower()}}}]*\}}")
    if strict:  # four options: an explicit ANSWER line, "answer is X" / "answer: X", boxed, a closing mark
        return [(re.compile(rf"ANSWER:\s*({opt})"), 0),
                (re.compile(rf"[Aa]nswer\s*(?:is\s*:?\s*|:\s*)\*{{0,2}}\s*\(?({opt})\)?\*{{0,2}}"), 0),
                (boxed, 0), (tail, 1)]
    return [(re.compile(rf"[Aa]nswer is:?\s*\*{{0,2}}\(?({opt})\)?\*{{0,2}}"), 0), (boxed, 0), (tail, 1),
            (re.compile(rf"(?:^|\n)\s*\(?({opt})[.)]\s*$", re.MULTILINE), 2),
            (re.compile(rf"[Aa]nswer:?\s*\(?({opt})\)?"), 0)]


def _pick_choice(text: str | None, rules) -> str:
    if not text:
        return "?"
    part = _final_part(text)
    for pattern, mode in rules:
        if mode == 1:  # the closing mark must end the answer
            m = pattern.search(part.strip())
            if m:
                return (m.group(1) or m.group(2)).upper()
        elif mode == 2:  # the last option standing alone on a line
            hits = pattern.findall(part)
            if hits:
                return hits[-1].upper()
        else:
            m = pattern.search(part)
            if m:
                return m.group(1).upper()
    return "?"


_GPQA_RULES = _choice_rules("D", strict=True)
_MMLU_PRO_RULES = _choice_rules("J", strict=False)


def parse_gpqa_answer(text: str | None) -> str:
    return _pick_choice(text, _GPQA_RULES)


def parse_mmlu_pro_answer(text: str | None) -> str:
    return _pick_choice(text, _MMLU_PRO_RULES)


# ---------------------------------------------------- LiveCodeBench code
_CHANNEL = re.compile(r"<\|channel\|>\s*(?P<name>[^<\n]+)\s*<\|message\|>(?P<body>.*?)(?=(?:<\|channel\|>|<\|end\|>|$))",
                      re.IGNORECASE | re.DOTALL)
_SPECIAL = re.compile(r"<\|[^|]+(?:\|[^|]+)*\|>")
_PY_BLOCK = re.compile(r"```(?:python3?|py)?\s*\n(.*?)```", re.IGNORECASE | re.DOTALL)
_TOP_DEF = re.compile(r"^(def |async def |class |import |from \S+ import )")
_TOP_IMPORT = re.compile(r"^(import |from \S+ import )")
_DEFINES = re.compile(r"^(def |async def |class )", re.MULTILINE)
_HAS_CODE = re.compile(r"^(def |async def |class |import |from \S+ import )", re.MULTILINE)


def top_level_code(code: str) -> str:
    """Top-level definitions with their bodies and the import lines; drops
    example calls and prose around them (the code itself when nothing qualifies)."""
    kept: list[str] = []
    inside = False
    for line in code.split("\n"):
        bare = line.lstrip()
        indented = line[:1].isspace()
        if not indented and _TOP_DEF.match(bare):
            inside = True
            kept.append(line)
        elif inside:
            if not bare or indented:
                kept.append(line)
            else:
                inside = False  # a top-level statement ends the definition and is dropped
        elif not bare:
            if kept:
                kept.append(line)
        elif _TOP_IMPORT.match(bare):
            kept.append(line)
    while kept and not kept[-1].strip():
        kept.pop()
    return "\n".join(kept) if kept else code


def parse_lcb_code(text: str | None) -> str | None:
    if text is None:
        return None
    segments = list(_CHANNEL.finditer(text))
    if segments:
        final = [m for m in segments if m.group("name").strip().lower() in ("final", "answer")]
        text = (final or segments)[-1].group("body")
    text = _SPECIAL.sub("", text).strip()
    blocks = _PY_BLOCK.findall(text)
    if blocks:
        defining = [b for b in blocks if _DEFINES.search(b)]
        return top_level_code((defining or blocks)[-1])
    candidate = top_level_code(text)
    return candidate if _HAS_CODE.search(candidate) else None


PARSERS = {
    "passthrough": strip_reasoning,
    "noop": lambda text: text,
    "identity": lambda text: text,
    "boxed": last_boxed,
    "mc_answer": extract_mc_answer,
    "multiple_choice_answer": extract_mc_answer,
    "gpqa_answer": parse_gpqa_answer,
    "mmlu_pro_answer": parse_mmlu_pro_answer,
    "code_completion": extract_code,
    "humaneval": extract_code,
    "lcb_code": parse_lcb_code,
}
CHOICE_PARSERS = frozenset({"mc_answer", "multiple_choice_answer", "gpqa_answer", "mmlu_pro_answer"})
CODE_PARSERS = frozenset({"code_completion", "humaneval", "lcb_code"})


def parse_generation(parser: str, text: str | None):
    if parser not in PARSERS:
        raise ValueError(f"unknown parser {parser!r}; known: {sorted(PARSERS)}")
    return PARSERS[parser](text)
