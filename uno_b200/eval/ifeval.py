"""IFEval instruction-following grader.

Grades a response against the verifiable instructions of the IFEval
benchmark (Zhou et al., 2023), the grader the reference wires in for its
``ifeval`` task (``evaluation/graders/ifeval.py:33-130``): every row carries
``instruction_id_list`` and one ``kwargs`` dict per instruction; a response
follows an instruction when its checker holds.  Two modes, as in IFEval:

* strict -- the response as generated (after the reasoning block);
* loose  -- the instruction counts as followed if it holds for any of eight
  variants of the response: as is, without its first line, without its last
  line, without both, and each of those with ``*`` removed.

The checkers are written here from the benchmark's published definitions
(counts with the relations ``less than`` / ``at least``, markdown
conventions for bullets, highlights, sections and paragraphs, ...).  The
language check uses the Unicode script of the letters for non-Latin
languages and a stop-word vote for Latin-script ones, so grading needs no
network model and is deterministic.
"""

from __future__ import annotations

import json
import re
from typing import Any, Callable

# ------------------------------------------------------------------ helpers
_WORD = re.compile(r"\b\w+(?:['’]\w+)?\b", re.UNICODE)


def _words(text: str) -> list[str]:
    return _WORD.findall(text)


def _compare(count: int, relation: str | None, n: int) -> bool:
    if relation in (None, "at least"):
        return count >= n
    if relation == "less than":
        return count < n
    raise ValueError(f"unknown relation {relation!r}")


def _sentences(text: str) -> list[str]:
    text = re.sub(r"\b(?:Mr|Mrs|Ms|Dr|Prof|Sr|Jr|St|vs|etc|e\.g|i\.e)\.", lambda m: m.group(0)[:-1], text)
    parts = re.split(r"(?<=[.!?])\s+|\n+", text.strip())
    return [p for p in parts if re.search(r"\w", p)]


def _paragraphs_by_divider(text: str) -> list[str]:
    return re.split(r"\s?\*\*\*\s?", text)


# ------------------------------------------------------------------ language
_SCRIPTS = {  # language -> unicode ranges of its script
    "ar": [(0x0600, 0x06FF)], "fa": [(0x0600, 0x06FF)], "ur": [(0x0600, 0x06FF)],
    "ru": [(0x0400, 0x04FF)], "bg": [(0x0400, 0x04FF)], "uk": [(0x0400, 0x04FF)],
    "hi": [(0x0900, 0x097F)], "mr": [(0x0900, 0x097F)], "ne": [(0x0900, 0x097F)],
    "bn": [(0x0980, 0x09FF)], "pa": [(0x0A00, 0x0A7F)], "gu": [(0x0A80, 0x0AFF)],
    "ta": [(0x0B80, 0x0BFF)], "te": [(0x0C00, 0x0C7F)], "kn": [(0x0C80, 0x0CFF)],
    "th": [(0x0E00, 0x0E7F)], "ko": [(0xAC00, 0xD7AF), (0x1100, 0x11FF)],
    "ja": [(0x3040, 0x30FF)], "zh": [(0x4E00, 0x9FFF)], "he": [(0x0590, 0x05FF)],
    "el": [(0x0370, 0x03FF)],
}
_STOPWORDS = {
    "en": "the and of to is in that it for with as was on are be this by not you",
    "de": "der die und das ist nicht zu den mit sich des auf für ein eine",
    "fr": "le la les et des est une un pour que dans pas qui sur du avec",
    "es": "el la los las y que de en es un una por para con no se",
    "it": "il la che di e un una per non sono con del della gli le",
    "pt": "o a os as e que de um uma para com não se em do da",
    "fi": "ja on ei se että hän oli ovat kuin mutta myös tai niin",
    "sw": "na ya wa kwa ni za katika la kuwa hii cha hiyo lakini",
    "vi": "và của là có không được cho những một các người này với",
    "nl": "de het en een van is dat niet op te zijn voor met",
    "tr": "ve bir bu da için ile de ne değil gibi çok daha",
    "id": "dan yang di ini itu dengan untuk tidak dari ke pada",
}


def detect_language(text: str) -> str | None:
    letters = [c for c in text if c.isalpha()]
    if not letters:
        return None
    counts: dict[str, int] = {}
    for c in letters:
        o = ord(c)
        for lang, ranges in _SCRIPTS.items():
            if any(lo <= o <= hi for lo, hi in ranges):
                counts[lang] = counts.get(lang, 0) + 1
                break
    non_latin = sum(counts.values())
    if non_latin > len(letters) / 2:
        if counts.get("ja"):  # kana marks Japanese even when most characters are kanji
            return "ja"
        return max(counts, key=counts.get)
    words = [w.lower() for w in _words(text)]
    scores = {lang: sum(1 for w in words if w in set(sw.split())) for lang, sw in _STOPWORDS.items()}
    best = max(scores, key=scores.get)
    return best if scores[best] > 0 else "en"


def _same_language(detected: str | None, wanted: str) -> bool:
    if detected is None:
        return False
    groups = [{"ar", "fa", "ur"}, {"ru", "bg", "uk"}, {"hi", "mr", "ne"}]
    if detected == wanted:
        return True
    return any(detected in g and wanted in g for g in groups)


# ------------------------------------------------------------------ checkers
def _kw(k: dict, name: str, default=None):
    v = k.get(name, default)
    return default if v is None else v


def _keywords_existence(r: str, k: dict, prompt: str) -> bool:
    return all(re.search(re.escape(w), r, re.IGNORECASE) for w in _kw(k, "keywords", []))


def _keyword_frequency(r: str, k: dict, prompt: str) -> bool:
    n = len(re.findall(re.escape(k["keyword"]), r, re.IGNORECASE))
    return _compare(n, k.get("relation"), int(k["frequency"]))


def _forbidden_words(r: str, k: dict, prompt: str) -> bool:
    return not any(re.search(r"\b" + re.escape(w) + r"\b", r, re.IGNORECASE) for w in _kw(k, "forbidden_words", []))


def _letter_frequency(r: str, k: dict, prompt: str) -> bool:
    n = r.lower().count(str(k["letter"]).lower())
    return _compare(n, k.get("let_relation"), int(k["let_frequency"]))


def _response_language(r: str, k: dict, prompt: str) -> bool:
    return _same_language(detect_language(r), str(k["language"]))


def _number_sentences(r: str, k: dict, prompt: str) -> bool:
    return _compare(len(_sentences(r)), k.get("relation"), int(k["num_sentences"]))


def _number_paragraphs(r: str, k: dict, prompt: str) -> bool:
    parts = _paragraphs_by_divider(r)
    n = int(k["num_paragraphs"])
    # empty pieces are allowed only at the ends (a leading / trailing divider)
    for i, p in enumerate(parts):
        if not p.strip() and 0 < i < len(parts) - 1:
            return False
    return len([p for p in parts if p.strip()]) == n


def _number_words(r: str, k: dict, prompt: str) -> bool:
    return _compare(len(_words(r)), k.get("relation"), int(k["num_words"]))


def _nth_paragraph_first_word(r: str, k: dict, prompt: str) -> bool:
    paras = [p for p in re.split(r"\n\s*\n", r) if p.strip()]
    if len(paras) != int(k["num_paragraphs"]):
        return False
    nth = int(k["nth_paragraph"])
    if not 1 <= nth <= len(paras):
        return False
    words = paras[nth - 1].strip().split()
    if not words:
        return False
    first = re.sub(r"^[^\w]+|[^\w]+$", "", words[0]).lower()
    return first == str(k["first_word"]).lower()


def _placeholders(r: str, k: dict, prompt: str) -> bool:
    return len(re.findall(r"\[.*?\]", r)) >= int(k["num_placeholders"])


def _postscript(r: str, k: dict, prompt: str) -> bool:
    marker = str(_kw(k, "postscript_marker", "P.S.")).strip()
    pat = r"\s*p\.\s?p\.\s?s.*$" if marker.lower() == "p.p.s" else r"\s*" + re.escape(marker.lower()) + r".*$"
    return re.search(pat, r.lower(), re.MULTILINE) is not None


def _bullet_lists(r: str, k: dict, prompt: str) -> bool:
    n = len(re.findall(r"^\s*\*[^\*].*$", r, re.MULTILINE)) + len(re.findall(r"^\s*-.*$", r, re.MULTILINE))
    return n == int(k["num_bullets"])


_CONSTRAINED = ("My answer is yes.", "My answer is no.", "My answer is maybe.")


def _constrained_response(r: str, k: dict, prompt: str) -> bool:
    return any(option in r.strip() for option in _CONSTRAINED)


def _highlighted_sections(r: str, k: dict, prompt: str) -> bool:
    n = sum(1 for h in re.findall(r"\*[^\n\*]*\*", r) if h.strip("*").strip())
    n += sum(1 for h in re.findall(r"\*\*[^\n\*]*\*\*", r) if h.strip("*").strip())
    return n >= int(k["num_highlights"])


def _multiple_sections(r: str, k: dict, prompt: str) -> bool:
    splitter = str(_kw(k, "section_spliter", "Section")).strip()
    parts = re.split(r"\s?" + re.escape(splitter) + r"\s?\d+\s?", r)
    return len(parts) - 1 >= int(k["num_sections"])


def _json_format(r: str, k: dict, prompt: str) -> bool:
    body = r.strip()
    body = re.sub(r"^```(?:json|Json|JSON)?\s*", "", body)
    body = re.sub(r"\s*```$", "", body)
    try:
        json.loads(body)
        return True
    except ValueError:
        return False


def _title(r: str, k: dict, prompt: str) -> bool:
    return any(t.strip() for t in re.findall(r"<<([^\n]+?)>>", r))


def _two_responses(r: str, k: dict, prompt: str) -> bool:
    parts = [p.strip() for p in r.split("******")]
    valid = [p for i, p in enumerate(parts) if p or (0 < i < len(parts) - 1)]
    if len(valid) != 2 or not all(valid):
        return False
    return valid[0] != valid[1]


def _repeat_prompt(r: str, k: dict, prompt: str) -> bool:
    return r.strip().lower().startswith(str(k["prompt_to_repeat"]).strip().lower())


def _end_checker(r: str, k: dict, prompt: str) -> bool:
    return r.strip().strip('"').lower().endswith(str(k["end_phrase"]).strip().lower())


def _capital_word_frequency(r: str, k: dict, prompt: str) -> bool:
    n = sum(1 for w in _words(r) if w.isupper())
    return _compare(n, k.get("capital_relation"), int(k["capital_frequency"]))


def _english_capital(r: str, k: dict, prompt: str) -> bool:
    return r.isupper() and detect_language(r) == "en"


def _english_lowercase(r: str, k: dict, prompt: str) -> bool:
    return r.islower() and detect_language(r) == "en"


def _no_comma(r: str, k: dict, prompt: str) -> bool:
    return "," not in r


def _quotation(r: str, k: dict, prompt: str) -> bool:
    body = r.strip()
    return len(body) > 1 and body[0] == '"' and body[-1] == '"'


CHECKERS: dict[str, Callable[[str, dict, str], bool]] = {
    "keywords:existence": _keywords_existence,
    "keywords:frequency": _keyword_frequency,
    "keywords:forbidden_words": _forbidden_words,
    "keywords:letter_frequency": _letter_frequency,
    "language:response_language": _response_language,
    "length_constraints:number_sentences": _number_sentences,
    "length_constraints:number_paragraphs": _number_paragraphs,
    "length_constraints:number_words": _number_words,
    "length_constraints:nth_paragraph_first_word": _nth_paragraph_first_word,
    "detectable_content:number_placeholders": _placeholders,
    "detectable_content:postscript": _postscript,
    "detectable_format:number_bullet_lists": _bullet_lists,
    "detectable_format:constrained_response": _constrained_response,
    "detectable_format:number_highlighted_sections": _highlighted_sections,
    "detectable_format:multiple_sections": _multiple_sections,
    "detectable_format:json_format": _json_format,
    "detectable_format:title": _title,
    "combination:two_responses": _two_responses,
    "combination:repeat_prompt": _repeat_prompt,
    "startend:end_checker": _end_checker,
    "change_case:capital_word_frequency": _capital_word_frequency,
    "change_case:english_capital": _english_capital,
    "change_case:english_lowercase": _english_lowercase,
    "punctuation:no_comma": _no_comma,
    "startend:quotation": _quotation,
}


def _loose_variants(r: str) -> list[str]:
    lines = r.split("\n")
    base = [r, "\n".join(lines[1:]).strip(), "\n".join(lines[:-1]).strip(), "\n".join(lines[1:-1]).strip()]
    return base + [v.replace("*", "") for v in base]


def check(instruction_id: str, response: str, kwargs: dict | None, prompt: str = "", loose: bool = False) -> bool:
    fn = CHECKERS.get(instruction_id)
    if fn is None:
        raise KeyError(f"unknown IFEval instruction {instruction_id!r}")
    kw = {k: v for k, v in (kwargs or {}).items() if v is not None}
    candidates = _loose_variants(response) if loose else [response]
    return any(c.strip() and fn(c, kw, prompt) for c in candidates)


def grade_ifeval(generation: str, ground_truth: Any, prompt: str = "") -> dict:
    """Per-instruction and prompt-level results in strict and loose mode; ``correct`` is strict prompt-level."""
    from uno_b200.eval.parsers import strip_reasoning

    if isinstance(ground_truth, str):
        ground_truth = json.loads(ground_truth)
    ids = list(ground_truth["instruction_id_list"])
    kwargs = list(ground_truth.get("kwargs") or [{}] * len(ids))
    response = strip_reasoning(generation or "")
    strict = [check(i, response, k, prompt) for i, k in zip(ids, kwargs)]
    loose = [check(i, response, k, prompt, loose=True) for i, k in zip(ids, kwargs)]
    return {"correct": all(strict), "strict_prompt_follow": all(strict), "strict_inst_follow": strict,
            "loose_prompt_follow": all(loose), "loose_inst_follow": loose}
