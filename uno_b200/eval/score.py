"""Grade a generations file and score it (``evaluation/score_generations.py``).

Routing by task: multiple-choice parsers grade letters; ``humaneval`` /
``mbpp`` (and any ``code_completion`` parser) run the sandboxed code grader;
LiveCodeBench rows run their stdin / functional tests (``eval/lcb.py``);
AA-LCR asks its judge for a JSON grade;
benchmarks with a judge use the LLM judge when a transport is given (else the
rows are reported as ungraded); ``ifeval`` uses the instruction checkers of ``eval/ifeval.py``;
everything else is graded as math (boxed answer equivalence).  Scores are
the mean correctness over all samples, the per-question mean, and the
generation throughput (TPS, TPF) copied from the generation summary.

CLI: ``python -m uno_b200.eval.score --generations FILE [--benchmark NAME]
[--data FILE] [--grades OUT] [--scores OUT] [--judge-base-url URL ...]``.
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any, Callable

from uno_b200.eval.benchmarks import get_benchmark
from uno_b200.eval.data import first_field, read_jsonl, ID_FIELDS
from uno_b200.eval.graders import JUDGED_TASKS, OMNISCIENCE_DENOMINATOR, grade_judged, grade_math, \
    grade_multiple_choice, grade_with_judge
from uno_b200.eval.parsers import CHOICE_PARSERS, CODE_PARSERS, parse_generation


def grade_row(row: dict, record: dict | None, *, task: str, parser: str, judge: Callable | None = None,
              judge_model: str | None = None, timeout: float = 10.0,
              judge_options: dict | None = None) -> dict[str, Any]:
    """Grade of one generation row; ``judge_options`` = temperature / max_tokens / reasoning_effort."""
    jopts = {k: v for k, v in (judge_options or {}).items() if v is not None}
    gen = row.get("generation", "")
    truth = row.get("ground_truth")
    if task == "ifeval":
        from uno_b200.eval.ifeval import grade_ifeval

        rec = record or {}
        prompt = rec.get("completion_input") or rec.get("prompt") or row.get("question") or ""
        return grade_ifeval(gen, truth if truth is not None else rec.get("ground_truth", rec), prompt)
    if task in ("lcb", "lcbv6", "livecodebench"):
        from uno_b200.eval.lcb import extract_python_code, generation_passed, parse_tests, run_generation

        codes = run_generation(extract_python_code(gen), parse_tests(truth), int(timeout))
        return {"correct": generation_passed(codes), "test_results": codes}
    if task in JUDGED_TASKS:
        rec = record or {}
        if task == "hle" and rec.get("answer_type") == "multipleChoice":  # letter answers need no judge
            from uno_b200.eval.parsers import extract_mc_answer

            gold = str(truth).strip()[:1].upper() if truth else None
            pick = extract_mc_answer(gen)
            return {"prediction": pick, "correct": pick is not None and pick == gold}
        if judge is None:
            return {"correct": None, "status": "ungraded: no judge endpoint"}
        question = str(rec.get("completion_input") or rec.get("problem") or row.get("question") or "")
        return grade_judged(task, question, gen, truth, transport=judge, model=judge_model or "judge", **jopts)
    if parser in CHOICE_PARSERS:
        return grade_multiple_choice(parse_generation(parser, gen), truth)
    if parser in CODE_PARSERS or task in ("humaneval", "mbpp"):
        if record is None:
            return {"correct": None, "status": "missing source record"}
        from uno_b200.eval.code_grading import grade_code_record

        parsed = parse_generation(parser, gen) if parser in CODE_PARSERS else None
        return grade_code_record(gen, parsed, record, timeout)
    if judge_model is not None:
        if judge is None:
            return {"correct": None, "status": "ungraded: no judge endpoint"}
        question = row.get("question") or (record or {}).get("question", "")
        return grade_with_judge(question, truth, gen, model=judge_model, transport=judge, **jopts)
    return grade_math(gen, truth)


FIXED_DENOMINATOR_TASKS = ("gpqa_diamond", "hle", "aa_lcr")


def pass_at_k(n: int, c: int, k: int) -> float:
    """Unbiased pass@k of a problem with ``c`` of ``n`` samples correct (``k`` capped at ``n``)."""
    from math import comb

    if k <= 0:
        return 0.0
    k = min(k, n)
    return 1.0 if n - c < k else 1.0 - comb(n - c, k) / comb(n, k)


def grouped_summary(per_problem: dict[str, list[bool]]) -> dict[str, Any]:
    """Problem count, samples per problem, and avg@k / pass@k for k = 1, 5, 10 (the
    reference scorer's summary keys): avg@k averages each problem's first k samples."""
    most = max((len(v) for v in per_problem.values()), default=0)
    out: dict[str, Any] = {"num_problems": len(per_problem), "max_samples_per_problem": most}
    for k in (1, 5, 10):
        if most < k:
            continue
        first_k = [x for v in per_problem.values() for x in v[:k]]
        out[f"avg_at_{k}"] = sum(first_k) / len(first_k) if first_k else float("nan")
        out[f"pass_at_{k}"] = sum(pass_at_k(len(v), sum(v), k) for v in per_problem.values()) / len(per_problem)
    return out


def expand_generation_rows(rows: list[dict]) -> list[dict]:
    """One row per generation with ``id`` = the source record and ``sample``.

    Reads this framework's rows and the reference runner's (``source_row``,
    ``sample_index``, an ``id`` of ``record:sampleN``, or a ``generations``
    list with one entry per sample)."""
    out = []
    for i, row in enumerate(rows):
        rid = row.get("source_row", row.get("id", i))
        gens = row.get("generations")
        if isinstance(gens, list):
            for k, g in enumerate(gens):
                out.append({**row, "id": rid, "sample": k, "generation": g})
            continue
        sample = row.get("sample", row.get("sample_index", 0))
        out.append({**row, "id": rid, "sample": sample})
    return out


def score_file(generations: str | Path, *, benchmark: str | None = None, data: str | Path | None = None,
               parser: str | None = None, grades_out: str | Path | None = None,
               scores_out: str | Path | None = None, summary: str | Path | None = None,
               judge: Callable | None = None, task: str | None = None,
               judge_model: str | None = None, timeout: float | None = None, workers: int = 1,
               judge_options: dict | None = None) -> dict[str, Any]:
    """Grade a generations file and write ``grades_out`` / ``scores_out``.

    ``timeout`` overrides the benchmark's per-test grader timeout; ``workers``
    grading threads run at once (code runs in its own sandbox subprocess and
    judge calls are network-bound, so threads overlap them)."""
    rows = expand_generation_rows(read_jsonl(generations))
    bench = get_benchmark(benchmark) if benchmark else None
    task = task or (bench.task if bench else "math")
    parser = parser or (bench.parser if bench else "passthrough")
    records = {}
    if data is not None:
        for i, rec in enumerate(read_jsonl(data)):
            rid = first_field(rec, ID_FIELDS)
            records[str(rid if rid is not None else i)] = rec
    limit = float(timeout) if timeout is not None else (bench.grader_timeout if bench else 10.0)
    model = judge_model or (bench.judge if bench else None)

    def one(row):
        g = grade_row(row, records.get(str(row.get("id"))), task=task, parser=parser, judge=judge,
                      judge_model=model, timeout=limit, judge_options=judge_options)
        return {"id": row.get("id"), "sample": row.get("sample"), **g}

    if workers > 1 and len(rows) > 1:
        from concurrent.futures import ThreadPoolExecutor

        with ThreadPoolExecutor(max_workers=int(workers)) as pool:
            grades = list(pool.map(one, rows))  # results keep the rows' order
    else:
        grades = [one(row) for row in rows]
    graded = [g for g in grades if g["correct"] is not None]
    per_q: dict[str, list[bool]] = {}
    for g in graded:
        per_q.setdefault(str(g["id"]), []).append(bool(g["correct"]))
    scores: dict[str, Any] = {
        "benchmark": bench.name if bench else None,
        "rows": len(rows),
        "graded": len(graded),
        "accuracy": sum(bool(g["correct"]) for g in graded) / len(graded) if graded else None,
        "question_accuracy": (sum(sum(v) / len(v) for v in per_q.values()) / len(per_q)) if per_q else None,
        "num_generations": len(graded),
        "num_correct": sum(bool(g["correct"]) for g in graded),
        **grouped_summary(per_q),
    }
    if task == "aa_omniscience":  # the benchmark's own metrics, over its full question count
        right = sum(1 for g in grades if g.get("grade") == 1)
        wrong = sum(1 for g in grades if g.get("grade") == -1)
        scores.update({"denominator": OMNISCIENCE_DENOMINATOR, "num_correct": right, "num_incorrect": wrong,
                       "accuracy": right / OMNISCIENCE_DENOMINATOR,
                       "non_hallucination_rate": 1.0 - wrong / OMNISCIENCE_DENOMINATOR,
                       "omniscience_index": (right - wrong) / OMNISCIENCE_DENOMINATOR})
    if bench is not None and task in FIXED_DENOMINATOR_TASKS:
        # the benchmark's full count: a missing generation counts as a wrong one
        samples = int(bench.num_samples)
        if summary is not None and Path(summary).is_file():
            gen_summary = json.loads(Path(summary).read_text())
            samples = int(gen_summary.get("num_samples_per_problem", gen_summary.get("num_samples", samples)))
        expected = bench.expected_rows * samples
        scores["fixed_denominator"] = expected
        scores["accuracy"] = scores["num_correct"] / expected
    if summary is not None and Path(summary).is_file():
        s = json.loads(Path(summary).read_text())
        for key in ("output_tokens_per_second", "decoder_tokens_per_sequence_forward", "total_output_tokens"):
            if key in s:
                scores[key] = s[key]
    if grades_out is not None:
        with open(grades_out, "w", encoding="utf-8") as fh:
            for g in grades:
                fh.write(json.dumps(g) + "\n")
    if scores_out is not None:
        Path(scores_out).write_text(json.dumps(scores, indent=2) + "\n")
    return scores


def judge_transport(base_url: str | None, api_key: str | None = None) -> Callable | None:
    """OpenAI-compatible chat transport of a judge endpoint (``/v1`` appended when missing)."""
    if not base_url:
        return None
    from uno_b200.eval.graders import http_chat_transport

    url = base_url.rstrip("/")
    return http_chat_transport(url if url.endswith("/v1") else url + "/v1", api_key)


def main(argv: list[str] | None = None) -> dict[str, Any]:
    import argparse
    import os

    ap = argparse.ArgumentParser(description="Grade a generations JSONL file and write its scores.")
    ap.add_argument("--generations", type=Path, required=True)
    ap.add_argument("--benchmark")
    ap.add_argument("--data", type=Path, help="the benchmark's records (code graders need them)")
    ap.add_argument("--task", help="grading task when no benchmark is named (default: math)")
    ap.add_argument("--parser")
    ap.add_argument("--grades", type=Path)
    ap.add_argument("--scores", type=Path)
    ap.add_argument("--generation-summary", type=Path, help="copies throughput figures into the scores")
    ap.add_argument("--timeout", type=float, help="per-test grader time limit")
    ap.add_argument("--grader-num-processes", type=int, default=1)
    ap.add_argument("--judge-model")
    ap.add_argument("--judge-base-url", default=os.environ.get("UNO_JUDGE_BASE_URL"))
    ap.add_argument("--judge-api-key", default=os.environ.get("UNO_JUDGE_API_KEY"))
    ap.add_argument("--judge-max-concurrency", type=int)
    ap.add_argument("--judge-temperature", type=float)
    ap.add_argument("--judge-max-tokens", type=int)
    ap.add_argument("--judge-reasoning-effort")
    args = ap.parse_args(argv)
    gen = args.generations
    scores = score_file(gen, benchmark=args.benchmark, data=args.data, parser=args.parser, task=args.task,
                        grades_out=args.grades or gen.with_name("grades.jsonl"),
                        scores_out=args.scores or gen.with_name("scores.json"), summary=args.generation_summary,
                        judge=judge_transport(args.judge_base_url, args.judge_api_key), judge_model=args.judge_model,
                        timeout=args.timeout,
                        workers=max(int(args.grader_num_processes or 1), int(args.judge_max_concurrency or 1)),
                        judge_options={"temperature": args.judge_temperature, "max_tokens": args.judge_max_tokens,
                                       "reasoning_effort": args.judge_reasoning_effort})
    print(json.dumps(scores, indent=2))
    return scores


if __name__ == "__main__":
    main()
