"""Evaluation runner: ``python -m uno_b200.eval.run --benchmark NAME --model DIR ...``.

Protocol of ``evaluation/run.py:196-613``:

* a registered benchmark fixes samples, temperature, top-p/top-k, completion
  budget, context length, concurrency, instruction, parser, chat-template
  arguments and the pinned dataset (rows + sha256); any departure is an
  *override* and is refused unless the run is labelled with
  ``--protocol-arm LABEL`` (the overrides are recorded in the summary);
* prompts are rendered with the tokenizer's chat template; samples are
  question-major (q0 s0..sN-1, q1 s0..);
* each request's completion budget is ``min(max_tokens, context - prompt -
  active-forward reserve)`` where the reserve is ``max(block, tree size)``;
  requests with no budget are skipped and reported;
* generations are appended to a JSONL file keyed by (id, sample), so an
  interrupted run resumes where it stopped; a summary JSON records TPS, TPF,
  the protocol and its overrides; grading and scoring follow unless
  ``--no-grade``.
"""

from __future__ import annotations

import argparse
import json
import os
import time
from pathlib import Path
from typing import Any

from uno_b200.eval.benchmarks import PROTOCOL_DATE, PROTOCOL_NAME, get_benchmark
from uno_b200.eval.data import ANSWER_FIELDS, ID_FIELDS, append_jsonl, first_field, load_records, \
    protocol_artifact_fingerprint, read_jsonl


def completion_budget(prompt_tokens: int, context_length: int, reserve: int, global_max: int | None) -> int:
    room = context_length - prompt_tokens - reserve
    return max(0, room if global_max is None else min(global_max, room))


def _int_list(value: str) -> list[int]:
    return [int(x) for x in str(value).split(",") if x.strip()]


def default_replicas(args) -> int:
    """``--data-parallel-size``, else one replica per visible GPU (at most 8) divided by the TP size."""
    if args.data_parallel_size is not None:
        return int(args.data_parallel_size)
    if args.device != "cuda":
        return 1
    import torch

    gpus = min(torch.cuda.device_count(), 8) if torch.cuda.is_available() else 1
    return max(1, gpus // max(1, int(args.tensor_parallel_size)))


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--benchmark")
    p.add_argument("--data", type=Path)
    p.add_argument("--model", required=True)
    p.add_argument("--tokenizer-path")
    p.add_argument("--model-revision")
    p.add_argument("--gated-lora-path")
    p.add_argument("--gated-lora-revision")
    p.add_argument("--gated-lora-subfolder")
    p.add_argument("--hf-cache-dir")
    p.add_argument("--hf-local-files-only", action="store_true")
    p.add_argument("--output", type=Path)
    p.add_argument("--grades", type=Path, help="grades JSONL (default: grades.jsonl beside --output)")
    p.add_argument("--scores", type=Path, help="scores JSON (default: scores.json beside --output)")
    p.add_argument("--summary-output", type=Path)
    p.add_argument("--limit", type=int)
    p.add_argument("--num-samples", "--repetitions", dest="num_samples", type=int,
                   help="generations per problem (default: the benchmark's)")
    p.add_argument("--temperature", type=float)
    p.add_argument("--top-p", type=float)
    p.add_argument("--top-k", type=int)
    p.add_argument("--max-tokens", type=int)
    p.add_argument("--max-model-len", type=int)
    p.add_argument("--max-num-seqs", type=int)
    p.add_argument("--max-num-batched-tokens", type=int)
    p.add_argument("--instruction")
    p.add_argument("--parser")
    p.add_argument("--chat-template-kwargs-json")
    p.add_argument("--protocol-arm")
    p.add_argument("--diffusion-block-size", type=int, default=8)
    p.add_argument("--tree-verify-size", type=int)
    p.add_argument("--tree-candidate-top-k", type=int, default=16)
    p.add_argument("--tensor-parallel-size", type=int, default=1)
    p.add_argument("--data-parallel-size", type=int,
                   help="engine replicas (default: one per visible GPU up to 8, as the reference's 8 on a full node; "
                        "1 on the CPU)")
    p.add_argument("--device", choices=("cuda", "cpu"), default="cuda")
    p.add_argument("--load-format", default="auto")
    p.add_argument("--mask-token-id", type=int)
    p.add_argument("--stop-token-ids")
    p.add_argument("--noise-mode", default="random_uniform")
    p.add_argument("--noise-salt", type=int)
    p.add_argument("--ignore-eos", action="store_true")
    p.add_argument("--save-token-ids", action="store_true", help="keep each generation's token ids in its row")
    p.add_argument("--no-progress", action="store_true")
    p.add_argument("--gpu-memory-utilization", type=float)
    p.add_argument("--attention-backend", choices=("fa2", "fa3", "fa4", "native"), default="native",
                   help="accepted for script compatibility; every value runs this framework's attention kernels")
    p.add_argument("--cuda-graph-block-sizes", type=_int_list, help="comma-separated forward lengths to capture")
    p.add_argument("--cuda-graph-batch-sizes", type=_int_list, help="comma-separated batch sizes to capture")
    p.add_argument("--torch-compile", action="store_true",
                   help="accepted for script compatibility; this framework runs hand-written kernels and "
                        "CUDA graphs, so the flag changes nothing")
    p.add_argument("--grader-timeout", type=float, help="per-test grader time limit (default: the benchmark's)")
    p.add_argument("--grader-num-processes", type=int, default=1, help="grading threads")
    p.add_argument("--skip-row-count-check", action="store_true")
    p.add_argument("--no-grade", "--skip-grading", dest="no_grade", action="store_true")
    p.add_argument("--judge-model", help="judge model for LLM-graded benchmarks (default: the benchmark's)")
    p.add_argument("--judge-base-url", default=os.environ.get("UNO_JUDGE_BASE_URL"),
                   help="OpenAI-compatible endpoint of the judge (env UNO_JUDGE_BASE_URL)")
    p.add_argument("--judge-api-key", default=os.environ.get("UNO_JUDGE_API_KEY"))
    p.add_argument("--judge-max-concurrency", type=int, help="concurrent judge requests")
    p.add_argument("--judge-temperature", type=float)
    p.add_argument("--judge-max-tokens", type=int)
    p.add_argument("--judge-reasoning-effort")
    p.add_argument("--seed", type=int)
    return p


def resolve_protocol(args, bench) -> dict[str, Any]:
    """Fill unset options from the benchmark; collect departures from it."""
    defaults = {"num_samples": bench.num_samples if bench else 1, "temperature": bench.temperature if bench else 1.0,
                "top_k": bench.top_k if bench else None, "top_p": bench.top_p if bench else None,
                "max_tokens": bench.max_tokens if bench else None,
                "max_model_len": bench.max_model_len if bench else 32768,
                "max_num_seqs": bench.max_num_seqs if bench else 256,
                "instruction": bench.instruction if bench else "",
                "parser": bench.parser if bench else "passthrough"}
    overrides = {}
    for name, default in defaults.items():
        got = getattr(args, name)
        if got is None:
            setattr(args, name, default)
        elif bench is not None and got != default:
            overrides[name] = {"canonical": default, "actual": got}
    if args.max_num_batched_tokens is None:
        args.max_num_batched_tokens = args.max_model_len
    elif bench is not None and args.max_num_batched_tokens != args.max_model_len:
        overrides["max_num_batched_tokens"] = {"canonical": args.max_model_len, "actual": args.max_num_batched_tokens}
    return overrides


def main(argv: list[str] | None = None) -> dict[str, Any]:
    args = build_parser().parse_args(argv)
    from uno_b200.generation import format_chat_prompt, resolve_model_sources
    from uno_b200.utils.hf_compat import load_model_config, load_tokenizer
    from uno_b200.utils.hub import resolve_hf_snapshot
    from uno_b200.utils.model_tokens import resolve_model_token_ids

    model, adapter = resolve_model_sources(args.model, args.gated_lora_path, model_revision=args.model_revision,
                                           gated_lora_subfolder=args.gated_lora_subfolder,
                                           hf_cache_dir=args.hf_cache_dir,
                                           hf_local_files_only=args.hf_local_files_only)
    bench = get_benchmark(args.benchmark) if args.benchmark else None
    overrides = resolve_protocol(args, bench)
    chat_kwargs = dict(bench.chat_template_kwargs) if bench else {}
    if args.chat_template_kwargs_json:
        extra = json.loads(args.chat_template_kwargs_json)
        if not isinstance(extra, dict):
            raise ValueError("--chat-template-kwargs-json must be a JSON object")
        chat_kwargs.update(extra)
        if bench and chat_kwargs != dict(bench.chat_template_kwargs):
            overrides["chat_template_kwargs"] = {"canonical": dict(bench.chat_template_kwargs), "actual": chat_kwargs}
    if args.data is None:
        if bench is None:
            raise ValueError("--data is required when --benchmark is not set")
        # the prepared file under UNO_EVAL_DATA_DIR, prepared now when it is missing (pinned bundle
        # from UNO_EVAL_PROTOCOL_SOURCE_DIR or the Hub, public datasets otherwise)
        from uno_b200.eval.prepare import prepare_benchmark_data

        args.data = prepare_benchmark_data(bench.name, output_dir=bench.data_path.parent)
    if not Path(args.data).is_file():
        raise FileNotFoundError(f"dataset not found: {args.data} (set UNO_EVAL_DATA_DIR or pass --data)")
    if bench is not None:
        if args.limit is not None:
            overrides["limit"] = {"canonical": None, "actual": args.limit}
        rows, sha = protocol_artifact_fingerprint(args.data)
        if rows != bench.expected_rows or sha != bench.data_sha256:
            overrides["data"] = {"canonical": {"rows": bench.expected_rows, "sha256": bench.data_sha256},
                                 "actual": {"rows": rows, "sha256": sha}}
    if overrides and not args.protocol_arm:
        raise ValueError(f"Canonical protocol overrides ({', '.join(sorted(overrides))}) require --protocol-arm LABEL")
    if args.num_samples < 1:
        raise ValueError("--num-samples must be positive")

    name = bench.name if bench else Path(args.data).stem
    out = args.output or Path(f"{name}-generations.jsonl")
    summary_path = args.summary_output or out.with_name(f"{out.stem.removesuffix('-generations')}-generation-summary.json")
    records = load_records(args.data, args.limit)
    if bench and args.limit is None and not args.skip_row_count_check and len(records) != bench.expected_rows:
        raise ValueError(f"{bench.name} expects {bench.expected_rows} rows, but {args.data} contains {len(records)}.")

    if str(model).startswith("preset:"):
        from uno_b200.models.presets import resolve_preset

        cfg, model_dir = resolve_preset(str(model)[len("preset:"):]), None
    else:
        model_dir = resolve_hf_snapshot(model, revision=args.model_revision, cache_dir=args.hf_cache_dir,
                                        local_files_only=args.hf_local_files_only, artifact_name="model")
        cfg = load_model_config(model_dir)
    tokenizer = load_tokenizer(args.tokenizer_path or model_dir, cfg)
    stops = [int(x) for x in args.stop_token_ids.split(",")] if args.stop_token_ids else None
    mask_id, stop_ids, _ = resolve_model_token_ids(model_dir or cfg, tokenizer, mask_token_id=args.mask_token_id,
                                                   stop_token_ids=stops, noise_mode=args.noise_mode)

    items = []  # question-major
    for idx, rec in enumerate(records):
        msgs = rec.get("chat_input")
        if not isinstance(msgs, list) or not msgs:
            raise ValueError(f"Record {idx} needs a nonempty chat_input")
        ids, text, eff = format_chat_prompt(tokenizer, msgs, args.instruction, chat_kwargs)
        rid = first_field(rec, ID_FIELDS)
        rid = idx if rid is None else rid
        for s in range(args.num_samples):
            items.append({"id": rid, "sample": s, "prompt_ids": ids, "prompt": text,
                          "ground_truth": first_field(rec, ANSWER_FIELDS), "chat_input": msgs,
                          "completion_input": rec.get("completion_input")})
    done = set()
    if out.is_file():
        for row in read_jsonl(out):
            done.add((str(row["id"]), int(row["sample"])))
    reserve = max(args.diffusion_block_size, args.tree_verify_size or 0)
    pending, skipped = [], []
    for it in items:
        if (str(it["id"]), it["sample"]) in done:
            continue
        budget = completion_budget(len(it["prompt_ids"]), args.max_model_len, reserve, args.max_tokens)
        (pending if budget > 0 else skipped).append((it, budget))

    from uno_b200.llm import LLM
    from uno_b200.sampling_params import SamplingParams

    stats: dict[str, Any] = {}
    elapsed = 0.0
    total_tokens = 0
    if pending:
        llm = LLM(model_dir or model, tokenizer_path=args.tokenizer_path or model_dir, gated_lora_path=adapter,
                  device=args.device, load_format=args.load_format, tensor_parallel_size=args.tensor_parallel_size,
                  data_parallel_size=default_replicas(args), max_num_seqs=args.max_num_seqs,
                  max_model_len=args.max_model_len, max_num_batched_tokens=args.max_num_batched_tokens,
                  max_diffusion_block_size=args.diffusion_block_size,
                  cuda_graph_block_sizes=args.cuda_graph_block_sizes or sorted({1, args.diffusion_block_size}),
                  attention_backend=args.attention_backend,
                  **({"cuda_graph_batch_sizes": args.cuda_graph_batch_sizes} if args.cuda_graph_batch_sizes else {}),
                  tree_verify_size=args.tree_verify_size, tree_candidate_top_k=args.tree_candidate_top_k,
                  gated_lora_revision=args.gated_lora_revision, hf_cache_dir=args.hf_cache_dir,
                  hf_local_files_only=args.hf_local_files_only,
                  **({"gpu_memory_utilization": args.gpu_memory_utilization}
                     if args.gpu_memory_utilization is not None else {}),
                  **({"seed": args.seed} if args.seed is not None else {}))
        sp = SamplingParams(temperature=args.temperature, top_p=args.top_p, top_k=args.top_k,
                            max_tokens=max(b for _, b in pending), stop_token_ids=stop_ids, mask_token_id=mask_id,
                            noise_mode=args.noise_mode, noise_salt=args.noise_salt, ignore_eos=args.ignore_eos,
                            diffusion_block_size=args.diffusion_block_size)
        t0 = time.perf_counter()
        try:
            outs = llm.generate([it["prompt_ids"] for it, _ in pending], sp,
                                request_max_tokens=[b for _, b in pending], use_tqdm=not args.no_progress)
            elapsed = time.perf_counter() - t0
            stats = dict(getattr(llm, "last_generate_stats", {}))
        finally:
            llm.exit()
        rows = []
        for (it, budget), o in zip(pending, outs):
            total_tokens += len(o["token_ids"])
            row = {"id": it["id"], "sample": it["sample"], "question": it["prompt"],
                   "generation": o["text"], "token_count": len(o["token_ids"]), "budget": budget,
                   "ground_truth": it["ground_truth"], "stats": o.get("stats", {}),
                   # the reference runner's row keys, so that its scorer reads these files too
                   "source_row": it["id"], "sample_index": it["sample"], "problem": it["prompt"],
                   "rendered_prompt": it["prompt"], "chat_input": it["chat_input"],
                   "prompt_token_count": len(it["prompt_ids"]), "output_token_count": len(o["token_ids"]),
                   "context_length": args.max_model_len, "active_forward_reserve": reserve,
                   "resolved_max_tokens": budget}
            if it["completion_input"] is not None:
                row["completion_input"] = it["completion_input"]
            if args.save_token_ids:
                row["token_ids"] = list(o["token_ids"])
            rows.append(row)
        append_jsonl(out, rows)
    forwards = int(stats.get("forwards", 0))
    summary = {"protocol": PROTOCOL_NAME, "protocol_date": PROTOCOL_DATE, "benchmark": bench.name if bench else None,
               "protocol_arm": args.protocol_arm, "overrides": overrides, "model": args.model,
               "gated_lora_path": adapter, "requests": len(items), "generated": len(pending),
               "num_problems": len(records), "num_samples_per_problem": args.num_samples,
               "num_generations": len(items),
               "resumed": len(done), "skipped_no_budget": [[s["id"], s["sample"]] for s, _ in skipped],
               "total_output_tokens": total_tokens, "elapsed_seconds": elapsed,
               "output_tokens_per_second": total_tokens / elapsed if elapsed else 0.0,
               "decoder_stats": stats,
               "decoder_tokens_per_sequence_forward": int(stats.get("accepts", 0)) / forwards if forwards else 0.0}
    Path(summary_path).write_text(json.dumps(summary, indent=2) + "\n")
    if not args.no_grade:
        from uno_b200.eval.score import judge_transport, score_file

        judge = judge_transport(args.judge_base_url, args.judge_api_key)
        workers = max(int(args.grader_num_processes or 1), int(args.judge_max_concurrency or 1))
        summary["scores"] = score_file(out, benchmark=args.benchmark, data=args.data, parser=args.parser,
                                       grades_out=args.grades or out.with_name("grades.jsonl"),
                                       scores_out=args.scores or out.with_name("scores.json"), summary=summary_path,
                                       judge=judge, judge_model=args.judge_model, timeout=args.grader_timeout,
                                       workers=workers,
                                       judge_options={"temperature": args.judge_temperature,
                                                      "max_tokens": args.judge_max_tokens,
                                                      "reasoning_effort": args.judge_reasoning_effort})
    return summary


if __name__ == "__main__":
    print(json.dumps(main(), indent=2))
