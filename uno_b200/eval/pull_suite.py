"""Pull-based multi-node evaluation: one coordinator, many generation workers.

Behaviour of ``evaluation/pull_suite.py:357-1132``:

* the coordinator expands every (benchmark, record, sample) into a job,
  drops the jobs already present in the results file (idempotent resume),
  and serves a job queue and a result queue over a ``multiprocessing``
  manager (TCP, authkey);
* the run *manifest* (protocol settings, model, dataset fingerprints) is
  hashed; a worker whose manifest hash differs is refused, so results of
  different configurations never mix;
* workers connect with retries until a deadline, pull jobs in small batches,
  generate (an :class:`~uno_b200.engine.async_engine.AsyncLLMEngine`-backed
  generator in production, any callable in tests) and push one result per
  job; a ``None`` job tells a worker to stop;
* the coordinator appends every result to the JSONL results file as it
  arrives (flushed per row) and stops the workers when all jobs are done.

CLI: ``python -m uno_b200.eval.pull_suite jobs|coordinator|worker|score ...``:

* ``jobs`` expands registered benchmarks into the job file and writes the run
  manifest (model, block size, each benchmark's data fingerprint, and the
  sampling settings, which every worker takes from the manifest);
* ``score`` splits the collected results per benchmark and grades each one
  (``uno_b200.eval.score``), leaving ``<benchmark>/{generations,grades}.jsonl``
  and ``scores.json`` beside them.

``uno_b200/eval/run_pull_suite_slurm.sh`` runs the four roles in one Slurm
allocation (``submit_pull_suite.sh`` submits one allocation per benchmark).

Every option falls back to the ``NANO_*`` variable of the reference launcher
(:data:`SUITE_ENV`), so its environment-driven scripts run unchanged.  A run
keeps the benchmark's canonical settings unless it is labelled with a protocol
arm (:func:`resolve_suite`).  Workers report output token counts, and the
coordinator writes ``suite_summary.json`` beside the results: output tokens per
second and per GPU of this invocation and of all invocations of a resumed run.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import queue
import time
from multiprocessing.managers import BaseManager
from pathlib import Path
from typing import Any, Callable

_JOBS: "queue.Queue | None" = None
_RESULTS: "queue.Queue | None" = None
_MANIFEST: dict = {"digest": None}


def _jobs():
    return _JOBS


def _results():
    return _RESULTS


def _manifest():
    return _MANIFEST["digest"]


def _init_server(digest: str) -> None:
    global _JOBS, _RESULTS
    _JOBS, _RESULTS = queue.Queue(), queue.Queue()
    _MANIFEST["digest"] = digest


class SuiteManager(BaseManager):
    pass


SuiteManager.register("jobs", callable=_jobs)
SuiteManager.register("results", callable=_results)
SuiteManager.register("manifest", callable=_manifest)


def manifest_digest(manifest: dict) -> str:
    return hashlib.sha256(json.dumps(manifest, sort_keys=True, separators=(",", ":")).encode()).hexdigest()


def job_key(job: dict) -> tuple:
    return (str(job["benchmark"]), str(job["id"]), int(job["sample"]))


def completed_keys(path: str | Path) -> set:
    done = set()
    if Path(path).is_file():
        with open(path, encoding="utf-8") as fh:
            for line in fh:
                if line.strip():
                    done.add(job_key(json.loads(line)))
    return done


def run_coordinator(jobs: list[dict], results_path: str | Path, manifest: dict, address: tuple[str, int],
                    authkey: bytes, num_workers: int, timeout: float = 3600.0) -> dict[str, Any]:
    """Serve the pending jobs and collect their results (blocks until done)."""
    digest = manifest_digest(manifest)
    done = completed_keys(results_path)
    pending = [j for j in jobs if job_key(j) not in done]
    mgr = SuiteManager(address=address, authkey=authkey)
    mgr.start(initializer=_init_server, initargs=(digest,))
    try:
        jq, rq = mgr.jobs(), mgr.results()
        for job in pending:
            jq.put(job)
        got, deadline, out_tokens, t0 = 0, time.time() + timeout, 0, time.perf_counter()
        with open(results_path, "a", encoding="utf-8") as fh:
            while got < len(pending):
                try:
                    row = rq.get(timeout=1.0)
                except queue.Empty:
                    if time.time() > deadline:
                        raise TimeoutError(f"{len(pending) - got} jobs unfinished after {timeout} s")
                    continue
                if "worker_done" in row:  # a worker that found the queue empty and left early
                    continue
                if job_key(row) in done:  # a retried job finished twice: keep the first
                    continue
                done.add(job_key(row))
                fh.write(json.dumps(row, ensure_ascii=False) + "\n")
                fh.flush()
                got += 1
                out_tokens += int(row.get("output_token_count", 0))
        elapsed = time.perf_counter() - t0
        for _ in range(num_workers):
            jq.put(None)
        # every worker acknowledges its stop marker before the server goes away
        acked, ack_deadline = 0, time.time() + 30.0
        while acked < num_workers and time.time() < ack_deadline:
            try:
                row = rq.get(timeout=1.0)
            except queue.Empty:
                continue
            acked += int("worker_done" in row)
    finally:
        mgr.shutdown()
    summary = {"jobs": len(jobs), "resumed": len(jobs) - len(pending), "completed": got, "manifest": digest}
    summary.update(write_suite_summary(Path(results_path).with_name("suite_summary.json"), manifest, num_workers,
                                       {"num_generations": got, "output_tokens": out_tokens,
                                        "elapsed_seconds": elapsed}))
    return summary


def _rate(tokens: float, seconds: float, gpus: int = 1) -> float:
    return tokens / seconds / gpus if seconds and gpus else 0.0


def write_suite_summary(path: Path, manifest: dict, workers: int, invocation: dict) -> dict[str, Any]:
    """Throughput of this coordinator invocation and of every invocation of the run so far (a
    resumed run appends to the list), per second and per GPU (one worker = one GPU) -- the
    suite summary of ``evaluation/pull_suite.py:920-994``."""
    previous = []
    if path.is_file():
        previous = list(json.loads(path.read_text()).get("invocations", []))
    invocation = {**invocation, "worker_count": int(workers)}
    runs = previous + [invocation]
    busy = [r for r in runs if int(r.get("num_generations", 0)) > 0]
    busy_tokens = sum(int(r["output_tokens"]) for r in busy)
    busy_seconds = sum(float(r["elapsed_seconds"]) for r in busy)
    tokens, seconds = int(invocation["output_tokens"]), float(invocation["elapsed_seconds"])
    out = {"model": manifest.get("model"), "gated_lora_path": manifest.get("gated_lora_path"),
           "benchmarks": [e["name"] for e in manifest.get("benchmarks", [])], "worker_count": int(workers),
           "invocation_num_generations": int(invocation["num_generations"]), "invocation_output_tokens": tokens,
           "invocation_elapsed_seconds": seconds,
           "invocation_output_tokens_per_second": _rate(tokens, seconds),
           "invocation_output_tokens_per_second_per_gpu": _rate(tokens, seconds, workers),
           "generation_invocation_output_tokens": busy_tokens,
           "generation_invocation_elapsed_seconds": busy_seconds,
           "generation_invocation_output_tokens_per_second": _rate(busy_tokens, busy_seconds),
           "generation_invocation_output_tokens_per_second_per_gpu": _rate(busy_tokens, busy_seconds, workers),
           "invocations": runs}
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_suffix(".tmp")
    tmp.write_text(json.dumps(out, indent=2) + "\n")
    os.replace(tmp, path)
    return {k: v for k, v in out.items() if k != "invocations"}


def connect(address: tuple[str, int], authkey: bytes, deadline_s: float = 120.0) -> SuiteManager:
    end = time.time() + deadline_s
    while True:
        mgr = SuiteManager(address=address, authkey=authkey)
        try:
            mgr.connect()
            return mgr
        except (ConnectionRefusedError, OSError):
            if time.time() > end:
                raise
            time.sleep(0.5)


def run_worker(address: tuple[str, int], authkey: bytes, manifest: dict,
               generate: Callable[[list[dict]], list[str]], batch: int = 8, connect_deadline: float = 120.0) -> int:
    """Pull jobs until told to stop; ``generate`` maps jobs to generation texts."""
    mgr = connect(address, authkey, connect_deadline)
    want = manifest_digest(manifest)
    have = mgr.manifest()._getvalue()  # the manager hands back a proxy of the digest string
    if have != want:
        raise RuntimeError(f"manifest mismatch: coordinator {have}, worker {want}")
    jq, rq = mgr.jobs(), mgr.results()
    handled = 0
    stop = False
    while not stop:
        jobs = []
        try:
            job = jq.get(timeout=5.0)
        except queue.Empty:
            continue
        except (EOFError, ConnectionError, BrokenPipeError):
            return handled  # the coordinator finished and closed the queues
        while True:
            if job is None:
                stop = True
                break
            jobs.append(job)
            if len(jobs) >= batch:
                break
            try:
                job = jq.get_nowait()
            except queue.Empty:
                break
        if jobs:
            outs = generate(jobs)
            for job, out in zip(jobs, outs):
                row = {**{k: job[k] for k in ("benchmark", "id", "sample")}, "ground_truth": job.get("ground_truth"),
                       "worker": os.getpid()}
                if isinstance(out, str):
                    row["generation"] = out
                else:  # an engine result: text, token ids and decoder statistics
                    ids = list(out.token_ids)
                    row.update(generation=out.text, output_token_count=len(ids), stats=dict(out.stats))
                    if job.get("save_token_ids"):
                        row["token_ids"] = ids
                rq.put(row)
            handled += len(jobs)
    rq.put({"worker_done": os.getpid(), "handled": handled})
    return handled


def build_jobs(benchmarks: list[str], tokenizer, *, data_root: str | Path | None = None,
               num_samples: int | None = None, limit: int | None = None, context_length: int | None = None,
               max_tokens: int | None = None, reserve: int = 8) -> tuple[list[dict], list[dict]]:
    """Jobs of a suite run and the benchmark entries of its manifest.

    Per benchmark: its records (the registry's pinned file, or the file of the
    same name under ``data_root``), the canonical prompt rendering (chat
    template, instruction, chat-template kwargs), ``num_samples`` samples of
    each record (the benchmark's own count by default), and each job's
    completion budget -- the context length less the prompt and ``reserve``
    slots of the largest decode forward (the diffusion block), capped by the
    output limit -- as ``eval.run`` computes it.  Records whose prompt leaves no budget get no job.
    """
    from uno_b200.eval.benchmarks import get_benchmark
    from uno_b200.eval.data import ANSWER_FIELDS, ID_FIELDS, first_field, load_records, \
        protocol_artifact_fingerprint
    from uno_b200.eval.run import completion_budget
    from uno_b200.generation import format_chat_prompt

    jobs: list[dict] = []
    entries: list[dict] = []
    for name in benchmarks:
        bench = get_benchmark(name)
        path = Path(data_root) / bench.data_path.name if data_root else bench.data_path
        records = load_records(path, limit)
        rows, sha = protocol_artifact_fingerprint(path)
        samples = int(num_samples or bench.num_samples)
        context = int(context_length or bench.max_model_len)
        cap = int(max_tokens or bench.max_tokens)
        skipped = 0
        for idx, rec in enumerate(records):
            msgs = rec.get("chat_input")
            if not isinstance(msgs, list) or not msgs:
                raise ValueError(f"{bench.name} record {idx} needs a nonempty chat_input")
            ids, _, _ = format_chat_prompt(tokenizer, msgs, bench.instruction, dict(bench.chat_template_kwargs))
            rid = first_field(rec, ID_FIELDS)
            budget = completion_budget(len(ids), context, reserve, cap)
            if budget <= 0:
                skipped += 1
                continue
            for sample in range(samples):
                jobs.append({"benchmark": bench.name, "id": idx if rid is None else rid, "sample": sample,
                             "prompt_ids": ids, "max_tokens": budget,
                             "ground_truth": first_field(rec, ANSWER_FIELDS)})
        entries.append({"name": bench.name, "data": str(path), "rows": rows, "sha256": sha, "num_samples": samples,
                        "context_length": context, "max_tokens": cap, "skipped_no_budget": skipped,
                        "sampling": {"temperature": bench.temperature, "top_p": bench.top_p, "top_k": bench.top_k}})
    return jobs, entries


def suite_sampling(entries: list[dict], overrides: dict | None = None) -> dict:
    """The one sampling setting of a run: the benchmarks' canonical one, or explicit overrides."""
    chosen = {k: v for k, v in (overrides or {}).items() if v is not None}
    for key in ("temperature", "top_p", "top_k"):
        if key in chosen:
            continue
        values = {json.dumps(e["sampling"][key]) for e in entries}
        if len(values) > 1:
            raise ValueError(f"the benchmarks disagree on {key}; run them in separate allocations or set it")
        chosen[key] = entries[0]["sampling"][key] if entries else None
    return chosen


def score_results(results: str | Path, manifest: dict, out_dir: str | Path, judge=None) -> dict[str, Any]:
    """Split the results file per benchmark and grade each part."""
    from uno_b200.eval.data import read_jsonl
    from uno_b200.eval.score import score_file

    out_dir = Path(out_dir)
    by_bench: dict[str, list[dict]] = {}
    for row in read_jsonl(results):
        by_bench.setdefault(str(row["benchmark"]), []).append(row)
    summary = {}
    for entry in manifest.get("benchmarks", []):
        name = entry["name"]
        rows = sorted(by_bench.get(name, []), key=lambda r: (str(r["id"]), int(r["sample"])))
        bdir = out_dir / name
        bdir.mkdir(parents=True, exist_ok=True)
        gen = bdir / "generations.jsonl"
        gen.write_text("".join(json.dumps(r, ensure_ascii=False) + "\n" for r in rows), encoding="utf-8")
        summary[name] = score_file(gen, benchmark=name, data=entry["data"], grades_out=bdir / "grades.jsonl",
                                   scores_out=bdir / "scores.json", judge=judge)
    return summary


def engine_generator(model: str, sampling_params, **engine_kwargs) -> Callable[[list[dict]], list[str]]:
    """Generation callable backed by one AsyncLLMEngine (continuous batching across pulls)."""
    from uno_b200.engine.async_engine import AsyncLLMEngine
    from uno_b200.llm import LLM

    engine = AsyncLLMEngine(LLM(model, **engine_kwargs), sampling_params)
    engine.start()

    def generate(jobs: list[dict]) -> list[str]:
        futs = [engine.submit(j["prompt_ids"], request_id=f"{j['benchmark']}/{j['id']}/{j['sample']}",
                              max_tokens=j.get("max_tokens")) for j in jobs]
        return [f.result() for f in futs]

    generate.engine = engine
    return generate


# Options read from the environment variables of the reference's pull-suite launcher when the
# command line leaves them unset (``evaluation/pull_suite.py:105-285``).
SUITE_ENV = {
    "model": "NANO_MODEL", "model_revision": "NANO_MODEL_REVISION", "tokenizer_path": "NANO_TOKENIZER_PATH",
    "tokenizer_revision": "NANO_TOKENIZER_REVISION", "gated_lora_path": "NANO_GATED_LORA_PATH",
    "gated_lora_revision": "NANO_GATED_LORA_REVISION", "hf_cache_dir": "NANO_HF_CACHE_DIR",
    "hf_local_files_only": "NANO_HF_LOCAL_FILES_ONLY", "protocol_arm": "NANO_PROTOCOL_ARM",
    "data_root": "NANO_DATA_ROOT", "num_samples": "NANO_NUM_SAMPLES", "limit": "NANO_LIMIT",
    "max_num_seqs": "NANO_MAX_NUM_SEQS", "context_length": "NANO_CONTEXT_LENGTH",
    "max_num_batched_tokens": "NANO_MAX_NUM_BATCHED_TOKENS", "gpu_memory_utilization": "NANO_GPU_MEMORY_UTILIZATION",
    "attention_backend": "NANO_ATTENTION_BACKEND", "max_tokens": "NANO_MAX_TOKENS", "temperature": "NANO_TEMPERATURE",
    "top_k": "NANO_TOP_K", "top_p": "NANO_TOP_P", "diffusion_block_size": "NANO_DIFFUSION_BLOCK_SIZE",
    "tree_verify_size": "NANO_TREE_VERIFY_SIZE", "tree_candidate_top_k": "NANO_TREE_CANDIDATE_TOP_K",
    "torch_compile": "NANO_TORCH_COMPILE", "noise_mode": "NANO_NOISE_MODE", "noise_salt": "NANO_NOISE_SALT",
    "ignore_eos": "NANO_IGNORE_EOS", "mask_token_id": "NANO_MASK_TOKEN_ID", "stop_token_ids": "NANO_STOP_TOKEN_IDS",
    "cuda_graph_block_sizes": "NANO_CUDA_GRAPH_BLOCK_SIZES", "cuda_graph_batch_sizes": "NANO_CUDA_GRAPH_BATCH_SIZES",
    "save_token_ids": "NANO_SAVE_TOKEN_IDS", "benchmark": "NANO_BENCHMARKS",
}
_FLAGS = {"hf_local_files_only", "torch_compile", "ignore_eos", "save_token_ids"}
_INT_LISTS = {"stop_token_ids", "cuda_graph_block_sizes", "cuda_graph_batch_sizes"}


def _flag(raw: str) -> bool:
    return raw.strip().lower() in {"1", "true", "yes", "on"}


def _ints(raw: str) -> list[int]:
    return [int(x) for x in str(raw).replace(",", " ").split()]


def apply_env(args, env=None) -> None:
    """Fill every option the command line left unset from its ``NANO_*`` variable."""
    env = os.environ if env is None else env
    for dest, var in SUITE_ENV.items():
        raw = env.get(var)
        if raw is None or not raw.strip() or getattr(args, dest) not in (None, False, []):
            continue
        if dest in _FLAGS:
            value = _flag(raw)
        elif dest in _INT_LISTS:
            value = _ints(raw)
        elif dest == "benchmark":
            value = raw.replace(",", " ").split()
        else:
            value = raw if dest in _TEXT else (float(raw) if dest in _FLOATS else int(raw))
        setattr(args, dest, value)
    for dest, value in SUITE_DEFAULTS.items():
        if getattr(args, dest) is None:
            setattr(args, dest, value)


SUITE_DEFAULTS = {"diffusion_block_size": 16, "tree_candidate_top_k": 16, "noise_mode": "random_uniform",
                  "attention_backend": "native", "gpu_memory_utilization": 0.9}
_TEXT = {"model", "model_revision", "tokenizer_path", "tokenizer_revision", "gated_lora_path", "gated_lora_revision",
         "hf_cache_dir", "protocol_arm", "data_root", "attention_backend", "noise_mode"}
_FLOATS = {"gpu_memory_utilization", "temperature", "top_p"}


def resolve_suite(args) -> dict[str, Any]:
    """Canonical settings of a single-benchmark run; departures need ``--protocol-arm``.

    A canonical run covers exactly one benchmark with that benchmark's samples,
    context, budget, batch and sampling, and all of its records
    (``evaluation/pull_suite.py:155-185,295-303``).  A labelled protocol arm may
    span several benchmarks with one uniform setting.  Returns the departures.
    """
    from uno_b200.eval.benchmarks import get_benchmark

    names = list(dict.fromkeys(get_benchmark(b).name for b in args.benchmark))
    if len(names) != len(args.benchmark):
        raise SystemExit(f"benchmarks listed twice: {args.benchmark}")
    if len(names) != 1 and not args.protocol_arm:
        raise SystemExit("a canonical run evaluates one benchmark (one allocation each, submit_pull_suite.sh); "
                         "name a --protocol-arm to run several with one setting")
    if args.limit is not None and args.limit < 1:
        raise SystemExit("--limit must be positive")
    if args.num_samples is not None and args.num_samples < 1:
        raise SystemExit("--num-samples must be positive")
    departures: dict[str, Any] = {}
    bench = get_benchmark(names[0]) if len(names) == 1 else None
    canonical = {"num_samples": bench.num_samples, "context_length": bench.max_model_len,
                 "max_tokens": bench.max_tokens, "max_num_seqs": bench.max_num_seqs,
                 "temperature": bench.temperature, "top_k": bench.top_k, "top_p": bench.top_p} if bench else {}
    for name, value in canonical.items():
        got = getattr(args, name)
        if got is None:
            setattr(args, name, value)
        elif got != value:
            departures[name] = {"canonical": value, "actual": got}
    if args.max_num_seqs is None:
        args.max_num_seqs = 64
    context = args.context_length
    if args.max_num_batched_tokens is None:
        args.max_num_batched_tokens = context
    elif bench is not None and args.max_num_batched_tokens != context:
        departures["max_num_batched_tokens"] = {"canonical": context, "actual": args.max_num_batched_tokens}
    if args.limit is not None:
        departures["limit"] = {"canonical": None, "actual": args.limit}
    if departures and not args.protocol_arm:
        raise SystemExit("departures from the canonical protocol need --protocol-arm (NANO_PROTOCOL_ARM): "
                         + ", ".join(f"{k}={v['actual']!r} (canonical {v['canonical']!r})"
                                     for k, v in departures.items()))
    if args.tree_verify_size is not None and args.torch_compile:
        raise SystemExit("tree verification runs without --torch-compile")
    return departures


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("role", choices=("jobs", "coordinator", "worker", "score"))
    ap.add_argument("--address", help="coordinator HOST:PORT (listen or connect; default from "
                                      "NANO_PULL_COORDINATOR_HOST / _PORT, else 127.0.0.1:50123)")
    ap.add_argument("--authkey", default=os.environ.get("UNO_SUITE_AUTHKEY", os.environ.get("NANO_PULL_AUTH_KEY",
                                                                                               "uno-b200")))
    ap.add_argument("--connect-timeout", type=float, default=float(os.environ.get("NANO_PULL_CONNECT_TIMEOUT", 120)))
    ap.add_argument("--jobs", type=Path, help="JSONL of jobs (written by the jobs role, read by the coordinator)")
    ap.add_argument("--manifest", type=Path, help="JSON run manifest shared by all roles (default: "
                                                  "$NANO_RESULTS_ROOT/$NANO_RUN_NAME/run_manifest.json)")
    ap.add_argument("--output", type=Path, help="results JSONL (default: results.jsonl beside the manifest)")
    ap.add_argument("--num-workers", type=int, default=1)
    ap.add_argument("--model", help="model directory, hub id or preset")
    ap.add_argument("--model-revision")
    ap.add_argument("--tokenizer-path")
    ap.add_argument("--tokenizer-revision")
    ap.add_argument("--gated-lora-path")
    ap.add_argument("--gated-lora-revision")
    ap.add_argument("--hf-cache-dir")
    ap.add_argument("--hf-local-files-only", action="store_true")
    ap.add_argument("--protocol-arm", help="label of a run that departs from the canonical protocol")
    ap.add_argument("--benchmark", action="append", default=[], help="jobs: a registered benchmark (repeatable)")
    ap.add_argument("--data-root", help="jobs: directory of the prepared benchmark files")
    ap.add_argument("--num-samples", type=int)
    ap.add_argument("--limit", type=int)
    ap.add_argument("--context-length", type=int)
    ap.add_argument("--max-tokens", type=int)
    ap.add_argument("--max-num-seqs", type=int)
    ap.add_argument("--max-num-batched-tokens", type=int)
    ap.add_argument("--gpu-memory-utilization", type=float)
    ap.add_argument("--attention-backend", help="accepted for script compatibility (one attention implementation)")
    ap.add_argument("--temperature", type=float, help="jobs: override the benchmarks' temperature")
    ap.add_argument("--top-p", type=float)
    ap.add_argument("--top-k", type=int)
    ap.add_argument("--diffusion-block-size", type=int)
    ap.add_argument("--tree-verify-size", type=int)
    ap.add_argument("--tree-candidate-top-k", type=int)
    ap.add_argument("--torch-compile", action="store_true", help="accepted for script compatibility")
    ap.add_argument("--noise-mode")
    ap.add_argument("--noise-salt", type=int)
    ap.add_argument("--ignore-eos", action="store_true")
    ap.add_argument("--mask-token-id", type=int)
    ap.add_argument("--stop-token-ids", type=_ints, help="comma-separated stop token ids")
    ap.add_argument("--cuda-graph-block-sizes", type=_ints)
    ap.add_argument("--cuda-graph-batch-sizes", type=_ints)
    ap.add_argument("--save-token-ids", action="store_true")
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--out-dir", type=Path, help="score: directory of the per-benchmark grades")
    return ap


def _paths(args) -> None:
    run_dir = None
    if os.environ.get("NANO_RESULTS_ROOT") and os.environ.get("NANO_RUN_NAME"):
        run_dir = Path(os.environ["NANO_RESULTS_ROOT"]) / os.environ["NANO_RUN_NAME"]
    if args.manifest is None:
        if run_dir is None:
            raise SystemExit("--manifest is required (or NANO_RESULTS_ROOT and NANO_RUN_NAME)")
        args.manifest = run_dir / "run_manifest.json"
    if args.output is None:
        args.output = args.manifest.with_name("results.jsonl")
    if args.jobs is None:
        args.jobs = args.manifest.with_name("jobs.jsonl")
    if args.address is None:
        host = os.environ.get("NANO_PULL_COORDINATOR_HOST", "127.0.0.1")
        args.address = f"{host}:{os.environ.get('NANO_PULL_COORDINATOR_PORT', '50123')}"


def jobs_role(args) -> dict:
    from uno_b200.generation import resolve_model_sources
    from uno_b200.utils.hf_compat import load_model_config, load_tokenizer
    from uno_b200.utils.hub import resolve_hf_snapshot
    from uno_b200.utils.model_tokens import resolve_model_token_ids

    if not args.benchmark or not args.model:
        raise SystemExit("jobs needs --benchmark (or NANO_BENCHMARKS) and --model (or NANO_MODEL)")
    departures = resolve_suite(args)
    model, adapter = resolve_model_sources(args.model, args.gated_lora_path)
    model_dir = resolve_hf_snapshot(model, revision=args.model_revision, cache_dir=args.hf_cache_dir,
                                    local_files_only=args.hf_local_files_only, artifact_name="model")
    tokenizer = load_tokenizer(args.tokenizer_path or model_dir, load_model_config(model_dir))
    mask_id, stop_ids, _ = resolve_model_token_ids(model_dir, tokenizer, mask_token_id=args.mask_token_id,
                                                   stop_token_ids=args.stop_token_ids, noise_mode=args.noise_mode)
    reserve = max(args.diffusion_block_size, args.tree_verify_size or 0)  # the largest decode forward's slots
    jobs, entries = build_jobs(args.benchmark, tokenizer, data_root=args.data_root, num_samples=args.num_samples,
                               limit=args.limit, context_length=args.context_length, max_tokens=args.max_tokens,
                               reserve=reserve)
    if args.save_token_ids:
        for job in jobs:
            job["save_token_ids"] = True
    block = args.diffusion_block_size
    manifest = {"model": args.model, "model_revision": args.model_revision, "gated_lora_path": adapter,
                "gated_lora_revision": args.gated_lora_revision, "tokenizer_path": args.tokenizer_path,
                "tokenizer_revision": args.tokenizer_revision or (args.model_revision if not args.tokenizer_path
                                                                  else None),
                "diffusion_block_size": block, "protocol_arm": args.protocol_arm, "overrides": departures,
                "benchmarks": entries,
                "sampling": suite_sampling(entries, {"temperature": args.temperature, "top_p": args.top_p,
                                                     "top_k": args.top_k}),
                "engine": {"max_num_seqs": args.max_num_seqs, "max_model_len": args.context_length,
                           "max_num_batched_tokens": args.max_num_batched_tokens,
                           "gpu_memory_utilization": args.gpu_memory_utilization,
                           "max_diffusion_block_size": max(block, args.tree_verify_size or 0),
                           "tree_verify_size": args.tree_verify_size,
                           "tree_candidate_top_k": args.tree_candidate_top_k,
                           "cuda_graph_block_sizes": args.cuda_graph_block_sizes or sorted({1, block}),
                           "cuda_graph_batch_sizes": args.cuda_graph_batch_sizes},
                "request": {"mask_token_id": mask_id, "stop_token_ids": stop_ids, "noise_mode": args.noise_mode,
                            "noise_salt": args.noise_salt, "ignore_eos": bool(args.ignore_eos)}}
    args.jobs.parent.mkdir(parents=True, exist_ok=True)
    args.jobs.write_text("".join(json.dumps(j) + "\n" for j in jobs), encoding="utf-8")
    args.manifest.parent.mkdir(parents=True, exist_ok=True)
    args.manifest.write_text(json.dumps(manifest, indent=2, sort_keys=True) + "\n", encoding="utf-8")
    return {"jobs": len(jobs), "manifest": manifest_digest(manifest)}


def worker_settings(manifest: dict, args) -> tuple[Any, dict]:
    """``(SamplingParams, LLM keyword arguments)`` of a worker, all from the run manifest."""
    from uno_b200.sampling_params import SamplingParams

    samp, req, eng = manifest.get("sampling", {}), manifest.get("request", {}), dict(manifest.get("engine", {}))
    block = int(manifest.get("diffusion_block_size", 16))
    sp = SamplingParams(temperature=samp.get("temperature", 1.0), top_p=samp.get("top_p"), top_k=samp.get("top_k"),
                        diffusion_block_size=block, mask_token_id=req.get("mask_token_id", args.mask_token_id),
                        stop_token_ids=req.get("stop_token_ids"), noise_mode=req.get("noise_mode", "random_uniform"),
                        noise_salt=req.get("noise_salt"), ignore_eos=bool(req.get("ignore_eos", False)),
                        max_tokens=1 << 30)
    kwargs = {k: v for k, v in eng.items() if v is not None}
    kwargs.setdefault("max_diffusion_block_size", block)
    for key in ("model_revision", "gated_lora_revision"):
        if manifest.get(key):
            kwargs[key] = manifest[key]
    if manifest.get("tokenizer_path"):
        kwargs["tokenizer_path"] = manifest["tokenizer_path"]
    if args.hf_cache_dir:
        kwargs["hf_cache_dir"] = args.hf_cache_dir
    if args.hf_local_files_only:
        kwargs["hf_local_files_only"] = True
    return sp, {"device": args.device, "gated_lora_path": manifest.get("gated_lora_path"), **kwargs}


def main(argv=None):
    args = build_parser().parse_args(argv)
    apply_env(args)
    _paths(args)
    host, port = args.address.rsplit(":", 1)
    address, authkey = (host, int(port)), args.authkey.encode()
    if args.role == "jobs":
        print(json.dumps(jobs_role(args)))
        return
    manifest = json.loads(args.manifest.read_text())
    if args.role == "score":
        print(json.dumps(score_results(args.output, manifest, args.out_dir or args.output.parent), indent=2))
    elif args.role == "coordinator":
        jobs = [json.loads(line) for line in args.jobs.read_text().splitlines() if line.strip()]
        print(json.dumps(run_coordinator(jobs, args.output, manifest, address, authkey, args.num_workers)))
    else:
        sp, kwargs = worker_settings(manifest, args)
        gen = engine_generator(args.model or manifest["model"], sp, **kwargs)
        try:
            print(json.dumps({"handled": run_worker(address, authkey, manifest, gen,
                                                    connect_deadline=args.connect_timeout)}))
        finally:
            gen.engine.shutdown()


if __name__ == "__main__":
    main()
