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
        got, deadline = 0, time.time() + timeout
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
    return {"jobs": len(jobs), "resumed": len(jobs) - len(pending), "completed": got, "manifest": digest}


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
            texts = generate(jobs)
            for job, text in zip(jobs, texts):
                rq.put({**{k: job[k] for k in ("benchmark", "id", "sample")}, "generation": text,
                        "ground_truth": job.get("ground_truth"), "worker": os.getpid()})
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
        return [f.result().text for f in futs]

    generate.engine = engine
    return generate


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("role", choices=("jobs", "coordinator", "worker", "score"))
    ap.add_argument("--address", default="127.0.0.1:50123", help="coordinator HOST:PORT (listen or connect)")
    ap.add_argument("--authkey", default=os.environ.get("UNO_SUITE_AUTHKEY", "uno-b200"))
    ap.add_argument("--jobs", type=Path, help="JSONL of jobs (written by the jobs role, read by the coordinator)")
    ap.add_argument("--manifest", type=Path, required=True, help="JSON run manifest shared by all roles")
    ap.add_argument("--output", type=Path, default=Path("suite-results.jsonl"), help="results JSONL")
    ap.add_argument("--num-workers", type=int, default=1)
    ap.add_argument("--model", help="model directory, hub id or preset")
    ap.add_argument("--tokenizer-path")
    ap.add_argument("--benchmark", action="append", default=[], help="jobs: a registered benchmark (repeatable)")
    ap.add_argument("--data-root", help="jobs: directory of the prepared benchmark files")
    ap.add_argument("--num-samples", type=int)
    ap.add_argument("--limit", type=int)
    ap.add_argument("--context-length", type=int)
    ap.add_argument("--max-tokens", type=int)
    ap.add_argument("--temperature", type=float, help="jobs: override the benchmarks' temperature")
    ap.add_argument("--top-p", type=float)
    ap.add_argument("--top-k", type=int)
    ap.add_argument("--diffusion-block-size", type=int, default=8)
    ap.add_argument("--mask-token-id", type=int)
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--out-dir", type=Path, help="score: directory of the per-benchmark grades")
    args = ap.parse_args(argv)
    host, port = args.address.rsplit(":", 1)
    address, authkey = (host, int(port)), args.authkey.encode()
    if args.role == "jobs":
        from uno_b200.generation import resolve_model_sources
        from uno_b200.utils.hf_compat import load_model_config, load_tokenizer
        from uno_b200.utils.hub import resolve_hf_snapshot

        if not args.benchmark or not args.model or not args.jobs:
            raise SystemExit("jobs needs --benchmark, --model and --jobs")
        model, adapter = resolve_model_sources(args.model, None)
        model_dir = resolve_hf_snapshot(model, artifact_name="model")
        tokenizer = load_tokenizer(args.tokenizer_path or model_dir, load_model_config(model_dir))
        jobs, entries = build_jobs(args.benchmark, tokenizer, data_root=args.data_root, num_samples=args.num_samples,
                                   limit=args.limit, context_length=args.context_length, max_tokens=args.max_tokens,
                                   reserve=args.diffusion_block_size)  # the largest decode forward's slots
        manifest = {"model": args.model, "gated_lora_path": adapter, "diffusion_block_size": args.diffusion_block_size,
                    "benchmarks": entries,
                    "sampling": suite_sampling(entries, {"temperature": args.temperature, "top_p": args.top_p,
                                                         "top_k": args.top_k})}
        args.jobs.parent.mkdir(parents=True, exist_ok=True)
        args.jobs.write_text("".join(json.dumps(j) + "\n" for j in jobs), encoding="utf-8")
        args.manifest.write_text(json.dumps(manifest, indent=2, sort_keys=True) + "\n", encoding="utf-8")
        print(json.dumps({"jobs": len(jobs), "manifest": manifest_digest(manifest)}))
        return
    manifest = json.loads(args.manifest.read_text())
    if args.role == "score":
        print(json.dumps(score_results(args.output, manifest, args.out_dir or args.output.parent), indent=2))
    elif args.role == "coordinator":
        jobs = [json.loads(line) for line in args.jobs.read_text().splitlines() if line.strip()]
        print(json.dumps(run_coordinator(jobs, args.output, manifest, address, authkey, args.num_workers)))
    else:
        from uno_b200.sampling_params import SamplingParams

        samp = manifest.get("sampling", {})
        block = int(manifest.get("diffusion_block_size", args.diffusion_block_size))
        sp = SamplingParams(temperature=samp.get("temperature", 1.0), top_p=samp.get("top_p"),
                            top_k=samp.get("top_k"), diffusion_block_size=block,
                            mask_token_id=args.mask_token_id, max_tokens=1 << 30)
        gen = engine_generator(args.model or manifest["model"], sp, device=args.device,
                               gated_lora_path=manifest.get("gated_lora_path"), max_diffusion_block_size=block)
        try:
            print(json.dumps({"handled": run_worker(address, authkey, manifest, gen)}))
        finally:
            gen.engine.shutdown()


if __name__ == "__main__":
    main()
