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

CLI: ``python -m uno_b200.eval.pull_suite coordinator|worker ...``.
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
    ap.add_argument("role", choices=("coordinator", "worker"))
    ap.add_argument("--address", default="127.0.0.1:50123")
    ap.add_argument("--authkey", default=os.environ.get("UNO_SUITE_AUTHKEY", "uno-b200"))
    ap.add_argument("--jobs", type=Path, help="coordinator: JSONL of jobs (benchmark, id, sample, prompt_ids, ...)")
    ap.add_argument("--manifest", type=Path, required=True, help="JSON run manifest shared by all roles")
    ap.add_argument("--output", type=Path, default=Path("suite-results.jsonl"))
    ap.add_argument("--num-workers", type=int, default=1)
    ap.add_argument("--model", help="worker: model directory or preset")
    ap.add_argument("--temperature", type=float, default=1.0)
    ap.add_argument("--diffusion-block-size", type=int, default=8)
    ap.add_argument("--mask-token-id", type=int)
    ap.add_argument("--device", default="cuda")
    args = ap.parse_args(argv)
    host, port = args.address.rsplit(":", 1)
    address, authkey = (host, int(port)), args.authkey.encode()
    manifest = json.loads(args.manifest.read_text())
    if args.role == "coordinator":
        jobs = [json.loads(line) for line in args.jobs.read_text().splitlines() if line.strip()]
        print(json.dumps(run_coordinator(jobs, args.output, manifest, address, authkey, args.num_workers)))
    else:
        from uno_b200.sampling_params import SamplingParams

        sp = SamplingParams(temperature=args.temperature, diffusion_block_size=args.diffusion_block_size,
                            mask_token_id=args.mask_token_id, max_tokens=1 << 30)
        gen = engine_generator(args.model, sp, device=args.device, max_diffusion_block_size=args.diffusion_block_size)
        try:
            print(json.dumps({"handled": run_worker(address, authkey, manifest, gen)}))
        finally:
            gen.engine.shutdown()


if __name__ == "__main__":
    main()
