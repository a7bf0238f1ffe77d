"""Data-parallel replica process: ``python -m uno_b200.dp_worker <fd>``.

One replica is one independent engine (its own tensor-parallel group, KV cache
and scheduler) on the GPU slice that the parent put in ``CUDA_VISIBLE_DEVICES``.
It talks to the parent (:class:`uno_b200.llm.ReplicaSet`) over the inherited
duplex pipe ``fd`` with tagged tuples:

parent -> replica
    ``("init", model, tokenizer_path, engine_kwargs)``  build the engine (first message)
    ``("work", prompts, sampling_params, generate_kwargs, stream)``  one generate call
    ``("quit",)``  release the engine and exit

replica -> parent
    ``("up",)``  the engine is built
    ``("tick", [stats, ...])``  decode statistics of requests that just finished (only with ``stream``)
    ``("done", outputs, totals)``  outputs in prompt order and the summed decode statistics
    ``("fault", phase, traceback_text)``  ``phase`` is ``"init"`` or ``"work"``

A failed ``work`` message leaves the replica serving; a failed ``init`` ends it.
The reference replica loop is ``nano_vllm_uno/dp_worker.py:18-55``.
"""

from __future__ import annotations

import sys
import traceback
from multiprocessing.connection import Connection

from uno_b200.engine.sequence import DECODE_STAT_KEYS


def sum_decode_stats(outputs) -> dict[str, int]:
    """Per-key totals of the ``stats`` dicts of a list of generate outputs."""
    totals = dict.fromkeys(DECODE_STAT_KEYS, 0)
    for out in outputs:
        for key, value in out["stats"].items():
            if key in totals:
                totals[key] += int(value)
    return totals


def _serve(conn: Connection, engine) -> None:
    while True:
        msg = conn.recv()
        if msg[0] == "quit":
            return
        if msg[0] != "work":
            conn.send(("fault", "work", f"unknown message tag {msg[0]!r}"))
            continue
        _, prompts, sp, gen_kwargs, stream = msg
        report = (lambda finished: conn.send(("tick", list(finished)))) if stream else None
        try:
            outputs = engine.generate(prompts, sp, progress_callback=report, **gen_kwargs)
        except BaseException:  # the caller decides; this replica keeps serving
            conn.send(("fault", "work", traceback.format_exc()))
        else:
            conn.send(("done", outputs, sum_decode_stats(outputs)))


def main(fd: int) -> None:
    conn = Connection(fd)
    engine = None
    try:
        tag, model, tokenizer_path, engine_kwargs = conn.recv()
        if tag != "init":
            raise RuntimeError(f"expected an init message, got {tag!r}")
        from uno_b200.engine.llm_engine import LLMEngine

        engine = LLMEngine(model, tokenizer_path, **engine_kwargs)
        conn.send(("up",))
        _serve(conn, engine)
    except BaseException:
        try:
            conn.send(("fault", "init" if engine is None else "work", traceback.format_exc()))
        except (BrokenPipeError, EOFError, OSError):
            pass  # the parent is gone
    finally:
        try:
            if engine is not None:
                engine.exit()
        finally:
            conn.close()


if __name__ == "__main__":
    main(int(sys.argv[1]))
