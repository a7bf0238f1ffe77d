"""Data-parallel replica process (``python -m uno_b200.dp_worker <fd>``).

Protocol of ``nano_vllm_uno/dp_worker.py:18-55`` over an inherited pipe fd:
receive ``(model, tokenizer_path, kwargs)``, build an :class:`LLMEngine`, reply
``(True, None)``; then serve ``("generate", prompts, sp, kwargs, report)``
(optionally streaming ``("progress", stats)`` messages) until ``("exit",)``.
Failures are reported as ``(False, traceback)``.
"""

from __future__ import annotations

import sys
import traceback
from multiprocessing.connection import Connection

from uno_b200.engine.sequence import DECODE_STAT_KEYS


def aggregate_output_stats(outputs) -> dict[str, int]:
    return {k: sum(int(o["stats"][k]) for o in outputs) for k in DECODE_STAT_KEYS}


def main(fd: int) -> None:
    from uno_b200.engine.llm_engine import LLMEngine

    conn = Connection(fd)
    engine = None
    try:
        model, tokenizer_path, kwargs = conn.recv()
        engine = LLMEngine(model, tokenizer_path, **kwargs)
        conn.send((True, None))
        while True:
            cmd = conn.recv()
            if cmd[0] == "exit":
                break
            _, prompts, sp, gen_kwargs, report = cmd
            try:
                cb = (lambda stats: conn.send(("progress", stats))) if report else None
                outs = engine.generate(prompts, sp, progress_callback=cb, **gen_kwargs)
                conn.send((True, (outs, aggregate_output_stats(outs))))
            except BaseException:
                conn.send((False, traceback.format_exc()))
    except BaseException:
        try:
            conn.send((False, traceback.format_exc()))
        except (BrokenPipeError, EOFError, OSError):
            pass
    finally:
        if engine is not None:
            engine.exit()
        conn.close()


if __name__ == "__main__":
    main(int(sys.argv[1]))
