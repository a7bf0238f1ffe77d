"""Thread-driven front end over one synchronous :class:`LLMEngine`.

Behaviour of ``nano_vllm_uno/engine/async_engine.py:13-211``:

* ``start()`` launches one daemon thread that owns the engine; ``submit()``
  is thread-safe and returns a ``concurrent.futures.Future`` resolving to a
  :class:`GenerationResult` when that request finishes;
* every request of one front end shares a single :class:`SamplingParams`
  (the decode step batches them together); ``max_tokens`` may differ per
  request;
* a fatal engine error fails every pending future with that error and makes
  later ``submit()`` calls raise; ``shutdown()`` stops the thread after the
  current step, fails unfinished requests and releases the engine.

The loop sleeps on a condition variable while the engine has nothing
scheduled, so an idle front end costs no CPU.
"""

from __future__ import annotations

import collections
import concurrent.futures
import threading
import uuid
from dataclasses import dataclass
from typing import Any

from uno_b200.sampling_params import SamplingParams


@dataclass(frozen=True)
class GenerationResult:
    request_id: str
    text: str
    token_ids: list[int]
    stats: dict[str, int]


@dataclass
class _Request:
    request_id: str
    prompt: str | list[int]
    future: concurrent.futures.Future
    max_tokens: int | None = None


class AsyncLLMEngine:
    """Run one synchronous engine behind a persistent request inbox."""

    def __init__(self, engine: Any, sampling_params: SamplingParams) -> None:
        self.engine = engine
        self.sampling_params = sampling_params
        self._cv = threading.Condition()
        self._inbox: collections.deque[_Request] = collections.deque()
        self._stop = False
        self._accepting = False
        self._thread: threading.Thread | None = None
        self._fatal: BaseException | None = None
        self._by_seq: dict[int, _Request] = {}

    # ------------------------------------------------------------ control
    def start(self) -> None:
        with self._cv:
            if self._thread is not None:
                if self._thread.is_alive():
                    return
                raise RuntimeError("AsyncLLMEngine cannot be restarted after shutdown")
            self._accepting = True
            self._thread = threading.Thread(target=self._loop, name="uno-b200-engine", daemon=True)
            self._thread.start()

    def submit(self, prompt: str | list[int], *, request_id: str | None = None,
               max_tokens: int | None = None) -> concurrent.futures.Future:
        with self._cv:
            if not self._accepting:
                if self._fatal is not None:
                    raise RuntimeError("AsyncLLMEngine has failed") from self._fatal
                raise RuntimeError("AsyncLLMEngine is not running")
            fut: concurrent.futures.Future = concurrent.futures.Future()
            self._inbox.append(_Request(request_id or uuid.uuid4().hex, prompt, fut, max_tokens))
            self._cv.notify()
            return fut

    def shutdown(self, timeout: float | None = 30.0) -> None:
        with self._cv:
            self._accepting = False
            thread = self._thread
            if thread is None:
                return
            self._stop = True
            self._cv.notify()
        thread.join(timeout=timeout)
        if thread.is_alive():
            raise TimeoutError("Timed out waiting for AsyncLLMEngine to stop")

    @property
    def is_running(self) -> bool:
        with self._cv:
            t = self._thread
            return bool(self._accepting and self._fatal is None and t is not None and t.is_alive())

    @property
    def fatal_error(self) -> BaseException | None:
        with self._cv:
            return self._fatal

    # ------------------------------------------------------------- thread
    def _take_inbox(self) -> tuple[list[_Request], bool]:
        """Block while idle; return the new requests and whether to stop."""
        with self._cv:
            while not self._inbox and not self._stop and self.engine.is_finished():
                self._cv.wait()
            batch = list(self._inbox)
            self._inbox.clear()
            return batch, self._stop

    def _admit(self, req: _Request) -> None:
        if not req.future.set_running_or_notify_cancel():
            return  # cancelled before it reached the engine
        try:
            seq_id = self.engine.add_request(req.prompt, self.sampling_params, max_tokens=req.max_tokens)
        except BaseException as exc:  # a bad request fails alone
            req.future.set_exception(exc)
            return
        if seq_id in self._by_seq:
            err = RuntimeError(f"Duplicate scheduler sequence id: {seq_id}")
            req.future.set_exception(err)
            raise err
        self._by_seq[seq_id] = req

    def _finish(self, outputs) -> None:
        for seq_id, token_ids, stats in outputs:
            req = self._by_seq.pop(seq_id, None)
            if req is None:
                raise RuntimeError(f"Completed scheduler sequence {seq_id} has no pending request")
            out = self.engine.finalize_output(token_ids, stats, self.sampling_params)
            req.future.set_result(GenerationResult(request_id=req.request_id, text=str(out["text"]),
                                                   token_ids=list(out["token_ids"]), stats=dict(out["stats"])))

    def _fail_all(self, error: BaseException) -> None:
        pending = list(self._by_seq.values())
        self._by_seq.clear()
        with self._cv:
            pending += list(self._inbox)
            self._inbox.clear()
        for req in pending:
            if not req.future.done():
                req.future.set_exception(error)

    def _loop(self) -> None:
        try:
            while True:
                batch, stop = self._take_inbox()
                if stop:
                    break
                for req in batch:
                    self._admit(req)
                if not self.engine.is_finished():
                    outputs, _ = self.engine.step()
                    self._finish(outputs)
        except BaseException as exc:
            with self._cv:
                self._fatal = exc
            self._fail_all(exc)
        finally:
            with self._cv:
                self._accepting = False
            self._fail_all(RuntimeError("AsyncLLMEngine stopped before request completion"))
            self.engine.exit()
