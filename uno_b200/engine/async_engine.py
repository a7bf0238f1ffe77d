"""Thread-driven front end over one synchronous :class:`LLMEngine`.

Public behaviour of ``nano_vllm_uno/engine/async_engine.py:13-211``:
``AsyncLLMEngine(engine, sampling_params)`` with ``start()``,
``submit(prompt, *, request_id=None, max_tokens=None) -> Future[GenerationResult]``,
``shutdown(timeout=30.0)``, ``is_running`` and ``fatal_error``.  Every request
shares the front end's :class:`SamplingParams` (one decode batch); ``max_tokens``
may differ per request.

Design: callers append to an inbox guarded by a condition variable; one daemon
thread (the *pump*) owns the engine.  Each turn it moves the inbox into the
engine, runs one ``engine.step()`` and settles the futures of the requests
that finished.  The :class:`_Ledger` maps the engine's sequence ids to the
callers' futures.  When idle the pump sleeps on the condition variable.  An
exception from the engine is fatal: every open future receives it, ``submit``
refuses new work, and the engine is released; a request whose own prompt is
rejected fails alone.
"""

from __future__ import annotations

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


class _Ledger:
    """Requests inside the engine, keyed by the engine's sequence id (pump thread only)."""

    def __init__(self) -> None:
        self._open: dict[int, _Request] = {}

    def enter(self, engine, sp: SamplingParams, req: _Request) -> None:
        if not req.future.set_running_or_notify_cancel():
            return  # the caller cancelled it while it waited in the inbox
        try:
            seq_id = engine.add_request(req.prompt, sp, max_tokens=req.max_tokens)
        except BaseException as exc:  # a malformed request fails on its own
            req.future.set_exception(exc)
            return
        clash = self._open.get(seq_id)
        if clash is not None:
            err = RuntimeError(f"engine reused sequence id {seq_id}, still held by request {clash.request_id}")
            req.future.set_exception(err)
            raise err
        self._open[seq_id] = req

    def settle(self, engine, sp: SamplingParams, finished) -> None:
        for seq_id, token_ids, stats in finished:
            req = self._open.pop(seq_id, None)
            if req is None:
                raise RuntimeError(f"engine finished sequence {seq_id}, which no submitted request owns")
            out = engine.finalize_output(token_ids, stats, sp)
            req.future.set_result(GenerationResult(req.request_id, str(out.get("text", "")),
                                                   list(out["token_ids"]), dict(out["stats"])))

    def drain(self) -> list[_Request]:
        reqs = list(self._open.values())
        self._open.clear()
        return reqs


class AsyncLLMEngine:
    """Run one synchronous engine behind a persistent request inbox."""

    def __init__(self, engine: Any, sampling_params: SamplingParams) -> None:
        self.engine = engine
        self.sampling_params = sampling_params
        self._cv = threading.Condition()
        self._inbox: list[_Request] = []
        self._state = "new"  # new -> running -> stopping -> stopped (or failed)
        self._fatal: BaseException | None = None
        self._pump: threading.Thread | None = None
        self._ledger = _Ledger()

    # ------------------------------------------------------------- callers
    def start(self) -> None:
        with self._cv:
            if self._state == "running":
                return
            if self._state != "new":
                raise RuntimeError(f"AsyncLLMEngine is {self._state}; a front end cannot be started twice")
            self._state = "running"
            self._pump = threading.Thread(target=self._pump_main, name="uno-b200-async-engine", daemon=True)
            self._pump.start()

    def submit(self, prompt: str | list[int], *, request_id: str | None = None,
               max_tokens: int | None = None) -> concurrent.futures.Future:
        with self._cv:
            if self._state != "running":
                if self._fatal is not None:
                    raise RuntimeError("AsyncLLMEngine failed and accepts no more requests") from self._fatal
                raise RuntimeError(f"AsyncLLMEngine is not running (state: {self._state})")
            fut: concurrent.futures.Future = concurrent.futures.Future()
            self._inbox.append(_Request(request_id or uuid.uuid4().hex, prompt, fut, max_tokens))
            self._cv.notify()
        return fut

    def shutdown(self, timeout: float | None = 30.0) -> None:
        with self._cv:
            pump = self._pump
            if self._state == "running":
                self._state = "stopping"
            self._cv.notify()
        if pump is None:
            return
        pump.join(timeout)
        if pump.is_alive():
            raise TimeoutError(f"the AsyncLLMEngine thread did not stop within {timeout} s")

    @property
    def is_running(self) -> bool:
        with self._cv:
            return self._state == "running" and self._pump is not None and self._pump.is_alive()

    @property
    def fatal_error(self) -> BaseException | None:
        with self._cv:
            return self._fatal

    # ---------------------------------------------------------------- pump
    def _next_turn(self) -> list[_Request] | None:
        """New requests for this turn, or None when the pump must stop; sleeps while idle."""
        with self._cv:
            while self._state == "running" and not self._inbox and self.engine.is_finished():
                self._cv.wait()
            if self._state != "running":
                return None
            batch, self._inbox = self._inbox, []
            return batch

    def _pump_main(self) -> None:
        sp = self.sampling_params
        try:
            while (batch := self._next_turn()) is not None:
                for req in batch:
                    self._ledger.enter(self.engine, sp, req)
                if not self.engine.is_finished():
                    finished, _ = self.engine.step()
                    self._ledger.settle(self.engine, sp, finished)
        except BaseException as exc:
            with self._cv:
                self._fatal = exc
                self._state = "failed"
            self._abandon(exc)
        finally:
            with self._cv:
                if self._state != "failed":
                    self._state = "stopped"
            self._abandon(RuntimeError("AsyncLLMEngine shut down before this request finished"))
            self.engine.exit()

    def _abandon(self, error: BaseException) -> None:
        with self._cv:
            waiting, self._inbox = self._inbox, []
        for req in self._ledger.drain() + waiting:
            if not req.future.done():
                req.future.set_exception(error)
