"""User-facing ``LLM``: the engine plus a ``greedy`` switch and data-parallel replicas.

API of ``nano_vllm_uno/llm.py:21-266``: ``LLM(model, tokenizer_path=None,
data_parallel_size=1, **engine_kwargs)`` and ``generate(prompts,
sampling_params=None, *, greedy=None, request_max_tokens=None, use_tqdm=True,
detokenize=True)``; ``last_generate_stats`` holds the summed decode statistics
of the latest call.

With ``data_parallel_size = R > 1`` the object drives a :class:`ReplicaSet`
instead of an in-process engine: ``R`` engine processes
(``python -m uno_b200.dp_worker``), each on its own slice of
``tensor_parallel_size`` visible GPUs and its own rendezvous port.  Prompt ``i``
goes to replica ``i mod R``; outputs come back in prompt order.
"""

from __future__ import annotations

import atexit
import os
import subprocess
import sys
from dataclasses import replace
from multiprocessing import Pipe
from multiprocessing.connection import wait
from typing import Any

from tqdm.auto import tqdm

from uno_b200.engine.llm_engine import LLMEngine
from uno_b200.engine.sequence import DECODE_STAT_KEYS
from uno_b200.sampling_params import SamplingParams


def with_greedy_flag(sp: SamplingParams, greedy: bool | None) -> SamplingParams:
    """``greedy=True``: arg-max decoding over the full vocabulary; ``False``: make sure the
    temperature is positive; ``None``: ``sp`` as given."""
    if greedy is None:
        return sp
    if greedy:
        return replace(sp, temperature=0.0, top_k=None, top_p=None)
    return replace(sp, temperature=1.0) if sp.temperature == 0.0 else sp


def _zero_stats() -> dict[str, int]:
    return dict.fromkeys(DECODE_STAT_KEYS, 0)


class ReplicaError(RuntimeError):
    """A data-parallel replica failed; the message carries its traceback."""


def _stop_process(proc: subprocess.Popen, grace_s: float) -> None:
    """Wait up to ``grace_s`` for a clean exit, then SIGTERM, then SIGKILL."""
    for action, wait_s in ((None, grace_s), (proc.terminate, 5.0), (proc.kill, None)):
        if proc.poll() is not None:
            return
        if action is not None:
            action()
        try:
            proc.wait(timeout=wait_s)
        except subprocess.TimeoutExpired:
            continue


class _Replica:
    """Handle of one replica process and its end of the pipe."""

    def __init__(self, index: int, devices: list[str] | None, port: int, init_msg: tuple):
        self.index = index
        self.devices = devices
        ours, theirs = Pipe(duplex=True)
        env = dict(os.environ, TORCH_DISTRIBUTED_PORT=str(port))
        if devices is not None:
            env["CUDA_VISIBLE_DEVICES"] = ",".join(devices)
        self.proc = subprocess.Popen([sys.executable, "-m", "uno_b200.dp_worker", str(theirs.fileno())],
                                     env=env, pass_fds=(theirs.fileno(),))
        theirs.close()
        self.conn = ours
        self.conn.send(init_msg)

    def label(self) -> str:
        where = f"GPUs {','.join(self.devices)}" if self.devices else "CPU"
        return f"replica {self.index} ({where})"

    def wait_up(self) -> None:
        try:
            msg = self.conn.recv()
        except EOFError:
            raise ReplicaError(f"{self.label()} exited while building its engine") from None
        if msg[0] != "up":
            raise ReplicaError(f"{self.label()} could not build its engine:\n{msg[-1]}")

    def close(self, grace_s: float = 30.0) -> None:
        try:
            self.conn.send(("quit",))
        except (BrokenPipeError, EOFError, OSError):
            pass
        self.conn.close()
        _stop_process(self.proc, grace_s)


class ReplicaSet:
    """``count`` independent engines, each on ``tp`` GPUs of the visible set."""

    def __init__(self, count: int, model, tokenizer_path, engine_kwargs: dict):
        tp = int(engine_kwargs.get("tensor_parallel_size", 1))
        on_cpu = engine_kwargs.get("device", "cuda") == "cpu"
        visible = os.environ.get("CUDA_VISIBLE_DEVICES")
        pool = [d.strip() for d in visible.split(",") if d.strip()] if visible else [str(i) for i in range(count * tp)]
        if not on_cpu and len(pool) < count * tp:
            raise ValueError(f"{count} replicas x tensor_parallel_size {tp} need {count * tp} visible GPUs; "
                             f"CUDA_VISIBLE_DEVICES offers {len(pool)}")
        port0 = int(os.environ.get("TORCH_DISTRIBUTED_PORT", 20000 + os.getpid() % 20000))
        init_msg = ("init", model, tokenizer_path, engine_kwargs)
        self.replicas: list[_Replica] = []
        try:
            for r in range(count):
                devices = None if on_cpu else pool[r * tp:(r + 1) * tp]
                self.replicas.append(_Replica(r, devices, port0 + r, init_msg))
            for rep in self.replicas:  # all replicas build their engines concurrently
                rep.wait_up()
        except BaseException:
            self.close()
            raise

    def generate(self, prompts: list, sp: SamplingParams, limits: list[int] | None, gen_kwargs: dict,
                 pbar) -> tuple[list, dict[str, int]]:
        n = len(self.replicas)
        pending: dict = {}
        for rep in self.replicas:
            idx = list(range(rep.index, len(prompts), n))
            if not idx:
                continue
            kw = dict(gen_kwargs)
            if limits is not None:
                kw["request_max_tokens"] = [int(limits[i]) for i in idx]
            rep.conn.send(("work", [prompts[i] for i in idx], sp, kw, pbar is not None))
            pending[rep.conn] = (rep, idx)
        ordered: list = [None] * len(prompts)
        totals, seen = _zero_stats(), _zero_stats()
        while pending:
            for conn in wait(list(pending)):
                rep, idx = pending[conn]
                try:
                    msg = conn.recv()
                except EOFError:
                    raise ReplicaError(f"{rep.label()} exited during generate") from None
                if msg[0] == "tick":
                    for st in msg[1]:
                        for k in DECODE_STAT_KEYS:
                            seen[k] += int(st[k])
                    pbar.update(len(msg[1]))
                    pbar.set_postfix({"TPF": f"{seen['accepts'] / max(1, seen['forwards']):.2f}"})
                    continue
                if msg[0] == "fault":
                    raise ReplicaError(f"{rep.label()} failed during generate:\n{msg[-1]}")
                _, outputs, stats = msg
                if len(outputs) != len(idx):
                    raise ReplicaError(f"{rep.label()} answered {len(outputs)} of its {len(idx)} prompts")
                for i, out in zip(idx, outputs):
                    ordered[i] = out
                for k in DECODE_STAT_KEYS:
                    totals[k] += int(stats[k])
                del pending[conn]
        return ordered, totals

    def close(self) -> None:
        replicas, self.replicas = self.replicas, []
        for rep in replicas:
            rep.close()


class LLM(LLMEngine):
    def __init__(self, model, tokenizer_path=None, data_parallel_size: int = 1, **kwargs: Any):
        replicas = int(data_parallel_size)
        if replicas < 1:
            raise ValueError(f"data_parallel_size must be at least 1, got {data_parallel_size}")
        self.data_parallel_size = replicas
        self.last_generate_stats: dict[str, int] = {}
        self._replica_set: ReplicaSet | None = None
        if replicas == 1:
            super().__init__(model, tokenizer_path, **kwargs)
            return
        self._exited = False
        self._replica_set = ReplicaSet(replicas, model, tokenizer_path, kwargs)
        atexit.register(self.exit)

    def generate(self, prompts, sampling_params: SamplingParams | None = None, *, greedy: bool | None = None,
                 request_max_tokens: list[int] | None = None, use_tqdm: bool = True, detokenize: bool = True,
                 **kwargs: Any):
        if isinstance(sampling_params, list):
            raise ValueError("generate() takes a single SamplingParams shared by every prompt of the call, "
                             "not a list")
        sp = with_greedy_flag(sampling_params if sampling_params is not None else SamplingParams(), greedy)
        if self._replica_set is None:
            outputs = super().generate(prompts, sp, request_max_tokens=request_max_tokens, use_tqdm=use_tqdm,
                                       detokenize=detokenize, **kwargs)
            self.last_generate_stats = _zero_stats()
            for out in outputs:
                for k in DECODE_STAT_KEYS:
                    self.last_generate_stats[k] += int(out["stats"][k])
            return outputs
        if request_max_tokens is not None and len(request_max_tokens) != len(prompts):
            raise ValueError(f"request_max_tokens has {len(request_max_tokens)} entries for {len(prompts)} prompts")
        if not prompts:
            self.last_generate_stats = _zero_stats()
            return []
        pbar = tqdm(total=len(prompts), desc="Generating", dynamic_ncols=True) if use_tqdm else None
        try:
            outputs, totals = self._replica_set.generate(list(prompts), sp, request_max_tokens,
                                                         {**kwargs, "use_tqdm": False, "detokenize": detokenize},
                                                         pbar)
        finally:
            if pbar is not None:
                pbar.close()
        self.last_generate_stats = totals
        return outputs

    def exit(self):
        if getattr(self, "_replica_set", None) is None:
            return super().exit()
        if self._exited:
            return
        self._exited = True
        self._replica_set.close()
