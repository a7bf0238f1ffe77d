"""User-facing ``LLM``: engine + ``greedy`` flag + data-parallel replicas.

Same contract as ``nano_vllm_uno/llm.py:21-266``: with ``data_parallel_size > 1``
the constructor starts one ``python -m uno_b200.dp_worker`` process per
replica, each pinned to its own ``CUDA_VISIBLE_DEVICES`` slice of
``tensor_parallel_size`` GPUs; ``generate`` shards prompts round-robin,
aggregates progress and TPF statistics over pipes, and re-assembles outputs in
prompt order.  A replica failure surfaces its traceback; shutdown escalates
exit -> terminate -> kill.
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


class LLM(LLMEngine):
    def __init__(self, model, tokenizer_path=None, data_parallel_size: int = 1, **kwargs: Any):
        self.data_parallel_size = int(data_parallel_size)
        if self.data_parallel_size < 1:
            raise ValueError("data_parallel_size must be >= 1")
        self.last_generate_stats: dict[str, int] = {}
        if self.data_parallel_size == 1:
            super().__init__(model, tokenizer_path, **kwargs)
            return
        self._exited = False
        self._dp_workers: list = []
        tp = int(kwargs.get("tensor_parallel_size", 1))
        base_port = int(os.environ.get("TORCH_DISTRIBUTED_PORT", 20000 + os.getpid() % 20000))
        visible = os.environ.get("CUDA_VISIBLE_DEVICES")
        on_cpu = kwargs.get("device", "cuda") == "cpu"
        gpus = ([g.strip() for g in visible.split(",")] if visible
                else [str(i) for i in range(self.data_parallel_size * tp)])
        if not on_cpu and len(gpus) < self.data_parallel_size * tp:
            raise ValueError(
                f"data_parallel_size={self.data_parallel_size} and tensor_parallel_size={tp} "
                f"require {self.data_parallel_size * tp} visible GPUs, got {len(gpus)}"
            )
        try:
            for r in range(self.data_parallel_size):
                parent, child = Pipe()
                env = os.environ.copy()
                if not on_cpu:
                    env["CUDA_VISIBLE_DEVICES"] = ",".join(gpus[r * tp:(r + 1) * tp])
                env["TORCH_DISTRIBUTED_PORT"] = str(base_port + r)
                proc = subprocess.Popen([sys.executable, "-m", "uno_b200.dp_worker", str(child.fileno())],
                                        env=env, pass_fds=(child.fileno(),))
                child.close()
                self._dp_workers.append((proc, parent))
                parent.send((model, tokenizer_path, kwargs))
            for r, (_, conn) in enumerate(self._dp_workers):
                ok, result = conn.recv()
                if not ok:
                    raise RuntimeError(f"data-parallel replica {r} failed to start:\n{result}")
        except BaseException:
            self.exit()
            raise
        atexit.register(self.exit)

    def generate(self, prompts, sampling_params: SamplingParams | None = None, *, greedy: bool | None = None,
                 request_max_tokens: list[int] | None = None, use_tqdm: bool = True, detokenize: bool = True,
                 **kwargs: Any):
        if sampling_params is None:
            sampling_params = SamplingParams()
        if isinstance(sampling_params, list):
            raise ValueError(
                "LLM.generate() accepts exactly one SamplingParams object per call. "
                "All prompts in the call share that sampling configuration."
            )
        sp = sampling_params
        if greedy is not None:
            if greedy:
                sp = replace(sp, temperature=0.0, top_k=None, top_p=None)
            elif sp.temperature == 0.0:
                sp = replace(sp, temperature=1.0)
        if self.data_parallel_size == 1:
            outputs = super().generate(prompts, sp, request_max_tokens=request_max_tokens,
                                       use_tqdm=use_tqdm, detokenize=detokenize, **kwargs)
            self.last_generate_stats = {k: sum(int(o["stats"][k]) for o in outputs) for k in DECODE_STAT_KEYS}
            return outputs
        if not prompts:
            self.last_generate_stats = {k: 0 for k in DECODE_STAT_KEYS}
            return []
        if request_max_tokens is not None and len(request_max_tokens) != len(prompts):
            raise ValueError("request_max_tokens must contain one value per prompt")
        shards: list[list] = [[] for _ in self._dp_workers]
        for i, prompt in enumerate(prompts):
            limit = None if request_max_tokens is None else int(request_max_tokens[i])
            shards[i % len(shards)].append((i, prompt, limit))
        active = {}
        for r, shard in enumerate(shards):
            if not shard:
                continue
            idx, ps, limits = zip(*shard)
            wkw = {**kwargs, "use_tqdm": False, "detokenize": detokenize}
            if request_max_tokens is not None:
                wkw["request_max_tokens"] = list(limits)
            conn = self._dp_workers[r][1]
            conn.send(("generate", list(ps), sp, wkw, use_tqdm))
            active[conn] = (r, idx)
        ordered: list = [None] * len(prompts)
        totals = {k: 0 for k in DECODE_STAT_KEYS}
        progress = {k: 0 for k in DECODE_STAT_KEYS}
        pbar = tqdm(total=len(prompts), desc="Generating", dynamic_ncols=True) if use_tqdm else None
        try:
            while active:
                for conn in wait(list(active)):
                    r, idx = active[conn]
                    msg = conn.recv()
                    if msg[0] == "progress":
                        for st in msg[1]:
                            for k in DECODE_STAT_KEYS:
                                progress[k] += int(st[k])
                        if pbar is not None:
                            pbar.update(len(msg[1]))
                            f = progress["forwards"]
                            pbar.set_postfix({"TPF": f"{(progress['accepts'] / f if f else 0.0):.2f}"})
                        continue
                    ok, result = msg
                    if not ok:
                        raise RuntimeError(f"data-parallel replica {r} failed during generate:\n{result}")
                    outs, stats = result
                    if len(outs) != len(idx):
                        raise RuntimeError(f"data-parallel replica {r} returned an unexpected output count")
                    for i, o in zip(idx, outs):
                        ordered[i] = o
                    for k in DECODE_STAT_KEYS:
                        totals[k] += int(stats[k])
                    del active[conn]
        finally:
            if pbar is not None:
                pbar.close()
        self.last_generate_stats = totals
        return ordered

    def exit(self):
        if self.data_parallel_size == 1:
            return super().exit()
        if getattr(self, "_exited", False):
            return
        self._exited = True
        for proc, conn in getattr(self, "_dp_workers", []):
            try:
                conn.send(("exit",))
                conn.close()
            except (BrokenPipeError, EOFError, OSError):
                pass
            try:
                proc.wait(timeout=30)
            except subprocess.TimeoutExpired:
                pass
            if proc.poll() is None:
                proc.terminate()
                try:
                    proc.wait(timeout=5)
                except subprocess.TimeoutExpired:
                    proc.kill()
                    proc.wait()
        self._dp_workers = []
