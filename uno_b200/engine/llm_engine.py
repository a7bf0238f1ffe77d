"""Synchronous engine: tokenizer, TP ranks, scheduler, step loop.

Public surface of ``nano_vllm_uno/engine/llm_engine.py:30-318``:
``add_request``, ``step``, ``is_finished``, ``generate``, ``finalize_output``,
``get_stats``, ``reset_decode_timing``/``get_decode_timing`` and ``exit``.
A step is one scheduler batch: a prefill (which also samples each request's
first completion token) or one Psi-Spec decode cycle for the running batch.
All requests that are active together share one ``SamplingParams`` object.
"""

from __future__ import annotations

import atexit
import logging
import os
import socket
import sys
from time import perf_counter, perf_counter_ns
from typing import Callable

import torch
import torch.multiprocessing as mp
from tqdm.auto import tqdm

from uno_b200.config import Config
from uno_b200.engine.scheduler import Scheduler
from uno_b200.engine.sequence import Sequence
from uno_b200.sampling_params import SamplingParams
from uno_b200.utils.hf_compat import load_tokenizer

logger = logging.getLogger(__name__)


def strip_trailing_stops(token_ids: list[int], stops: set[int]) -> list[int]:
    """``token_ids`` without the run of stop tokens at its end (the decoder commits the stop token)."""
    keep = len(token_ids)
    for tok in reversed(token_ids):
        if tok not in stops:
            break
        keep -= 1
    return list(token_ids[:keep])


def resolve_special_tokens(config: Config, tokenizer_path=None):
    """Load the tokenizer and record EOS / PAD ids on ``config`` (PAD falls back to EOS)."""
    tok_path = tokenizer_path or (config.model if os.path.isdir(str(config.model)) else None)
    tokenizer = load_tokenizer(tok_path, config.hf_config)
    eos = getattr(tokenizer, "eos_token_id", None)
    pad = getattr(tokenizer, "pad_token_id", None)
    config.eos = -1 if eos is None else int(eos)
    config.pad = int(pad) if pad is not None else max(config.eos, 0)
    return tokenizer


# Engine keyword arguments that are refused, with the reason given to the caller.
_REFUSED_KWARGS = {
    "gated_lora": "gated_lora is not a setting: it is on exactly when gated_lora_path names an adapter",
    "lora_path": "lora_path is not supported: pass the draft adapter as gated_lora_path",
    "lora_mode": "lora_mode is not supported: the adapter always gates on the draft noise rows (gated_lora_path)",
}


def normalize_engine_kwargs(kwargs: dict) -> dict:
    """Validated copy of the engine keyword arguments.

    ``diffusion_block_size`` is accepted as an alias of ``max_diffusion_block_size``."""
    refused = [name for name in _REFUSED_KWARGS if name in kwargs]
    if refused:
        raise TypeError("; ".join(_REFUSED_KWARGS[name] for name in refused))
    out = dict(kwargs)
    if "diffusion_block_size" in out:
        if "max_diffusion_block_size" in out:
            raise TypeError("diffusion_block_size is an alias of max_diffusion_block_size; give one of them")
        out["max_diffusion_block_size"] = out.pop("diffusion_block_size")
    return out


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _reap(rank: int, proc, grace_s: float = 30.0) -> None:
    """Join a TP worker process, escalating to terminate and then kill."""
    proc.join(timeout=grace_s)
    for action in (proc.terminate, proc.kill):
        if not proc.is_alive():
            return
        logger.warning("TP worker %d is still alive; sending %s", rank, action.__name__)
        action()
        proc.join(timeout=5)


class LLMEngine:
    def __init__(self, model, tokenizer_path=None, **kwargs):
        config = Config(model, **normalize_engine_kwargs(kwargs))
        self._exited = False
        self.config = config
        Sequence.block_size = config.kvcache_block_size
        self.tokenizer = resolve_special_tokens(config, tokenizer_path)
        if config.device == "cuda":
            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        self.ps: list = []
        self.control = None
        self.rank = int(os.environ.get("RANK", 0)) if config.distributed_init == "env" else 0
        port = self._spawn_tp_workers() if config.distributed_init == "spawn" else None
        from uno_b200.engine.model_runner import ModelRunner
        from uno_b200.engine.worker import init_distributed

        self.control = init_distributed(config, self.rank, port)
        self.model_runner = ModelRunner(config, self.rank, self.control)
        if self.control is not None:
            import torch.distributed as dist

            dist.barrier(group=self.control.group)  # every rank has built its runner
        self.scheduler = Scheduler(config)
        self.sampling_params: SamplingParams | None = None
        self._decode_step_wall_ns: list[int] = []
        atexit.register(self.exit)

    def _spawn_tp_workers(self) -> int | None:
        """Start ranks 1..TP-1 as spawned processes; returns their rendezvous port."""
        world = self.config.tensor_parallel_size
        if world == 1:
            return None
        from uno_b200.engine.worker import worker_main

        port = int(os.environ.get("TORCH_DISTRIBUTED_PORT", _free_port()))
        ctx = mp.get_context("spawn")
        for rank in range(1, world):
            proc = ctx.Process(target=worker_main, args=(self.config, rank, port), daemon=False)
            proc.start()
            self.ps.append(proc)
        return port

    # ----------------------------------------------------------- rpc
    def call(self, method: str, *args):
        """Run ``method`` on every TP rank (rank 0 broadcasts the command)."""
        if self.control is not None and self.rank == 0:
            self.control.send(method, args)
        return getattr(self.model_runner, method)(*args)

    def exit(self) -> None:
        if getattr(self, "_exited", True):
            return
        self._exited = True
        sys.stdout.write(f"Engine stats: preemptions={self.scheduler.num_preemptions}\n")  # one write: ranks share stdout
        sys.stdout.flush()
        try:
            self.call("exit")
        except Exception:  # pragma: no cover - best-effort teardown
            logger.exception("shutting down the model runners failed")
        workers, self.ps = self.ps, []
        for rank, proc in enumerate(workers, start=1):
            _reap(rank, proc)
        import torch.distributed as dist

        if self.control is not None:
            self.control.close()
            if dist.is_initialized():
                dist.destroy_process_group()

    def get_stats(self) -> dict[str, int]:
        return {"preemptions": self.scheduler.num_preemptions}

    # ------------------------------------------------------- requests
    def _validate_sampling_params(self, sp: SamplingParams) -> None:
        if sp.diffusion_block_size > self.config.max_diffusion_block_size:
            raise ValueError(f"diffusion_block_size {sp.diffusion_block_size} is larger than this engine was "
                             f"built for (max_diffusion_block_size={self.config.max_diffusion_block_size})")

    def add_request(self, prompt: str | list[int], sampling_params: SamplingParams, *,
                    max_tokens: int | None = None) -> int:
        self._validate_sampling_params(sampling_params)
        if self.scheduler.is_finished():
            self.sampling_params = sampling_params
            if sampling_params.seed is not None:
                self.call("reseed", int(sampling_params.seed))
        elif self.sampling_params is not sampling_params:
            raise ValueError("requests that run together must use the same SamplingParams object; submit a "
                             "different one after the running batch has finished")
        if isinstance(prompt, str):
            prompt = self.tokenizer.encode(prompt)
        if max_tokens is not None and int(max_tokens) < 1:
            raise ValueError(f"max_tokens of a request must be at least 1, got {max_tokens}")
        seq = Sequence(list(prompt), max_completion_tokens=max_tokens)
        self.scheduler.add(seq)
        return seq.seq_id

    def step(self):
        t0 = perf_counter_ns() if self.config.decode_timing else 0
        sp = self.sampling_params
        if sp is None:
            raise RuntimeError("step() needs a request: add_request() sets the batch's SamplingParams")
        seqs, is_prefill = self.scheduler.schedule(sp)
        n_prefill = sum(len(s) - s.num_cached_tokens for s in seqs) if is_prefill else 0
        result = self.call("run", seqs, is_prefill, sp)
        for seq in seqs:
            self.scheduler.block_manager.publish_computed_prefix_blocks(seq)
        self.scheduler.postprocess(seqs, result, sp)
        n_new = sum(len(r) for r in result)
        outputs = [(s.seq_id, s.completion_token_ids, dict(s.stats)) for s in seqs if s.is_finished]
        if self.config.decode_timing and not is_prefill:
            self._decode_step_wall_ns.append(perf_counter_ns() - t0)
        return outputs, (n_prefill if is_prefill else -n_new)

    def is_finished(self) -> bool:
        return self.scheduler.is_finished()

    def reset_decode_timing(self) -> None:
        self._decode_step_wall_ns.clear()
        self.call("reset_decode_timing")

    def get_decode_timing(self) -> dict:
        timing = self.call("get_decode_timing")
        gpu_by_step: dict[int, float] = {}
        for r in timing["forward_records"]:
            gpu_by_step[int(r["step_index"])] = gpu_by_step.get(int(r["step_index"]), 0.0) + float(r["gpu_ms"])
        wall = [v / 1e6 for v in self._decode_step_wall_ns]
        gpu = [gpu_by_step.get(i, 0.0) for i in range(1, len(wall) + 1)]
        return {
            "enabled": bool(timing["enabled"]),
            "timing_scope": "decode_steps_only",
            "model_gpu_scope": "backbone_and_lm_head",
            "step_wall_ms": wall,
            "model_gpu_ms": gpu,
            "exposed_non_model_ms": [w - g for w, g in zip(wall, gpu)],
            "forward_records": timing["forward_records"],
        }

    def finalize_output(self, token_ids, stats, sampling_params: SamplingParams, detokenize: bool = True):
        """Output dict of one finished request: token ids without trailing stop tokens, its decode
        statistics, and (``detokenize``) the text."""
        stops = set(sampling_params.stop_token_ids or ())
        stops.add(self.scheduler.eos)
        ids = strip_trailing_stops(list(token_ids), stops)
        out = {"token_ids": ids, "stats": stats}
        if detokenize:
            out["text"] = self.tokenizer.decode(ids)
        return out

    def generate(self, prompts, sampling_params: SamplingParams, use_tqdm: bool = True,
                 detokenize: bool = True, progress_callback: Callable | None = None,
                 request_max_tokens: list[int] | None = None):
        """Run ``prompts`` to completion; outputs in prompt order.

        ``progress_callback`` receives the decode statistics of the requests that
        finished in a step; ``request_max_tokens`` overrides ``max_tokens`` per prompt."""
        if isinstance(sampling_params, list):
            raise ValueError("generate() takes a single SamplingParams shared by every prompt of the call, "
                             "not a list")
        self._validate_sampling_params(sampling_params)
        if request_max_tokens is not None and len(request_max_tokens) != len(prompts):
            raise ValueError(f"request_max_tokens has {len(request_max_tokens)} entries for {len(prompts)} prompts")
        limits = request_max_tokens if request_max_tokens is not None else [None] * len(prompts)
        order = [self.add_request(p, sampling_params, max_tokens=None if m is None else int(m))
                 for p, m in zip(prompts, limits)]
        finished: dict[int, tuple] = {}
        bar = _ProgressBar(len(prompts)) if use_tqdm else None
        try:
            while not self.is_finished():
                t = perf_counter()
                done, n = self.step()
                if bar is not None:
                    bar.step(n, perf_counter() - t, len(done))
                for seq_id, toks, stats in done:
                    finished[seq_id] = (toks, stats)
                if done and progress_callback is not None:
                    progress_callback([stats for _, _, stats in done])
        finally:
            if bar is not None:
                bar.close()
        return [self.finalize_output(*finished[i], sampling_params, detokenize=detokenize) for i in order]


class _ProgressBar:
    """tqdm bar over requests with the latest prefill and decode rates (tokens per second)."""

    def __init__(self, total: int):
        self.bar = tqdm(total=total, desc="Generating", dynamic_ncols=True)
        self.rates = {"Prefill": 0.0, "Decode": 0.0}

    def step(self, n_tokens: int, seconds: float, n_finished: int) -> None:
        # step() reports prefill tokens as a positive count and decoded tokens as a negative one
        self.rates["Prefill" if n_tokens > 0 else "Decode"] = abs(n_tokens) / max(seconds, 1e-9)
        self.bar.set_postfix({k: f"{int(v)}tok/s" for k, v in self.rates.items()})
        if n_finished:
            self.bar.update(n_finished)

    def close(self) -> None:
        self.bar.close()
