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


def _trim_terminal_stop_tokens(token_ids: list[int], stops: set[int]) -> list[int]:
    end = len(token_ids)
    while end > 0 and token_ids[end - 1] in stops:
        end -= 1
    return token_ids[:end]


def resolve_special_tokens(config: Config, tokenizer_path=None):
    """Load the tokenizer and record EOS / PAD ids on ``config``."""
    tok_path = tokenizer_path or (config.model if os.path.isdir(str(config.model)) else None)
    tokenizer = load_tokenizer(tok_path, config.hf_config)
    eos = getattr(tokenizer, "eos_token_id", None)
    config.eos = -1 if eos is None else int(eos)
    pad = getattr(tokenizer, "pad_token_id", None)
    config.pad = int(pad) if pad is not None else max(config.eos, 0)
    return tokenizer


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class LLMEngine:
    def __init__(self, model, tokenizer_path=None, **kwargs):
        if "gated_lora" in kwargs:
            raise TypeError("gated_lora is derived from gated_lora_path and cannot be set directly")
        removed = {"lora_path", "lora_mode"}.intersection(kwargs)
        if removed:
            raise TypeError(
                f"Removed LoRA argument(s): {', '.join(sorted(removed))}. "
                "Use gated_lora_path to enable draft-noise-only LoRA."
            )
        if "diffusion_block_size" in kwargs:
            if "max_diffusion_block_size" in kwargs:
                raise TypeError("Pass only max_diffusion_block_size or diffusion_block_size, not both")
            kwargs["max_diffusion_block_size"] = kwargs.pop("diffusion_block_size")
        self._exited = False
        config = Config(model, **kwargs)
        self.config = config
        Sequence.block_size = config.kvcache_block_size
        self.tokenizer = resolve_special_tokens(config, tokenizer_path)

        self.ps: list = []
        self.control = None
        world = config.tensor_parallel_size
        if config.device == "cuda":
            local = int(os.environ.get("LOCAL_RANK", 0))
            torch.cuda.set_device(local)
        if world > 1 and config.distributed_init == "spawn":
            port = int(os.environ.get("TORCH_DISTRIBUTED_PORT", _free_port()))
            ctx = mp.get_context("spawn")
            from uno_b200.engine.worker import worker_main

            for rank in range(1, world):
                p = ctx.Process(target=worker_main, args=(config, rank, port), daemon=False)
                p.start()
                self.ps.append(p)
        else:
            port = None
        from uno_b200.engine.model_runner import ModelRunner
        from uno_b200.engine.worker import init_distributed

        self.rank = int(os.environ.get("RANK", 0)) if config.distributed_init == "env" else 0
        self.control = init_distributed(config, self.rank, port)
        self.model_runner = ModelRunner(config, self.rank, self.control)
        if self.control is not None:
            import torch.distributed as dist

            dist.barrier(group=self.control.group)
        self.scheduler = Scheduler(config)
        self.sampling_params: SamplingParams | None = None
        self._decode_step_wall_ns: list[int] = []
        atexit.register(self.exit)

    # ----------------------------------------------------------- rpc
    def call(self, method: str, *args):
        """Run ``method`` on every TP rank (rank 0 broadcasts the command)."""
        if self.control is not None and self.rank == 0:
            payload = args
            if method == "run":
                seqs, is_prefill, sp = args
                payload = ([s.to_worker_state(include_token_ids=is_prefill) for s in seqs], is_prefill, sp)
            self.control.send(method, payload)
        return getattr(self.model_runner, method)(*args)

    def exit(self) -> None:
        if getattr(self, "_exited", True):
            return
        self._exited = True
        print(f"Engine stats: preemptions={self.scheduler.num_preemptions}", flush=True)
        try:
            self.call("exit")
        except Exception:  # pragma: no cover
            logger.exception("exit failed")
        for rank, p in enumerate(self.ps, start=1):
            p.join(timeout=30)
            if p.is_alive():
                logger.warning("Worker %d did not exit; terminating it", rank)
                p.terminate()
                p.join(timeout=5)
                if p.is_alive():
                    p.kill()
        self.ps.clear()
        import torch.distributed as dist

        if self.control is not None and dist.is_initialized():
            dist.destroy_process_group()

    def get_stats(self) -> dict[str, int]:
        return {"preemptions": self.scheduler.num_preemptions}

    # ------------------------------------------------------- requests
    def _validate_sampling_params(self, sp: SamplingParams) -> None:
        if sp.diffusion_block_size > self.config.max_diffusion_block_size:
            raise ValueError(
                f"SamplingParams.diffusion_block_size={sp.diffusion_block_size} exceeds engine "
                f"capacity max_diffusion_block_size={self.config.max_diffusion_block_size}"
            )

    def add_request(self, prompt: str | list[int], sampling_params: SamplingParams, *,
                    max_tokens: int | None = None) -> int:
        self._validate_sampling_params(sampling_params)
        if self.scheduler.is_finished():
            self.sampling_params = sampling_params
            if sampling_params.seed is not None:
                self.call("reseed", int(sampling_params.seed))
        elif self.sampling_params is not sampling_params:
            raise ValueError("All active requests must share one SamplingParams object")
        if isinstance(prompt, str):
            prompt = self.tokenizer.encode(prompt)
        if max_tokens is not None and int(max_tokens) < 1:
            raise ValueError("per-request max_tokens must be positive")
        seq = Sequence(list(prompt), max_completion_tokens=max_tokens)
        self.scheduler.add(seq)
        return seq.seq_id

    def step(self):
        t0 = perf_counter_ns() if self.config.decode_timing else 0
        sp = self.sampling_params
        if sp is None:
            raise RuntimeError("Cannot step without active sampling parameters")
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
        stops = {self.scheduler.eos, *(sampling_params.stop_token_ids or [])}
        token_ids = _trim_terminal_stop_tokens(list(token_ids), stops)
        out = {"token_ids": token_ids, "stats": stats}
        if detokenize:
            out["text"] = self.tokenizer.decode(token_ids)
        return out

    def generate(self, prompts, sampling_params: SamplingParams, use_tqdm: bool = True,
                 detokenize: bool = True, progress_callback: Callable | None = None,
                 request_max_tokens: list[int] | None = None):
        if isinstance(sampling_params, list):
            raise ValueError(
                "generate() accepts exactly one SamplingParams object per call. "
                "All prompts in the call share that sampling configuration."
            )
        self._validate_sampling_params(sampling_params)
        if request_max_tokens is not None and len(request_max_tokens) != len(prompts):
            raise ValueError("request_max_tokens must contain one value per prompt")
        pbar = tqdm(total=len(prompts), desc="Generating", dynamic_ncols=True) if use_tqdm else None
        ids = [
            self.add_request(p, sampling_params,
                             max_tokens=None if request_max_tokens is None else int(request_max_tokens[i]))
            for i, p in enumerate(prompts)
        ]
        done: dict[int, tuple] = {}
        prefill_tps = decode_tps = 0.0
        while not self.is_finished():
            t = perf_counter()
            output, n = self.step()
            if pbar is not None:
                dt = perf_counter() - t
                if n > 0:
                    prefill_tps = n / dt
                else:
                    decode_tps = -n / dt
                pbar.set_postfix({"Prefill": f"{int(prefill_tps)}tok/s", "Decode": f"{int(decode_tps)}tok/s"})
            for seq_id, toks, stats in output:
                done[seq_id] = (toks, stats)
            if output:
                if pbar is not None:
                    pbar.update(len(output))
                if progress_callback is not None:
                    progress_callback([s for _, _, s in output])
        if pbar is not None:
            pbar.close()
        return [self.finalize_output(*done[i], sampling_params, detokenize=detokenize) for i in ids]
