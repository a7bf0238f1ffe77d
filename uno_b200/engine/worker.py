"""Tensor-parallel worker processes and their set-up.

Reference: followers block on an ``mp.Event`` and read pickled commands from a
64 MiB POSIX shared-memory segment (``nano_vllm_uno/engine/model_runner.py:154-255``).
Here rank 0 writes each command into a fixed-layout shared-memory slot
(``engine/control.py``) and every follower executes the same method on its own
:class:`ModelRunner`; a gloo group carries set-up and barriers, the data plane
(activations, logits) stays on NCCL and the fused peer-memory kernels.  The
same code path serves engines that spawn their own ranks and jobs started by
``torchrun`` (``distributed_init="env"``).
"""

from __future__ import annotations

import logging
import os
import traceback

import torch
import torch.distributed as dist

from uno_b200.engine.control import ChannelControlPlane
from uno_b200.parallel import state as tp

logger = logging.getLogger(__name__)


def init_distributed(config, rank: int, port: int | None = None):
    """Create the process group (NCCL data plane + gloo control plane)."""
    world = config.tensor_parallel_size
    if world == 1:
        tp.set_tp_state(0, 1)
        return None
    on_gpu = config.device == "cuda"
    if on_gpu:
        local = int(os.environ.get("LOCAL_RANK", rank))
        torch.cuda.set_device(local)
    if config.distributed_init == "env":
        init_method = None  # torchrun exported MASTER_ADDR/PORT/RANK/WORLD_SIZE
    else:
        init_method = f"tcp://127.0.0.1:{port}"
    backend = "nccl" if on_gpu else "gloo"
    tp.init_tp(world, rank, backend=backend, init_method=init_method)
    control = dist.new_group(backend="gloo") if on_gpu else dist.group.WORLD
    minutes = float(os.environ.get("TORCH_DISTRIBUTED_TIMEOUT_MINUTES", "10"))
    return ChannelControlPlane.create(control, rank, world, timeout_s=60.0 * minutes)


def follower_loop(runner, control: ChannelControlPlane) -> None:
    try:
        while True:
            method, args = control.recv()
            getattr(runner, method)(*args)
            if method == "exit":
                break
    finally:
        control.close()


def worker_main(config, rank: int, port: int, ready=None) -> None:
    """Entry point of a spawned TP rank (rank >= 1)."""
    from uno_b200.engine.model_runner import ModelRunner

    control = None
    try:
        control = init_distributed(config, rank, port)
        runner = ModelRunner(config, rank, control)
        dist.barrier(group=control.group)
        follower_loop(runner, control)
    except BaseException:
        logger.error("TP rank %d failed:\n%s", rank, traceback.format_exc())
        raise
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:  # pragma: no cover - teardown best effort
                pass


def serve_follower(model, tokenizer_path=None, **kwargs) -> None:
    """Run a follower TP rank of a ``torchrun`` job until rank 0 exits.

    Rank 0 builds ``LLM(model, distributed_init="env", **kwargs)``; every other
    rank calls this with the same arguments.
    """
    from uno_b200.config import Config
    from uno_b200.engine.model_runner import ModelRunner
    from uno_b200.engine.sequence import Sequence as _Seq

    kwargs = dict(kwargs)
    kwargs["distributed_init"] = "env"
    if "diffusion_block_size" in kwargs:
        kwargs["max_diffusion_block_size"] = kwargs.pop("diffusion_block_size")
    config = Config(model, **kwargs)
    _Seq.block_size = config.kvcache_block_size
    from uno_b200.engine.llm_engine import resolve_special_tokens

    resolve_special_tokens(config, tokenizer_path)
    rank = int(os.environ["RANK"])
    if config.device == "cuda":
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    control = init_distributed(config, rank)
    runner = ModelRunner(config, rank, control)
    dist.barrier(group=control.group)
    follower_loop(runner, control)
