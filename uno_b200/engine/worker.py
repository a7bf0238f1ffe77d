"""Tensor-parallel worker processes and the rank-0 -> followers control plane.

Reference: followers block on an ``mp.Event`` and read pickled commands from a
64 MiB POSIX shared-memory segment (``nano_vllm_uno/engine/model_runner.py:154-255``).
Here the command channel is a gloo process group on the host: rank 0 calls
``broadcast_object_list`` with ``(method, args)`` and every follower executes
the same method on its own :class:`ModelRunner`.  The data plane (activations,
logits) stays on NCCL.  The same code path serves engines that spawn their
own ranks and jobs started by ``torchrun`` (``distributed_init="env"``).
"""

from __future__ import annotations

import logging
import os
import traceback

import torch
import torch.distributed as dist

from uno_b200.engine.sequence import Sequence
from uno_b200.parallel import state as tp

logger = logging.getLogger(__name__)


class ControlPlane:
    def __init__(self, group, rank: int, world: int):
        self.group = group
        self.rank = rank
        self.world = world

    def send(self, method: str, args: tuple) -> None:
        dist.broadcast_object_list([method, args], src=0, group=self.group)

    def recv(self):
        box = [None, None]
        dist.broadcast_object_list(box, src=0, group=self.group)
        return box[0], box[1]


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
    return ControlPlane(control, rank, world)


def follower_loop(runner, control: ControlPlane) -> None:
    while True:
        method, args = control.recv()
        if method == "run":
            states, is_prefill, sp = args
            args = ([Sequence.from_worker_state(s) for s in states], is_prefill, sp)
        fn = getattr(runner, method)
        fn(*args)
        if method == "exit":
            break


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
