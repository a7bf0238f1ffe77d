"""LoRA-only AdamW with ZeRO-2 sharding and fused collectives.

Behaviour of the reference optimizer path (DeepSpeed stage 2 over the LoRA
parameters, ``training/configs/deepspeed_zero2.json:18-27``; AdamW with
decoupled weight decay, ``training/train.py:285-290``; global grad-norm clip):
gradients are averaged over the data-parallel ranks, clipped by their global
L2 norm, and each rank updates the Adam moments of its 1/world shard only;
the updated parameters then reach every rank.

Storage: all trainable tensors become views of ONE flat fp32 parameter buffer
and their ``.grad`` views of one flat gradient buffer.  On CUDA both live in a
symmetric workspace shared over CUDA IPC, and one kernel (``fused_adamw`` in
``ops/csrc/optim.cu``) reads the peers' gradients of its shard, reduces,
clips, applies AdamW and stores the new values into every rank's parameter
buffer.  On CPU (and as the reference) the same step runs as
``reduce_scatter`` -> norm ``all_reduce`` -> AdamW -> ``all_gather``.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist
from torch import nn


def _align(n: int, a: int) -> int:
    return -(-n // a) * a


class ShardedLoraAdamW:
    def __init__(self, params: list[nn.Parameter], lr: float = 1e-4, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.0, max_grad_norm: float = 1.0, group=None, fused: bool | None = None):
        self.params = [p for p in params]
        if not self.params:
            raise ValueError("no trainable parameters")
        self.device = self.params[0].device
        self.group = group if (group is not None and dist.is_initialized()) else None
        self.world = dist.get_world_size(self.group) if self.group is not None else 1
        self.rank = dist.get_rank(self.group) if self.group is not None else 0
        self.lr, self.betas, self.eps = float(lr), (float(betas[0]), float(betas[1])), float(eps)
        self.weight_decay, self.max_grad_norm = float(weight_decay), float(max_grad_norm)
        self.fused = (self.device.type == "cuda") if fused is None else bool(fused)
        numel = sum(p.numel() for p in self.params)
        self.n = _align(numel, 4 * self.world)
        self.shard = self.n // self.world
        self.step_count = 0
        self._ws = None
        if self.fused:
            self._alloc_symmetric()
        else:
            self.flat = torch.zeros(self.n, device=self.device, dtype=torch.float32)
            self.flat_grad = torch.zeros(self.n, device=self.device, dtype=torch.float32)
        off = 0
        with torch.no_grad():
            for p in self.params:
                k = p.numel()
                view = self.flat[off:off + k].view_as(p)
                view.copy_(p.detach().float())
                p.data = view
                p.grad = self.flat_grad[off:off + k].view_as(p)
                off += k
        self.m = torch.zeros(self.shard, device=self.device, dtype=torch.float32)
        self.v = torch.zeros(self.shard, device=self.device, dtype=torch.float32)
        self._scratch = torch.empty(self.shard, device=self.device, dtype=torch.float32)
        self._norm = torch.zeros(1, device=self.device, dtype=torch.float32)

    # ------------------------------------------------------------ storage
    def _alloc_symmetric(self) -> None:
        from uno_b200.ops.cuda import ext
        from uno_b200.parallel.symm import _RawBuffer

        ctl = int(ext().opt_ctl_bytes())
        self.ctl_off = 0
        self.params_off = _align(ctl, 4096)
        self.grads_off = _align(self.params_off + 4 * self.n, 4096)
        nbytes = _align(self.grads_off + 4 * self.n, 4096)
        out = ext().symm_alloc(nbytes)
        self._ptr = int(out[0])
        handle = [int(b) for b in out[1:]]
        handles = [None] * self.world
        if self.group is not None:
            dist.all_gather_object(handles, handle, group=self.group)
        else:
            handles = [handle]
        self._ws = [self._ptr if j == self.rank else int(ext().symm_open(handles[j])) for j in range(self.world)]
        raw = torch.as_tensor(_RawBuffer(self._ptr, nbytes), device=self.device)
        self.flat = raw[self.params_off:self.params_off + 4 * self.n].view(torch.float32)
        self.flat_grad = raw[self.grads_off:self.grads_off + 4 * self.n].view(torch.float32)
        if self.group is not None:
            dist.barrier(group=self.group)

    def close(self) -> None:
        if self._ws is None:
            return
        from uno_b200.ops.cuda import ext

        torch.cuda.synchronize(self.device)
        if self.group is not None:
            dist.barrier(group=self.group)
        for j, ptr in enumerate(self._ws):
            ext().symm_close(ptr, j == self.rank)
        self._ws = None

    # --------------------------------------------------------------- step
    def zero_grad(self) -> None:
        self.flat_grad.zero_()

    def set_lr(self, lr: float) -> None:
        self.lr = float(lr)

    @torch.no_grad()
    def step(self) -> float:
        """One optimizer step; returns the global gradient norm before clipping."""
        self.step_count += 1
        b1, b2 = self.betas
        if self.fused:
            from uno_b200.ops.cuda import ext

            ext().fused_adamw(self._ws, self.rank, self.params_off, self.grads_off, self.ctl_off, self.n, self.m,
                              self.v, self._scratch, self._norm, self.lr, b1, b2, self.eps, self.weight_decay,
                              self.max_grad_norm, self.step_count)
            return float(self._norm.item())
        lo = self.rank * self.shard
        if self.world > 1:
            g = torch.empty(self.shard, device=self.device, dtype=torch.float32)
            dist.reduce_scatter_tensor(g, self.flat_grad, group=self.group)
            g /= self.world
        else:
            g = self.flat_grad[lo:lo + self.shard].clone()
        sq = (g.double() ** 2).sum().reshape(1)
        if self.world > 1:
            dist.all_reduce(sq, group=self.group)
        norm = float(math.sqrt(float(sq.item())))
        coef = min(1.0, self.max_grad_norm / (norm + 1e-6)) if self.max_grad_norm > 0 else 1.0
        g *= coef
        p = self.flat[lo:lo + self.shard]
        self.m.mul_(b1).add_(g, alpha=1 - b1)
        self.v.mul_(b2).addcmul_(g, g, value=1 - b2)
        bc1, bc2 = 1 - b1 ** self.step_count, 1 - b2 ** self.step_count
        p.mul_(1 - self.lr * self.weight_decay)
        p.addcdiv_(self.m / bc1, (self.v / bc2).sqrt_().add_(self.eps), value=-self.lr)
        if self.world > 1:
            dist.all_gather_into_tensor(self.flat, p.clone(), group=self.group)
        return norm

    # ------------------------------------------------------- checkpoints
    def state_dict(self) -> dict:
        return {"step": self.step_count, "m": self.m.cpu(), "v": self.v.cpu(), "world": self.world,
                "rank": self.rank, "n": self.n}

    def load_state_dict(self, state: dict) -> None:
        if int(state["world"]) != self.world or int(state["n"]) != self.n:
            raise ValueError("optimizer state was saved with a different world size or parameter layout")
        self.step_count = int(state["step"])
        self.m.copy_(state["m"])
        self.v.copy_(state["v"])
