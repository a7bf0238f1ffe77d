"""FSDP-style sharding of the frozen base weights for LoRA training.

Every projection weight ``W [N, K]`` is split by output rows across the
data-parallel ranks: rank ``j`` keeps rows ``[j N/world, (j+1) N/world)`` and
their transpose in ONE symmetric allocation that the other ranks open over
CUDA IPC.  Before a projection's GEMM the training code copies every owner's
block peer-to-local into one reusable buffer (``gather_rows`` / ``gather_cols``
in ``uno_b200.train.native``: contiguous copies on the copy engines over
NVLink), so the GEMM reads each weight byte from local HBM once per row tile.
Streaming the owners' rows straight into the GEMM's TMA loads was measured
first and re-read the weights over NVLink once per 128-row tile (0.47 / 0.28
scaling efficiency at 2 / 4 GPUs for 8,192-row training GEMMs).

Per-rank memory for the frozen projections drops to ``2 / world`` of one full
copy (rows + transposed rows), plus one gathered projection (W and W^T).  The reference does not shard the base
(DeepSpeed ZeRO-2 over the LoRA parameters only,
``training/configs/deepspeed_zero2.json:18-27``); this module is the
FSDP configuration of the training target.

Weights are written once before a barrier and never change, so the GEMMs need
no flags to read them.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from uno_b200.train.native import WeightShard


def _align(n: int, a: int = 4096) -> int:
    return -(-n // a) * a


class ShardedWeights:
    def __init__(self, entries: list[tuple[str, torch.Tensor]], group=None):
        from uno_b200.ops.cuda import ext
        from uno_b200.parallel.symm import _RawBuffer

        self.group = group if (group is not None and dist.is_initialized()) else None
        self.world = dist.get_world_size(self.group) if self.group is not None else 1
        self.rank = dist.get_rank(self.group) if self.group is not None else 0
        self.device = entries[0][1].device
        layout = {}
        off = 0
        for name, w in entries:
            N, K = w.shape
            if N % self.world or (N // self.world) % 64:
                raise ValueError(f"{name}: {N} rows do not split into 64-row multiples over {self.world} ranks")
            rows = N // self.world
            w_off = off
            wt_off = _align(w_off + rows * K * 2, 256)
            off = _align(wt_off + rows * K * 2, 256)
            layout[name] = (N, K, rows, w_off, wt_off)
        self.nbytes = _align(max(off, 4096))
        out = ext().symm_alloc(self.nbytes)
        self._ptr = int(out[0])
        handle = [int(b) for b in out[1:]]
        handles = [handle]
        if self.group is not None:
            handles = [None] * self.world
            dist.all_gather_object(handles, handle, group=self.group)
        self._bases = [self._ptr if j == self.rank else int(ext().symm_open(handles[j])) for j in range(self.world)]
        # views of every rank's region (used only as operands of this framework's own kernels)
        self._views = [torch.as_tensor(_RawBuffer(b, self.nbytes), device=self.device) for b in self._bases]
        own = self._views[self.rank]
        with torch.no_grad():
            for name, w in entries:
                N, K, rows, w_off, wt_off = layout[name]
                mine = w.detach()[self.rank * rows:(self.rank + 1) * rows].to(torch.bfloat16)
                own[w_off:w_off + rows * K * 2].view(torch.bfloat16).view(rows, K).copy_(mine)
                own[wt_off:wt_off + rows * K * 2].view(torch.bfloat16).view(K, rows).copy_(mine.t())
        torch.cuda.synchronize(self.device)
        if self.group is not None:
            dist.barrier(group=self.group)
        self.layout = layout

    def shards(self, name: str) -> list[WeightShard]:
        N, K, rows, w_off, wt_off = self.layout[name]
        out = []
        for j, v in enumerate(self._views):
            W = v[w_off:w_off + rows * K * 2].view(torch.bfloat16).view(rows, K)
            Wt = v[wt_off:wt_off + rows * K * 2].view(torch.bfloat16).view(K, rows)
            out.append(WeightShard(j * rows, (j + 1) * rows, W, Wt))
        return out

    def local_bytes(self) -> int:
        return self.nbytes

    def close(self) -> None:
        if self._bases is None:
            return
        from uno_b200.ops.cuda import ext

        torch.cuda.synchronize(self.device)
        if self.group is not None:
            dist.barrier(group=self.group)
        self._views = []
        for j, ptr in enumerate(self._bases):
            ext().symm_close(ptr, j == self.rank)
        self._bases = None
