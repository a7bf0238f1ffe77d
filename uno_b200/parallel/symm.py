"""Symmetric peer-memory workspace for the fused tensor-parallel collectives.

Every TP rank allocates one workspace of the same layout with ``cudaMalloc``,
publishes its CUDA IPC handle over the host control group and opens the
handles of its peers, so kernels can store directly into any rank's memory
over NVLink (no NCCL on the hot path).  Layout (see ``ops/csrc/comm.cu``):

* ``[0, 4096)`` control words (epoch counter, CTA counter, arrive/done flags);
* ``recv``: ``tp x R x H`` bf16 receive slots for row-parallel partial rows;
* ``gather``: ``T_max x H`` bf16 gathered activations (normalised rows that
  their owners broadcast to every rank);
* ``vp``: the vocab-parallel sampling exchange region (per-row partials and
  flags of ``ops/csrc/vocab_parallel.cu``) for up to ``max_logit_rows`` rows.

:class:`FusedTPComm` is consumed by ``uno_b200.ops.cuda``: row-parallel GEMMs
and the vocab-parallel embedding send their partial rows into the owners'
receive slots from their epilogues, and ``reduce_norm`` runs the fused
reduce + residual + RMSNorm + all-gather kernel.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


class _RawBuffer:
    """Expose a raw device allocation to torch via ``__cuda_array_interface__``."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {
            "shape": (int(nbytes),),
            "typestr": "|u1",
            "data": (int(ptr), False),
            "version": 3,
            "strides": None,
        }


def _align(n: int, a: int = 4096) -> int:
    return -(-n // a) * a


class FusedTPComm:
    def __init__(self, rank: int, world: int, control_group, max_tokens: int, hidden: int, device,
                 max_logit_rows: int | None = None):
        from uno_b200.ops.cuda import ext

        if world > 8:
            raise ValueError("fused TP collectives support at most 8 ranks")
        self.rank, self.world = int(rank), int(world)
        self.hidden = int(hidden)
        self.max_tokens = int(max_tokens)
        self.device = torch.device(device)
        R = -(-self.max_tokens // self.world)
        self.recv_off = 4096
        recv_bytes = self.world * R * self.hidden * 2
        self.gather_off = _align(self.recv_off + recv_bytes)
        gather_bytes = self.world * R * self.hidden * 2
        self.vp_off = _align(self.gather_off + gather_bytes)
        self.max_logit_rows = int(max_logit_rows or self.max_tokens)
        self.nbytes = _align(self.vp_off + int(ext().vp_region_bytes(self.max_logit_rows)))
        out = ext().symm_alloc(self.nbytes)
        self.ptr = int(out[0])
        handle = [int(b) for b in out[1:]]
        handles: list = [None] * self.world
        dist.all_gather_object(handles, handle, group=control_group)
        self.peers = [self.ptr if j == self.rank else int(ext().symm_open(handles[j])) for j in range(self.world)]
        raw = torch.as_tensor(_RawBuffer(self.ptr + self.gather_off, gather_bytes), device=self.device)
        self.gather = raw.view(torch.bfloat16).view(self.world * R, self.hidden)
        self._closed = False
        dist.barrier(group=control_group)

    def vp_args(self) -> tuple[list[int], int, int]:
        """``(exchange region of every rank, rank, max rows)`` for the vocab-parallel sampling kernels."""
        return [p + self.vp_off for p in self.peers], self.rank, self.max_logit_rows

    def rows_per_rank(self, T: int) -> int:
        return -(-int(T) // self.world)

    def rs_args(self, T: int):
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed the fused TP workspace ({self.max_tokens})")
        return (self.peers, self.rank, self.recv_off)

    def gather_wait_args(self, a: torch.Tensor) -> tuple[int, int]:
        """``(workspace base, rows per rank)`` when ``a`` lives in the gathered buffer, else ``(0, 0)``.

        A GEMM reading gathered rows waits, per tile, for the ranks that own
        them to finish broadcasting (the reduce kernel itself does not wait)."""
        ptr = a.data_ptr()
        lo = self.ptr + self.gather_off
        if lo <= ptr < lo + self.gather.numel() * 2:
            return self.ptr, self.rows_per_rank(a.shape[0])
        return 0, 0

    def reduce_norm(self, T: int, residual: torch.Tensor | None, weight, eps: float, groups: int,
                    final: bool = False):
        """Sum partials of owned rows (+ residual), RMSNorm, broadcast rows.

        Returns ``(gathered normed rows [T, H], residual shard [R, H])``.  The
        kernel returns before the peers' rows have landed; GEMMs reading the
        gathered rows wait for their owners tile by tile.  ``final`` (the last
        norm of a forward, whose rows leave the fused path) waits for all rows.
        """
        from uno_b200.ops.cuda import ext

        add = residual is not None
        if residual is None:
            residual = torch.empty(self.rows_per_rank(T), self.hidden, device=self.device, dtype=torch.bfloat16)
        ext().reduce_norm_gather(self.peers, self.rank, int(T), self.hidden, self.recv_off, self.gather_off,
                                 residual, add, weight, int(groups), float(eps), bool(final))
        return self.gather[:T], residual

    def embedding_scatter(self, ids: torch.Tensor, table: torch.Tensor, vocab_start: int) -> None:
        from uno_b200.ops.cuda import ext

        ext().embedding_scatter(self.peers, self.rank, ids.reshape(-1).contiguous(), table, int(vocab_start),
                                self.recv_off, self.gather_off)

    def close(self) -> None:
        if self._closed:
            return
        from uno_b200.ops.cuda import ext

        self._closed = True
        torch.cuda.synchronize()
        for j, p in enumerate(self.peers):
            if j != self.rank:
                ext().symm_close(p, False)
        ext().symm_close(self.ptr, True)
