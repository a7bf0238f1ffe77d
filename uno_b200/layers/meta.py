"""Per-forward metadata passed explicitly through the model.

The reference keeps this in a process-global mutable ``Context``
(``nano_vllm_uno/utils/context.py:7-94``).  Here it is an explicit argument so
that a captured CUDA graph, an eager forward and a CPU oracle forward can run
side by side without global state.

Visibility rule shared by every decode-time mode (block decode and tree
verify): for request ``b`` the first ``prefix_lens[b]`` cached tokens are
visible to every query of the forward, and query ``i`` additionally sees the
forward's own key ``j`` (stored at logical position ``prefix + j``) iff bit
``j`` of ``suffix_mask[b, i]`` is set.  A linear block uses the causal masks
``(2 << i) - 1``; a tree uses ancestor-or-self masks.  Prefill is plain causal
attention over ``cu_seqlens``.
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import Enum, auto

import torch


class Mode(Enum):
    PREFILL = auto()
    BLOCK = auto()
    TREE = auto()


@dataclass
class ForwardMeta:
    mode: Mode
    positions: torch.Tensor            # [T] int64 RoPE positions
    slot_mapping: torch.Tensor         # [T] int64 physical KV slot (-1 = do not store)
    block_tables: torch.Tensor         # [B, max_pages] int32 (-1 padded)
    # prefill
    cu_seqlens_q: torch.Tensor | None = None   # [B+1] int32
    cu_seqlens_k: torch.Tensor | None = None   # [B+1] int32 (cached prefix + new)
    max_seqlen_q: int = 0
    max_seqlen_k: int = 0
    # block / tree
    prefix_lens: torch.Tensor | None = None    # [B] int32 tokens before this forward
    suffix_mask: torch.Tensor | None = None    # [B, Q] int64 visibility bitmask
    seqlen_q: int = 0                          # queries per request (L or Q)
    # gated LoRA: 1.0 rows use the adapter, 0.0 rows the base model; None = off
    lora_mask: torch.Tensor | None = None      # [T] float32
    # prefill computes logits only at these rows (last token of each request)
    logits_indices: torch.Tensor | None = None
    # upper bound on keys any request of this forward can see (split planning)
    max_kv: int = 0

    @property
    def batch_size(self) -> int:
        return int(self.block_tables.shape[0])

    @property
    def lora_enabled(self) -> bool:
        return self.lora_mask is not None


def causal_suffix_masks(L: int, device=None) -> torch.Tensor:
    """``[L]`` int64 masks: query i sees block keys 0..i."""
    if L > 64:
        raise ValueError("block decode supports at most 64 queries per request")
    masks = [(2 << i) - 1 for i in range(L)]
    masks = [m - (1 << 64) if m >= (1 << 63) else m for m in masks]
    return torch.tensor(masks, dtype=torch.int64, device=device)


def ancestor_masks(parents: torch.Tensor) -> torch.Tensor:
    """``[B, Q]`` int64 ancestor-or-self bitmasks from parent indices (root = -1)."""
    B, Q = parents.shape
    if Q > 64:
        raise ValueError("tree masks support at most 64 nodes")
    par = parents.detach().to("cpu", torch.int64).tolist()
    out = []
    for row in par:
        masks = [0] * Q
        for i in range(Q):
            p = row[i]
            m = 1 << i
            if p >= 0:
                if p >= i:
                    raise ValueError("tree nodes must be in parent-before-child order")
                m |= masks[p]
            masks[i] = m
        # reinterpret bit 63 as a signed int64
        out.append([m - (1 << 64) if m >= (1 << 63) else m for m in masks])
    return torch.tensor(out, dtype=torch.int64, device=parents.device)
