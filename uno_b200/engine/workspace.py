"""Persistent device buffers for decode forwards (shared by eager and graph runs).

Reference: ``nano_vllm_uno/engine/block_forward_workspace.py:6-113``.  All
metadata a decode forward reads lives at fixed addresses so a captured CUDA
graph replays with fresh contents.  The host stages one pinned buffer and issues
a single host-to-device copy per forward.
"""

from __future__ import annotations

import numpy as np
import torch

from uno_b200.layers.meta import ForwardMeta, Mode


class DecodeWorkspace:
    # Packed int64 staging layout (one H2D copy): see ``stage``.
    def __init__(self, max_seqs: int, max_q: int, max_pages: int, device, page_size: int):
        self.max_seqs = int(max_seqs)
        self.max_q = int(max_q)
        self.max_pages = int(max_pages)
        self.page_size = int(page_size)
        self.device = torch.device(device)
        T = self.max_seqs * self.max_q
        self.max_tokens = T
        # int64 section: ids, positions, slots, suffix masks, prefix lens
        self._n64 = 4 * T + self.max_seqs
        self._n32 = self.max_seqs * self.max_pages
        pin = self.device.type == "cuda"
        self.host64 = torch.zeros(self._n64, dtype=torch.int64, pin_memory=pin)
        self.host32 = torch.zeros(self._n32, dtype=torch.int32, pin_memory=pin)
        self.host_lora = torch.zeros(T, dtype=torch.float32, pin_memory=pin)
        self.dev64 = torch.zeros(self._n64, dtype=torch.int64, device=self.device)
        self.dev32 = torch.zeros(self._n32, dtype=torch.int32, device=self.device)
        self.lora_mask = torch.zeros(T, dtype=torch.float32, device=self.device)
        self.input_ids = self.dev64[0:T]
        self.positions = self.dev64[T:2 * T]
        self.slot_mapping = self.dev64[2 * T:3 * T]
        self.suffix_mask_flat = self.dev64[3 * T:4 * T]
        self.prefix_lens64 = self.dev64[4 * T:4 * T + self.max_seqs]
        self.prefix_lens = torch.zeros(self.max_seqs, dtype=torch.int32, device=self.device)
        self.block_tables = self.dev32.view(self.max_seqs, self.max_pages)
        h = self.host64.numpy()
        self.h_ids = h[0:T]
        self.h_pos = h[T:2 * T]
        self.h_slot = h[2 * T:3 * T]
        self.h_mask = h[3 * T:4 * T]
        self.h_prefix = h[4 * T:4 * T + self.max_seqs]
        self.h_tables = self.host32.numpy().reshape(self.max_seqs, self.max_pages)
        self.h_lora = self.host_lora.numpy()

    def upload(self, lora: bool, n_tokens: int) -> None:
        self.dev64.copy_(self.host64, non_blocking=True)
        self.dev32.copy_(self.host32, non_blocking=True)
        if lora:
            self.lora_mask[:n_tokens].copy_(self.host_lora[:n_tokens], non_blocking=True)
        self.prefix_lens.copy_(self.prefix_lens64)

    def meta(self, mode: Mode, B: int, Q: int, lora: bool, max_kv: int = 0) -> ForwardMeta:
        T = B * Q
        return ForwardMeta(
            mode=mode,
            positions=self.positions[:T],
            slot_mapping=self.slot_mapping[:T],
            block_tables=self.block_tables[:B],
            prefix_lens=self.prefix_lens[:B],
            suffix_mask=self.suffix_mask_flat[:T].view(B, Q),
            seqlen_q=Q,
            lora_mask=self.lora_mask[:T] if lora else None,
            max_kv=max_kv or self.max_pages * self.page_size,
        )


def slots_for(block_table: list[int], start: int, count: int, page: int) -> np.ndarray:
    pos = np.arange(start, start + count, dtype=np.int64)
    table = np.asarray(block_table, dtype=np.int64)
    return table[pos // page] * page + pos % page
