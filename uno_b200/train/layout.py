"""Block-diffusion training layout: one forward over paired noisy/clean copies.

The reference delegates this to the checkpoint's remote code
(``prepare_for_bd_training``, ``training/modeling.py:93-113``, called from
``training/trainer.py:186-203``); it is restated here from its documented
behaviour:

* every packed sequence (positions restart at 0) contributes its *noisy* copy
  followed by its *clean* copy, so a row of length S becomes 2S
  (``training/modeling.py:71-88``);
* noise: each block of ``block_size`` positions draws ``t ~ U(0, 1)`` and
  ``p = eps + (1 - eps) t``; every supervised token (label != IGNORE) of the
  block is replaced, with probability ``p``, by a uniform id in
  ``[1, mask_token_id)`` (the inference noise, ``engine/noise.py:24-26``);
* visibility: a noisy token sees the clean tokens strictly before its block
  and every noisy token of its own block; a clean token sees the clean tokens
  at or before its position; nothing crosses packed sequences;
* the gated LoRA is active on the noisy copy only.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from uno_b200.train.config import IGNORE_INDEX


@dataclass
class UnoBatch:
    ids: torch.Tensor          # [B, 2S] noisy/clean copies per packed sequence
    positions: torch.Tensor    # [B, 2S]
    noisy: torch.Tensor        # [B, 2S] bool: token belongs to a noisy copy
    segment: torch.Tensor      # [B, 2S] packed-sequence index inside the row
    noisy_index: torch.Tensor  # [B, S] where original token i sits in the noisy copy
    clean_index: torch.Tensor  # [B, S] where it sits in the clean copy
    noised: torch.Tensor       # [B, S] bool: token i was replaced by noise
    p_mask: torch.Tensor       # [n_noised] noise probability of each noised token (row-major)
    block_size: int

    def attention_mask(self) -> torch.Tensor:
        """Dense visibility ``[B, 2S, 2S]`` (True = may attend)."""
        return visibility(self.segment, self.positions, self.noisy, self.block_size)

    def gather_regions(self, hidden: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Split ``hidden [B, 2S, H]`` into noisy and clean states in original token order."""
        h = hidden.shape[-1]
        noisy = hidden.gather(1, self.noisy_index[..., None].expand(-1, -1, h))
        clean = hidden.gather(1, self.clean_index[..., None].expand(-1, -1, h))
        return noisy, clean


def visibility(segment, positions, noisy, block_size: int) -> torch.Tensor:
    sq, sk = segment[:, :, None], segment[:, None, :]
    pq, pk = positions[:, :, None], positions[:, None, :]
    nq, nk = noisy[:, :, None], noisy[:, None, :]
    bq = pq // block_size
    vis = (nq & nk & (pk // block_size == bq)) | (nq & ~nk & (pk < bq * block_size)) | (~nq & ~nk & (pk <= pq))
    return vis & (sq == sk)


def build_uno_batch(input_ids: torch.Tensor, labels: torch.Tensor, position_ids: torch.Tensor | None = None, *,
                    block_size: int, mask_token_id: int, generator: torch.Generator | None = None,
                    eps: float = 1e-3) -> UnoBatch:
    if block_size <= 0:
        raise ValueError("block_size must be positive")
    if mask_token_id <= 1:
        raise ValueError("mask_token_id must be > 1 (noise ids are drawn from [1, mask_token_id))")
    B, S = input_ids.shape
    dev = input_ids.device
    ar = torch.arange(S, device=dev)
    if position_ids is None:
        position_ids = ar.expand(B, S)
    position_ids = position_ids.long()
    starts = position_ids == 0
    starts[:, 0] = True
    seg = starts.long().cumsum(1) - 1
    # consecutive block numbering: a block starts at a new sequence or a new position block
    blk = position_ids // block_size
    block_start = starts.clone()
    block_start[:, 1:] |= blk[:, 1:] != blk[:, :-1]
    block_num = block_start.long().cumsum(1) - 1

    t = torch.rand(B, S, generator=generator, device=dev).gather(1, block_num)
    p = eps + (1.0 - eps) * t
    eligible = labels != IGNORE_INDEX
    noised = eligible & (torch.rand(B, S, generator=generator, device=dev) < p)
    noise_ids = torch.randint(1, mask_token_id, (B, S), generator=generator, device=dev)
    noisy_ids = torch.where(noised, noise_ids, input_ids)

    # placement: sequence [start, start+len) -> noisy at 2*start.., clean at 2*start+len..
    seg_start = torch.where(starts, ar.expand(B, S), torch.zeros_like(position_ids)).cummax(1).values
    seg_len = torch.zeros(B, S, dtype=torch.long, device=dev).scatter_add_(1, seg, torch.ones_like(seg))
    length = seg_len.gather(1, seg)
    noisy_index = seg_start + ar                      # = 2*start + (i - start)
    clean_index = seg_start + length + ar             # = 2*start + len + (i - start)

    def place(noisy_val, clean_val):
        out = torch.empty(B, 2 * S, dtype=noisy_val.dtype, device=dev)
        out.scatter_(1, noisy_index, noisy_val)
        out.scatter_(1, clean_index, clean_val)
        return out

    return UnoBatch(
        ids=place(noisy_ids, input_ids),
        positions=place(position_ids, position_ids),
        noisy=place(torch.ones(B, S, dtype=torch.bool, device=dev), torch.zeros(B, S, dtype=torch.bool, device=dev)),
        segment=place(seg, seg),
        noisy_index=noisy_index,
        clean_index=clean_index,
        noised=noised,
        p_mask=p[noised],
        block_size=int(block_size),
    )


def shift_labels_for_next_token(labels: torch.Tensor, position_ids: torch.Tensor) -> torch.Tensor:
    """Next-token labels; positions that end a packed sequence get IGNORE
    (``training/losses.py:9-18``)."""
    shifted = torch.full_like(labels, IGNORE_INDEX)
    shifted[:, :-1] = labels[:, 1:]
    shifted[:, :-1].masked_fill_(position_ids[:, :-1] >= position_ids[:, 1:], IGNORE_INDEX)
    return shifted
