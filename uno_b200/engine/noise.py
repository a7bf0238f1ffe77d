"""Draft-row noise for the Psi-Spec draft forward.

Semantics of ``nano_vllm_uno/engine/noise.py:10-179``:

* ``random_uniform``: ids uniform in ``[1, mask_token_id)`` (the Uno training
  noise, bounded by the vocabulary);
* ``mask``: every noise slot holds ``mask_token_id``;
* ``deterministic_uniform``: a splitmix64-style hash of (prompt hash, salt,
  completion length, seed token, sequence length, slot) so that the noise is
  independent of batching and scheduling (reproducibility tests).
"""

from __future__ import annotations

import numpy as np
import torch

from uno_b200.engine.sequence import Sequence
from uno_b200.sampling_params import SamplingParams

_M64 = 0xFFFFFFFFFFFFFFFF


def noise_bounds(sp: SamplingParams, vocab_size: int) -> tuple[int, int]:
    mask = sp.mask_token_id
    if mask is None or int(mask) <= 1:
        raise ValueError(
            "two-pass decoding requires mask_token_id on SamplingParams; noise "
            "tokens must be bounded by the diffusion-training mask token."
        )
    return 1, min(int(mask), int(vocab_size))


def splitmix64(value: int) -> int:
    """Finaliser of splitmix64 (Steele, Lea & Flood 2014)."""
    z = value & _M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
    return (z ^ (z >> 31)) & _M64


def prompt_seed(seq: Sequence) -> int:
    if seq.noise_seed is None:
        h = 0xD6E8FEB86659FD93
        for t in seq.prompt_token_ids:
            h = splitmix64(h ^ int(t))
        seq.noise_seed = h
    return seq.noise_seed


def deterministic_noise(seq: Sequence, count: int, low: int, high: int, seed_token: int,
                        sp: SamplingParams) -> list[int]:
    span = max(1, high - low)
    salt = seq.seq_id if sp.noise_salt is None else sp.noise_salt
    base = (
        prompt_seed(seq) * 0x9E3779B185EBCA87
        + int(salt) * 0xD1B54A32D192ED03
        + seq.num_completion_tokens * 0xC2B2AE3D27D4EB4F
        + int(seed_token) * 0x165667B19E3779F9
        + len(seq) * 0x85EBCA77C2B2AE63
    )
    return [low + splitmix64(base + s * 0x27D4EB2F165667C5) % span for s in range(count)]


def build_draft_batch(seqs: list[Sequence], block_len: int, sp: SamplingParams, *, vocab_size: int,
                      generator: torch.Generator | None = None) -> np.ndarray:
    """Host ``[B, L]`` int64 rows ``[seed, noise_1 .. noise_{L-1}]``."""
    B = len(seqs)
    out = np.empty((B, block_len), dtype=np.int64)
    out[:, 0] = [s.token_ids[-1] for s in seqs]
    if block_len <= 1:
        return out
    low, high = noise_bounds(sp, vocab_size)
    if sp.noise_mode == "random_uniform":
        out[:, 1:] = torch.randint(low, high, (B, block_len - 1), generator=generator).numpy()
    elif sp.noise_mode == "mask":
        out[:, 1:] = high
    else:
        for i, seq in enumerate(seqs):
            out[i, 1:] = deterministic_noise(seq, block_len - 1, low, high, seq.token_ids[-1], sp)
    return out
