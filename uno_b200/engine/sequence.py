"""Request state: tokens, KV frontier, page table and decode statistics.

Behavioural twin of the reference ``Sequence`` (``nano_vllm_uno/engine/sequence.py:22-145``):
the logical sequence is ``token_ids``; ``num_cached_tokens`` is the KV frontier
(how many leading tokens have K/V resident in the paged cache); the final token
of a running sequence is normally *uncached* and is the seed of the next
forward.  ``stats`` carries the TPF accounting keys (forwards, accepts,
lookaheads).
"""

from __future__ import annotations

from enum import Enum, auto
from itertools import count

DECODE_STAT_KEYS = ("forwards", "accepts", "lookaheads")


def new_decode_stats() -> dict[str, int]:
    return {key: 0 for key in DECODE_STAT_KEYS}


class SequenceStatus(Enum):
    WAITING = auto()
    RUNNING = auto()
    FINISHED = auto()


class Sequence:
    block_size = 256
    _ids = count()

    __slots__ = (
        "seq_id",
        "status",
        "token_ids",
        "num_prompt_tokens",
        "num_cached_tokens",
        "block_table",
        "stats",
        "max_completion_tokens",
        "noise_seed",
    )

    def __init__(self, token_ids: list[int], max_completion_tokens: int | None = None):
        if not token_ids:
            raise ValueError("a sequence needs at least one prompt token")
        self.seq_id = next(Sequence._ids)
        self.status = SequenceStatus.WAITING
        self.token_ids = [int(t) for t in token_ids]
        self.num_prompt_tokens = len(self.token_ids)
        self.num_cached_tokens = 0
        self.block_table: list[int] = []
        self.stats = new_decode_stats()
        self.max_completion_tokens = (
            None if max_completion_tokens is None else int(max_completion_tokens)
        )
        self.noise_seed: int | None = None

    # ------------------------------------------------------------------ views
    def __len__(self) -> int:
        return len(self.token_ids)

    def __getitem__(self, key):
        return self.token_ids[key]

    @property
    def num_tokens(self) -> int:
        return len(self.token_ids)

    @property
    def last_token(self) -> int:
        return self.token_ids[-1]

    @property
    def is_finished(self) -> bool:
        return self.status is SequenceStatus.FINISHED

    @property
    def num_completion_tokens(self) -> int:
        return len(self.token_ids) - self.num_prompt_tokens

    @property
    def prompt_token_ids(self) -> list[int]:
        return self.token_ids[: self.num_prompt_tokens]

    @property
    def completion_token_ids(self) -> list[int]:
        return self.token_ids[self.num_prompt_tokens :]

    @property
    def num_cached_blocks(self) -> int:
        return self.num_cached_tokens // self.block_size

    @property
    def num_blocks(self) -> int:
        return -(-len(self.token_ids) // self.block_size)

    @property
    def last_block_num_tokens(self) -> int:
        return len(self.token_ids) - (self.num_blocks - 1) * self.block_size

    def block(self, i: int) -> list[int]:
        if not 0 <= i < self.num_blocks:
            raise IndexError(i)
        return self.token_ids[i * self.block_size : (i + 1) * self.block_size]

    # -------------------------------------------------------------- mutation
    def extend_tokens(self, tokens: list[int]) -> None:
        if tokens:
            self.token_ids.extend(int(t) for t in tokens)

    def rollback_kv_to(self, target: int) -> None:
        """Move the KV frontier back to ``target`` without touching tokens.

        The frontier may never drop below ``len - 1`` (the seed token is the
        only token allowed to be uncached) nor rise above its current value.
        """
        low = max(0, len(self) - 1)
        if not low <= target <= self.num_cached_tokens:
            raise ValueError(
                "Invalid KV rollback target: "
                f"minimum={low}, target={target}, current={self.num_cached_tokens}"
            )
        self.num_cached_tokens = target

    def __repr__(self) -> str:  # pragma: no cover - debugging aid
        return (
            f"Sequence(id={self.seq_id}, len={len(self)}, cached={self.num_cached_tokens}, "
            f"blocks={len(self.block_table)}, status={self.status.name})"
        )
