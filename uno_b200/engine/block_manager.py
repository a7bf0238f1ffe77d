"""Paged KV-cache page allocator with a hashed prefix cache.

Same contract as the reference ``BlockManager`` (``nano_vllm_uno/engine/block_manager.py:25-196``):

* pages hold ``block_size`` tokens and are reference counted;
* a full page whose K/V is complete is *published* under a chained 64-bit hash
  of its tokens (hash of page i folds in the hash of page i-1), so identical
  prompt prefixes share pages;
* freed pages keep their hash and can be re-activated by a later prefix hit
  until they are handed out again;
* decode reserves the pages for the whole draft/verify span up front so the
  model runner never allocates inside a forward.

Only the last token of a sequence may be uncached, so at most ``len - 1``
tokens are eligible for prefix reuse.
"""

from __future__ import annotations

from collections import deque

import numpy as np
import xxhash

from uno_b200.engine.sequence import Sequence


class Block:
    __slots__ = ("block_id", "ref_count", "hash", "token_ids")

    def __init__(self, block_id: int):
        self.block_id = block_id
        self.ref_count = 0
        self.hash = -1
        self.token_ids: list[int] = []


def chain_hash(token_ids: list[int], prefix: int = -1) -> int:
    """xxh64 over the little-endian int64 tokens, seeded by the parent hash."""
    h = xxhash.xxh64()
    if prefix != -1:
        h.update(int(prefix).to_bytes(8, "little"))
    h.update(np.asarray(token_ids, dtype=np.int64).tobytes())
    return h.intdigest()


class BlockManager:
    def __init__(self, num_blocks: int, block_size: int):
        if num_blocks < 1:
            raise ValueError("the KV cache needs at least one page")
        self.block_size = int(block_size)
        self.blocks = [Block(i) for i in range(num_blocks)]
        self.hash_to_block_id: dict[int, int] = {}
        self.free_block_ids: deque[int] = deque(range(num_blocks))
        self.used_block_ids: set[int] = set()

    # ----------------------------------------------------------- internals
    compute_hash = staticmethod(chain_hash)

    @property
    def num_free_blocks(self) -> int:
        return len(self.free_block_ids)

    def _take_free_block(self) -> Block:
        block_id = self.free_block_ids.popleft()
        block = self.blocks[block_id]
        if block.ref_count != 0:
            raise RuntimeError(f"free page {block_id} still referenced")
        # The page is being repurposed: drop its prefix-cache entry.
        if block.hash != -1 and self.hash_to_block_id.get(block.hash) == block_id:
            del self.hash_to_block_id[block.hash]
        block.ref_count = 1
        block.hash = -1
        block.token_ids = []
        self.used_block_ids.add(block_id)
        return block

    def _release_block(self, block_id: int) -> None:
        self.used_block_ids.discard(block_id)
        self.free_block_ids.append(block_id)

    def _cached_prefix(self, seq: Sequence):
        """Yield (page index, hash, page id) for the reusable leading pages."""
        h = -1
        cacheable = max(0, len(seq) - 1)
        for i in range(seq.num_blocks):
            end = min((i + 1) * self.block_size, len(seq))
            if end - i * self.block_size != self.block_size or end > cacheable:
                return
            tokens = seq.block(i)
            h = chain_hash(tokens, h)
            block_id = self.hash_to_block_id.get(h, -1)
            if block_id == -1 or self.blocks[block_id].token_ids != tokens:
                return
            yield i, h, block_id

    # ------------------------------------------------------------- prefill
    def plan_prefix_cache_and_check_capacity(self, seq: Sequence) -> int | None:
        """Number of reusable prefix pages, or None when the prompt does not fit."""
        hits = 0
        needed = seq.num_blocks
        for _, _, block_id in self._cached_prefix(seq):
            hits += 1
            if block_id in self.used_block_ids:
                needed -= 1  # shared with a live sequence: costs no free page
        if len(self.free_block_ids) < needed:
            return None
        return hits

    def allocate(self, seq: Sequence, num_cached_blocks: int) -> None:
        if seq.block_table:
            raise RuntimeError(f"seq {seq.seq_id} already owns pages")
        if not 0 <= num_cached_blocks <= seq.num_blocks:
            raise ValueError("invalid cached page count")
        h = -1
        for i in range(num_cached_blocks):
            tokens = seq.block(i)
            h = chain_hash(tokens, h)
            block_id = self.hash_to_block_id[h]
            block = self.blocks[block_id]
            if block.token_ids != tokens:
                raise RuntimeError("prefix cache hash collision")
            if block_id in self.used_block_ids:
                block.ref_count += 1
            else:
                # Re-activate a free page that still holds valid K/V.
                block.ref_count = 1
                self.free_block_ids.remove(block_id)
                self.used_block_ids.add(block_id)
            seq.block_table.append(block_id)
        for _ in range(num_cached_blocks, seq.num_blocks):
            seq.block_table.append(self._take_free_block().block_id)
        seq.num_cached_tokens = num_cached_blocks * self.block_size

    # ------------------------------------------------------------- publish
    def publish_computed_prefix_blocks(self, seq: Sequence) -> None:
        """Publish full pages whose K/V is complete after this step."""
        end = min(seq.num_cached_tokens // self.block_size, seq.num_blocks, len(seq.block_table))
        start = end
        while start > 0 and self.blocks[seq.block_table[start - 1]].hash == -1:
            start -= 1
        if start == end:
            return
        h = self.blocks[seq.block_table[start - 1]].hash if start > 0 else -1
        for i in range(start, end):
            tokens = seq.block(i)
            h = chain_hash(tokens, h)
            block = self.blocks[seq.block_table[i]]
            block.hash = h
            block.token_ids = tokens
            self.hash_to_block_id[h] = block.block_id

    def deallocate(self, seq: Sequence) -> None:
        for block_id in reversed(seq.block_table):
            block = self.blocks[block_id]
            block.ref_count -= 1
            if block.ref_count == 0:
                self._release_block(block_id)
            elif block.ref_count < 0:
                raise RuntimeError(f"page {block_id} released twice")
        seq.num_cached_tokens = 0
        seq.block_table.clear()

    # -------------------------------------------------------------- decode
    def num_blocks_needed_for_forward(self, seq: Sequence, num_forward_tokens: int = 1) -> int:
        if num_forward_tokens <= 0:
            return 0
        if not seq.block_table:
            raise RuntimeError("forward sizing requires an admitted sequence")
        total = len(seq) + num_forward_tokens
        return max(0, -(-total // self.block_size) - len(seq.block_table))

    def has_enough_blocks_for_forward(self, seq: Sequence, num_forward_tokens: int = 1) -> bool:
        return len(self.free_block_ids) >= self.num_blocks_needed_for_forward(seq, num_forward_tokens)

    def reserve_blocks_for_forward(self, seq: Sequence, num_forward_tokens: int) -> int:
        extra = self.num_blocks_needed_for_forward(seq, num_forward_tokens)
        if extra > len(self.free_block_ids):
            raise RuntimeError(
                f"Cannot reserve {extra} KV blocks for seq_id={seq.seq_id}; "
                f"only {len(self.free_block_ids)} are free"
            )
        for _ in range(extra):
            seq.block_table.append(self._take_free_block().block_id)
        return extra
