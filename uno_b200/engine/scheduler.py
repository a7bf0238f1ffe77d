"""Prefill-first, unchunked scheduler with decode-time page reservation.

Mirrors the reference policy (``nano_vllm_uno/engine/scheduler.py:9-135``):

* a step is either a prefill batch (waiting requests admitted FIFO while the
  prompt tokens not served by the prefix cache fit ``max_num_batched_tokens``)
  or a decode batch of running requests;
* prefill is never chunked: a single prompt larger than the budget is an error;
* decode reserves pages for ``max(block_len, tree_verify_size)`` extra tokens
  per request, preempting from the tail of the running queue when pages run
  out (``fail_on_preemption`` turns a preemption into an error);
* a preempted request frees its pages and returns to the front of the queue
  (recomputation).
"""

from __future__ import annotations

from collections import deque

from uno_b200.engine.block_manager import BlockManager
from uno_b200.engine.sequence import Sequence, SequenceStatus
from uno_b200.sampling_params import SamplingParams


class Scheduler:
    def __init__(self, config):
        self.max_num_seqs = int(config.max_num_seqs)
        self.max_num_batched_tokens = int(config.max_num_batched_tokens)
        self.eos = config.eos
        self.fail_on_preemption = bool(config.fail_on_preemption)
        self.tree_verify_size = config.tree_verify_size
        self.block_manager = BlockManager(config.num_kvcache_blocks, config.kvcache_block_size)
        self.waiting: deque[Sequence] = deque()
        self.running: deque[Sequence] = deque()
        self.num_preemptions = 0
        self.num_prefill_batches = 0
        self.prefill_batch_sizes: list[int] = []
        self.decode_batch_sizes: list[int] = []

    def is_finished(self) -> bool:
        return not self.waiting and not self.running

    def add(self, seq: Sequence) -> None:
        self.waiting.append(seq)

    def forward_reserve(self, sampling_params: SamplingParams) -> int:
        return max(int(sampling_params.diffusion_block_size), int(self.tree_verify_size or 0))

    def schedule(self, sampling_params: SamplingParams) -> tuple[list[Sequence], bool]:
        batch = self._schedule_prefill()
        if batch:
            self.num_prefill_batches += 1
            self.prefill_batch_sizes.append(len(batch))
            return batch, True
        batch = self._schedule_decode(sampling_params)
        self.decode_batch_sizes.append(len(batch))
        return batch, False

    def _schedule_prefill(self) -> list[Sequence]:
        batch: list[Sequence] = []
        tokens = 0
        slots = max(0, self.max_num_seqs - len(self.running))
        bm = self.block_manager
        while self.waiting and len(batch) < slots:
            seq = self.waiting[0]
            hits = bm.plan_prefix_cache_and_check_capacity(seq)
            if hits is None:
                break
            uncached = len(seq) - hits * bm.block_size
            if uncached > self.max_num_batched_tokens:
                raise ValueError(
                    "Prompt exceeds the non-chunked prefill budget: "
                    f"{uncached} uncached tokens > "
                    f"max_num_batched_tokens={self.max_num_batched_tokens}"
                )
            if tokens + uncached > self.max_num_batched_tokens:
                break
            bm.allocate(seq, hits)
            tokens += uncached
            seq.status = SequenceStatus.RUNNING
            self.waiting.popleft()
            self.running.append(seq)
            batch.append(seq)
        return batch

    def _schedule_decode(self, sampling_params: SamplingParams) -> list[Sequence]:
        reserve = self.forward_reserve(sampling_params)
        bm = self.block_manager
        batch: list[Sequence] = []
        while self.running and len(batch) < self.max_num_seqs:
            seq = self.running.popleft()
            admitted = True
            while not bm.has_enough_blocks_for_forward(seq, reserve):
                if self.running:
                    self.preempt(self.running.pop())
                else:
                    self.preempt(seq)
                    admitted = False
                    break
            if admitted:
                bm.reserve_blocks_for_forward(seq, reserve)
                batch.append(seq)
        if not batch:
            raise RuntimeError(
                "No request fits in the KV cache even after preempting all others; "
                "increase the cache size or lower max_model_len"
            )
        self.running.extendleft(reversed(batch))
        return batch

    def preempt(self, seq: Sequence) -> None:
        self.num_preemptions += 1
        if self.fail_on_preemption:
            raise RuntimeError(
                "Scheduler preemption disabled for this run: "
                f"seq_id={seq.seq_id}, len={len(seq)}, "
                f"free_blocks={self.block_manager.num_free_blocks}"
            )
        seq.status = SequenceStatus.WAITING
        self.block_manager.deallocate(seq)
        self.waiting.appendleft(seq)

    def reset_stats(self) -> None:
        self.num_preemptions = 0
        self.num_prefill_batches = 0
        self.prefill_batch_sizes.clear()
        self.decode_batch_sizes.clear()

    def postprocess(
        self,
        seqs: list[Sequence],
        token_ids_batch: list[list[int]],
        sampling_params: SamplingParams,
    ) -> None:
        """Finish requests that emitted a stop token or reached their budget."""
        stops = set(sampling_params.stop_token_ids or [])
        if self.eos is not None and self.eos >= 0:
            stops.add(self.eos)
        for seq, new_tokens in zip(seqs, token_ids_batch):
            hit_stop = not sampling_params.ignore_eos and any(t in stops for t in new_tokens)
            limit = (
                seq.max_completion_tokens
                if seq.max_completion_tokens is not None
                else sampling_params.max_tokens
            )
            if hit_stop or seq.num_completion_tokens >= limit:
                seq.status = SequenceStatus.FINISHED
                self.block_manager.deallocate(seq)
                self.running.remove(seq)
