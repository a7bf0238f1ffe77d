"""Psi-Spec two-pass decoding (draft forward + verify forward per cycle).

Algorithm of ``nano_vllm_uno/engine/two_pass_decoding.py:100-817``:

Linear sampler, block length L:

1. **Draft** forward on ``[seed, noise_1 .. noise_{L-1}]`` with the gated LoRA
   active on the noise rows only.  Row 0 is the exact AR distribution of the
   next token (the base model sees only committed context), so ``clean`` is an
   exact target sample; rows 1.. give the draft distributions ``q`` and the
   proposals ``spec_i``.  The noise K/V is discarded afterwards.
2. **Verify** forward on ``[clean, spec_1 .. spec_{L-1}]`` with LoRA off.  Row
   ``i`` gives the target ``p`` for ``spec_{i+1}``; the last row gives a
   *lookahead* sample.  Proposals are accepted left to right with probability
   ``min(1, p/q)``; the first rejection is replaced by a residual resample.
   At most ``L + 1`` tokens commit per two forwards.
3. One device-to-host copy of ``[committed..., length]`` rows per cycle.

Tree sampler: the draft rows provide per-depth top-K candidates from which a
best-first tree of ``tree_verify_size`` nodes is built; one tree-masked
forward scores every node; a target token is sampled at every node and walked
through the tree; the accepted path's K/V is compacted in place.

Stats per request: ``forwards += 2``, ``accepts += committed``,
``lookaheads += committed > L`` (TPF = accepts / forwards).
"""

from __future__ import annotations

from typing import Callable

import numpy as np
import torch

from uno_b200.engine.draft_tree import build_draft_tree_batch, walk_tree
from uno_b200.engine.noise import build_draft_batch
from uno_b200.engine.sampling import Sampler
from uno_b200.engine.sequence import Sequence
from uno_b200.sampling_params import SamplingParams
from uno_b200.utils.trace import nvtx


class TwoPassDecoder:
    def __init__(
        self,
        run_block: Callable,
        eos_token_id: int,
        pad_token_id: int,
        vocab_size: int,
        device: torch.device,
        sampler: Sampler,
        gated_lora: bool = False,
        run_tree: Callable | None = None,
        compact_tree_kv: Callable | None = None,
        tree_verify_size: int | None = None,
        tree_candidate_top_k: int = 16,
        noise_seed: int = 0,
    ):
        self.run_block = run_block
        self.eos_token_id = int(eos_token_id) if eos_token_id is not None else -1
        self.pad_token_id = int(pad_token_id) if pad_token_id is not None else 0
        self.vocab_size = int(vocab_size)
        self.device = torch.device(device)
        self.sampler = sampler
        self.gated_lora = bool(gated_lora)
        self.run_tree = run_tree
        self.compact_tree_kv = compact_tree_kv
        self.tree_verify_size = tree_verify_size
        self.tree_candidate_top_k = int(tree_candidate_top_k)
        if tree_verify_size is not None and (run_tree is None or compact_tree_kv is None):
            raise ValueError("tree verification requires run_tree and compact_tree_kv callbacks")
        self.noise_gen = torch.Generator()
        self.noise_gen.manual_seed(int(noise_seed))

    # ------------------------------------------------------------------ cycle
    @torch.inference_mode()
    def run_cycle(self, seqs: list[Sequence], sp: SamplingParams, apply: bool = True) -> list[list[int]]:
        if not seqs:
            return []
        L = int(sp.diffusion_block_size)
        with nvtx("draft"):
            proposal, draft_logits, q_sparse = self.draft_stage(seqs, L, sp)
        if self.tree_verify_size is None:
            with nvtx("verify"):
                payload = self.verify_stage(seqs, proposal, draft_logits, q_sparse, sp)
        else:
            with nvtx("tree"):
                payload = self.tree_verify_stage(seqs, proposal[:, 0], draft_logits, L, sp)
        rows = payload.cpu().numpy()  # the single host synchronisation of the cycle
        accepted = [[] for _ in seqs]
        if apply:
            self.apply_committed_rows(seqs, accepted, rows, L)
        return accepted

    @staticmethod
    def apply_committed_rows(seqs, accepted, rows: np.ndarray, block_len: int) -> None:
        for seq, out, row in zip(seqs, accepted, rows):
            n = int(row[-1])
            committed = [int(t) for t in row[:n]]
            if seq.max_completion_tokens is not None:
                remaining = max(0, seq.max_completion_tokens - seq.num_completion_tokens)
                committed = committed[:remaining]
            if committed:
                seq.extend_tokens(committed)
                out.extend(committed)
            seq.stats["forwards"] += 2
            seq.stats["accepts"] += len(committed)
            seq.stats["lookaheads"] += int(len(committed) > block_len)
            target = max(0, len(seq) - 1)
            seq.rollback_kv_to(target)

    # ------------------------------------------------------------------ draft
    def draft_stage(self, seqs, L: int, sp: SamplingParams):
        B = len(seqs)
        host = build_draft_batch(seqs, L, sp, vocab_size=self.vocab_size, generator=self.noise_gen)
        draft_tokens = torch.from_numpy(host).to(self.device, non_blocking=True)
        use_lora = self.gated_lora and L > 1
        logits = self.run_block(seqs, draft_tokens, lora=use_lora)  # [B, L, V]
        q_sparse = None
        if self.tree_verify_size is None:
            proposal = torch.empty((B, L), dtype=torch.int64, device=logits.device)
            clean, _ = self.sampler.sample(logits[:, 0, :], sp)
            proposal[:, 0] = clean
            if L > 1:
                spec_rows = logits[:, 1:, :]  # strided [B, L-1, V] rows: the CUDA samplers read them in place
                if not spec_rows.is_cuda:
                    spec_rows = spec_rows.reshape(-1, logits.shape[-1])
                spec, q_sparse = self.sampler.sample(spec_rows, sp)
                proposal[:, 1:] = spec.view(B, L - 1)
        else:
            # Under vocab parallelism the logits stay sharded: the root is sampled by the
            # vocab-parallel sampler and the tree builder merges per-shard candidates.
            proposal = torch.zeros((B, L), dtype=torch.int64, device=logits.device)
            root, _ = self.sampler.sample(logits[:, 0, :], sp)
            proposal[:, 0] = root
        draft_logits = logits[:, 1:, :]
        # Drop the noise K/V: only the seed stays cached.
        for seq in seqs:
            seq.rollback_kv_to(len(seq))
        return proposal, draft_logits, q_sparse

    # ----------------------------------------------------------------- verify
    def verify_stage(self, seqs, proposal, draft_logits, q_sparse, sp: SamplingParams):
        B, L = proposal.shape
        logits = self.run_block(seqs, proposal, lora=False)
        lookahead, _ = self.sampler.sample(logits[:, -1, :], sp)
        on_gpu = proposal.is_cuda
        if L == 1:
            if on_gpu:
                return self._payload_gpu(proposal, lookahead, sp)
            accepted = torch.ones((B, 0), dtype=torch.bool, device=proposal.device)
            corr = proposal[:, 1:]
        elif sp.greedy:
            target = self._argmax(logits[:, : L - 1, :])
            if on_gpu:
                return self._payload_gpu(proposal, lookahead, sp, target=target)
            accepted = proposal[:, 1:] == target
            corr = target
        else:
            V = self.sampler.vocab_size(logits)
            Vs = logits.shape[-1]  # the local vocabulary shard under vocab-parallel sampling
            clean = logits[:, : L - 1, :]
            draft = draft_logits[:, : L - 1, :]
            if not clean.is_cuda:
                clean, draft = clean.reshape(-1, Vs), draft.reshape(-1, Vs)
            spec = proposal[:, 1:].reshape(-1)
            if sp.filtered(V):
                if q_sparse is None:
                    raise RuntimeError("Filtered draft verification requires the sampled sparse q")
                acc, c = self.sampler.verify_filtered(clean, spec, sp, q_sparse)
            else:
                acc, c = self.sampler.verify_unfiltered(clean, draft, spec, sp.temperature)
            if on_gpu:
                return self._payload_gpu(proposal, lookahead, sp, accepted=acc, corr=c)
            accepted = acc.view(B, L - 1).bool()
            corr = c.view(B, L - 1)
        return self.build_payload(proposal, accepted, corr, lookahead, sp)

    def _payload_gpu(self, proposal, lookahead, sp: SamplingParams, **kw):
        """Payload assembly and stop truncation in one kernel (``cuda.cycle_payload``)."""
        from uno_b200.ops import cuda

        stops = () if sp.ignore_eos else tuple([self.eos_token_id] + [int(t) for t in sp.stop_token_ids or []])
        return cuda.cycle_payload(proposal, lookahead, stops, **kw)

    def _argmax(self, logits):
        shape = logits.shape
        rows = logits if logits.is_cuda else logits.reshape(-1, shape[-1])
        return self.sampler.argmax(rows).view(shape[:-1])

    def build_payload(self, proposal, accepted, corr, lookahead, sp: SamplingParams):
        """``[B, L+2]`` int64: committed tokens (L+1 slots) then the length."""
        B, L = proposal.shape
        dev = proposal.device
        payload = torch.empty((B, L + 2), dtype=torch.int64, device=dev)
        committed = payload[:, : L + 1]
        committed[:, :L] = proposal
        committed[:, L] = lookahead.to(torch.int64)
        if L > 1:
            reject = ~accepted
            rejected = reject.any(dim=1)
            first = torch.argmax(reject.to(torch.int64), dim=1)
            cols = (first + 1)[:, None]
            repl = corr.to(torch.int64).gather(1, first[:, None])
            committed.scatter_(1, cols, torch.where(rejected[:, None], repl, committed.gather(1, cols)))
            lengths = torch.where(rejected, first + 2, torch.full_like(first, L + 1))
        else:
            lengths = torch.full((B,), L + 1, dtype=torch.int64, device=dev)
        payload[:, -1] = self.truncate_at_stop(committed, lengths, sp)
        return payload

    def truncate_at_stop(self, committed, lengths, sp: SamplingParams):
        if sp.ignore_eos:
            return lengths
        pos = torch.arange(committed.shape[1], device=committed.device)[None, :]
        valid = pos < lengths[:, None]
        stop = committed.eq(self.eos_token_id)
        for t in sp.stop_token_ids or []:
            stop |= committed.eq(int(t))
        stop &= valid
        hit = stop.any(dim=1)
        first = torch.argmax(stop.to(torch.int64), dim=1)
        return torch.where(hit, first + 1, lengths)

    # ------------------------------------------------------------------- tree
    def tree_verify_stage(self, seqs, root_tokens, draft_logits, L: int, sp: SamplingParams):
        B = len(seqs)
        Q = int(self.tree_verify_size)
        sharded = self.sampler.vocab_size(draft_logits) != draft_logits.shape[-1]
        shard = self.sampler.shard if sharded else None
        tree = build_draft_tree_batch(root_tokens, draft_logits, max_nodes=Q,
                                      candidate_top_k=self.tree_candidate_top_k,
                                      temperature=sp.temperature, shard=shard)
        logits = self.run_tree(seqs, tree.token_ids, tree.depths, tree.parent_indices)  # [B, Q, V]
        targets, _ = self.sampler.sample(logits.reshape(-1, logits.shape[-1]), sp)
        targets = targets.view(B, Q)
        committed, accepted_nodes, lengths = walk_tree(
            tree.token_ids, tree.parent_indices, targets, max_depth=L - 1, pad_token_id=self.pad_token_id)
        lengths = self.truncate_at_stop(committed, lengths, sp)
        cache_lengths = (lengths - 1).clamp(min=0, max=L)
        self.compact_tree_kv(seqs, accepted_nodes, cache_lengths, Q)
        payload = torch.empty((B, committed.shape[1] + 1), dtype=torch.int64, device=committed.device)
        payload[:, :-1] = committed
        payload[:, -1] = lengths
        return payload
