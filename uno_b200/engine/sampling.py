"""Token sampling and Psi-Spec verification primitives.

Semantics follow ``nano_vllm_uno/layers/sampler.py:14-133`` and
``nano_vllm_uno/engine/two_pass_decoding.py:56-97, 711-817``:

* greedy: argmax;
* unfiltered stochastic: categorical sample of ``softmax(logits / T)`` by the
  Gumbel-max trick;
* top-k (optionally followed by nucleus) and exact top-p: sparse renormalised
  distributions ``(ids, probs)``; the draft's sparse ``q`` is kept so the
  verifier can compute ``p(s)/q(s)`` on the same support;
* verify (speculative sampling, Leviathan et al. 2023 / Chen et al. 2023):
  accept draft token ``s`` with probability ``min(1, p(s)/q(s))``; on reject,
  resample from ``norm(max(p - q, 0))``.  Every committed token is therefore an
  exact sample of the target model (lossless).

On CUDA the hot variants (full-vocab Gumbel sampling, argmax, fused verify)
run the framework's Philox-keyed kernels; on CPU they run here with a torch
generator.  Randomness is keyed by ``(seed, counter)`` so every TP rank that
runs the same call draws the same numbers without a broadcast.

Filtered distributions on CUDA (bf16 logits) never leave the device as a
candidate list: ``cuda.filtered_sample`` selects the top-k / nucleus set of
each row exactly (radix select over the row) and keeps, per row, the key of
the last kept token with the row max and kept mass (:class:`FilteredRows`);
``cuda.filtered_verify`` recomputes the target's set and evaluates p and q
from those numbers and the two logits rows.  Elsewhere the sparse ``(ids,
probs)`` form below is used.

Vocab-parallel mode (tensor parallelism with the fused NVLink collectives):
the lm_head leaves each rank a ``[rows, V/tp]`` logits shard and
:class:`VocabShard` tells the sampler where it sits.  Greedy, unfiltered
sampling and the unfiltered verify then run the vocab-parallel kernels, which
exchange a few numbers per row between ranks instead of the logits; the
Philox noise is keyed by global token id, so the tokens equal those of the
same logits on one GPU.  Top-k / top-p merge each rank's best candidates
(``engine/vp_filtered.py``: exact, with the logits gathered only for a batch
the candidates cannot decide); the draft tree merges per-shard top-K
candidates (``draft_tree.shard_candidate_log_probs``).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch

from uno_b200.sampling_params import SamplingParams
from uno_b200.utils.trace import nvtx


@dataclass
class FilteredRows:
    """A filtered draft distribution on CUDA: the logits rows it was sampled
    from and the per-row ``(last-kept key, max, kept mass)`` params."""

    rows: torch.Tensor
    params: torch.Tensor


def filter_args(sp: SamplingParams, vocab: int) -> tuple[int, float]:
    """``(top_k, top_p)`` of a filtered request; 0 and 1.0 switch a filter off."""
    k = int(sp.top_k) if sp.uses_top_k(vocab) else 0
    if not k and sp.top_k is not None and sp.uses_top_p():
        raise ValueError("top_k must be smaller than the model vocabulary")
    return k, float(sp.top_p) if sp.uses_top_p() else 1.0


def native_filtered(logits: torch.Tensor) -> bool:
    """bf16 logits rows the filtered kernels can read in place."""
    if not logits.is_cuda or logits.dtype != torch.bfloat16 or logits.dim() not in (2, 3):
        return False
    if logits.stride(-1) != 1 or logits.shape[-1] % 8 or logits.shape[-1] >= 1 << 18 or logits.data_ptr() % 16:
        return False
    return all(st % 8 == 0 for st in logits.stride()[:-1])


@dataclass
class VocabShard:
    """This rank's slice ``[start, start + logits.shape[-1])`` of a ``vocab``-sized vocabulary."""

    start: int
    vocab: int
    gather: Callable[[torch.Tensor], torch.Tensor]  # shard -> full logits (all-gather over the last dim)


class Sampler:
    """Stateful sampler: one RNG stream (seed, counter) shared by all ranks."""

    def __init__(self, seed: int = 0, shard: VocabShard | None = None):
        self.seed = int(seed) & 0xFFFFFFFF
        self.counter = 0
        self._gen: torch.Generator | None = None
        self.shard = shard

    def _sharded(self, logits: torch.Tensor) -> bool:
        return self.shard is not None and logits.shape[-1] != self.shard.vocab

    def full(self, logits: torch.Tensor) -> torch.Tensor:
        """Full-vocabulary logits (gathers a vocab-parallel shard)."""
        return self.shard.gather(logits) if self._sharded(logits) else logits

    def vocab_size(self, logits: torch.Tensor) -> int:
        return self.shard.vocab if self._sharded(logits) else logits.shape[-1]

    def argmax(self, logits: torch.Tensor) -> torch.Tensor:
        if self._sharded(logits):
            from uno_b200.ops import cuda

            return cuda.vp_sample(logits, 1.0, self.seed, 0, self.shard.start, greedy=True)
        return argmax(logits)

    def reseed(self, seed: int) -> None:
        self.seed = int(seed) & 0xFFFFFFFF
        self.counter = 0
        self._gen = None

    def _next(self) -> int:
        self.counter += 1
        return self.counter

    def _cpu_gen(self) -> torch.Generator:
        if self._gen is None:
            self._gen = torch.Generator()
            self._gen.manual_seed(self.seed)
        return self._gen

    # ---------------------------------------------------------------- sampling
    def sample(self, logits: torch.Tensor, sp: SamplingParams):
        """Return ``(tokens [N] int64, sparse_q or None)``."""
        with nvtx("sample"):
            return self._sample(logits, sp)

    def _sample(self, logits: torch.Tensor, sp: SamplingParams):
        V = self.vocab_size(logits)
        if sp.greedy:
            return self.argmax(logits), None
        if self._sharded(logits):
            if not sp.filtered(V):
                return self.sample_full(logits, sp.temperature), None
            from uno_b200.engine import vp_filtered

            k, p = filter_args(sp, V)
            key = self._next()
            return vp_filtered.sample(logits.reshape(-1, logits.shape[-1]), k, p, sp.temperature, self.shard.start,
                                      self.shard.gather, self.seed, key)
        if sp.filtered(V):
            k, p = filter_args(sp, V)
            if native_filtered(logits):
                from uno_b200.ops import cuda

                key = self._next()
                tokens, params = cuda.filtered_sample(logits, 1.0 / sp.temperature, k, p, self.seed, key)
                return tokens, FilteredRows(logits, params)
            rows = logits.reshape(-1, V)
            if k:
                ids, probs = sparse_top_k(rows, sp.temperature, k, sp.top_p)
            else:
                ids, probs = sparse_top_p(rows, sp.temperature, p)
            off = self.sample_probs(probs)
            return ids.gather(1, off[:, None]).view(-1), (ids, probs)
        return self.sample_full(logits, sp.temperature), None

    def sample_full(self, logits: torch.Tensor, temperature: float) -> torch.Tensor:
        key = self._next()
        if logits.is_cuda:
            from uno_b200.ops import cuda

            if self._sharded(logits):
                return cuda.vp_sample(logits, 1.0 / temperature, self.seed, key, self.shard.start)
            return cuda.sample_gumbel(logits, 1.0 / temperature, self.seed, key)
        probs = torch.softmax(logits.float() / temperature, dim=-1)
        return self.sample_probs(probs)

    def sample_probs(self, probs: torch.Tensor) -> torch.Tensor:
        """Gumbel-max over explicit probabilities: argmax(p / Exp(1))."""
        self._next()
        if probs.is_cuda:
            noise = torch.empty_like(probs).exponential_(1)
        else:
            noise = torch.empty_like(probs).exponential_(1, generator=self._cpu_gen())
        return probs.div(noise.clamp_min_(1e-10)).argmax(dim=-1)

    def uniform(self, n: int, device) -> torch.Tensor:
        self._next()
        if torch.device(device).type == "cuda":
            return torch.rand(n, device=device)
        return torch.rand(n, generator=self._cpu_gen()).to(device)

    # ----------------------------------------------------------- verification
    def verify_unfiltered(self, clean_logits: torch.Tensor, draft_logits: torch.Tensor,
                          spec: torch.Tensor, temperature: float):
        """Fused p/q accept test + residual resample on raw logits rows."""
        key = self._next()
        if clean_logits.is_cuda:
            from uno_b200.ops import cuda

            if self._sharded(clean_logits):
                return cuda.vp_verify(clean_logits, draft_logits, spec, 1.0 / temperature, self.seed, key,
                                      self.shard.start)
            return cuda.fused_verify(clean_logits, draft_logits, spec, 1.0 / temperature, self.seed, key)
        return verify_reference(clean_logits, draft_logits, spec, temperature, self._cpu_gen())

    def verify_filtered(self, clean_logits: torch.Tensor, spec: torch.Tensor, sp: SamplingParams,
                        draft_distribution):
        if self._sharded(clean_logits) and not isinstance(draft_distribution, FilteredRows):
            from uno_b200.engine import vp_filtered

            k, p = filter_args(sp, self.shard.vocab)
            key = self._next()
            return vp_filtered.verify(clean_logits.reshape(-1, clean_logits.shape[-1]), spec, draft_distribution, k, p,
                                      sp.temperature, self.shard.start, self.shard.gather, self.seed, key)
        clean_logits = self.full(clean_logits)
        V = clean_logits.shape[-1]
        if isinstance(draft_distribution, FilteredRows):
            from uno_b200.ops import cuda

            if not native_filtered(clean_logits):
                raise RuntimeError("the draft was sampled by the filtered kernel; the target rows must be too")
            k, p = filter_args(sp, V)
            key = self._next()
            return cuda.filtered_verify(clean_logits, draft_distribution.rows, draft_distribution.params, spec,
                                        1.0 / sp.temperature, k, p, self.seed, key)
        clean_logits = clean_logits.reshape(-1, V)
        if sp.top_k is None:
            clean_ids, clean_probs = sparse_top_p(clean_logits, sp.temperature, float(sp.top_p))
            dense_vocab = V
        else:
            clean_ids, clean_probs = sparse_top_k(clean_logits, sp.temperature, int(sp.top_k), sp.top_p)
            dense_vocab = None
        draft_ids, draft_probs = draft_distribution
        u = self.uniform(clean_probs.shape[0], clean_probs.device)
        accepted, corr_probs = sparse_verify_tensors(clean_ids, clean_probs, draft_ids, draft_probs,
                                                     spec, u, dense_vocab)
        off = self.sample_probs(corr_probs)
        return accepted, clean_ids.gather(1, off[:, None]).view(-1)


# --------------------------------------------------------------------------
def argmax(logits: torch.Tensor) -> torch.Tensor:
    if logits.is_cuda:
        from uno_b200.ops import cuda

        return cuda.argmax(logits)
    return logits.argmax(dim=-1)


def ranked_top(logits: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """The ``k`` largest logits per row with their ids, value descending.  On the CPU equal
    values keep the lowest id first (a stable sort), the ranking of the CUDA filtered kernels."""
    if logits.is_cuda:
        return torch.topk(logits, k=int(k), dim=-1, sorted=True)
    values, ids = torch.sort(logits, dim=-1, descending=True, stable=True)
    return values[..., : int(k)], ids[..., : int(k)]


def sparse_top_k(logits: torch.Tensor, temperature: float, k: int, top_p: float | None):
    if (logits.is_cuda and logits.dtype == torch.bfloat16 and logits.dim() == 2 and int(k) <= 32
            and logits.is_contiguous()):
        # one kernel pass per row: top-k ids with their log-softmax values (sorted, lowest id on ties)
        from uno_b200.ops.cuda import ext

        n = logits.shape[0]
        ids = torch.empty(n, int(k), device=logits.device, dtype=torch.int64)
        lp = torch.empty(n, int(k), device=logits.device, dtype=torch.float32)
        ext().topk_lse(logits, int(k), 1.0 / float(temperature), ids, lp)
        probs = torch.softmax(lp, dim=-1)  # renormalised over the k candidates
    else:
        values, ids = ranked_top(logits, int(k))
        probs = torch.softmax(values.float() / float(temperature), dim=-1)
    if top_p is not None and float(top_p) < 1.0:
        cdf = probs.cumsum(dim=-1)
        probs = probs.masked_fill((cdf - probs) > float(top_p), 0.0)
        probs = probs / probs.sum(dim=-1, keepdim=True).clamp_min(1e-12)
    return ids, probs


def sparse_top_p(logits: torch.Tensor, temperature: float, top_p: float, initial_k: int = 256):
    """Exact nucleus on an adaptively grown candidate set (doubling until the
    retained mass reaches ``top_p`` for every row)."""
    V = logits.shape[-1]
    log_z = torch.logsumexp(logits.float() / float(temperature), dim=-1, keepdim=True)
    k = min(int(initial_k), V)
    ranked = None if logits.is_cuda else ranked_top(logits, V)  # CPU: one stable sort serves every k
    while True:
        values, ids = ranked_top(logits, k) if ranked is None else (ranked[0][..., :k], ranked[1][..., :k])
        probs = torch.exp(values.float() / float(temperature) - log_z)
        if k == V or bool((probs.sum(dim=-1) >= float(top_p)).all()):
            break
        k = min(2 * k, V)
    cdf = probs.cumsum(dim=-1)
    probs = probs.masked_fill((cdf - probs) > float(top_p), 0.0)
    probs = probs / probs.sum(dim=-1, keepdim=True).clamp_min(1e-12)
    return ids, probs


def sparse_verify_tensors(clean_ids, clean_probs, draft_ids, draft_probs, spec, u, dense_vocab):
    """Accept flags and correction distribution on the target's sparse support."""
    p_s = torch.where(clean_ids.eq(spec[:, None]), clean_probs, 0.0).sum(dim=1)
    q_s = torch.where(draft_ids.eq(spec[:, None]), draft_probs, 0.0).sum(dim=1)
    ratio = torch.where(q_s > 0, p_s / q_s.clamp_min(1e-30), torch.zeros_like(p_s))
    accepted = u.lt(ratio.clamp(max=1.0))
    if dense_vocab is None:
        q_on_clean = torch.where(clean_ids[:, :, None].eq(draft_ids[:, None, :]),
                                 draft_probs[:, None, :], 0.0).sum(dim=2)
    else:
        q_dense = draft_probs.new_zeros((draft_probs.shape[0], dense_vocab))
        q_dense.scatter_add_(1, draft_ids, draft_probs)
        q_on_clean = q_dense.gather(1, clean_ids)
    corr = (clean_probs - q_on_clean).clamp_min(0.0)
    total = corr.sum(dim=1, keepdim=True)
    corr = torch.where(total > 0, corr / total.clamp_min(1e-12), clean_probs)
    return accepted, corr


def verify_reference(clean_logits, draft_logits, spec, temperature, gen: torch.Generator | None = None):
    """fp32 oracle of the fused verify kernel (``engine/fused_verify_kernel.py:8-98``)."""
    p = torch.softmax(clean_logits.float() / temperature, dim=-1)
    q = torch.softmax(draft_logits.float() / temperature, dim=-1)
    idx = spec.long()[:, None]
    ps, qs = p.gather(1, idx).squeeze(1), q.gather(1, idx).squeeze(1)
    ratio = torch.where(qs > 0, ps / qs.clamp_min(1e-30), torch.zeros_like(ps))
    u = torch.rand(ps.shape[0], generator=gen).to(ps.device)
    accepted = (ratio >= 1.0) | (u < ratio)
    resid = (p - q).clamp_min(0.0)
    noise = torch.empty_like(resid).exponential_(1, generator=gen).clamp_min(1e-10)
    corr = resid.div(noise).argmax(dim=-1)
    # If p == q exactly the residual is empty; sample from p instead.
    empty = resid.sum(dim=-1) <= 0
    if bool(empty.any()):
        corr = torch.where(empty, p.div(noise).argmax(dim=-1), corr)
    corr = torch.where(accepted, torch.zeros_like(corr), corr)
    return accepted.to(torch.int32), corr
