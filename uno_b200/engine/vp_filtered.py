"""Top-k / top-p sampling and verification on vocabulary-parallel logits, without gathering them.

Under tensor parallelism each rank holds the logits of its vocabulary slice.
The reference gathers the full rows to rank 0 before filtering
(``nano_vllm_uno/layers/embed_head.py:62-65``, ``layers/sampler.py:21-90``,
``engine/two_pass_decoding.py:56-97``).  Here every rank sends only what a
filter can keep:

1. each rank ranks its shard (value descending, lowest id first on ties) and
   keeps its best ``C`` logits, and its shard's log-normaliser at the
   temperature;
2. one all-gather moves ``C`` ids, ``C`` scaled logits and the normaliser per
   row and rank (``tp * (2C + 1)`` float64s a row, against ``V`` bf16 logits);
3. every rank merges the same ``tp * C`` candidates into global log-probs
   (scaled logit minus the logsumexp of the shard normalisers), orders them
   like a full-vocabulary sort, and applies the request's top-k and nucleus
   exactly as ``engine/sampling.py`` ``sparse_top_k`` / ``sparse_top_p`` do on
   full rows.

The merged set decides a row exactly when the last candidate the filter needs
lies strictly above every rank's ``C``-th logit (the *floor*): every token
above the floor is a candidate, so the sorted prefix the filter reads is the
full vocabulary's.  A batch with a row that fails this (a nucleus wider than
the candidates, or a tie across the floor) asks again with four times the
candidates while they stay smaller than the logits, then gathers the logits;
the check is the one host read of each exchange.

Draws are counter-based (a splitmix64 hash of seed, call, stream, row and
global token id), so every rank takes the same decisions from the same merged
candidates without exchanging them.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

# Candidates a rank contributes to a nucleus-only request; a top-k request sends max(k, TOP_K_MIN).
TOP_P_CANDIDATES = 256
TOP_K_MIN = 64

_GOLDEN = 0x9E3779B97F4A7C15
_ROW = 0xD1B54A32D192ED03
_COL = 0xABC98388FB8FAC03


def _i64(v: int) -> int:
    v &= (1 << 64) - 1
    return v - (1 << 64) if v >= 1 << 63 else v


def _srl(x: torch.Tensor, s: int) -> torch.Tensor:
    """Logical right shift of int64 lanes."""
    return (x >> s) & ((1 << (64 - s)) - 1)


def _mix(x: torch.Tensor) -> torch.Tensor:
    """splitmix64 finaliser (Steele, Lea & Flood 2014) on wrapping int64 lanes."""
    x = (x ^ _srl(x, 30)) * _i64(0xBF58476D1CE4E5B9)
    x = (x ^ _srl(x, 27)) * _i64(0x94D049BB133111EB)
    return x ^ _srl(x, 31)


def _mix_int(v: int) -> int:
    v &= (1 << 64) - 1
    v = ((v ^ (v >> 30)) * 0xBF58476D1CE4E5B9) & ((1 << 64) - 1)
    v = ((v ^ (v >> 27)) * 0x94D049BB133111EB) & ((1 << 64) - 1)
    return v ^ (v >> 31)


def counter_uniform(seed: int, key: int, stream: int, rows: torch.Tensor, cols: torch.Tensor) -> torch.Tensor:
    """Uniform float64 draws in (0, 1), one per (row, col) lane, from (seed, key, stream)."""
    base = _mix_int(_mix_int((int(seed) & 0xFFFFFFFF) * _GOLDEN + int(key)) + int(stream) * _GOLDEN)
    h = _mix(rows.long() * _i64(_ROW) + cols.long() * _i64(_COL) + _i64(base))
    return (_srl(h, 11).double() + 0.5) * (2.0 ** -53)


def _draw(probs: torch.Tensor, ids: torch.Tensor, seed: int, key: int, stream: int) -> torch.Tensor:
    """Gumbel-max over explicit probabilities: the column maximising p / Exp(1), the
    exponential keyed by the row and the candidate's global id."""
    rows = torch.arange(probs.shape[0], device=probs.device)[:, None].expand_as(ids)
    e = -torch.log(counter_uniform(seed, key, stream, rows, ids))
    return (probs.double() / e).argmax(dim=1)


@dataclass
class Candidates:
    """Merged candidates of every rank, ordered like a full-vocabulary sort."""

    ids: torch.Tensor    # [N, W] int64 global ids
    logp: torch.Tensor   # [N, W] float64 global log-probs at the temperature
    floor: torch.Tensor  # [N] float64: the highest rank-local C-th log-prob (-inf when a shard fits whole)


def shard_candidates(rows: torch.Tensor, count: int, inv_t: float, vocab_start: int, gather) -> Candidates:
    """Each rank's best ``count`` logits of its shard ``rows [N, Vs]``, exchanged with ``gather``
    (an all-gather over the last dimension of the tensor-parallel group) and merged."""
    N, Vs = rows.shape
    C = min(int(count), Vs)
    from uno_b200.engine.sampling import ranked_top

    if C == Vs:  # the whole shard: one stable sort
        vals, ids = torch.sort(rows, dim=1, descending=True, stable=True)
    else:
        vals, ids = ranked_top(rows, C)
    scaled = vals.double() * float(inv_t)
    # the shard's log-normaliser in fp32 (one pass over the shard; the merge runs in fp64)
    lse = torch.logsumexp(rows.float() * float(inv_t), dim=1, keepdim=True).double()
    packed = torch.cat([(ids + int(vocab_start)).double(), scaled, lse], dim=1)
    everyone = gather(packed)
    tp = everyone.shape[1] // (2 * C + 1)
    everyone = everyone.view(N, tp, 2 * C + 1)
    g_lse = torch.logsumexp(everyone[..., 2 * C], dim=1, keepdim=True)
    g_ids = everyone[..., :C].round().long().reshape(N, tp * C)
    logp = (everyone[..., C:2 * C] - g_lse[..., None]).reshape(N, tp * C)
    if C < Vs:
        floor = (everyone[..., 2 * C - 1] - g_lse).amax(dim=1)
    else:
        floor = torch.full((N,), -math.inf, dtype=torch.float64, device=rows.device)
    order = torch.argsort(g_ids, dim=1, stable=True)
    g_ids, logp = g_ids.gather(1, order), logp.gather(1, order)
    order = torch.argsort(logp, dim=1, descending=True, stable=True)
    return Candidates(g_ids.gather(1, order), logp.gather(1, order), floor)


def filtered_support(c: Candidates, top_k: int, top_p: float):
    """``(ids, probs, exact, kept)`` of the filter on the merged candidates: the support with the
    renormalised kept probabilities (zero outside the filter), whether each row is decided
    exactly, and the number of kept tokens per row."""
    W = c.ids.shape[1]
    if top_k:
        k = min(int(top_k), W)
        ids, logp = c.ids[:, :k], c.logp[:, :k]
        probs = torch.softmax(logp, dim=1)
        edge = logp[:, k - 1]  # the renormalisation reads the whole top-k
    else:
        ids, logp = c.ids, c.logp
        probs = torch.exp(logp)
    if top_p < 1.0:
        cdf = probs.cumsum(dim=1)
        keep = (cdf - probs) <= float(top_p)
        probs = probs.masked_fill(~keep, 0.0)
        if not top_k:
            last = keep.sum(dim=1).clamp_min(1) - 1
            edge = logp.gather(1, last[:, None]).squeeze(1)
            reached = cdf.gather(1, last[:, None]).squeeze(1) > float(top_p)
            edge = torch.where(reached, edge, torch.full_like(edge, -math.inf))
    elif not top_k:
        edge = torch.full((ids.shape[0],), -math.inf, dtype=torch.float64, device=ids.device)
    probs = probs / probs.sum(dim=1, keepdim=True).clamp_min(1e-300)
    exact = torch.isneginf(c.floor) | (edge > c.floor)
    return ids, probs, exact, (probs > 0).sum(dim=1)


def _supports(rows: torch.Tensor, top_k: int, top_p: float, inv_t: float, vocab_start: int, gather):
    """Kept ``(ids, probs)`` of every row, trimmed to the widest row's kept count.  A batch the
    candidates do not decide retries with four times the candidates while they stay smaller
    than the logits, then gathers the logits and sorts the full rows."""
    N, Vs = rows.shape
    count = max(int(top_k), TOP_K_MIN) if top_k else TOP_P_CANDIDATES
    while True:
        c = shard_candidates(rows, count, inv_t, vocab_start, gather)
        ids, probs, exact, kept = filtered_support(c, top_k, top_p)
        ok, width = torch.stack([exact.all().long(), kept.max()]).tolist()
        if ok:
            break
        count *= 4
        if count >= Vs or (2 * count + 1) * 8 > Vs * rows.element_size():
            full = gather(rows)
            c = shard_candidates(full, full.shape[1], inv_t, 0, lambda x: x)
            ids, probs, _, kept = filtered_support(c, top_k, top_p)
            width = int(kept.max())
            break
    order = torch.argsort(probs, dim=1, descending=True, stable=True)[:, :max(int(width), 1)]
    return ids.gather(1, order), probs.gather(1, order)


def sample(rows: torch.Tensor, top_k: int, top_p: float, temperature: float, vocab_start: int, gather,
           seed: int, key: int):
    """``(tokens [N], (ids, probs))`` drawn from the filtered distribution of vocabulary-parallel
    rows."""
    ids, probs = _supports(rows, top_k, top_p, 1.0 / float(temperature), vocab_start, gather)
    pick = _draw(probs, ids, seed, key, 4)
    return ids.gather(1, pick[:, None]).squeeze(1), (ids, probs)


def lookup(ids: torch.Tensor, probs: torch.Tensor, want: torch.Tensor) -> torch.Tensor:
    """Probability of each ``want[n, j]`` under the sparse row ``(ids[n], probs[n])`` (0 when absent)."""
    order = torch.argsort(ids, dim=1)
    sid, sp = ids.gather(1, order), probs.gather(1, order)
    pos = torch.searchsorted(sid, want.contiguous()).clamp_max(sid.shape[1] - 1)
    return torch.where(sid.gather(1, pos).eq(want), sp.gather(1, pos), torch.zeros((), dtype=sp.dtype,
                                                                                    device=sp.device))


def verify(rows: torch.Tensor, spec: torch.Tensor, draft: tuple[torch.Tensor, torch.Tensor], top_k: int,
           top_p: float, temperature: float, vocab_start: int, gather, seed: int, key: int):
    """Ψ-Spec accept test ``u < min(1, p(s)/q(s))`` and residual draw from ``max(p - q, 0)`` on the
    target's filtered support, with the draft's sparse ``(ids, probs)``."""
    ids, p = _supports(rows, top_k, top_p, 1.0 / float(temperature), vocab_start, gather)
    q_ids, q = draft
    spec = spec.reshape(-1, 1).long()
    p_s = lookup(ids, p, spec).squeeze(1)
    q_s = lookup(q_ids, q.double(), spec).squeeze(1)
    ratio = torch.where(q_s > 0, p_s / q_s.clamp_min(1e-300), torch.zeros_like(p_s))
    n = torch.arange(ids.shape[0], device=ids.device)
    u = counter_uniform(seed, key, 5, n, torch.zeros_like(n))
    accepted = u < ratio.clamp(max=1.0)
    resid = (p - lookup(q_ids, q.double(), ids)).clamp_min(0.0)
    total = resid.sum(dim=1, keepdim=True)
    resid = torch.where(total > 0, resid / total.clamp_min(1e-300), p)
    pick = _draw(resid, ids, seed, key, 6)
    return accepted.to(torch.int32), ids.gather(1, pick[:, None]).squeeze(1)
