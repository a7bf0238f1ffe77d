"""Draft trees for tree-verified Psi-Spec (CPU twins of the device kernels).

* :func:`build_tree_from_candidates` -- best-first, fixed-budget, prefix-closed
  tree over per-depth top-K draft candidates.  A candidate's priority is its
  cumulative draft log-probability; ties break by (depth, rank, token id,
  parent index), all ascending (``nano_vllm_uno/engine/draft_tree.py:51-150``).
  Nodes are emitted parent-before-child, node 0 is the root.
* :func:`walk_tree` -- follow target samples through the tree: from the root,
  the committed token at each step is the target sample at the current node;
  descend into the child carrying that token if one exists.  Every committed
  token is a target sample, so the walk is lossless
  (``nano_vllm_uno/engine/draft_tree.py:370-421``).
* :func:`tree_kv_moves` -- logical source/destination positions that compact
  the accepted path's K/V to the contiguous frontier
  (``nano_vllm_uno/engine/tree_kv_copy.py:8-96``).
"""

from __future__ import annotations

import heapq
import math
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class DraftTree:
    token_ids: tuple[int, ...]
    parent_indices: tuple[int, ...]
    depths: tuple[int, ...]
    log_masses: tuple[float, ...]

    @property
    def num_nodes(self) -> int:
        return len(self.token_ids)


@dataclass
class DraftTreeBatch:
    token_ids: torch.Tensor       # [B, Q] int64
    parent_indices: torch.Tensor  # [B, Q] int64 (root: -1)
    depths: torch.Tensor          # [B, Q] int64
    log_masses: torch.Tensor      # [B, Q] float32


def build_tree_from_candidates(root_token: int, top_tokens, top_log_probs, max_nodes: int) -> DraftTree:
    depth_count = len(top_tokens)
    if len(top_log_probs) != depth_count:
        raise ValueError("top_tokens and top_log_probs must have the same depth")
    if max_nodes < 1:
        raise ValueError("max_nodes must include at least the root")
    for d, (toks, lps) in enumerate(zip(top_tokens, top_log_probs)):
        if not toks or len(toks) != len(lps):
            raise ValueError(f"candidate row {d} must contain equally sized non-empty lists")
    tokens = [int(root_token)]
    parents = [-1]
    depths = [0]
    masses = [0.0]
    children: list[dict[int, int]] = [{}]
    heap: list[tuple[float, int, int, int, int]] = []

    def expose(node: int) -> None:
        d = depths[node]
        if d >= depth_count:
            return
        for rank, (tok, lp) in enumerate(zip(top_tokens[d], top_log_probs[d])):
            tok = int(tok)
            if tok in children[node]:
                continue
            mass = masses[node] + float(lp)
            if math.isnan(mass):
                raise ValueError("draft candidate log probabilities must not be NaN")
            heapq.heappush(heap, (-mass, d + 1, rank, tok, node))

    expose(0)
    while len(tokens) < max_nodes and heap:
        neg_mass, d, _rank, tok, parent = heapq.heappop(heap)
        if tok in children[parent]:
            continue
        idx = len(tokens)
        tokens.append(tok)
        parents.append(parent)
        depths.append(d)
        masses.append(-neg_mass)
        children.append({})
        children[parent][tok] = idx
        expose(idx)
    return DraftTree(tuple(tokens), tuple(parents), tuple(depths), tuple(masses))


def candidate_log_probs(draft_logits: torch.Tensor, k: int, temperature: float):
    """Top-K token ids and their log-softmax values per draft row ``[B, D, V]``."""
    scaled = draft_logits.float()
    if temperature > 0:
        scaled = scaled / float(temperature)
    values, ids = torch.topk(scaled, k=min(int(k), scaled.shape[-1]), dim=-1, sorted=True)
    return ids, values - torch.logsumexp(scaled, dim=-1, keepdim=True)


def shard_candidate_log_probs(shard_logits: torch.Tensor, k: int, temperature: float, vocab_start: int,
                              gather) -> tuple[torch.Tensor, torch.Tensor]:
    """:func:`candidate_log_probs` of the full vocabulary from this rank's shard ``[B, D, V/tp]``.

    Each rank takes the top-K of its shard with log-softmax values over the
    shard, recovers the shard's log-normaliser from its best candidate, and
    ``gather`` (an all-gather over the last dimension of the tensor-parallel
    group) exchanges those K ids, K values and one normaliser per row -- not the
    logits.  Every rank then merges the same ``tp * K`` candidates: global
    log-probability = shard log-probability + shard normaliser - logsumexp of
    the normalisers, and the best K of them.  The reference gathers the full
    logits to rank 0 for this (``nano_vllm_uno/layers/embed_head.py:62-65``).
    """
    B, D, Vs = shard_logits.shape
    K = min(int(k), Vs)
    rows = shard_logits.reshape(B * D, Vs)
    inv_t = 1.0 / float(temperature) if temperature > 0 else 1.0
    if rows.is_cuda and rows.dtype == torch.bfloat16 and K <= 32:
        from uno_b200.ops.cuda import ext

        rows = rows.contiguous()
        ids = torch.empty(B * D, K, device=rows.device, dtype=torch.int64)
        lp = torch.empty(B * D, K, device=rows.device, dtype=torch.float32)
        ext().topk_lse(rows, K, inv_t, ids, lp)
    else:
        ids, lp = candidate_log_probs(rows[:, None, :], K, temperature)
        ids, lp = ids[:, 0], lp[:, 0].float()
    # x_best / T - log_softmax(x_best) = the shard's log-normaliser
    lse = rows.gather(1, ids[:, :1]).float() * inv_t - lp[:, :1]
    packed = torch.cat([(ids + int(vocab_start)).double(), lp.double(), lse.double()], dim=1)
    everyone = gather(packed)
    tp = everyone.shape[1] // (2 * K + 1)
    everyone = everyone.view(B * D, tp, 2 * K + 1)
    g_ids = everyone[..., :K].round().long()
    g_lse = everyone[..., 2 * K]
    shift = (g_lse - torch.logsumexp(g_lse, dim=1, keepdim=True))[..., None]
    cand = (everyone[..., K:2 * K] + shift).reshape(B * D, tp * K)
    vals, pos = torch.topk(cand, K, dim=1, sorted=True)
    out_ids = g_ids.reshape(B * D, tp * K).gather(1, pos)
    return out_ids.view(B, D, K), vals.float().view(B, D, K)


def build_draft_tree_batch(root_tokens: torch.Tensor, draft_logits: torch.Tensor, *, max_nodes: int,
                           candidate_top_k: int, temperature: float, shard=None) -> DraftTreeBatch:
    """Best-first draft trees from ``[B, depth, V]`` draft logits.  With ``shard``
    (a vocab-parallel ``VocabShard``) the logits are this rank's vocabulary
    slice and the candidates come from :func:`shard_candidate_log_probs`."""
    if root_tokens.dim() != 1:
        raise ValueError("root_tokens must have shape [B]")
    if draft_logits.dim() != 3 or draft_logits.shape[0] != root_tokens.shape[0]:
        raise ValueError("draft_logits must have shape [B, depth, vocab]")
    if candidate_top_k < 1:
        raise ValueError("candidate_top_k must be >= 1")
    candidates = None
    if shard is not None:
        candidates = shard_candidate_log_probs(draft_logits, candidate_top_k, temperature, shard.start, shard.gather)
    if draft_logits.is_cuda:
        from uno_b200.ops import cuda

        return cuda.build_draft_tree(root_tokens, draft_logits, max_nodes, candidate_top_k, temperature,
                                     candidates=candidates)
    ids, lps = candidates if candidates is not None else candidate_log_probs(draft_logits, candidate_top_k,
                                                                             temperature)
    trees = [build_tree_from_candidates(r, t, lp, max_nodes)
             for r, t, lp in zip(root_tokens.tolist(), ids.tolist(), lps.tolist())]
    for tree in trees:
        if tree.num_nodes != max_nodes:
            raise ValueError(
                f"candidate set produced only {tree.num_nodes} tree nodes, but fixed tree "
                f"verification requires {max_nodes}; increase tree_candidate_top_k or "
                "lower tree_verify_size"
            )
    dev = root_tokens.device
    return DraftTreeBatch(
        token_ids=torch.tensor([t.token_ids for t in trees], dtype=torch.int64, device=dev),
        parent_indices=torch.tensor([t.parent_indices for t in trees], dtype=torch.int64, device=dev),
        depths=torch.tensor([t.depths for t in trees], dtype=torch.int64, device=dev),
        log_masses=torch.tensor([t.log_masses for t in trees], dtype=torch.float32, device=dev),
    )


def walk_tree(tree_tokens: torch.Tensor, parents: torch.Tensor, targets: torch.Tensor, *,
              max_depth: int, pad_token_id: int):
    """Return (committed [B, max_depth+2], accepted_nodes [B, max_depth+1], lengths [B])."""
    if tree_tokens.dim() != 2 or parents.shape != tree_tokens.shape or targets.shape != tree_tokens.shape:
        raise ValueError("tree tokens, parents, and target tokens must share [B, Q]")
    if max_depth < 0:
        raise ValueError("max_depth must be non-negative")
    if tree_tokens.is_cuda:
        from uno_b200.ops import cuda

        return cuda.walk_tree(tree_tokens, parents, targets, max_depth, pad_token_id)
    B, Q = tree_tokens.shape
    n_cached = max_depth + 1
    committed = torch.full((B, n_cached + 1), int(pad_token_id), dtype=tree_tokens.dtype)
    accepted = torch.full((B, n_cached), -1, dtype=torch.int64)
    lengths = torch.ones(B, dtype=torch.int64)
    tt, pp, tg = tree_tokens.tolist(), parents.tolist(), targets.tolist()
    for b in range(B):
        committed[b, 0] = tt[b][0]
        accepted[b, 0] = 0
        cur = 0
        for step in range(1, n_cached + 1):
            sampled = tg[b][cur]
            committed[b, step] = sampled
            lengths[b] = step + 1
            if step > max_depth:
                break
            child = next((j for j in range(Q) if pp[b][j] == cur and tt[b][j] == sampled), -1)
            if child < 0:
                break
            accepted[b, step] = child
            cur = child
    return committed, accepted, lengths


def tree_kv_moves(accepted_nodes: torch.Tensor, cache_lengths: torch.Tensor, prefix_lens: torch.Tensor):
    """Logical (src, dst) positions per request; -1 where nothing moves."""
    B, P = accepted_nodes.shape
    offs = torch.arange(P, device=accepted_nodes.device)[None, :]
    valid = offs < cache_lengths.long()[:, None]
    src = torch.where(valid, prefix_lens.long()[:, None] + accepted_nodes.long(), -1)
    dst = torch.where(valid, prefix_lens.long()[:, None] + offs, -1)
    return src, dst
