"""Psi-Spec is lossless: committed tokens are distributed exactly as AR samples.

Unit level: the speculative accept/resample rule turns draft samples ``s ~ q``
into samples of the target ``p`` (unfiltered, top-k and top-p variants), and
the tree walk emits target samples.  Engine level (BASELINE config 1 model):
Psi-Spec with block 4 and plain AR decoding produce the same distribution of
completion prefixes (two-sample chi-square).
"""

import numpy as np
import pytest
import torch

from uno_b200.engine.draft_tree import walk_tree
from uno_b200.engine.sampling import Sampler, verify_reference
from uno_b200.sampling_params import SamplingParams


def chi2_stat(counts, probs):
    counts = np.asarray(counts, dtype=np.float64)
    probs = np.asarray(probs, dtype=np.float64)
    n = counts.sum()
    keep = probs * n >= 5
    exp = probs[keep] * n
    stat = ((counts[keep] - exp) ** 2 / exp).sum()
    # pool the sparse tail into one bin
    tail_o, tail_e = counts[~keep].sum(), probs[~keep].sum() * n
    if tail_e > 0:
        stat += (tail_o - tail_e) ** 2 / tail_e
    dof = int(keep.sum())
    return stat, dof


def chi2_threshold(dof):
    # generous bound (~p < 1e-4): mean dof, sd sqrt(2 dof)
    return dof + 6 * np.sqrt(2 * dof) + 10


def test_verify_reference_is_lossless():
    g = torch.Generator().manual_seed(0)
    V, n = 40, 40000
    p_log = torch.randn(V, generator=g) * 1.5
    q_log = torch.randn(V, generator=g) * 1.5
    q = torch.softmax(q_log, -1)
    spec = torch.multinomial(q, n, replacement=True, generator=g)
    acc, corr = verify_reference(p_log.repeat(n, 1), q_log.repeat(n, 1), spec, 1.0, g)
    out = torch.where(acc.bool(), spec, corr)
    counts = torch.bincount(out, minlength=V).numpy()
    stat, dof = chi2_stat(counts, torch.softmax(p_log, -1).numpy())
    assert stat < chi2_threshold(dof), (stat, dof)


@pytest.mark.parametrize("top_k,top_p", [(8, None), (None, 0.8), (12, 0.9)])
def test_filtered_verify_is_lossless(top_k, top_p):
    torch.manual_seed(1)
    V, n = 32, 30000
    sp = SamplingParams(temperature=0.9, top_k=top_k, top_p=top_p)
    p_log = torch.randn(1, V) * 2
    q_log = torch.randn(1, V) * 2
    sampler = Sampler(5)
    spec, q_sparse = sampler.sample(q_log.repeat(n, 1), sp)
    acc, corr = sampler.verify_filtered(p_log.repeat(n, 1), spec, sp, q_sparse)
    out = torch.where(acc, spec, corr)
    # target distribution: the filtered p
    ref_tokens, _ = Sampler(9).sample(p_log.repeat(n, 1), sp)
    c1 = torch.bincount(out, minlength=V).double()
    c2 = torch.bincount(ref_tokens, minlength=V).double()
    keep = (c1 + c2) >= 20
    stat = (((c1 - c2) ** 2) / (c1 + c2).clamp_min(1))[keep].sum().item()
    dof = int(keep.sum())
    assert stat < chi2_threshold(dof), (stat, dof)


def test_tree_walk_emits_target_samples():
    """With context-free targets the walk's first two tokens are iid ~ p."""
    g = torch.Generator().manual_seed(3)
    V, Q, n = 6, 7, 20000
    p = torch.tensor([0.3, 0.25, 0.2, 0.1, 0.1, 0.05])
    tokens = torch.tensor([[0, 1, 2, 3, 1, 2, 0]]).repeat(n, 1)
    parents = torch.tensor([[-1, 0, 0, 0, 1, 1, 2]]).repeat(n, 1)
    targets = torch.multinomial(p, n * Q, replacement=True, generator=g).view(n, Q)
    committed, _, lengths = walk_tree(tokens, parents, targets, max_depth=2, pad_token_id=0)
    for col in (1, 2):
        rows = lengths > col  # position col was emitted
        counts = torch.bincount(committed[rows, col], minlength=V).numpy()
        stat, dof = chi2_stat(counts, p.numpy())
        assert stat < chi2_threshold(dof), (col, stat)
    assert (lengths >= 2).all()


def _completion_prefixes(llm, prompt, sp, reps, batch, k):
    import dataclasses

    out = []
    for rep in range(reps):
        # a seeded SamplingParams restarts the RNG streams: use a fresh seed per call
        sp_rep = dataclasses.replace(sp, seed=sp.seed * 1000 + rep)
        res = llm.generate([prompt] * batch, sp_rep, use_tqdm=False, detokenize=False)
        out.extend(tuple(r["token_ids"][:k]) for r in res)
    return out


@pytest.mark.slow
def test_engine_psi_spec_matches_ar_in_law():
    """Config-1 model: completion prefixes of Psi-Spec (block 4) vs AR decoding."""
    from uno_b200 import LLM

    llm = LLM("preset:tiny-qwen3", device="cpu", max_num_seqs=64, max_model_len=128,
              kvcache_block_size=64, dummy_lora_rank=8, dummy_lora_alpha=16, max_diffusion_block_size=4)
    # Sharpen the output distribution so a few thousand samples cover it.
    llm.model_runner.model.lm_head.weight.data.mul_(40.0)
    prompt = [5, 17, 300, 42, 7, 99, 1000, 3]
    k = 4
    spec_sp = SamplingParams(temperature=1.0, max_tokens=k, diffusion_block_size=4, mask_token_id=4095,
                             ignore_eos=True, seed=11)
    ar_sp = SamplingParams(temperature=1.0, max_tokens=k, diffusion_block_size=1, mask_token_id=4095,
                           ignore_eos=True, seed=12)
    a = _completion_prefixes(llm, prompt, spec_sp, 24, 64, k)
    b = _completion_prefixes(llm, prompt, ar_sp, 24, 64, k)
    llm.exit()
    # compare per-position marginals and the (t1, t2, t3) joint
    for key in [lambda t: t[1], lambda t: t[2], lambda t: t[3], lambda t: t[1:4]]:
        ca, cb = {}, {}
        for t in a:
            ca[key(t)] = ca.get(key(t), 0) + 1
        for t in b:
            cb[key(t)] = cb.get(key(t), 0) + 1
        bins = [x for x in set(ca) | set(cb) if ca.get(x, 0) + cb.get(x, 0) >= 20]
        if len(bins) < 2:
            continue
        stat = sum((ca.get(x, 0) - cb.get(x, 0)) ** 2 / (ca.get(x, 0) + cb.get(x, 0)) for x in bins)
        assert stat < chi2_threshold(len(bins)), (stat, len(bins))
    # Psi-Spec must actually accept drafts (TPF > AR's 1 token per forward)
    assert llm.last_generate_stats  # populated


def test_cpu_filtered_ranking_keeps_lowest_ids_on_ties():
    """The sparse CPU path ranks equal logits lowest id first, as the CUDA filtered kernels do."""
    from uno_b200.engine.sampling import sparse_top_k, sparse_top_p

    logits = torch.zeros(1, 64)
    logits[0, 40] = 3.0
    ids, probs = sparse_top_k(logits, 1.0, 5, None)
    assert ids[0].tolist() == [40, 0, 1, 2, 3]
    ids, probs = sparse_top_p(logits, 1.0, 0.5)
    kept = ids[0][probs[0] > 0].tolist()
    assert kept[0] == 40 and kept[1:] == list(range(len(kept) - 1))
