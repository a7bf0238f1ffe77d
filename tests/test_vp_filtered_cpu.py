"""Top-k / top-p sampling and verification on vocabulary shards (``engine/vp_filtered.py``).

The merged candidates of the shards must give the same filtered support and
probabilities as the full-vocabulary sparse filters of ``engine/sampling.py``;
wide nuclei and ties across the candidate floor must take the retry and gather
paths and stay exact; draws must follow the filtered law and the verify must be
lossless; every gloo rank must take the same decisions.
"""

import math
import multiprocessing as mp
import socket

import pytest
import torch

from uno_b200.engine import vp_filtered as vpf
from uno_b200.engine.sampling import sparse_top_k, sparse_top_p


def _shards_gather(full: torch.Tensor, world: int, count: int, inv_t: float):
    """Merged candidates of ``world`` simulated ranks holding equal slices of ``full``."""
    Vs = full.shape[1] // world
    packs = []

    def make_gather(r):
        def gather(packed):
            packs.append(packed)
            return packed
        return gather

    for r in range(world):
        vpf.shard_candidates(full[:, r * Vs:(r + 1) * Vs], count, inv_t, r * Vs, make_gather(r))
    everyone = torch.cat(packs, dim=1)
    return vpf.shard_candidates(full[:, :Vs], count, inv_t, 0, lambda _: everyone)


def _dense(ids, probs, V):
    out = torch.zeros(ids.shape[0], V, dtype=torch.float64)
    out.scatter_add_(1, ids, probs.double())
    return out


@pytest.mark.parametrize("top_k,top_p,world", [(5, 1.0, 2), (40, 1.0, 4), (20, 0.8, 2), (0, 0.9, 2), (0, 0.5, 4)])
def test_merged_support_matches_full_vocabulary(top_k, top_p, world):
    g = torch.Generator().manual_seed(top_k * 7 + world)
    V, T = 512, 0.7
    full = (torch.randn(6, V, generator=g) * 4).to(torch.bfloat16).float()
    c = _shards_gather(full, world, max(top_k, 64) if top_k else 64, 1 / T)
    ids, probs, exact, _ = vpf.filtered_support(c, top_k, top_p)
    if top_k:
        want_ids, want_p = sparse_top_k(full, T, top_k, top_p if top_p < 1 else None)
    else:
        want_ids, want_p = sparse_top_p(full, T, top_p)
    ok = exact.tolist()
    got, want = _dense(ids, probs, V), _dense(want_ids, want_p, V)
    for r in range(full.shape[0]):
        if ok[r]:
            assert torch.allclose(got[r], want[r], atol=1e-5), r
    assert any(ok)


def test_wide_nucleus_and_floor_ties_stay_exact():
    V, T = 4096, 1.0
    flat = torch.zeros(3, V)  # every token equal: the nucleus is 90 % of the vocabulary
    flat[1, :7] = 2.0  # a tie of seven across a 4-candidate floor
    flat[2] = torch.randn(V, generator=torch.Generator().manual_seed(3)) * 0.1
    world = 2
    Vs = V // world
    for top_k, top_p in ((0, 0.9), (3, 1.0)):
        outs = []
        for r in range(world):
            calls = []

            def gather(x, r=r, calls=calls):
                calls.append(x.shape)
                parts = []
                for q in range(world):
                    parts.append(x if q == r else _peer_pack(flat, q, Vs, x, T))
                return torch.cat(parts, dim=-1)

            outs.append(vpf._supports(flat[:, r * Vs:(r + 1) * Vs], top_k, top_p, 1 / T, r * Vs, gather))
            # the candidates grow fourfold while they weigh less than the logits, then the logits are gathered
            widths = [shape[1] for shape in calls]
            assert widths[0] == 2 * (64 if top_k else 256) + 1 and widths[-1] == Vs and len(widths) >= 2
            assert all(b == 4 * (a - 1) + 1 for a, b in zip(widths[:-2], widths[1:-1]))
        ids, probs = outs[0]
        assert torch.equal(ids, outs[1][0]) and torch.equal(probs, outs[1][1])
        if top_k:
            want_ids, want_p = sparse_top_k(flat, T, top_k, None)
        else:
            want_ids, want_p = sparse_top_p(flat, T, top_p)
        assert torch.allclose(_dense(ids, probs, V), _dense(want_ids, want_p, V), atol=1e-9)


def _peer_pack(full, q, Vs, like, T):
    """What rank ``q`` sends for an exchange shaped like ``like`` (its candidates or its logits)."""
    shard = full[:, q * Vs:(q + 1) * Vs]
    if like.shape[1] == Vs:  # the logits gather
        return shard.to(like.dtype)
    C = (like.shape[1] - 1) // 2
    box = []
    vpf.shard_candidates(shard, C, 1 / T, q * Vs, lambda x: box.append(x) or x)
    return box[0]


def test_counter_uniform_is_uniform_and_keyed():
    rows = torch.arange(200)[:, None].expand(200, 500)
    cols = torch.arange(500)[None, :].expand(200, 500)
    u = vpf.counter_uniform(7, 3, 4, rows, cols)
    assert float(u.min()) > 0 and float(u.max()) < 1
    counts = torch.histc(u.float(), bins=20, min=0, max=1)
    expected = u.numel() / 20
    chi2 = float(((counts - expected) ** 2 / expected).sum())
    assert chi2 < 60  # 19 degrees of freedom
    assert torch.equal(u, vpf.counter_uniform(7, 3, 4, rows, cols))
    assert not torch.equal(u, vpf.counter_uniform(7, 4, 4, rows, cols))


def _chi2(counts: torch.Tensor, probs: torch.Tensor) -> tuple[float, int]:
    n = float(counts.sum())
    mask = probs * n >= 5
    exp = probs[mask] * n
    return float(((counts[mask] - exp) ** 2 / exp).sum()), int(mask.sum()) - 1


def test_sample_follows_filtered_law_and_verify_is_lossless():
    V, T, N = 64, 0.8, 20000
    g = torch.Generator().manual_seed(11)
    target = torch.randn(V, generator=g) * 2
    draft = target + torch.randn(V, generator=g)
    world, Vs = 2, V // 2
    ident = lambda x: x  # noqa: E731 -- one rank holding the whole vocabulary
    for top_k, top_p in ((10, 1.0), (0, 0.85), (12, 0.9)):
        rows_t, rows_d = target.expand(N, V).contiguous(), draft.expand(N, V).contiguous()
        tok, (q_ids, q) = vpf.sample(rows_d, top_k, top_p, T, 0, ident, seed=5, key=1)
        if top_k:
            w_ids, w_p = sparse_top_k(rows_d[:1], T, top_k, top_p if top_p < 1 else None)
            p_ids, p_p = sparse_top_k(rows_t[:1], T, top_k, top_p if top_p < 1 else None)
        else:
            w_ids, w_p = sparse_top_p(rows_d[:1], T, top_p)
            p_ids, p_p = sparse_top_p(rows_t[:1], T, top_p)
        law_q = _dense(w_ids, w_p, V)[0]
        chi2, dof = _chi2(torch.bincount(tok, minlength=V).double(), law_q)
        assert chi2 < dof + 6 * math.sqrt(2 * dof) + 10, (top_k, top_p, chi2, dof)
        acc, corr = vpf.verify(rows_t, tok, (q_ids, q), top_k, top_p, T, 0, ident, seed=5, key=2)
        out = torch.where(acc.bool(), tok, corr)
        law_p = _dense(p_ids, p_p, V)[0]
        chi2, dof = _chi2(torch.bincount(out, minlength=V).double(), law_p)
        assert chi2 < dof + 6 * math.sqrt(2 * dof) + 10, (top_k, top_p, chi2, dof)
    del world, Vs


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, box):
    import torch.distributed as dist

    from uno_b200.engine.sampling import Sampler, VocabShard
    from uno_b200.sampling_params import SamplingParams

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)

    def gather(x):
        parts = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(parts, x.contiguous())
        return torch.cat(parts, dim=-1)

    V = 256
    Vs = V // world
    full = torch.randn(8, 3, V, generator=torch.Generator().manual_seed(0)) * 3
    draft = full + torch.randn(8, 3, V, generator=torch.Generator().manual_seed(1))
    shard = lambda x: x[..., rank * Vs:(rank + 1) * Vs]  # noqa: E731
    out = []
    for sp in (SamplingParams(temperature=0.7, top_k=8), SamplingParams(temperature=1.0, top_p=0.9),
               SamplingParams(temperature=0.9, top_k=30, top_p=0.8)):
        s = Sampler(seed=3, shard=VocabShard(rank * Vs, V, gather))
        tok, q = s.sample(shard(draft).reshape(-1, Vs), sp)
        acc, corr = s.verify_filtered(shard(full).reshape(-1, Vs), tok, sp, q)
        # one process holding the whole vocabulary draws the same tokens (draws keyed by global id)
        k, p = (sp.top_k or 0), (sp.top_p if sp.top_p is not None else 1.0)
        tok1, q1 = vpf.sample(draft.reshape(-1, V), k, p, sp.temperature, 0, lambda x: x, 3, 1)
        acc1, corr1 = vpf.verify(full.reshape(-1, V), tok1, q1, k, p, sp.temperature, 0, lambda x: x, 3, 2)
        same = tok.tolist() == tok1.tolist() and acc.tolist() == acc1.tolist() and corr.tolist() == corr1.tolist()
        out.append((tok.tolist(), acc.tolist(), corr.tolist(), bool((tok >= 0).all() and (tok < V).all()), same))
    box.put((rank, out))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sampler_on_gloo_ranks_takes_identical_decisions(world):
    ctx = mp.get_context("spawn")
    box = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, box)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(box.get(timeout=180) for _ in range(world))
    for p in procs:
        p.join(60)
    assert all(got[r] == got[0] for r in range(world))
    assert all(case[3] and case[4] for case in got[0])
