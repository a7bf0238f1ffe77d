"""Filtered (top-k / top-p) sampling and sparse verification kernels (GPU only).

The kept set, row max and kept mass of ``filtered.cu`` are checked against a
float64 reference over the same ranking (value descending, lowest id first);
the sample and verify laws by chi-square tests, including the Sampler-level
lossless test of ``tests/test_lossless.py`` run on the CUDA path.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"
V_BIG = 151936


@pytest.fixture(scope="module")
def C():
    from uno_b200.ops import cuda

    cuda.ext()
    yield cuda


def _reference(C, row, inv_temp, k, p):
    """float64 kept count, normalised exclusive prefix mass and weights of one bf16 row."""
    keys = C.filtered_keys(row[None])[0].cpu()
    order = torch.argsort(keys, descending=True)
    y = (row.float().cpu() * torch.tensor(inv_temp, dtype=torch.float32)).double()[order]
    w = torch.exp(y - y.max())
    if k:
        total = w[:k].sum()
        excl = torch.cumsum(w[:k], 0) - w[:k]
        n = k if p >= 1.0 else int((excl / total <= p).sum())
        return n, excl / total, order, w
    total = w.sum()
    excl = torch.cumsum(w, 0) - w
    return int((excl / total <= p).sum()), excl / total, order, w


def _check_rows(C, x, inv_temp, k, p, tol=2e-5):
    tokens, params = C.filtered_sample(x, inv_temp, k, p, 11, 3)
    kept = C.filtered_kept(x, params)
    _, m, S = C.unpack_filtered_params(params)
    torch.cuda.synchronize()
    for r in range(x.shape[0]):
        row = x[r]
        n_ref, excl, order, w = _reference(C, row, inv_temp, k, p)
        n_got = int(kept[r].sum())
        lo, hi = sorted((n_ref, n_got))
        if lo != hi:  # only tokens whose preceding mass sits on the cut may differ
            assert k == 0 or p < 1.0, (r, n_ref, n_got)
            assert float((excl[lo:hi] - p).abs().max()) < tol, (r, n_ref, n_got)
        assert bool(kept[r, tokens[r]]), "the sample must come from the kept set"
        ids = order[:n_got]
        assert bool(kept[r].cpu()[ids].all())
        want_m = float((row.float() * torch.tensor(inv_temp, device=DEV)).max())
        assert float(m[r]) == want_m
        want_S = float(w[:n_got].sum())
        assert abs(float(S[r]) - want_S) <= 1e-5 * want_S, (r, float(S[r]), want_S)


@pytest.mark.parametrize("inv_temp,k,p", [
    (1.0, 0, 0.9), (1.0, 0, 0.95), (1.0, 0, 0.5), (1.0 / 0.6, 0, 0.95), (1.0, 1, 1.0), (1.0, 50, 1.0),
    (1.0, 1000, 1.0), (1.0, 20000, 1.0), (1.0, 50, 0.9), (1.0 / 0.7, 1000, 0.5),
])
def test_filtered_selection_matches_float64(C, inv_temp, k, p):
    torch.manual_seed(k * 7 + int(p * 100))
    x = (torch.randn(4, V_BIG, device=DEV) * 3).to(torch.bfloat16)
    _check_rows(C, x, inv_temp, k, p)


def test_filtered_selection_resolves_ties_by_id(C):
    """Nucleus through a value shared by ~150k tokens: the lowest ids are kept first."""
    x = torch.zeros(2, V_BIG, device=DEV, dtype=torch.bfloat16)
    x[:, 1000:1005] = 5.0
    x[1, 70000:70100] = 2.0
    _check_rows(C, x, 1.0, 0, 0.95)
    _check_rows(C, x, 1.0, 100000, 1.0)


def test_filtered_selection_crowded_boundary_bin(C):
    """Top-k inside a narrow band of distinct values: the boundary bin is re-binned over exact keys."""
    torch.manual_seed(5)
    x = ((torch.rand(3, V_BIG, device=DEV) - 0.5) * 0.02).to(torch.bfloat16)
    x[:, 7] = 5.0
    _check_rows(C, x, 1.0, 100000, 1.0)
    _check_rows(C, x, 1.0, 100000, 0.5)
    _check_rows(C, x, 1.0, 0, 0.3)


def test_filtered_small_vocab_and_strided_rows(C):
    torch.manual_seed(2)
    x = (torch.randn(6, 4096, device=DEV) * 2).to(torch.bfloat16)
    _check_rows(C, x, 1.0, 0, 0.9)
    _check_rows(C, x, 1.0, 64, 0.8)
    blk = (torch.randn(3, 5, 4096, device=DEV) * 2).to(torch.bfloat16)
    view = blk[:, 1:, :]  # strided [B, L-1, V] rows, read in place
    t1, p1 = C.filtered_sample(view, 1.0, 16, 0.9, 4, 9)
    t2, p2 = C.filtered_sample(view.reshape(-1, 4096).contiguous(), 1.0, 16, 0.9, 4, 9)
    assert torch.equal(p1, p2)
    assert torch.equal(t1, t2)


def _chi2(counts, probs):
    counts = np.asarray(counts, dtype=np.float64)
    probs = np.asarray(probs, dtype=np.float64)
    n = counts.sum()
    keep = probs * n >= 5
    exp = probs[keep] * n
    stat = ((counts[keep] - exp) ** 2 / exp).sum()
    tail_o, tail_e = counts[~keep].sum(), probs[~keep].sum() * n
    if tail_e > 0:
        stat += (tail_o - tail_e) ** 2 / tail_e
    dof = int(keep.sum())
    return stat, dof + 6 * np.sqrt(2 * max(dof, 1)) + 10


def _filtered_probs(C, row, inv_temp, k, p):
    n, _, order, w = _reference(C, row, inv_temp, k, p)
    probs = torch.zeros(row.shape[-1], dtype=torch.float64)
    probs[order[:n]] = w[:n] / w[:n].sum()
    return probs.numpy()


@pytest.mark.parametrize("k,p", [(0, 0.8), (40, 1.0), (40, 0.9)])
def test_filtered_sample_law(C, k, p):
    torch.manual_seed(3)
    V, R = 1024, 8192
    row = (torch.randn(V, device=DEV) * 2).to(torch.bfloat16)
    rows = row[None].expand(R, V)  # every row reads the same logits with its own noise
    counts = np.zeros(V)
    for call in range(4):
        tok, _ = C.filtered_sample(rows, 1.0, k, p, 21, 100 + call)
        counts += np.bincount(tok.cpu().numpy(), minlength=V)
    stat, bound = _chi2(counts, _filtered_probs(C, row, 1.0, k, p))
    assert stat < bound, (stat, bound)


@pytest.mark.parametrize("k,p", [(0, 0.8), (40, 1.0), (24, 0.9)])
def test_filtered_verify_law(C, k, p):
    """Draft s ~ q, then accept / resample: the committed token is distributed as the filtered p."""
    torch.manual_seed(4)
    V, R = 1024, 8192
    c_row = (torch.randn(V, device=DEV) * 2).to(torch.bfloat16)
    d_row = (c_row.float() + torch.randn(V, device=DEV)).to(torch.bfloat16)
    clean, draft = c_row[None].expand(R, V), d_row[None].expand(R, V)
    counts = np.zeros(V)
    accepted = 0
    for call in range(4):
        spec, params = C.filtered_sample(draft, 1.0, k, p, 5, 2 * call)
        acc, corr = C.filtered_verify(clean, draft, params, spec, 1.0, k, p, 5, 2 * call + 1)
        out = torch.where(acc.bool(), spec, corr)
        counts += np.bincount(out.cpu().numpy(), minlength=V)
        accepted += int(acc.sum())
    pc = _filtered_probs(C, c_row, 1.0, k, p)
    qd = _filtered_probs(C, d_row, 1.0, k, p)
    stat, bound = _chi2(counts, pc)
    assert stat < bound, (stat, bound)
    rate = accepted / (4 * R)
    want = float(np.minimum(pc, qd).sum())
    assert abs(rate - want) < 0.02, (rate, want)


@pytest.mark.parametrize("top_k,top_p", [(8, None), (None, 0.8), (12, 0.9)])
def test_sampler_filtered_verify_is_lossless_on_cuda(top_k, top_p):
    """The Sampler-level lossless test of the CPU suite, on the CUDA kernels."""
    from uno_b200.engine.sampling import FilteredRows, Sampler
    from uno_b200.sampling_params import SamplingParams

    torch.manual_seed(1)
    V, n = 32, 30000
    sp = SamplingParams(temperature=0.9, top_k=top_k, top_p=top_p)
    p_log = (torch.randn(1, V) * 2).to(DEV, torch.bfloat16)
    q_log = (torch.randn(1, V) * 2).to(DEV, torch.bfloat16)
    sampler = Sampler(5)
    spec, q_sparse = sampler.sample(q_log.repeat(n, 1), sp)
    assert isinstance(q_sparse, FilteredRows)
    acc, corr = sampler.verify_filtered(p_log.repeat(n, 1), spec, sp, q_sparse)
    out = torch.where(acc.bool(), spec, corr)
    ref_tokens, _ = Sampler(9).sample(p_log.repeat(n, 1), sp)
    c1 = torch.bincount(out, minlength=V).double().cpu()
    c2 = torch.bincount(ref_tokens, minlength=V).double().cpu()
    keep = (c1 + c2) >= 20
    stat = (((c1 - c2) ** 2) / (c1 + c2).clamp_min(1))[keep].sum().item()
    dof = int(keep.sum())
    assert stat < dof + 6 * np.sqrt(2 * dof) + 10, (stat, dof)
