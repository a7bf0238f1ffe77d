"""Vocab-parallel draft-tree candidates on gloo ranks (CPU).

Each rank keeps a vocabulary shard of the same logits; the merged top-K
candidates must equal the single-rank top-K over the full vocabulary, with the
same log-probabilities, and every rank must hold the same result.
"""

import multiprocessing as mp
import socket


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, box):
    import torch
    import torch.distributed as dist

    from uno_b200.engine.draft_tree import candidate_log_probs, shard_candidate_log_probs

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)

    def gather(x):
        parts = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(parts, x.contiguous())
        return torch.cat(parts, dim=-1)

    out = []
    for trial, (B, D, V, K, T) in enumerate(((2, 3, 64, 4, 1.0), (3, 7, 512, 16, 0.7), (1, 2, 96, 24, 0.0))):
        g = torch.Generator().manual_seed(trial)
        full = torch.randn(B, D, V, generator=g) * 3
        Vs = V // world
        shard = full[:, :, rank * Vs:(rank + 1) * Vs]
        ids, lp = shard_candidate_log_probs(shard, K, T, rank * Vs, gather)
        want_ids, want_lp = candidate_log_probs(full, K, T)
        out.append((torch.equal(ids, want_ids), float((lp - want_lp).abs().max()), ids.tolist()))
    box.put((rank, out))
    dist.destroy_process_group()


def test_shard_candidates_match_full_vocabulary():
    ctx = mp.get_context("spawn")
    box = ctx.Queue()
    port, world = _port(), 2
    procs = [ctx.Process(target=_worker, args=(r, world, port, box)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(box.get(timeout=180) for _ in range(world))
    for p in procs:
        p.join(60)
    for trial in range(3):
        for r in range(world):
            same_ids, err, _ = got[r][trial]
            assert same_ids, (r, trial)
            assert err < 1e-5, (r, trial, err)
        assert got[0][trial][2] == got[1][trial][2]
