"""Helper launched by tests/test_tp_gpu.py under torch.distributed.run.

Every rank builds the same full logits from a common seed, keeps its vocabulary
shard, and runs the vocab-parallel sample / arg-max / verify kernels over the
fused-collective workspace; the results must equal the single-GPU kernels on
the full rows (samples and arg-max exactly, verify decisions up to summation
order, which these inputs do not reach).  The draft-tree candidates merged from
the shards must equal the top-K of the full rows, and build the same trees.
Top-k / top-p sampling and verification merged from the shards must take the
same decisions as the same merge over the full rows.
"""

import os
import sys
from types import SimpleNamespace

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from uno_b200.ops import cuda  # noqa: E402
from uno_b200.parallel.symm import FusedTPComm  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
    ctrl = dist.new_group(backend="gloo")
    comm = FusedTPComm(rank, world, ctrl, max_tokens=256, hidden=256, device="cuda", max_logit_rows=600)
    cuda.set_tp_comm(comm)
    V = 4096 * world
    Vs = V // world
    g = torch.Generator(device="cuda").manual_seed(5)
    failures = []
    for trial, rows in enumerate((7, 64, 300, 600)):
        full = (torch.randn(rows, V, device="cuda", generator=g) * 3).bfloat16()
        # draft logits close to the target so that both accepts and rejects occur
        draft = (full.float() + torch.randn(rows, V, device="cuda", generator=g) * 1.5).bfloat16()
        spec = cuda.sample_gumbel(draft, 1.0, 11, 100 + trial)
        shard = full[:, rank * Vs:(rank + 1) * Vs]
        dshard = draft[:, rank * Vs:(rank + 1) * Vs]
        want_g = cuda.argmax(full)
        got_g = cuda.vp_sample(shard.contiguous(), 1.0, 0, 0, rank * Vs, greedy=True)
        want_s = cuda.sample_gumbel(full, 0.8, 7, trial)
        got_s = cuda.vp_sample(shard.contiguous(), 0.8, 7, trial, rank * Vs)
        acc_w, corr_w = cuda.fused_verify(full, draft, spec, 1.0, 9, trial)
        acc_g, corr_g = cuda.vp_verify(shard.contiguous(), dshard.contiguous(), spec, 1.0, 9, trial, rank * Vs)
        torch.cuda.synchronize()
        if not torch.equal(want_g, got_g):
            failures.append(f"argmax rows={rows}")
        if not torch.equal(want_s, got_s):
            failures.append(f"sample rows={rows}")
        if not torch.equal(acc_w, acc_g):
            failures.append(f"accept rows={rows}: {(acc_w != acc_g).sum().item()} differ")
        rej = acc_w == 0
        if not torch.equal(corr_w[rej], corr_g[rej]):
            failures.append(f"resample rows={rows}: {(corr_w[rej] != corr_g[rej]).sum().item()} differ")
        if not (0 < int(acc_w.sum()) < rows or rows < 16):
            failures.append(f"rows={rows}: accept mix not exercised ({int(acc_w.sum())})")
    # draft-tree candidates: per-shard top-K merged over the group == top-K of the full rows
    from uno_b200.engine.draft_tree import build_draft_tree_batch, shard_candidate_log_probs

    def gather(x):
        parts = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(parts, x.contiguous())
        return torch.cat(parts, dim=-1)

    for B, D, K in ((1, 7, 4), (8, 7, 16)):
        full = (torch.randn(B, D + 1, V, device="cuda", generator=g) * 3).bfloat16()
        draft = full[:, 1:]
        ids, lp = shard_candidate_log_probs(draft[:, :, rank * Vs:(rank + 1) * Vs], K, 1.0, rank * Vs, gather)
        want_ids = torch.empty(B * D, K, device="cuda", dtype=torch.int64)
        want_lp = torch.empty(B * D, K, device="cuda", dtype=torch.float32)
        cuda.ext().topk_lse(draft.reshape(B * D, V).contiguous(), K, 1.0, want_ids, want_lp)
        if not torch.equal(ids.reshape(B * D, K), want_ids):
            failures.append(f"tree candidates B={B} K={K}: ids differ")
        if float((lp.reshape(B * D, K) - want_lp).abs().max()) > 1e-4:
            failures.append(f"tree candidates B={B} K={K}: log-probs differ")
        roots = torch.arange(B, device="cuda", dtype=torch.int64) + 3
        t_full = build_draft_tree_batch(roots, draft, max_nodes=16, candidate_top_k=K, temperature=1.0)

        t_vp = build_draft_tree_batch(roots, draft[:, :, rank * Vs:(rank + 1) * Vs], max_nodes=16,
                                      candidate_top_k=K, temperature=1.0,
                                      shard=SimpleNamespace(start=rank * Vs, gather=gather))
        if not (torch.equal(t_full.token_ids, t_vp.token_ids) and torch.equal(t_full.parent_indices,
                                                                               t_vp.parent_indices)):
            failures.append(f"tree B={B} K={K}: trees differ")
    # top-k / top-p: merged shard candidates (NCCL all-gather) == the same merge on the full rows
    from uno_b200.engine import vp_filtered as vpf

    def nccl_gather(x):
        parts = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(parts, x.contiguous())
        return torch.cat(parts, dim=-1)

    full = (torch.randn(48, V, device="cuda", generator=g) * 3).bfloat16()
    draft = (full.float() + torch.randn(48, V, device="cuda", generator=g)).bfloat16()
    for k, p in ((20, 1.0), (0, 0.9), (50, 0.8)):
        sh = lambda x: x[:, rank * Vs:(rank + 1) * Vs].contiguous()  # noqa: E731
        tok, q = vpf.sample(sh(draft), k, p, 0.7, rank * Vs, nccl_gather, 3, 1)
        acc, corr = vpf.verify(sh(full), tok, q, k, p, 0.7, rank * Vs, nccl_gather, 3, 2)
        tok1, q1 = vpf.sample(draft, k, p, 0.7, 0, lambda x: x, 3, 1)
        acc1, corr1 = vpf.verify(full, tok1, q1, k, p, 0.7, 0, lambda x: x, 3, 2)
        if not (torch.equal(tok, tok1) and torch.equal(acc, acc1) and torch.equal(corr, corr1)):
            failures.append(f"filtered k={k} p={p}: shard merge differs from the full rows")
    err = cuda.error_flag()
    if err:
        failures.append(f"device error flag {err}")
    results = [None] * world
    dist.all_gather_object(results, failures, group=ctrl)
    comm.close()
    dist.barrier(group=ctrl)
    dist.destroy_process_group()
    if rank == 0:
        bad = [f"rank {r}: {f}" for r, fs in enumerate(results) for f in fs]
        print("VP_FAIL " + "; ".join(bad) if bad else "VP_OK", flush=True)


if __name__ == "__main__":
    main()
