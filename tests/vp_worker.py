"""Helper launched by tests/test_tp_gpu.py under torch.distributed.run.

Every rank builds the same full logits from a common seed, keeps its vocabulary
shard, and runs the vocab-parallel sample / arg-max / verify kernels over the
fused-collective workspace; the results must equal the single-GPU kernels on
the full rows (samples and arg-max exactly, verify decisions up to summation
order, which these inputs do not reach).
"""

import os
import sys

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
