"""Helper launched by tests/test_tp_gpu.py under torch.distributed.run.

Every rank feeds different gradients to the fused ZeRO-2 LoRA AdamW kernel;
rank 0 compares the parameters every rank ends with against torch.optim.AdamW
on the rank-averaged, globally clipped gradients.
"""

import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from uno_b200.ops import cuda  # noqa: E402
from uno_b200.train.optim import ShardedLoraAdamW  # noqa: E402

SHAPES = [(64, 4096), (4096, 64), (1000,), (3, 7)]


def grads(rank, steps):
    g = torch.Generator(device="cuda").manual_seed(100 + rank)
    return [[torch.randn(*sh, device="cuda", generator=g) * (5.0 if s == 0 else 1e-3) for sh in SHAPES]
            for s in range(steps)]


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
    init = [torch.linspace(-1, 1, int(torch.tensor(sh).prod()), device="cuda").view(*sh) for sh in SHAPES]
    params = [torch.nn.Parameter(t.clone()) for t in init]
    opt = ShardedLoraAdamW(params, lr=1e-2, weight_decay=0.01, max_grad_norm=1.0, group=dist.group.WORLD)
    assert opt.fused
    steps = 4
    norms = []
    for s, gs in enumerate(grads(rank, steps)):
        opt.zero_grad()
        for p, g in zip(params, gs):
            p.grad += g
        norms.append(opt.step())
    torch.cuda.synchronize()
    got = torch.cat([p.detach().reshape(-1) for p in params])
    everyone = [torch.empty_like(got) for _ in range(world)]
    dist.all_gather(everyone, got)
    ok = True
    if rank == 0:
        ref = [torch.nn.Parameter(t.clone()) for t in init]
        topt = torch.optim.AdamW(ref, lr=1e-2, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
        per_rank = [grads(r, steps) for r in range(world)]
        for s in range(steps):
            for i, p in enumerate(ref):
                p.grad = sum(per_rank[r][s][i] for r in range(world)) / world
            torch.nn.utils.clip_grad_norm_(ref, 1.0)
            topt.step()
        want = torch.cat([p.detach().reshape(-1) for p in ref])
        for r, t in enumerate(everyone):
            err = (t - want).abs().max().item()
            print(f"rank {r}: max |param - torch AdamW| = {err:.3e}", flush=True)
            ok &= err < 1e-5
        ok &= norms[0] > 1.0 and cuda.error_flag() == 0
    opt.close()
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print("OPT_OK" if ok else "OPT_FAIL", flush=True)


if __name__ == "__main__":
    main()
