"""Helper launched by tests/test_tp_gpu.py under torch.distributed.run.

Every rank builds the same small model and LoRA; the native training forward
and backward run once with replicated frozen weights and once with the weights
row-sharded over the ranks (GEMMs read the peers' rows over NVLink).  Hidden
states and LoRA gradients must agree.
"""

import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from test_train_gpu import _setup  # noqa: E402


def run(fsdp: bool, group):
    from uno_b200.train.forward import uno_hidden_states
    from uno_b200.train.native import build_projections

    # every projection's output rows split into 64-row multiples over up to 8 ranks
    model, lora, opt, ub = _setup(head_dim=128, hidden=512, heads=8, kv_heads=4, inter=1024)
    proj, sharded = build_projections(model, lora, group=group, fsdp=fsdp)
    for layer in proj:
        for p in layer.values():
            p.refresh(0)
    opt.zero_grad()
    h = uno_hidden_states(model, lora, ub.ids, ub.positions, ub.attention_mask(), ub.noisy, native=proj)
    w = torch.randn(h.shape, device="cuda", generator=torch.Generator(device="cuda").manual_seed(9))
    (h.float() * w).sum().backward()
    torch.cuda.synchronize()
    out = h.detach().float(), opt.flat_grad.clone()
    opt.close()
    if sharded is not None:
        sharded.close()
    return out


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
    h0, g0 = run(False, None)
    h1, g1 = run(True, dist.group.WORLD)
    from uno_b200.ops import cuda

    hd = ((h1 - h0).norm() / h0.norm()).item()
    gd = ((g1 - g0).norm() / g0.norm()).item()
    ok = torch.tensor([1 if (hd < 1e-2 and gd < 2e-2 and cuda.error_flag() == 0) else 0], device="cuda")
    print(f"rank {rank}: hidden rel {hd:.2e} grad rel {gd:.2e}", flush=True)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    dist.destroy_process_group()
    if rank == 0:
        print("FSDP_OK" if ok.item() == 1 else "FSDP_FAIL", flush=True)


if __name__ == "__main__":
    main()
