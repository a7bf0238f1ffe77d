"""Fused tensor-parallel kernels timed on N ranks (one process per GPU).

``python -m torch.distributed.run --nproc-per-node N -m uno_b200.parallel.comm_cases``

Every case is timed with CUDA events around ``--iters`` back-to-back
iterations after warm-up, on every rank, and reported as the MAX over ranks
(rank 0 prints one JSON line per case).  The roofline of a fused
compute + collective path is the slower of its FLOPs at the measured GEMM
peak and its NVLink bytes per GPU at the measured peer-copy bandwidth:

* ``rowpar_rs_norm_ag`` -- the row-parallel o_proj GEMM whose epilogue sends
  each partial row to its owner (reduce-scatter), then the reduce + residual
  + RMSNorm + all-gather kernel (Qwen3-8B decode step: 512 rows, hidden 4096);
* ``reduce_norm_gather`` -- that second kernel alone;
* ``vp_verify`` -- vocab-parallel Psi-Spec verify of 448 rows (HBM-bound: each
  rank reads its two V/N logit shards; the exchange is a few bytes per row).
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

GEMM_PEAK = 1665e12  # measured cuBLAS bf16 burst on this pool
HBM_BW = 6549e9      # measured copy bandwidth
NVLINK_BW = 770e9    # measured peer copy, per direction per GPU


def _time(fn, iters: int) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / iters * 1e3], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--iters", type=int, default=50)
    args = ap.parse_args(argv)
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("nccl", device_id=torch.device("cuda", torch.cuda.current_device()))
    ctrl = dist.new_group(backend="gloo")
    from uno_b200.ops import cuda as C
    from uno_b200.parallel.symm import FusedTPComm

    T, H, Kin = 512, 4096, 4096 // world
    comm = FusedTPComm(rank, world, ctrl, max_tokens=T, hidden=H, device="cuda", max_logit_rows=512)
    C.set_tp_comm(comm)
    torch.manual_seed(rank)
    x = torch.randn(T, Kin, device="cuda").bfloat16()
    w = torch.randn(H, Kin, device="cuda").bfloat16() * 0.02
    norm_w = torch.ones(H, device="cuda").bfloat16()
    residual = torch.randn(comm.rows_per_rank(T), H, device="cuda").bfloat16()
    R = comm.rows_per_rank(T)
    rows_bytes = R * H * 2
    out = []

    def rs_then_norm():
        C._gemm(x, w, C.EPI_STORE, rs=comm.rs_args(T))
        comm.reduce_norm(T, residual, norm_w, 1e-6, 1)

    us = _time(rs_then_norm, args.iters)
    flops = 2 * T * H * Kin
    nv = (world - 1) * rows_bytes * 2  # partial rows out (RS) + normalised rows out (AG), per GPU
    roof = max(flops / GEMM_PEAK, nv / NVLINK_BW) * 1e6
    out.append({"case": "rowpar_rs_norm_ag", "shape": f"{T}x{H}x{Kin} tp={world}", "us": round(us, 2),
                "roofline_us": round(roof, 2), "frac_of_roofline": round(roof / us, 3),
                "nvlink_bytes_per_gpu": nv, "flops": flops})

    us = _time(lambda: comm.reduce_norm(T, residual, norm_w, 1e-6, 1), args.iters)
    nv = (world - 1) * rows_bytes
    roof = nv / NVLINK_BW * 1e6
    out.append({"case": "reduce_norm_gather", "shape": f"{T}x{H} tp={world}", "us": round(us, 2),
                "roofline_us": round(roof, 2), "frac_of_roofline": round(roof / us, 3), "nvlink_bytes_per_gpu": nv})

    V = 151936
    Vs = V // world
    rows = 448
    clean = (torch.randn(rows, Vs, device="cuda") * 3).bfloat16()
    draft = (clean.float() + 1).bfloat16()
    spec = torch.randint(0, V, (rows,), device="cuda", generator=torch.Generator(device="cuda").manual_seed(1))
    us = _time(lambda: C.vp_verify(clean, draft, spec, 1.0, 1, 2, rank * Vs), args.iters)
    hbm = rows * Vs * 2 * 2
    roof = hbm / HBM_BW * 1e6
    out.append({"case": "vp_verify", "shape": f"{rows} rows x V/{world}={Vs}", "us": round(us, 2),
                "roofline_us": round(roof, 2), "frac_of_roofline": round(roof / us, 3), "hbm_bytes_per_gpu": hbm})
    err = torch.tensor([C.error_flag()], device="cuda")
    dist.all_reduce(err, op=dist.ReduceOp.MAX)
    if rank == 0:
        for rec in out:
            print(json.dumps(rec), flush=True)
        print(json.dumps({"device_error_flag": int(err.item())}), flush=True)
    C.set_tp_comm(None)
    comm.close()
    dist.barrier(group=ctrl)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
