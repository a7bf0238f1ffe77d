"""Headline benchmark: Uno-Qwen3-8B Psi-Spec output tokens/s (linear sampler).

Config: Qwen3-8B architecture with random-init weights and a
random rank-64 conditional-LoRA adapter on every linear, bf16; 64 concurrent
requests with prompt lengths uniform in [128, 1024] and Zipf(1.1) token ids;
temperature 1.0; diffusion block size 8; 256-token KV pages; CUDA graphs for
decode batch sizes 1..64.  ``--gpus N`` runs tensor parallel degree N (strong
scaling: the same 64-request batch is split across N GPUs), one process per GPU
under ``torch.distributed.run``.

A *step* is one engine decode step: one Psi-Spec cycle (draft forward + verify
forward + accept/resample) for every running request.  ``value`` is committed
output tokens per second over exactly ``--steps`` steps after ``--warmup``
steps, timed with CUDA events on every rank (barrier + synchronize on both
sides) and reduced with MAX over ranks.  The per-step working set (16 GB of
weights plus the KV cache) is far larger than L2, so no L2 flush is needed.
``e2e`` is the same metric through the public ``LLM.generate`` API over the
whole workload (prefill included), wall-clock, which copies each step's inputs
host->device from pinned memory and reads committed tokens back every step.

``--impl reference`` runs the unmodified reference package from
``baseline/_ref`` through its own ``LLM`` API on the same workload.

``--sampler tree`` measures BASELINE config 3 (per-request tok/s of the tree
sampler) and ``--config uno-0.9b-dp`` config 4 (one 0.9B replica per GPU,
weak scaling).
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "Uno-Qwen3-8B Psi-Spec output tok/s at TP=1/2/4/8; per-request tok/s; TPF"
# The reference publishes one throughput figure: about 5,200 tok/s for Uno (Psi-Spec), read
# off its results chart (hardware unspecified).
BASELINE_TOKS = 5200.0
VOCAB = 151936
MASK_ID = 151669


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--block", type=int, default=8)
    ap.add_argument("--new-tokens", type=int, default=2048)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--top-k", type=int, default=None, help="filtered sampling (not the headline config)")
    ap.add_argument("--top-p", type=float, default=None, help="filtered sampling (not the headline config)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-tokens", type=int, default=0, help="override new tokens for the e2e run")
    ap.add_argument("--sampler", default="linear", choices=["linear", "tree"],
                    help="tree: BASELINE config 3 (64-node tree of depth 8, per-request tok/s; default batch 1)")
    ap.add_argument("--breakdown", type=int, default=0, metavar="S",
                    help="after the timed region, profile S more decode steps on rank 0 and print a per-step "
                         "breakdown (wall, model GPU, exposed host time, kernel busy time, top kernels)")
    ap.add_argument("--config", default="qwen3-8b", choices=["qwen3-8b", "uno-0.9b-dp"],
                    help="uno-0.9b-dp: BASELINE config 4 (0.9B dense model, one data-parallel replica per GPU, "
                         "256 requests per replica, prompts U[64,512], 1024 new tokens, block 16, LoRA rank 32)")
    args = ap.parse_args()
    if args.config == "uno-0.9b-dp":
        if args.batch == 64:
            args.batch = 256
        if args.block == 8:
            args.block = 16
        if args.new_tokens == 2048:
            args.new_tokens = 1024
    if args.sampler == "tree":
        # config 3: prompt 512 Zipf ids, 4096 new tokens, depth 8 (block 9), 64 nodes, top-4 candidates
        if args.batch == 64:
            args.batch = 1
        if args.block == 8:
            args.block = 9
        if args.new_tokens == 2048:
            args.new_tokens = 4096
    return args


def make_prompts(batch: int, seed: int, fixed_len: int | None = None, lo: int = 128,
                 hi: int = 1024) -> list[list[int]]:
    rng = np.random.default_rng(seed)
    perm = rng.permutation(VOCAB - 2) + 1
    lens = rng.integers(lo, hi + 1, size=batch) if fixed_len is None else np.full(batch, fixed_len)
    prompts = []
    for n in lens:
        ranks = rng.zipf(1.1, size=int(n)) - 1
        prompts.append([int(perm[r % len(perm)]) for r in ranks])
    return prompts


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, path: str):
        self.path = path
        self.proc = None

    def start(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader",
                                          "-lms", "50"], stdout=self.fh, stderr=subprocess.DEVNULL)
            time.sleep(0.3)  # let the sampler start before the timed region
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1].split()[0]))
                smax.append(float(parts[2].split()[0]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": []}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}


def engine_kwargs(args, tp: int) -> dict:
    ladder = list(range(1, 9)) + list(range(10, 33, 2)) + list(range(40, 65, 4)) + list(range(80, 257, 16))
    dp = getattr(args, "config", "qwen3-8b") == "uno-0.9b-dp"
    return dict(
        tensor_parallel_size=tp,
        max_num_seqs=args.batch,
        max_model_len=1024 + args.new_tokens + 64,
        max_num_batched_tokens=16384,
        kvcache_block_size=256,
        max_diffusion_block_size=args.block,
        cuda_graph_block_sizes=sorted({1, args.block}),
        cuda_graph_batch_sizes=[b for b in ladder if b <= args.batch],
        dummy_lora_rank=32 if dp else 64,
        dummy_lora_alpha=64.0 if dp else 128.0,
        gpu_memory_utilization=0.90,
        seed=args.seed,
    ) | ({"tree_verify_size": 64, "tree_candidate_top_k": 4} if getattr(args, "sampler", "linear") == "tree" else {})


def emit(obj) -> None:
    """One JSON line in a single write, so that another rank's output cannot split it."""
    sys.stdout.write(json.dumps(obj) + "\n")
    sys.stdout.flush()


def _filter_note(args) -> str:
    parts = ([f"top-k {args.top_k}"] if args.top_k else []) + ([f"top-p {args.top_p}"] if args.top_p else [])
    return (", " + ", ".join(parts)) if parts else ""


def run_dp_replicas(args):
    """one independent 0.9B replica per GPU (weak scaling over N replicas).

    Every rank times ``--steps`` steps of its own replica with CUDA events; the
    job's value is the sum of the committed tokens over the slowest rank's time
    (max over ranks), gathered over a gloo group."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("gloo")
    sys.path.insert(0, ROOT)
    from uno_b200 import LLM, SamplingParams

    llm = LLM("preset:uno-0.9b", **engine_kwargs(args, 1))
    sp = SamplingParams(temperature=1.0, max_tokens=args.new_tokens, diffusion_block_size=args.block,
                        mask_token_id=MASK_ID, ignore_eos=True, seed=args.seed + rank)
    prompts = make_prompts(args.batch, args.seed + 1000 * rank, None, 64, 512)
    for p in prompts:
        llm.add_request(p, sp)
    while llm.scheduler.waiting:
        llm.step()
    for _ in range(args.warmup):
        llm.step()
    clocks = ClockSampler(os.environ.get("UNO_BENCH_CLOCKS_CSV", "/tmp/bench_clocks.csv"))
    if world > 1:
        dist.barrier()
    clocks.start()
    llm.call("timer_start")
    tokens = 0
    stats0 = {k: sum(s.stats[k] for s in llm.scheduler.running) for k in ("forwards", "accepts")}
    for _ in range(args.steps):
        _, n = llm.step()
        tokens += -n
    ms = llm.call("timer_stop")
    clock_info = clocks.stop()
    stats1 = {k: sum(s.stats[k] for s in llm.scheduler.running) for k in ("forwards", "accepts")}
    running = len(llm.scheduler.running)
    launches = count_launches(llm)
    t = torch.tensor([float(tokens), ms], dtype=torch.float64)
    if world > 1:
        tot = t.clone()
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
        mx = t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        tokens_all, ms_max = float(tot[0]), float(mx[1])
    else:
        tokens_all, ms_max = float(tokens), ms
    e2e = None
    if not args.no_e2e:
        while not llm.is_finished():
            llm.step()
        sp2 = SamplingParams(temperature=1.0, max_tokens=args.e2e_tokens or args.new_tokens,
                             diffusion_block_size=args.block, mask_token_id=MASK_ID, ignore_eos=True,
                             seed=args.seed + 7 + rank)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        outs = llm.generate(prompts, sp2, use_tqdm=False, detokenize=False)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        e2 = torch.tensor([float(sum(len(o["token_ids"]) for o in outs)), dt], dtype=torch.float64)
        if world > 1:
            s2 = e2.clone()
            dist.all_reduce(s2, op=dist.ReduceOp.SUM)
            m2 = e2.clone()
            dist.all_reduce(m2, op=dist.ReduceOp.MAX)
            e2 = torch.tensor([float(s2[0]), float(m2[1])], dtype=torch.float64)
        ws = llm.model_runner.workspace
        e2e = {"value": float(e2[0]) / float(e2[1]), "unit": "tok/s", "seconds": float(e2[1]),
               "output_tokens": int(e2[0]),
               "h2d_bytes_per_step": int(ws.host64.numel() * 8 + ws.host32.numel() * 4) * 2 + args.batch * args.block * 4,
               "d2h_bytes_per_step": args.batch * (args.block + 2) * 8, "api": "uno_b200.LLM.generate"}
    if rank == 0:
        line = {
            "metric": "Uno 0.9B-class Psi-Spec system output tok/s, data-parallel replicas (config 4)",
            "value": tokens_all / (ms_max / 1e3), "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init weights, Zipf(1.1) prompt ids)",
            "config": {"model": "uno-0.9b (16 layers, hidden 2048, 16 heads, SwiGLU 5632) + rank-32 gated LoRA",
                       "global_batch": args.batch * world, "seq_len": "prompt U[64,512] + 1024 new",
                       "block_size": args.block, "sampler": "linear Psi-Spec, T=1.0", "kv_page": 256,
                       "parallelism": f"dp{world}", "running_requests_rank0": running,
                       "l2": "working set > L2 (1.8 GB weights + KV per step)"},
            "tpf": (stats1["accepts"] - stats0["accepts"]) / max(1, stats1["forwards"] - stats0["forwards"]),
            "clocks": clock_info, "e2e": e2e,
            "gpu_launches": launches * args.steps if launches is not None else None, "impl": "native",
        }
        emit(line)
    llm.exit()
    if world > 1:
        dist.destroy_process_group()


def run_native(args):
    import torch

    if args.config == "uno-0.9b-dp":
        return run_dp_replicas(args)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    sys.path.insert(0, ROOT)
    from uno_b200 import LLM, SamplingParams
    from uno_b200.engine.worker import serve_follower

    kw = engine_kwargs(args, world)
    if world > 1:
        kw["distributed_init"] = "env"
        os.environ.setdefault("TORCH_DISTRIBUTED_TIMEOUT_MINUTES", "5")
    if rank != 0:
        serve_follower("preset:qwen3-8b", **kw)
        return
    llm = LLM("preset:qwen3-8b", **kw)
    sp = SamplingParams(temperature=1.0, max_tokens=args.new_tokens, diffusion_block_size=args.block,
                        mask_token_id=MASK_ID, ignore_eos=True, seed=args.seed, top_k=args.top_k, top_p=args.top_p)
    tree = args.sampler == "tree"
    prompts = make_prompts(args.batch, args.seed, 512 if tree else None)

    # ---------------- device-timed steady-state decode steps
    for p in prompts:
        llm.add_request(p, sp)
    while llm.scheduler.waiting:
        llm.step()  # prefill (unchunked) until every request is admitted
    for _ in range(args.warmup):
        llm.step()
    clocks = ClockSampler(os.environ.get("UNO_BENCH_CLOCKS_CSV", "/tmp/bench_clocks.csv"))
    clocks.start()
    llm.call("timer_start")
    tokens = 0
    stats0 = {k: sum(s.stats[k] for s in llm.scheduler.running) for k in ("forwards", "accepts")}
    for _ in range(args.steps):
        outputs, n = llm.step()
        tokens += -n
    ms = llm.call("timer_stop")
    clock_info = clocks.stop()
    stats1 = {k: sum(s.stats[k] for s in llm.scheduler.running) for k in ("forwards", "accepts")}
    running = len(llm.scheduler.running)
    # launches per step: count kernels of one extra step under the profiler (not timed)
    launches = count_launches(llm)
    breakdown = step_breakdown(llm, args.breakdown) if args.breakdown else None
    # drain the remaining work so the engine is idle
    while not llm.is_finished():
        llm.step()

    # ---------------- end-to-end through the public API
    e2e = None
    if not args.no_e2e:
        new_tokens = args.e2e_tokens or args.new_tokens
        sp2 = SamplingParams(temperature=1.0, max_tokens=new_tokens, diffusion_block_size=args.block,
                             mask_token_id=MASK_ID, ignore_eos=True, seed=args.seed + 1, top_k=args.top_k,
                             top_p=args.top_p)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        outs = llm.generate(prompts, sp2, use_tqdm=False, detokenize=False)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        total = sum(len(o["token_ids"]) for o in outs)
        st = llm.last_generate_stats
        ws = llm.model_runner.workspace
        h2d = int(ws.host64.numel() * 8 + ws.host32.numel() * 4) * 2 + args.batch * args.block * 4
        e2e = {"value": total / dt / (len(prompts) if tree else 1),
               "unit": "tok/s per request" if tree else "tok/s", "seconds": dt, "output_tokens": total,
               "tpf": st.get("accepts", 0) / max(1, st.get("forwards", 0)),
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": args.batch * (args.block + 2) * 8,
               "api": "uno_b200.LLM.generate"}
    tps = tokens / (ms / 1e3)
    if tree:
        tps = tps / max(1, running)  # per-request tok/s
    d_acc = stats1["accepts"] - stats0["accepts"]
    d_fwd = stats1["forwards"] - stats0["forwards"]
    line = {
        "metric": METRIC + (" [tree sampler: per-request tok/s]" if tree else ""),
        "value": tps,
        "unit": "tok/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms / args.steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": (tps / BASELINE_TOKS) if (BASELINE_TOKS and not tree) else None,
        "dtype": "bf16",
        "data": "synthetic (random-init weights, Zipf(1.1) prompt ids)",
        "config": {"model": "Uno-Qwen3-8B (random init) + rank-64 gated LoRA", "global_batch": args.batch,
                   "seq_len": ("prompt 512 + 4096 new" if tree else "prompt U[128,1024] + 2048 new"),
                   "block_size": args.block,
                   "sampler": ("tree Psi-Spec, 64 nodes, depth 8, top-4 candidates, T=1.0" if tree
                               else "linear Psi-Spec, T=1.0") + _filter_note(args), "kv_page": 256,
                   "parallelism": f"tp{args.gpus}", "l2": "working set >> L2 (16 GB weights + KV per step)",
                   "running_requests": running},
        "tpf": d_acc / max(1, d_fwd),
        "clocks": clock_info,
        "e2e": e2e,
        "gpu_launches": launches * args.steps if launches is not None else None,
        "impl": "native",
    }
    emit(line)
    if breakdown is not None:
        emit({"breakdown": breakdown, "n_gpus": args.gpus})
    llm.exit()


def step_breakdown(llm, steps: int) -> dict | None:
    """Where one decode step's time goes on rank 0 (untimed diagnostic).

    Runs ``steps`` decode steps with the engine's decode timing on (CUDA events
    around each forward: backbone + lm_head) and under ``torch.profiler`` for
    the kernel list.  Reports per step: host wall time, model GPU time,
    ``exposed_non_model_ms`` (wall minus model GPU: sampling, verify, staging,
    control plane and host gaps), the union of kernel intervals (GPU busy) and
    the top kernels by device time."""
    import torch

    if llm.is_finished():
        return None
    from torch.profiler import ProfilerActivity, profile

    llm.config.decode_timing = True
    llm.reset_decode_timing()
    with profile(activities=[ProfilerActivity.CUDA, ProfilerActivity.CPU]) as prof:
        for _ in range(steps):
            if llm.is_finished():
                break
            llm.step()
        torch.cuda.synchronize()
    timing = llm.get_decode_timing()
    llm.config.decode_timing = False
    n = max(1, len(timing["step_wall_ms"]))
    kernels = [e for e in prof.events() if e.device_type.name == "CUDA"]
    spans = sorted((e.time_range.start, e.time_range.end) for e in kernels)
    busy, cur_s, cur_e = 0.0, None, None
    for a, b in spans:
        if cur_e is None or a > cur_e:
            if cur_e is not None:
                busy += cur_e - cur_s
            cur_s, cur_e = a, b
        else:
            cur_e = max(cur_e, b)
    if cur_e is not None:
        busy += cur_e - cur_s
    by_name: dict[str, list[float]] = {}
    for e in kernels:
        d = by_name.setdefault(e.name[:120], [0.0, 0])
        d[0] += e.time_range.end - e.time_range.start
        d[1] += 1
    top = sorted(by_name.items(), key=lambda kv: -kv[1][0])[:25]
    wall = sum(timing["step_wall_ms"]) / n
    return {
        "steps": n,
        "wall_ms_per_step": wall,
        "model_gpu_ms_per_step": sum(timing["model_gpu_ms"]) / n,
        "exposed_non_model_ms_per_step": sum(timing["exposed_non_model_ms"]) / n,
        "kernel_busy_ms_per_step": busy / 1e3 / n,
        "gpu_busy_fraction": busy / 1e3 / n / wall if wall > 0 else None,
        "top_kernels": [{"name": k, "ms_per_step": v[0] / 1e3 / n, "launches_per_step": v[1] / n} for k, v in top],
        "note": "profiled steps (not timed); per-kernel times under torch.profiler",
    }


def count_launches(llm):
    """Kernels of the extension launched by one decode step (profiled, untimed)."""
    import torch

    if llm.is_finished():
        return None
    try:
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            llm.step()
            torch.cuda.synchronize()
        names = [e.name for e in prof.events() if e.device_type.name == "CUDA"]
        return sum(1 for n in names if "uno::" in n)  # every kernel of the extension lives in namespace uno
    except Exception:  # pragma: no cover - profiler availability
        return None


def run_reference(args):
    if args.config != "qwen3-8b":
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps({"impl": "reference", "unavailable": "the reference arm is wired for the "
                              "Qwen3-8B headline configs only"}), flush=True)
        return
    if args.sampler == "tree":
        # The reference tree sampler requires attention_backend fa3 or fa4 (its config.py:134-138):
        # FA3 (flash_attn_interface / sgl_kernel) is Hopper-only and FA4 comes with SGLang; neither
        # is installed on this image.
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps({"impl": "reference", "unavailable": "reference tree sampler needs FA3 "
                              "(sm90-only) or FA4 via SGLang; neither is installed"}), flush=True)
        return
    from bench_reference import run  # the reference arm lives beside bench.py

    run(args)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_native(args)


if __name__ == "__main__":
    main()
