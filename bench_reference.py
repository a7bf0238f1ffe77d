"""Reference arm of ``bench.py``: the unmodified reference package (``nano_vllm_uno``).

The reference was installed offline into ``baseline/_ref``
(``pip install --no-index --no-deps --ignore-requires-python --target baseline/_ref``).
It has no random-init mode, so this arm first writes a checkpoint directory in
the Hugging Face layout it loads (``config.json``, a word-level
``tokenizer.json``, ``*.safetensors`` with N(0, 0.02) weights and unit norms,
and a PEFT adapter of rank 64 / alpha 128 on q,k,v,o,gate,up,down), then runs
the reference's own ``LLM`` API and stock code path on the same workload as the
native arm: 64 requests, block size 8, temperature 1.0, 256-token pages, CUDA
graphs for batch sizes 1..64 and block sizes {1, 8}, FlashAttention-2 backend.

Under ``torchrun`` with N ranks, rank 0 builds ``LLM(tensor_parallel_size=N)``
(the reference spawns its own TP workers on GPUs 1..N-1); other ranks wait for
rank 0's completion marker.  Device time is measured with CUDA events on rank
0's stream; every reference forward ends in NCCL collectives across the TP
ranks, so rank 0's elapsed time bounds the slowest rank.
"""

from __future__ import annotations

import json
import os
import socket
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(ROOT, "baseline", "_ref")
CKPT = os.environ.get("UNO_REF_CKPT", "/tmp/uno_ref_qwen3_8b")
METRIC = "Uno-Qwen3-8B Psi-Spec output tok/s at TP=1/2/4/8; per-request tok/s; TPF"


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def write_checkpoint(path: str, rank: int = 64, alpha: float = 128.0, std: float = 0.02, seed: int = 0) -> None:
    """Random Qwen3-8B checkpoint + tokenizer + PEFT adapter in the reference's format."""
    import torch
    from safetensors.torch import save_file
    from tokenizers import Tokenizer
    from tokenizers.models import WordLevel
    from tokenizers.pre_tokenizers import WhitespaceSplit
    from transformers import PreTrainedTokenizerFast, Qwen3Config

    done = os.path.join(path, ".complete")
    if os.path.exists(done):
        return
    os.makedirs(path, exist_ok=True)
    V, H, I, L, HQ, HKV, D = 151936, 4096, 12288, 36, 32, 8, 128
    cfg = Qwen3Config(vocab_size=V, hidden_size=H, intermediate_size=I, num_hidden_layers=L,
                      num_attention_heads=HQ, num_key_value_heads=HKV, head_dim=D, max_position_embeddings=40960,
                      rope_theta=1e6, rms_norm_eps=1e-6, tie_word_embeddings=False, attention_bias=False,
                      eos_token_id=151645, pad_token_id=151643, bos_token_id=151643)
    cfg.torch_dtype = "bfloat16"
    cfg.save_pretrained(path)
    vocab = {f"t{i}": i for i in range(V)}
    tok = Tokenizer(WordLevel(vocab, unk_token="t0"))
    tok.pre_tokenizer = WhitespaceSplit()
    fast = PreTrainedTokenizerFast(tokenizer_object=tok, eos_token="t151645", pad_token="t151643", unk_token="t0")
    fast.save_pretrained(path)
    gen = torch.Generator(device="cuda").manual_seed(seed)

    def rnd(*shape):
        return (torch.randn(*shape, device="cuda", generator=gen) * std).to(torch.bfloat16).cpu()

    ones = lambda n: torch.ones(n, dtype=torch.bfloat16)
    save_file({"model.embed_tokens.weight": rnd(V, H)}, os.path.join(path, "model-embed.safetensors"))
    save_file({"lm_head.weight": rnd(V, H), "model.norm.weight": ones(H)},
              os.path.join(path, "model-head.safetensors"))
    shapes = {"self_attn.q_proj": (HQ * D, H), "self_attn.k_proj": (HKV * D, H), "self_attn.v_proj": (HKV * D, H),
              "self_attn.o_proj": (H, HQ * D), "mlp.gate_proj": (I, H), "mlp.up_proj": (I, H),
              "mlp.down_proj": (H, I)}
    for li in range(L):
        t = {f"model.layers.{li}.{k}.weight": rnd(*s) for k, s in shapes.items()}
        t[f"model.layers.{li}.self_attn.q_norm.weight"] = ones(D)
        t[f"model.layers.{li}.self_attn.k_norm.weight"] = ones(D)
        t[f"model.layers.{li}.input_layernorm.weight"] = ones(H)
        t[f"model.layers.{li}.post_attention_layernorm.weight"] = ones(H)
        save_file(t, os.path.join(path, f"model-layer{li:02d}.safetensors"))
    adapter = os.path.join(path, "adapter")
    os.makedirs(adapter, exist_ok=True)
    at = {}
    for li in range(L):
        for k, (out_f, in_f) in shapes.items():
            pre = f"base_model.model.model.layers.{li}.{k}"
            at[pre + ".lora_A.weight"] = rnd(rank, in_f)
            at[pre + ".lora_B.weight"] = rnd(out_f, rank)
    save_file(at, os.path.join(adapter, "adapter_model.safetensors"))
    with open(os.path.join(adapter, "adapter_config.json"), "w") as fh:
        json.dump({"r": rank, "lora_alpha": alpha, "peft_type": "LORA",
                   "target_modules": ["q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"]},
                  fh)
    open(done, "w").close()


def _wait_for(path: str, timeout_s: float) -> None:
    t0 = time.time()
    while not os.path.exists(path):
        if time.time() - t0 > timeout_s:
            raise TimeoutError(f"rank 0 did not finish within {timeout_s}s")
        time.sleep(1.0)


def run(args) -> None:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    marker = os.path.join("/tmp", f"uno_ref_done_{os.environ.get('MASTER_PORT', 'single')}")
    if rank != 0:
        _wait_for(marker, 3600)
        return
    try:
        if os.path.exists(marker):
            os.unlink(marker)
        line = _run_rank0(args, world)
    except Exception as exc:  # report, do not crash the driver
        line = {"impl": "reference", "unavailable": f"{type(exc).__name__}: {str(exc).splitlines()[0][:300]}"}
    print(json.dumps(line), flush=True)
    open(marker, "w").close()


def locate_reference() -> tuple[str | None, str]:
    """Directory whose ``nano_vllm_uno`` package is the unmodified reference, and how it was found.

    Order: the offline install in ``baseline/_ref``; an importable ``nano_vllm_uno``
    installed elsewhere; a run-time offline install (``pip --no-index --no-deps``)
    from the reference source tree named by ``UNO_REF_SOURCE`` into
    ``baseline/_ref``.  Returns ``(None, reason)`` when none works.
    """
    if os.path.isdir(os.path.join(REF, "nano_vllm_uno")):
        return REF, "baseline/_ref"
    import importlib.util

    spec = importlib.util.find_spec("nano_vllm_uno")
    if spec is not None and spec.origin:
        return os.path.dirname(os.path.dirname(spec.origin)), "importable nano_vllm_uno"
    sources = [s for s in (os.environ.get("UNO_REF_SOURCE"),) if s]
    for src in sources:
        if not os.path.isfile(os.path.join(src, "pyproject.toml")):
            continue
        import subprocess

        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
               "--ignore-requires-python", "--target", REF, src]
        if os.path.isdir("/opt/wheelhouse"):
            cmd[5:5] = ["--find-links", "/opt/wheelhouse"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode == 0 and os.path.isdir(os.path.join(REF, "nano_vllm_uno")):
            return REF, f"installed at run time from {src}"
        tail = (r.stderr or r.stdout).strip().splitlines()[-1:] or ["no output"]
        return None, f"run-time install from {src} failed: {tail[0][:200]}"
    return None, ("baseline/_ref/nano_vllm_uno is missing, nano_vllm_uno is not importable and no reference "
                  "source tree is available for an offline install (set UNO_REF_SOURCE)")


def _run_rank0(args, world: int) -> dict:
    ref_dir, how = locate_reference()
    if ref_dir is None:
        return {"impl": "reference", "unavailable": how}
    import torch

    write_checkpoint(CKPT)
    torch.cuda.empty_cache()
    sys.path.insert(0, ref_dir)
    sys.path.insert(1, ROOT)
    os.environ["TORCH_DISTRIBUTED_PORT"] = str(_free_port())
    from nano_vllm_uno import LLM, SamplingParams

    from bench import MASK_ID, ClockSampler, make_prompts

    ladder = [b for b in list(range(1, 9)) + list(range(10, 33, 2)) + list(range(40, 65, 4)) if b <= args.batch]
    llm = LLM(CKPT, tokenizer_path=CKPT, tensor_parallel_size=world, gated_lora_path=os.path.join(CKPT, "adapter"),
              max_num_seqs=args.batch, max_model_len=1024 + args.new_tokens + 64, max_num_batched_tokens=16384,
              kvcache_block_size=256, max_diffusion_block_size=args.block, cuda_graph_block_sizes=[1, args.block],
              cuda_graph_batch_sizes=ladder, attention_backend="fa2", gpu_memory_utilization=0.9)
    sp = SamplingParams(temperature=1.0, max_tokens=args.new_tokens, diffusion_block_size=args.block,
                        mask_token_id=MASK_ID, ignore_eos=True)
    prompts = make_prompts(args.batch, args.seed)
    for p in prompts:
        llm.add_request(p, sp)
    while llm.scheduler.waiting:
        llm.step()
    for _ in range(args.warmup):
        llm.step()
    clocks = ClockSampler("/tmp/uno_ref_clocks.csv")
    clocks.start()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    tokens = 0
    for _ in range(args.steps):
        _, n = llm.step()
        tokens += -n
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    clock_info = clocks.stop()
    while not llm.is_finished():
        llm.step()
    e2e = None
    if not args.no_e2e:
        new_tokens = args.e2e_tokens or args.new_tokens
        sp2 = SamplingParams(temperature=1.0, max_tokens=new_tokens, diffusion_block_size=args.block,
                             mask_token_id=MASK_ID, ignore_eos=True)
        torch.cuda.synchronize()
        s0 = time.perf_counter()
        outs = llm.generate(prompts, sp2, use_tqdm=False, detokenize=False)
        torch.cuda.synchronize()
        dt = time.perf_counter() - s0
        total = sum(len(o["token_ids"]) for o in outs)
        st = llm.last_generate_stats
        e2e = {"value": total / dt, "unit": "tok/s", "seconds": dt, "output_tokens": total,
               "tpf": st.get("accepts", 0) / max(1, st.get("forwards", 0)), "api": "nano_vllm_uno.LLM.generate"}
    llm.exit()
    tps = tokens / (ms / 1e3)
    return {
        "metric": METRIC, "value": tps, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random-init checkpoint, Zipf(1.1) prompt ids)",
        "config": {"model": "Uno-Qwen3-8B (random init) + rank-64 gated LoRA", "global_batch": args.batch,
                   "block_size": args.block, "parallelism": f"tp{args.gpus}", "attention_backend": "fa2",
                   "l2": "working set >> L2"},
        "clocks": clock_info, "e2e": e2e, "impl": "reference",
        "reference_path": os.path.relpath(ref_dir, ROOT) if ref_dir.startswith(ROOT) else ref_dir,
        "reference_found": how,
    }
