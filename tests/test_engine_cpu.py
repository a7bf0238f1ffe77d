"""CPU (fp32 reference path) engine tests: config 1 end to end, TP over gloo, DP replicas."""

import os

import pytest
import torch

from uno_b200 import LLM, SamplingParams


def tiny_llm(**kw):
    base = dict(device="cpu", max_num_seqs=8, max_model_len=256, kvcache_block_size=64,
                dummy_lora_rank=8, dummy_lora_alpha=16, max_diffusion_block_size=4)
    base.update(kw)
    return LLM("preset:tiny-qwen3", **base)


def zipf_prompts(n, length, seed=0):
    g = torch.Generator().manual_seed(seed)
    import numpy as np

    rng = np.random.default_rng(seed)
    return [[int(x) % 4000 + 1 for x in rng.zipf(1.1, size=length)] for _ in range(n)]


def test_config1_end_to_end_linear():
    llm = tiny_llm()
    sp = SamplingParams(temperature=1.0, max_tokens=64, diffusion_block_size=4, mask_token_id=4095,
                        ignore_eos=True, seed=0)
    out = llm.generate(zipf_prompts(2, 32), sp, use_tqdm=False)
    st = llm.last_generate_stats
    llm.exit()
    assert all(len(o["token_ids"]) >= 64 for o in out)
    assert all(isinstance(o["text"], str) for o in out)
    # TPF accounting: 2 forwards per cycle, at least one token committed per cycle
    assert st["forwards"] % 2 == 0 and st["accepts"] >= st["forwards"] // 2


def test_seeded_runs_reproduce():
    sp = SamplingParams(temperature=1.0, max_tokens=20, diffusion_block_size=4, mask_token_id=4095,
                        ignore_eos=True, seed=5)
    a = tiny_llm()
    ra = [o["token_ids"] for o in a.generate(zipf_prompts(2, 16), sp, use_tqdm=False)]
    a.exit()
    b = tiny_llm()
    rb = [o["token_ids"] for o in b.generate(zipf_prompts(2, 16), sp, use_tqdm=False)]
    b.exit()
    assert ra == rb


def test_greedy_psi_spec_equals_greedy_ar():
    """Greedy Psi-Spec commits exactly the greedy AR continuation."""
    llm = tiny_llm()
    prompts = zipf_prompts(3, 20, seed=1)
    ar = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=24, diffusion_block_size=1,
                                              mask_token_id=4095, ignore_eos=True), use_tqdm=False)
    ps = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=24, diffusion_block_size=4,
                                              mask_token_id=4095, ignore_eos=True), use_tqdm=False)
    llm.exit()
    for a, b in zip(ar, ps):
        n = min(len(a["token_ids"]), len(b["token_ids"]))
        assert a["token_ids"][:n] == b["token_ids"][:n]


def test_tree_sampler_cpu():
    llm = tiny_llm(tree_verify_size=8, tree_candidate_top_k=3, max_diffusion_block_size=4)
    sp = SamplingParams(temperature=1.0, max_tokens=20, diffusion_block_size=4, mask_token_id=4095,
                        ignore_eos=True, seed=2)
    out = llm.generate(zipf_prompts(2, 12, seed=3), sp, use_tqdm=False)
    st = llm.last_generate_stats
    llm.exit()
    assert all(len(o["token_ids"]) >= 20 for o in out)
    assert st["accepts"] >= st["forwards"] // 2


def test_prefix_cache_reuse_and_stop_tokens():
    llm = tiny_llm(kvcache_block_size=64)
    prompt = list(range(1, 140))
    sp = SamplingParams(temperature=1.0, max_tokens=8, diffusion_block_size=4, mask_token_id=4095,
                        ignore_eos=True, seed=1)
    llm.generate([prompt], sp, use_tqdm=False)
    bm = llm.scheduler.block_manager
    assert len(bm.hash_to_block_id) >= 2  # two full prompt pages published
    out = llm.generate([prompt + [7]], sp, use_tqdm=False)
    assert len(out[0]["token_ids"]) >= 8
    # stop tokens end a request and are trimmed from the output
    first = out[0]["token_ids"][0]
    sp_stop = SamplingParams(temperature=0.0, max_tokens=30, diffusion_block_size=4, mask_token_id=4095,
                             stop_token_ids=[first])
    out2 = llm.generate([prompt + [7]], sp_stop, use_tqdm=False)
    llm.exit()
    assert first not in out2[0]["token_ids"][-1:]


def test_tensor_parallel_gloo_matches_single_rank():
    prompts = zipf_prompts(2, 24, seed=4)
    sp = SamplingParams(temperature=0.0, max_tokens=12, diffusion_block_size=4, mask_token_id=4095,
                        ignore_eos=True)
    one = tiny_llm()
    r1 = [o["token_ids"] for o in one.generate(prompts, sp, use_tqdm=False)]
    one.exit()
    two = tiny_llm(tensor_parallel_size=2)
    r2 = [o["token_ids"] for o in two.generate(prompts, sp, use_tqdm=False)]
    two.exit()
    for a, b in zip(r1, r2):
        n = min(len(a), len(b))
        # greedy decoding: fp32 reduction order may flip a near-tie late, so
        # require the leading tokens to agree
        assert a[:6] == b[:6]


def test_data_parallel_replicas_cpu():
    llm = LLM("preset:tiny-qwen3", data_parallel_size=2, device="cpu", max_num_seqs=4, max_model_len=128,
              kvcache_block_size=64, dummy_lora_rank=8, max_diffusion_block_size=4)
    sp = SamplingParams(temperature=1.0, max_tokens=10, diffusion_block_size=4, mask_token_id=4095,
                        ignore_eos=True, seed=0)
    out = llm.generate(zipf_prompts(5, 10), sp, use_tqdm=False)
    st = llm.last_generate_stats
    llm.exit()
    assert len(out) == 5 and all(len(o["token_ids"]) >= 10 for o in out)
    assert st["forwards"] > 0


def test_block_fp8_checkpoint_loads_dequantized(tmp_path):
    """A block-FP8 checkpoint (128x128 weight blocks + scale_inv) loads as its dequantized weights."""
    import json

    from safetensors.torch import save_file

    from uno_b200.models.decoder import build_model
    from uno_b200.utils.hf_compat import model_config_from_dict
    from uno_b200.parallel.state import set_tp_state
    from uno_b200.utils.loader import dummy_init, load_model

    set_tp_state(0, 1)  # single-rank shapes, whatever an earlier test left behind
    raw = dict(model_type="qwen3", vocab_size=512, hidden_size=256, intermediate_size=768, num_hidden_layers=1,
               num_attention_heads=4, num_key_value_heads=2, head_dim=64, eos_token_id=1, torch_dtype="float32")
    cfg = model_config_from_dict(raw)
    src = build_model(cfg)
    dummy_init(src, seed=3, std=0.05)
    sd = src.state_dict()
    hf = {n: t.contiguous() for n, t in sd.items() if "qkv_proj" not in n and "gate_up_proj" not in n}
    pre = "model.layers.0."
    qkv, gu = sd[pre + "self_attn.qkv_proj.weight"], sd[pre + "mlp.gate_up_proj.weight"]
    hf[pre + "self_attn.q_proj.weight"], hf[pre + "self_attn.k_proj.weight"], hf[pre + "self_attn.v_proj.weight"] = \
        qkv[:256].clone(), qkv[256:384].clone(), qkv[384:].clone()
    hf[pre + "mlp.gate_proj.weight"], hf[pre + "mlp.up_proj.weight"] = gu[:768].clone(), gu[768:].clone()

    def up(s):
        return s.repeat_interleave(128, 0).repeat_interleave(128, 1)

    deq = {}
    for name in [n for n in hf if n.endswith("_proj.weight")]:
        w = hf[name].float()
        scale = w.view(w.shape[0] // 128, 128, w.shape[1] // 128, 128).abs().amax(dim=(1, 3)).clamp_min(1e-8) / 448.0
        q = (w / up(scale)).to(torch.float8_e4m3fn)
        hf[name], hf[name + "_scale_inv"] = q, scale
        deq[name] = q.float() * up(scale)
    d = tmp_path / "fp8"
    d.mkdir()
    save_file(hf, str(d / "model.safetensors"))
    (d / "config.json").write_text(json.dumps(dict(raw, quantization_config={
        "quant_method": "fp8", "weight_block_size": [128, 128], "activation_scheme": "dynamic"})))
    dst = build_model(cfg)
    load_model(dst, str(d))
    got = dst.state_dict()
    want_qkv = torch.cat([deq[pre + f"self_attn.{x}_proj.weight"] for x in "qkv"])
    want_gu = torch.cat([deq[pre + "mlp.gate_proj.weight"], deq[pre + "mlp.up_proj.weight"]])
    assert torch.allclose(got[pre + "self_attn.qkv_proj.weight"], want_qkv)
    assert torch.allclose(got[pre + "mlp.gate_up_proj.weight"], want_gu)
    assert torch.allclose(got[pre + "mlp.down_proj.weight"], deq[pre + "mlp.down_proj.weight"])
    # quantisation error stays at the fp8 level
    assert ((want_qkv - qkv).abs().max() / qkv.abs().max()).item() < 0.07


def test_bench_configs_and_tool_modules_parse(monkeypatch):
    """bench.py maps each BASELINE config to its workload; the profiling tools import without a GPU."""
    import importlib
    import sys

    root = __import__("os").path.dirname(__import__("os").path.dirname(__import__("os").path.abspath(__file__)))
    sys.path.insert(0, root)
    bench = importlib.import_module("bench")
    monkeypatch.setattr(sys, "argv", ["bench.py"])
    a = bench.parse()
    assert (a.batch, a.block, a.new_tokens, a.config) == (64, 8, 2048, "qwen3-8b")
    monkeypatch.setattr(sys, "argv", ["bench.py", "--config", "uno-0.9b-dp"])
    a = bench.parse()
    assert (a.batch, a.block, a.new_tokens) == (256, 16, 1024)
    assert bench.engine_kwargs(a, 1)["dummy_lora_rank"] == 32
    monkeypatch.setattr(sys, "argv", ["bench.py", "--sampler", "tree"])
    a = bench.parse()
    assert (a.batch, a.block, a.new_tokens) == (1, 9, 4096)
    kc = importlib.import_module("uno_b200.ops.kernel_cases")
    assert set(kc.CASES) >= {"layer-gemms", "lm-head", "decode-attention", "sampling", "train-attention"}
    importlib.import_module("uno_b200.parallel.comm_cases")
