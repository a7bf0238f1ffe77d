"""End-to-end GPU model and engine checks against the fp32 CPU reference path."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def small_cfg():
    from uno_b200.utils.hf_compat import ModelConfig

    return ModelConfig(model_type="qwen3", vocab_size=2048, hidden_size=512, intermediate_size=1024,
                       num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2, head_dim=128,
                       max_position_embeddings=2048, eos_token_id=None, mask_token_id=2000)


def _models():
    from uno_b200.models.decoder import build_model
    from uno_b200.ops import cuda as C
    from uno_b200.utils.loader import dummy_init
    from uno_b200.utils.lora import dummy_lora

    cfg = small_cfg()
    cpu = build_model(cfg)
    dummy_init(cpu, seed=3, std=0.05)
    dummy_lora(cpu, rank=64, alpha=128, seed=4, std=0.05)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    with torch.device("cuda"):
        gpu = build_model(cfg)
    torch.set_default_dtype(prev)
    gpu.load_state_dict({k: v.to(torch.bfloat16) for k, v in cpu.state_dict().items()}, strict=False)
    for lc, lg in zip(cpu.modules(), gpu.modules()):
        for s in getattr(lc, "lora_slices", []):
            lg.add_lora_slice(s.A, s.B, s.scaling, s.out_start)
        if getattr(lc, "lora_slices", None):
            lg.pack_lora()
    C.prepare_model(gpu)
    return cfg, cpu, gpu


def _caches(cfg, device, dtype, pages=16, page=64):
    kv = torch.zeros(cfg.num_hidden_layers, 2, pages, cfg.num_key_value_heads, page, cfg.head_dim,
                     device=device, dtype=dtype)
    return kv


def _attach(model, kv):
    for i, attn in enumerate(model.attention_layers):
        attn.k_cache, attn.v_cache = kv[i, 0], kv[i, 1]


def _rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).norm() / b.norm()).item()


def test_model_prefill_and_block_decode_match_reference():
    from uno_b200.layers.meta import ForwardMeta, Mode, causal_suffix_masks

    cfg, cpu, gpu = _models()
    page = 64
    kv_c = _caches(cfg, "cpu", torch.float32)
    kv_g = _caches(cfg, "cuda", torch.bfloat16)
    _attach(cpu, kv_c)
    _attach(gpu, kv_g)
    lens = [37, 90]
    tables = torch.tensor([[0, 1, -1], [2, 3, 4]], dtype=torch.int32)
    ids = torch.randint(1, 2000, (sum(lens),))
    pos = torch.cat([torch.arange(n) for n in lens])
    slots = torch.cat([tables[b, torch.arange(n) // page].long() * page + torch.arange(n) % page
                       for b, n in enumerate(lens)])
    cu = torch.tensor([0, lens[0], sum(lens)], dtype=torch.int32)

    def meta_pf(dev):
        return ForwardMeta(mode=Mode.PREFILL, positions=pos.to(dev), slot_mapping=slots.to(dev),
                           block_tables=tables.to(dev), cu_seqlens_q=cu.to(dev), cu_seqlens_k=cu.to(dev),
                           max_seqlen_q=max(lens), max_seqlen_k=max(lens),
                           logits_indices=(cu[1:] - 1).long().to(dev))

    with torch.inference_mode():
        lc = cpu.compute_logits(cpu(ids, meta_pf("cpu")), meta_pf("cpu"))
        lg = gpu.compute_logits(gpu(ids.cuda(), meta_pf("cuda")), meta_pf("cuda"))
    assert _rel(lg, lc) < 3e-2
    # block decode of L=4 with LoRA on rows 1..3
    L = 4
    blk = torch.randint(1, 2000, (2, L))
    starts = torch.tensor(lens)
    bpos = (starts[:, None] + torch.arange(L)[None]).reshape(-1)
    bslots = torch.cat([tables[b, bpos.view(2, L)[b] // page].long() * page + bpos.view(2, L)[b] % page
                        for b in range(2)])
    mask = torch.tensor([0.0, 1, 1, 1] * 2)

    def meta_blk(dev, lora):
        return ForwardMeta(mode=Mode.BLOCK, positions=bpos.to(dev), slot_mapping=bslots.to(dev),
                           block_tables=tables.to(dev), prefix_lens=starts.to(torch.int32).to(dev),
                           suffix_mask=causal_suffix_masks(L, dev).repeat(2, 1), seqlen_q=L,
                           lora_mask=mask.to(dev) if lora else None, max_kv=200)

    for lora in (False, True):
        with torch.inference_mode():
            lc = cpu.compute_logits(cpu(blk.reshape(-1), meta_blk("cpu", lora)))
            lg = gpu.compute_logits(gpu(blk.reshape(-1).cuda(), meta_blk("cuda", lora)))
        assert _rel(lg, lc) < 3e-2, lora
    # LoRA must change the noisy rows and leave the seed rows untouched
    with torch.inference_mode():
        a = gpu.compute_logits(gpu(blk.reshape(-1).cuda(), meta_blk("cuda", False)))
        b = gpu.compute_logits(gpu(blk.reshape(-1).cuda(), meta_blk("cuda", True)))
    a, b = a.view(2, L, -1), b.view(2, L, -1)
    assert torch.allclose(a[:, 0].float(), b[:, 0].float(), atol=1e-2)
    assert (a[:, 1:] - b[:, 1:]).abs().max() > 1e-2


def test_engine_generate_graphs_and_eager_gpu():
    from uno_b200 import LLM, SamplingParams
    from uno_b200.ops import cuda as C

    cfg = small_cfg()
    prompts = [list(range(1, 40)), list(range(100, 130)), [5, 6, 7]]
    sp = SamplingParams(temperature=1.0, max_tokens=24, diffusion_block_size=4, mask_token_id=2000,
                        ignore_eos=True, seed=7)
    res = {}
    for eager in (True, False):
        llm = LLM(cfg, max_num_seqs=4, max_model_len=256, kvcache_block_size=64, dummy_lora_rank=64,
                  max_diffusion_block_size=4, cuda_graph_batch_sizes=[1, 2, 4], enforce_eager=eager,
                  gpu_memory_utilization=0.2, num_kvcache_blocks=64)
        out = llm.generate(prompts, sp, use_tqdm=False, detokenize=False)
        res[eager] = [o["token_ids"] for o in out]
        stats = llm.last_generate_stats
        if not eager:
            assert llm.model_runner.cuda_graph_hits > 0
        llm.exit()
        assert all(len(t) >= 24 for t in res[eager])
        assert stats["forwards"] > 0 and stats["accepts"] >= stats["forwards"] // 2
    # graphs replay the exact same kernels: identical samples
    assert res[True] == res[False]
    assert C.error_flag() == 0


def test_engine_tree_sampler_gpu():
    from uno_b200 import LLM, SamplingParams

    cfg = small_cfg()
    llm = LLM(cfg, max_num_seqs=2, max_model_len=256, kvcache_block_size=64, dummy_lora_rank=64,
              max_diffusion_block_size=5, tree_verify_size=16, tree_candidate_top_k=4,
              enforce_eager=True, gpu_memory_utilization=0.2, num_kvcache_blocks=32)
    sp = SamplingParams(temperature=1.0, max_tokens=20, diffusion_block_size=5, mask_token_id=2000,
                        ignore_eos=True, seed=3)
    out = llm.generate([[1, 2, 3, 4], [9, 8, 7]], sp, use_tqdm=False, detokenize=False)
    st = llm.last_generate_stats
    llm.exit()
    assert all(len(o["token_ids"]) >= 20 for o in out)
    assert st["accepts"] / st["forwards"] >= 0.5
