"""End to end against Hugging Face Transformers (CPU, fp32, BASELINE config 1 shape).

A random-init ``Qwen3ForCausalLM`` written with ``save_pretrained`` is loaded
by this framework from the same directory (HF safetensors layout and config).
Greedy decoding through ``LLM.generate`` -- plain autoregressive (block 1),
linear Psi-Spec with diffusion blocks of 4 and the tree sampler, whose output
is the AR greedy output whatever the drafts -- must reproduce ``transformers``' own greedy
``generate`` token for token.  The checkpoint carries no diffusion adapter, so
the engine adds a random gated LoRA for the drafts (``dummy_lora_rank``).
"""

import pytest
import torch

transformers = pytest.importorskip("transformers")

NEW = 24


@pytest.fixture(scope="module")
def hf_dir(tmp_path_factory):
    from transformers import Qwen3Config, Qwen3ForCausalLM

    torch.manual_seed(0)
    cfg = Qwen3Config(vocab_size=4096, hidden_size=256, intermediate_size=768, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=64, rope_theta=1e6,
                      rms_norm_eps=1e-6, max_position_embeddings=512, tie_word_embeddings=False)
    model = Qwen3ForCausalLM(cfg).eval()
    path = tmp_path_factory.mktemp("hf_qwen3_tiny")
    model.save_pretrained(path, safe_serialization=True)
    return path, model


PROMPTS = [[5, 17, 300, 42, 9, 1000, 7, 88], [1203, 4, 4, 77, 3050, 12, 600, 2, 31, 999, 18, 250]]


@pytest.mark.parametrize("block,tree", [(1, False), (4, False), (4, True)])
def test_greedy_generation_matches_transformers(hf_dir, block, tree):
    from uno_b200 import LLM, SamplingParams

    path, model = hf_dir
    want = []
    with torch.no_grad():
        for p in PROMPTS:
            ids = model.generate(torch.tensor([p]), max_new_tokens=NEW, do_sample=False, eos_token_id=None,
                                 pad_token_id=0)
            want.append(ids[0, len(p):].tolist())
    extra = {"tree_verify_size": 8, "tree_candidate_top_k": 3} if tree else {}
    llm = LLM(str(path), device="cpu", max_num_seqs=2, max_model_len=128, kvcache_block_size=64,
              dummy_lora_rank=8, max_diffusion_block_size=4, **extra)
    try:
        sp = SamplingParams(temperature=0.0, max_tokens=NEW, diffusion_block_size=block, mask_token_id=4000,
                            ignore_eos=True)
        got = [o["token_ids"][:NEW] for o in llm.generate(PROMPTS, sp, use_tqdm=False, detokenize=False)]
    finally:
        llm.exit()
    assert got == want
