"""Helper launched by tests/test_tp_gpu.py under torch.distributed.run.

Rank 0 builds a small tensor-parallel LLM, runs greedy and sampled Psi-Spec
generation and prints the tokens as one JSON line; other ranks serve as
followers.
"""

import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from uno_b200 import LLM, SamplingParams  # noqa: E402
from uno_b200.engine.worker import serve_follower  # noqa: E402
from uno_b200.utils.hf_compat import ModelConfig  # noqa: E402


def main():
    # 8 KV heads so that the model shards over up to 8 ranks
    cfg = ModelConfig(model_type="qwen3", vocab_size=4096, hidden_size=1024, intermediate_size=2048,
                      num_hidden_layers=3, num_attention_heads=16, num_key_value_heads=8, head_dim=128,
                      max_position_embeddings=2048, eos_token_id=None, mask_token_id=4000)
    eager = os.environ.get("TP_TEST_EAGER", "0") == "1"
    kw = dict(max_num_seqs=4, max_model_len=512, kvcache_block_size=64, dummy_lora_rank=64,
              max_diffusion_block_size=4, cuda_graph_batch_sizes=[1, 2, 4], enforce_eager=eager,
              gpu_memory_utilization=0.3, num_kvcache_blocks=64, distributed_init="env")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    kw["tensor_parallel_size"] = world
    if world == 1:
        kw.pop("distributed_init")
    if int(os.environ.get("RANK", "0")) != 0:
        serve_follower(cfg, **kw)
        return
    llm = LLM(cfg, **kw)
    prompts = [list(range(1, 70)), list(range(200, 230)), [5, 6, 7]]
    # one prefill over 300 rows: several GEMM row tiles, every rank owns rows
    long = [[(7 * i + 3 * j) % 3900 + 1 for j in range(100)] for i in range(3)]
    llm.generate(long, SamplingParams(temperature=0.0, max_tokens=1, diffusion_block_size=4, mask_token_id=4000,
                                      ignore_eos=True), use_tqdm=False)
    logits = llm.model_runner.last_prefill_logits.float().cpu()
    greedy = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=12, diffusion_block_size=4,
                                                  mask_token_id=4000, ignore_eos=True), use_tqdm=False)
    sampled = llm.generate(prompts, SamplingParams(temperature=1.0, max_tokens=24, diffusion_block_size=4,
                                                   mask_token_id=4000, ignore_eos=True, seed=3), use_tqdm=False)
    from uno_b200.ops import cuda

    print(json.dumps({"logits": logits.tolist(), "greedy": [o["token_ids"] for o in greedy],
                      "sampled": [o["token_ids"] for o in sampled],
                      "stats": llm.last_generate_stats, "err": cuda.error_flag()}), flush=True)
    llm.exit()


if __name__ == "__main__":
    main()
