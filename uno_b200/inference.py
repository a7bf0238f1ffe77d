"""Free-form inference CLI: ``python -m uno_b200.inference --model DIR --prompt TEXT``.

Same options and defaults as the reference's ``inference.py:24-145``
(temperature 1.0, top-k 50, top-p 0.95, block 8, CUDA graphs for block sizes
{1, block}); prints one JSON document with the generations, TPS and TPF.
``--prompt-ids`` accepts comma-separated token ids for checkpoints without a
tokenizer (synthetic models), and ``--device cpu`` runs the fp32 reference
path.
"""

from __future__ import annotations

import argparse
import json

from uno_b200.generation import format_chat_prompt, generate, resolve_model_sources
from uno_b200.sampling_params import SamplingParams


def _int_list(value: str | None) -> list[int] | None:
    if value is None:
        return None
    values = [int(v) for v in value.split(",") if v.strip()]
    if not values:
        raise argparse.ArgumentTypeError("expected comma-separated integers")
    return values


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--model", required=True)
    p.add_argument("--model-revision")
    p.add_argument("--tokenizer-path")
    adapter = p.add_mutually_exclusive_group()
    adapter.add_argument("--gated-lora-path")
    adapter.add_argument("--gated-lora-subfolder")
    p.add_argument("--gated-lora-revision")
    p.add_argument("--prompt", action="append", default=[])
    p.add_argument("--prompt-ids", action="append", type=_int_list, default=[])
    p.add_argument("--system-prompt", default="")
    p.add_argument("--max-tokens", type=int, default=256)
    p.add_argument("--max-model-len", type=int, default=32768)
    p.add_argument("--max-num-batched-tokens", type=int)
    p.add_argument("--max-num-seqs", type=int, default=4)
    p.add_argument("--temperature", type=float, default=1.0)
    p.add_argument("--top-k", type=int, default=50)
    p.add_argument("--top-p", type=float, default=0.95)
    p.add_argument("--diffusion-block-size", type=int, default=8)
    p.add_argument("--tree-verify-size", type=int)
    p.add_argument("--tree-candidate-top-k", type=int, default=32)
    p.add_argument("--attention-backend", choices=("fa2", "fa3", "fa4", "native"), default="fa2")
    p.add_argument("--tensor-parallel-size", type=int, default=1)
    p.add_argument("--data-parallel-size", type=int, default=1)
    p.add_argument("--gpu-memory-utilization", type=float, default=0.9)
    p.add_argument("--mask-token-id", type=int)
    p.add_argument("--stop-token-ids", type=_int_list)
    p.add_argument("--noise-mode", choices=("random_uniform", "deterministic_uniform", "mask"),
                   default="random_uniform")
    p.add_argument("--device", choices=("cuda", "cpu"), default="cuda")
    p.add_argument("--hf-cache-dir")
    p.add_argument("--hf-local-files-only", action="store_true")
    p.add_argument("--no-progress", action="store_true")
    return p


def main(argv: list[str] | None = None) -> dict:
    args = build_parser().parse_args(argv)
    if not args.prompt and not args.prompt_ids:
        raise SystemExit("give at least one --prompt or --prompt-ids")
    from uno_b200.utils.hf_compat import load_model_config, load_tokenizer
    from uno_b200.utils.hub import resolve_hf_snapshot
    from uno_b200.utils.model_tokens import resolve_model_token_ids

    model, adapter = resolve_model_sources(args.model, args.gated_lora_path, model_revision=args.model_revision,
                                           gated_lora_subfolder=args.gated_lora_subfolder,
                                           hf_cache_dir=args.hf_cache_dir,
                                           hf_local_files_only=args.hf_local_files_only)
    bundled = args.gated_lora_subfolder is not None
    model_revision = None if bundled else args.model_revision
    adapter_revision = None if bundled else args.gated_lora_revision
    if str(model).startswith("preset:"):
        from uno_b200.models.presets import resolve_preset

        hf_config, model_dir = resolve_preset(str(model)[len("preset:"):]), None
    else:
        model_dir = resolve_hf_snapshot(model, revision=model_revision, cache_dir=args.hf_cache_dir,
                                        local_files_only=args.hf_local_files_only, artifact_name="model")
        hf_config = load_model_config(model_dir)
    tokenizer_path = args.tokenizer_path or model_dir
    tokenizer = load_tokenizer(tokenizer_path, hf_config)
    mask_id, stop_ids, _ = resolve_model_token_ids(model_dir or hf_config, tokenizer,
                                                   mask_token_id=args.mask_token_id,
                                                   stop_token_ids=args.stop_token_ids, noise_mode=args.noise_mode)
    prompts = [format_chat_prompt(tokenizer, [{"role": "user", "content": text}], args.system_prompt)[0]
               for text in args.prompt]
    prompts += [list(ids) for ids in args.prompt_ids]
    sp = SamplingParams(temperature=args.temperature, top_k=args.top_k, top_p=args.top_p,
                        max_tokens=args.max_tokens, stop_token_ids=stop_ids, mask_token_id=mask_id,
                        noise_mode=args.noise_mode, diffusion_block_size=args.diffusion_block_size)
    outputs, metrics = generate(
        prompts, sp, model=model_dir or model, tokenizer_path=tokenizer_path,
        request_max_tokens=[args.max_tokens] * len(prompts), use_tqdm=not args.no_progress,
        model_revision=model_revision, hf_cache_dir=args.hf_cache_dir,
        hf_local_files_only=args.hf_local_files_only, data_parallel_size=args.data_parallel_size,
        tensor_parallel_size=args.tensor_parallel_size, max_num_seqs=args.max_num_seqs,
        max_model_len=args.max_model_len, max_num_batched_tokens=args.max_num_batched_tokens or args.max_model_len,
        gpu_memory_utilization=args.gpu_memory_utilization, attention_backend=args.attention_backend,
        max_diffusion_block_size=args.diffusion_block_size,
        cuda_graph_block_sizes=sorted({1, args.diffusion_block_size}), tree_verify_size=args.tree_verify_size,
        tree_candidate_top_k=args.tree_candidate_top_k, gated_lora_path=adapter,
        gated_lora_revision=adapter_revision, device=args.device)
    result = {"model": args.model, "gated_lora_path": adapter,
              "generations": [o["text"] for o in outputs], **metrics}
    print(json.dumps(result, indent=2, ensure_ascii=False))
    return result


if __name__ == "__main__":
    main()
