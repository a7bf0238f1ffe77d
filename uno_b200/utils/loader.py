"""Checkpoint loading: HF safetensors (or .bin) and random ("dummy") init.

Name mapping follows the reference loader (``nano_vllm_uno/utils/loader.py:15-55``):
``q_proj/k_proj/v_proj`` load into shards of ``qkv_proj`` and
``gate_proj/up_proj`` into shards of ``gate_up_proj`` through each parameter's
``weight_loader``, which also applies the tensor-parallel slicing.

``dummy_init`` fills weights with N(0, std) on their device (norm weights stay
1) from a seeded generator, so a benchmark needs no checkpoint on disk and every
TP rank draws the same full tensor before slicing its shard.
"""

from __future__ import annotations

import logging
import os
from glob import glob

import torch
from torch import nn

logger = logging.getLogger(__name__)


def _checkpoint_files(path: str) -> list[str]:
    files = sorted(glob(os.path.join(path, "*.safetensors")))
    if files:
        return files
    return sorted(glob(os.path.join(path, "*.bin")))


def iter_checkpoint(path: str):
    from safetensors import safe_open

    for file in _checkpoint_files(path):
        if file.endswith(".safetensors"):
            with safe_open(file, "pt", "cpu") as fh:
                for key in fh.keys():
                    yield key, fh.get_tensor(key)
        else:
            for key, value in torch.load(file, map_location="cpu").items():
                yield key, value


FP8_BLOCK = 128


def quantization_config(path: str) -> dict | None:
    """The checkpoint's ``quantization_config`` (``config.json``), validated; None when unquantized.

    Supported: ``quant_method: fp8`` with ``weight_block_size: [128, 128]`` and dynamic activations
    (the registry of ``nano_vllm_uno/layers/quantization.py:79-150``)."""
    import json

    cfg_path = os.path.join(path, "config.json")
    if not os.path.isfile(cfg_path):
        return None
    with open(cfg_path, encoding="utf-8") as fh:
        q = json.load(fh).get("quantization_config")
    if not q:
        return None
    method = q.get("quant_method")
    if method != "fp8":
        raise ValueError(f"unsupported quantization method {method!r} (registered: fp8)")
    if list(q.get("weight_block_size") or []) != [FP8_BLOCK, FP8_BLOCK]:
        raise ValueError("block FP8 checkpoints need weight_block_size=[128, 128]")
    if q.get("activation_scheme", "dynamic") != "dynamic":
        raise ValueError("block FP8 checkpoints need activation_scheme='dynamic'")
    return q


def dequantize_block_fp8(weight: torch.Tensor, scale_inv: torch.Tensor, dtype=torch.bfloat16) -> torch.Tensor:
    """``W[n, k] = fp8[n, k] * scale_inv[n // 128, k // 128]`` (128 x 128 weight blocks)."""
    N, K = weight.shape
    if N % FP8_BLOCK or K % FP8_BLOCK or scale_inv.shape != (N // FP8_BLOCK, K // FP8_BLOCK):
        raise ValueError(f"block FP8 weight {tuple(weight.shape)} does not match scales {tuple(scale_inv.shape)}")
    s = scale_inv.float().repeat_interleave(FP8_BLOCK, 0).repeat_interleave(FP8_BLOCK, 1)
    return (weight.float() * s).to(dtype)


def load_model(model: nn.Module, path: str) -> int:
    """Load every tensor of the checkpoint at ``path``; returns the count loaded.

    Block-FP8 checkpoints (``quantization_config.quant_method == "fp8"``) are
    dequantized to the model's dtype while loading: every ``*.weight`` stored
    as float8_e4m3 is multiplied by its ``*.weight_scale_inv`` blocks, then
    goes through the usual packing and tensor-parallel slicing, and the
    projections run on the bf16 kernels."""
    if not os.path.isdir(path):
        raise ValueError(f"load_model: not a directory: {path}")
    if not _checkpoint_files(path):
        raise FileNotFoundError(f"no *.safetensors or *.bin files in {path}")
    mapping = getattr(model, "packed_modules_mapping", {})
    scales = {}
    if quantization_config(path) is not None:
        scales = {name[: -len("_scale_inv")]: t for name, t in iter_checkpoint(path)
                  if name.endswith(".weight_scale_inv")}
    loaded = 0
    for name, tensor in iter_checkpoint(path):
        if name.endswith("rotary_emb.inv_freq") or name.endswith(".weight_scale_inv"):
            continue
        if tensor.dtype == torch.float8_e4m3fn:
            if name not in scales:
                raise ValueError(f"{name} is float8 but the checkpoint has no {name}_scale_inv")
            tensor = dequantize_block_fp8(tensor, scales[name], dtype=torch.float32)  # cast by the copy
        if name == "lm_head.weight" and model.config.tie_word_embeddings:
            continue
        for short, (packed, shard_id) in mapping.items():
            if short in name:
                param = model.get_parameter(name.replace(short, packed))
                param.weight_loader(param, tensor, shard_id)
                break
        else:
            param = model.get_parameter(name)
            loader = getattr(param, "weight_loader", None)
            if loader is None:
                param.data.copy_(tensor)
            else:
                loader(param, tensor)
        loaded += 1
    return loaded


@torch.no_grad()
def dummy_init(model: nn.Module, seed: int = 0, std: float = 0.02) -> None:
    """Random-init every 2-D weight from the full (unsharded) distribution.

    Each rank generates the full-size tensor with the same seed on the
    parameter's device and lets the parameter's ``weight_loader`` cut its shard,
    so the TP layout sees one consistent random model.
    """
    gen_device = next(model.parameters()).device
    gen = torch.Generator(device=gen_device)
    for idx, (name, param) in enumerate(model.named_parameters()):
        if param.dim() == 1:
            if name.endswith("bias"):
                param.data.zero_()
            else:
                param.data.fill_(1.0)
            continue
        gen.manual_seed(seed * 1_000_003 + idx)
        full_shape = _full_shape(model, name, param)
        full = torch.empty(full_shape, device=gen_device, dtype=torch.float32)
        full.normal_(0.0, std, generator=gen)
        full = full.to(param.dtype)
        loader = getattr(param, "weight_loader", None)
        if loader is None or full_shape == tuple(param.shape):
            param.data.copy_(full if full_shape == tuple(param.shape) else full[: param.shape[0]])
        else:
            _load_full(param, full, loader, model, name)


def _full_shape(model, name, param) -> tuple[int, ...]:
    module = model.get_submodule(name.rsplit(".", 1)[0])
    tp = getattr(module, "tp_size", 1)
    shape = list(param.shape)
    tp_dim = getattr(module, "tp_dim", None)
    if tp > 1:
        if tp_dim == 0 or module.__class__.__name__ in ("VocabParallelEmbedding", "ParallelLMHead"):
            shape[0] *= tp
        elif tp_dim == 1:
            shape[1] *= tp
    return tuple(shape)


def _load_full(param, full, loader, model, name) -> None:
    module = model.get_submodule(name.rsplit(".", 1)[0])
    from uno_b200.layers.linear import MergedColumnParallelLinear, QKVParallelLinear

    if isinstance(module, QKVParallelLinear):
        hd = module.head_size
        tp = module.tp_size
        q = module.num_heads * hd * tp
        kv = module.num_kv_heads * hd * tp
        loader(param, full[:q], "q")
        loader(param, full[q:q + kv], "k")
        loader(param, full[q + kv:], "v")
    elif isinstance(module, MergedColumnParallelLinear):
        off = 0
        for i, size in enumerate(module.output_sizes):
            loader(param, full[off:off + size], i)
            off += size
    else:
        loader(param, full)
