"""Gated-LoRA ("diffusion weights") adapter loading.

Reads a PEFT adapter directory: ``adapter_config.json`` (``r``, ``lora_alpha``,
``target_modules``) plus ``adapter_model*.safetensors`` (or ``.bin``) with keys
``base_model.model.model.layers.N.{self_attn,mlp}.X_proj.lora_{A,B}.weight``
(format of ``nano_vllm_uno/utils/lora.py:29-195`` and ``training/lora.py:66-133``).
Each pair becomes a slice of the fused module (q/k/v -> qkv_proj at the q/k/v
output offset; gate/up -> gate_up_proj at the shard offset; o/down as is) with
scaling ``alpha / r``.  Tensor parallel sharding: column-parallel layers keep A
whole and split B by rows; row-parallel layers split A by columns.

``dummy_lora`` attaches a random adapter of the given rank to every linear
(benchmarks with random-init weights).
"""

from __future__ import annotations

import json
import os
from glob import glob

import torch
from torch import nn

from uno_b200.layers.linear import MergedColumnParallelLinear, QKVParallelLinear

_QKV = ("q_proj", "k_proj", "v_proj")
_GATE_UP = {"gate_proj": 0, "up_proj": 1}


def _adapter_files(path: str) -> list[str]:
    files = sorted(glob(os.path.join(path, "adapter_model*.safetensors")))
    if not files:
        files = sorted(glob(os.path.join(path, "adapter_model*.bin")))
    if not files:
        raise FileNotFoundError(f"No adapter_model safetensors/bin file found in {path}")
    return files


def _load_tensors(path: str) -> dict[str, torch.Tensor]:
    from safetensors import safe_open

    out: dict[str, torch.Tensor] = {}
    for file in _adapter_files(path):
        if file.endswith(".safetensors"):
            with safe_open(file, "pt", "cpu") as fh:
                for key in fh.keys():
                    out[key] = fh.get_tensor(key)
        else:
            out.update(torch.load(file, map_location="cpu"))
    return out


def resolve_target(model: nn.Module, prefix: str):
    """Map ``model.layers.N.scope.proj`` to (fused module, output offset)."""
    parts = prefix.split(".")
    if len(parts) != 5 or parts[0] != "model" or parts[1] != "layers":
        raise ValueError(f"Unsupported LoRA tensor prefix: {prefix}")
    layer = model.model.layers[int(parts[2])]
    scope, proj = parts[3], parts[4]
    if scope == "self_attn" and proj in _QKV:
        mod = layer.self_attn.qkv_proj
        assert isinstance(mod, QKVParallelLinear)
        return mod, mod.shard_offset(proj[0])
    if scope == "self_attn" and proj == "o_proj":
        return layer.self_attn.o_proj, 0
    if scope == "mlp" and proj in _GATE_UP:
        mod = layer.mlp.gate_up_proj
        assert isinstance(mod, MergedColumnParallelLinear)
        return mod, mod.shard_offset(_GATE_UP[proj])
    if scope == "mlp" and proj == "down_proj":
        return layer.mlp.down_proj, 0
    raise ValueError(f"Unsupported LoRA target prefix: {prefix}")


def shard_lora(module, A: torch.Tensor, B: torch.Tensor):
    tp, rank = getattr(module, "tp_size", 1), getattr(module, "tp_rank", 0)
    if tp == 1:
        return A, B
    if module.tp_dim == 0:
        return A, B.chunk(tp, dim=0)[rank]
    if module.tp_dim == 1:
        return A.chunk(tp, dim=1)[rank], B
    raise ValueError(f"Cannot shard LoRA for {module}")


def _finish(modules) -> None:
    for m in modules:
        m.pack_lora()


def load_lora_adapter(model: nn.Module, path: str) -> dict:
    with open(os.path.join(path, "adapter_config.json"), "r", encoding="utf-8") as fh:
        cfg = json.load(fh)
    rank = int(cfg["r"])
    alpha = float(cfg["lora_alpha"])
    scaling = alpha / rank
    tensors = _load_tensors(path)
    touched, prefixes = set(), set()
    for key, A in tensors.items():
        if not key.endswith(".lora_A.weight"):
            continue
        stem = key[: -len(".lora_A.weight")]
        bkey = stem + ".lora_B.weight"
        if bkey not in tensors:
            raise KeyError(f"Missing LoRA B tensor for {key}: expected {bkey}")
        prefix = stem.removeprefix("base_model.model.")
        module, start = resolve_target(model, prefix)
        A_s, B_s = shard_lora(module, A, tensors[bkey])
        if module.tp_dim == 0 and module.tp_size > 1:
            pass  # start is already the local offset
        module.add_lora_slice(A_s, B_s, scaling, start)
        touched.add(module)
        prefixes.add(prefix)
    expected = set(cfg.get("target_modules") or [])
    missing = sorted(t for t in expected if not any(p == t or p.endswith("." + t) for p in prefixes))
    if missing:
        raise RuntimeError(f"LoRA adapter missing expected target modules: {missing}")
    _finish(touched)
    return {"path": path, "rank": rank, "alpha": alpha, "scaling": scaling,
            "num_slices": sum(len(m.lora_slices) for m in touched),
            "target_modules": sorted({p.split(".")[-1] for p in prefixes})}


@torch.no_grad()
def dummy_lora(model: nn.Module, rank: int, alpha: float | None = None, seed: int = 1,
               std: float = 0.02) -> dict:
    """Attach a random adapter of ``rank`` to q,k,v,o,gate,up,down of every layer."""
    alpha = float(alpha if alpha is not None else 2 * rank)
    scaling = alpha / rank
    dev = next(model.parameters()).device
    gen = torch.Generator(device=dev)
    touched = set()
    cfg = model.config
    q_out = cfg.num_attention_heads * cfg.head_dim
    kv_out = cfg.num_key_value_heads * cfg.head_dim
    shapes = {
        "q_proj": (cfg.hidden_size, q_out), "k_proj": (cfg.hidden_size, kv_out),
        "v_proj": (cfg.hidden_size, kv_out), "o_proj": (q_out, cfg.hidden_size),
        "gate_proj": (cfg.hidden_size, cfg.intermediate_size),
        "up_proj": (cfg.hidden_size, cfg.intermediate_size),
        "down_proj": (cfg.intermediate_size, cfg.hidden_size),
    }
    for li in range(cfg.num_hidden_layers):
        for proj, (fan_in, fan_out) in shapes.items():
            scope = "mlp" if proj in ("gate_proj", "up_proj", "down_proj") else "self_attn"
            module, start = resolve_target(model, f"model.layers.{li}.{scope}.{proj}")
            gen.manual_seed(seed * 7919 + li * 31 + list(shapes).index(proj))
            A = torch.empty(rank, fan_in, device=dev).normal_(0, std, generator=gen)
            B = torch.empty(fan_out, rank, device=dev).normal_(0, std, generator=gen)
            A_s, B_s = shard_lora(module, A, B)
            module.add_lora_slice(A_s, B_s, scaling, start)
            touched.add(module)
    _finish(touched)
    return {"rank": rank, "alpha": alpha, "scaling": scaling}


def save_lora_adapter(path: str, tensors: dict[str, torch.Tensor], rank: int, alpha: float,
                      target_modules: list[str], base_model: str | None = None) -> None:
    """Write a PEFT-format adapter directory (used by training and tests)."""
    from safetensors.torch import save_file

    os.makedirs(path, exist_ok=True)
    save_file({k: v.contiguous() for k, v in tensors.items()}, os.path.join(path, "adapter_model.safetensors"))
    with open(os.path.join(path, "adapter_config.json"), "w", encoding="utf-8") as fh:
        json.dump({"r": int(rank), "lora_alpha": float(alpha), "target_modules": list(target_modules),
                   "peft_type": "LORA", "base_model_name_or_path": base_model}, fh, indent=2)
