"""Trainable gated LoRA for the frozen decoder.

Equivalent of ``training/lora.py:66-179``: LoRA on q,k,v,o,gate,up,down
(``all``), PEFT initialisation (A: Kaiming-uniform with a = sqrt(5), B: zero),
fp32 parameters, scaling ``alpha / r``, and a *token-wise router*: the LoRA
branch of every projection is multiplied by a per-row mask (the noisy copy
of the Uno layout), so clean rows see the frozen base model only.

Adapters are written in the PEFT layout that the inference loader reads
(``base_model.model.model.layers.N.{self_attn,mlp}.X_proj.lora_{A,B}.weight``
plus ``adapter_config.json``), so a checkpoint serves directly as the
engine's ``gated_lora_path``.
"""

from __future__ import annotations

import math
import os

import torch
from torch import nn

from uno_b200.train.config import LoraSettings

_ATTN = ("q_proj", "k_proj", "v_proj", "o_proj")


def projection_shapes(cfg) -> dict[str, tuple[int, int]]:
    q_out = cfg.num_attention_heads * cfg.head_dim
    kv_out = cfg.num_key_value_heads * cfg.head_dim
    return {"q_proj": (cfg.hidden_size, q_out), "k_proj": (cfg.hidden_size, kv_out),
            "v_proj": (cfg.hidden_size, kv_out), "o_proj": (q_out, cfg.hidden_size),
            "gate_proj": (cfg.hidden_size, cfg.intermediate_size),
            "up_proj": (cfg.hidden_size, cfg.intermediate_size),
            "down_proj": (cfg.intermediate_size, cfg.hidden_size)}


class TrainableLoRA(nn.Module):
    """``A[layer][proj] [r, in]`` and ``B[layer][proj] [out, r]`` in fp32."""

    def __init__(self, cfg, settings: LoraSettings, device=None, seed: int = 0):
        super().__init__()
        settings.validate()
        self.settings = settings
        self.rank = settings.rank
        self.alpha = settings.resolved_alpha
        self.scaling = self.alpha / self.rank
        self.modules_ = settings.modules
        shapes = projection_shapes(cfg)
        gen = torch.Generator().manual_seed(seed)
        self.A = nn.ParameterDict()
        self.B = nn.ParameterDict()
        bound = 1.0  # kaiming_uniform(a=sqrt(5)) bound = 1 / sqrt(fan_in)
        for li in range(cfg.num_hidden_layers):
            for proj in self.modules_:
                fan_in, fan_out = shapes[proj]
                bound = 1.0 / math.sqrt(fan_in)
                a = (torch.rand(self.rank, fan_in, generator=gen) * 2 - 1) * bound
                self.A[self._key(li, proj)] = nn.Parameter(a.to(device))
                self.B[self._key(li, proj)] = nn.Parameter(torch.zeros(fan_out, self.rank, device=device))
        self.num_layers = cfg.num_hidden_layers

    @staticmethod
    def _key(layer: int, proj: str) -> str:
        return f"{layer}_{proj}"

    def has(self, layer: int, proj: str) -> bool:
        return self._key(layer, proj) in self.A

    def delta(self, layer: int, proj: str, x: torch.Tensor, row_mask: torch.Tensor | None) -> torch.Tensor:
        """``scaling * ((x A^T) * mask) B^T`` in fp32."""
        k = self._key(layer, proj)
        h = x.float() @ self.A[k].t()
        if row_mask is not None:
            h = h * row_mask.to(h.dtype)[..., None]
        return (h @ self.B[k].t()) * self.scaling

    # ------------------------------------------------------------- export
    def peft_state(self) -> dict[str, torch.Tensor]:
        out = {}
        for li in range(self.num_layers):
            for proj in self.modules_:
                scope = "self_attn" if proj in _ATTN else "mlp"
                stem = f"base_model.model.model.layers.{li}.{scope}.{proj}"
                out[f"{stem}.lora_A.weight"] = self.A[self._key(li, proj)].detach().float().cpu()
                out[f"{stem}.lora_B.weight"] = self.B[self._key(li, proj)].detach().float().cpu()
        return out

    def save(self, path: str, base_model: str | None = None) -> None:
        from uno_b200.utils.lora import save_lora_adapter

        save_lora_adapter(path, self.peft_state(), self.rank, self.alpha, list(self.modules_), base_model)

    @torch.no_grad()
    def load(self, path: str) -> None:
        from uno_b200.utils.lora import _load_tensors

        tensors = _load_tensors(path)
        for li in range(self.num_layers):
            for proj in self.modules_:
                scope = "self_attn" if proj in _ATTN else "mlp"
                stem = f"base_model.model.model.layers.{li}.{scope}.{proj}"
                self.A[self._key(li, proj)].copy_(tensors[f"{stem}.lora_A.weight"])
                self.B[self._key(li, proj)].copy_(tensors[f"{stem}.lora_B.weight"])


def adapter_exists(path: str) -> bool:
    return os.path.isfile(os.path.join(path, "adapter_config.json"))
