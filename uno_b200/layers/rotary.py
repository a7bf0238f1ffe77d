"""Rotary position embedding tables (default and YaRN).

Same math as the reference ``layers/rotary_embedding.py:8-148``: NeoX
half-split rotation, ``inv_freq = theta^(-2i/d)``; YaRN blends interpolated and
extrapolated frequencies with a linear ramp between the beta_fast/beta_slow
correction dimensions and scales cos/sin by the attention factor
(``0.1 ln(factor) + 1`` unless given).  The table is stored as one
``[max_pos, head_dim]`` fp32 tensor ``[cos | sin]`` that the fused
QKV epilogue kernel indexes by position.
"""

from __future__ import annotations

import math
from functools import lru_cache

import torch


def _yarn_params(rope_scaling: dict, max_position: int):
    factor = float(rope_scaling["factor"])
    if factor <= 0:
        raise ValueError(f"YaRN factor must be positive, got {factor}")
    original = int(rope_scaling.get("original_max_position_embeddings") or max_position)
    if original <= 0:
        raise ValueError("YaRN original_max_position_embeddings must be positive")
    attn = rope_scaling.get("attention_factor")
    if attn is None:
        attn = 1.0 if factor <= 1 else 0.1 * math.log(factor) + 1.0
    return (
        factor,
        original,
        float(attn),
        float(rope_scaling.get("beta_fast") or 32.0),
        float(rope_scaling.get("beta_slow") or 1.0),
        bool(rope_scaling.get("truncate", True)),
    )


def rope_inv_freq(rotary_dim: int, base: float, rope_scaling: dict | None, max_position: int):
    """Return (inv_freq [rotary_dim/2] fp32, attention_factor)."""
    exponents = torch.arange(0, rotary_dim, 2, dtype=torch.float32) / rotary_dim
    pos_freqs = float(base) ** exponents
    if rope_scaling is None:
        return 1.0 / pos_freqs, 1.0
    kind = rope_scaling.get("rope_type", rope_scaling.get("type"))
    if kind in (None, "default"):
        theta = rope_scaling.get("rope_theta")
        if theta is not None and float(theta) != float(base):
            raise NotImplementedError("default RoPE descriptor disagrees with rope_theta")
        return 1.0 / pos_freqs, 1.0
    if kind != "yarn":
        raise NotImplementedError(f"Unsupported rope_scaling={rope_scaling!r}")
    factor, original, attn, beta_fast, beta_slow, truncate = _yarn_params(rope_scaling, max_position)

    def correction_dim(rotations: float) -> float:
        return rotary_dim * math.log(original / (rotations * 2 * math.pi)) / (2 * math.log(base))

    low, high = correction_dim(beta_fast), correction_dim(beta_slow)
    if truncate:
        low, high = math.floor(low), math.ceil(high)
    low, high = max(low, 0), min(high, rotary_dim - 1)
    if low == high:
        high += 0.001
    ramp = ((torch.arange(rotary_dim // 2, dtype=torch.float32) - low) / (high - low)).clamp(0, 1)
    extrapolation = 1.0 / pos_freqs
    interpolation = 1.0 / (factor * pos_freqs)
    keep = 1.0 - ramp  # weight of the extrapolated (unscaled) frequency
    inv_freq = interpolation * (1.0 - keep) + extrapolation * keep
    return inv_freq, attn


@lru_cache(maxsize=8)
def _cos_sin_cpu(head_dim: int, max_position: int, base: float, scaling_key) -> torch.Tensor:
    rope_scaling = dict(scaling_key) if scaling_key is not None else None
    inv_freq, attn = rope_inv_freq(head_dim, base, rope_scaling, max_position)
    t = torch.arange(max_position, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    return torch.cat([freqs.cos() * attn, freqs.sin() * attn], dim=-1).contiguous()


def cos_sin_cache(head_dim: int, max_position: int, base: float, rope_scaling: dict | None,
                  device: torch.device | str = "cpu") -> torch.Tensor:
    """``[max_position, head_dim]`` fp32 table: first half cos, second half sin."""
    key = None
    if rope_scaling is not None:
        key = tuple(sorted((k, v) for k, v in rope_scaling.items() if not isinstance(v, (dict, list))))
    return _cos_sin_cpu(int(head_dim), int(max_position), float(base), key).to(device)
