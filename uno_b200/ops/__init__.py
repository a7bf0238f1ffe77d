"""Fused operator entry points.

Each op runs the hand-written sm_100a kernel for CUDA tensors and the fp32
PyTorch reference (``uno_b200.ops.reference``) for CPU tensors.  There is no
silent fallback: a CUDA tensor with the extension missing raises.
"""

from __future__ import annotations

import torch

from uno_b200.ops import reference as ref


def _cuda():
    from uno_b200.ops import cuda as _c

    return _c


def rms_norm(x, weight, eps, n_groups=1):
    if x.is_cuda:
        return _cuda().rms_norm(x, weight, eps, n_groups)
    return ref.rms_norm(x, weight, eps, n_groups)


def rms_norm_first(x, weight, eps, n_groups=1, final=False):
    """Norm that starts the residual stream: returns (normed, residual)."""
    if not isinstance(x, torch.Tensor) or x.is_cuda:
        return _cuda().rms_norm_first(x, weight, eps, n_groups, final)
    return ref.rms_norm(x, weight, eps, n_groups), x


def add_rms_norm(x, residual, weight, eps, n_groups=1, final=False):
    """``final``: last norm of a forward (completes the fused tensor-parallel gather)."""
    if not isinstance(x, torch.Tensor) or x.is_cuda:
        return _cuda().add_rms_norm(x, residual, weight, eps, n_groups, final)
    return ref.add_rms_norm(x, residual, weight, eps, n_groups)


def linear(x, layer, lora_mask=None):
    if x.is_cuda:
        return _cuda().linear(x, layer, lora_mask)
    return ref.linear(x, layer, lora_mask)


def gate_up_silu(x, layer, lora_mask=None):
    if x.is_cuda:
        return _cuda().gate_up_silu(x, layer, lora_mask)
    return ref.gate_up_silu(x, layer, lora_mask)


def qkv_rope_store(x, layer, lora_mask, positions, cos_sin, q_norm_w, k_norm_w, eps,
                   num_heads, num_kv_heads, head_dim, k_cache, v_cache, slot_mapping):
    fn = _cuda().qkv_rope_store if x.is_cuda else ref.qkv_rope_store
    return fn(x, layer, lora_mask, positions, cos_sin, q_norm_w, k_norm_w, eps,
              num_heads, num_kv_heads, head_dim, k_cache, v_cache, slot_mapping)


def attention(q, k_cache, v_cache, meta, scale):
    if q.is_cuda:
        return _cuda().attention(q, k_cache, v_cache, meta, scale)
    return ref.attention(q, k_cache, v_cache, meta, scale)


def embedding(ids, table, vocab_start=0):
    if ids.is_cuda:
        return _cuda().embedding(ids, table, vocab_start)
    return ref.embedding(ids, table, vocab_start)


def lm_head(x, weight):
    if x.is_cuda:
        return _cuda().lm_head(x, weight)
    return ref.lm_head(x, weight)


def is_cuda_available() -> bool:
    return torch.cuda.is_available()
