"""Differentiable forward of the frozen decoder plus trainable gated LoRA.

Runs the same layer math as the inference model (pre-norm residual blocks,
QKV with optional QK-norm, NeoX RoPE, GQA attention, SiLU-gated MLP, final
norm) over the concatenated noisy/clean Uno layout with an explicit
visibility mask, and adds the LoRA branch of every projection on rows whose
router mask is set.  Base weights are read from the inference model's
modules (no copy) and receive no gradient; activations of each layer can be
recomputed in backward (per-layer checkpointing, as the reference
checkpoints the modules that hold trainable parameters,
``training/checkpointing.py:12-52``).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint

from uno_b200.ops import reference as R
from uno_b200.train.lora import TrainableLoRA


def _proj(x, weight, bias, lora, li, name, mask):
    """Base projection (frozen) plus the gated LoRA delta of projection ``name``."""
    y = F.linear(x, weight, bias)
    if lora is not None and lora.has(li, name):
        y = y + lora.delta(li, name, x, mask).to(y.dtype)
    return y


def _layer(x, layer, li, lora, mask, positions, cos_sin, attn_mask, cfg):
    B, T, H = x.shape
    attn = layer.self_attn
    hq, hkv, hd = attn.num_heads, attn.num_kv_heads, attn.head_dim
    ln1 = layer.input_layernorm
    h = R.rms_norm(x, ln1.weight, ln1.eps, ln1.n_groups)
    qkv_w, qkv_b = attn.qkv_proj.weight, attn.qkv_proj.bias
    q_end, k_end = hq * hd, (hq + hkv) * hd
    qkv = F.linear(h, qkv_w, qkv_b)
    if lora is not None:
        parts = []
        for name, lo, hi in (("q_proj", 0, q_end), ("k_proj", q_end, k_end), ("v_proj", k_end, qkv.shape[-1])):
            seg = qkv[..., lo:hi]
            if lora.has(li, name):
                seg = seg + lora.delta(li, name, h, mask).to(seg.dtype)
            parts.append(seg)
        q, k, v = parts
    else:
        q, k, v = qkv[..., :q_end], qkv[..., q_end:k_end], qkv[..., k_end:]
    q = q.reshape(B, T, hq, hd)
    k = k.reshape(B, T, hkv, hd)
    v = v.reshape(B, T, hkv, hd)
    if attn.qk_norm:
        q = R.head_rms_norm(q, attn.q_norm.weight, attn.eps)
        k = R.head_rms_norm(k, attn.k_norm.weight, attn.eps)
    pos = positions.reshape(-1)
    q = R.apply_rope(q.reshape(B * T, hq, hd), pos, cos_sin).reshape(B, T, hq, hd)
    k = R.apply_rope(k.reshape(B * T, hkv, hd), pos, cos_sin).reshape(B, T, hkv, hd)
    o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                       attn_mask=attn_mask[:, None], scale=attn.scale, enable_gqa=hq != hkv)
    o = o.transpose(1, 2).reshape(B, T, hq * hd)
    o = _proj(o, attn.o_proj.weight, None, lora, li, "o_proj", mask)
    x = x + o
    ln2 = layer.post_attention_layernorm
    h = R.rms_norm(x, ln2.weight, ln2.eps, ln2.n_groups)
    mlp = layer.mlp
    inter = mlp.gate_up_proj.weight.shape[0] // 2
    gu = F.linear(h, mlp.gate_up_proj.weight)
    if lora is not None:
        g, u = gu[..., :inter], gu[..., inter:]
        if lora.has(li, "gate_proj"):
            g = g + lora.delta(li, "gate_proj", h, mask).to(g.dtype)
        if lora.has(li, "up_proj"):
            u = u + lora.delta(li, "up_proj", h, mask).to(u.dtype)
    else:
        g, u = gu[..., :inter], gu[..., inter:]
    a = F.silu(g) * u
    d = _proj(a, mlp.down_proj.weight, None, lora, li, "down_proj", mask)
    return x + d


def _layer_native(x, layer, proj, mask, positions, cos_sin, attn_mask, attn_meta=None):
    """The same layer with every projection on the tcgen05 GEMMs (``uno_b200.train.native``)."""
    from uno_b200.train.native import projection, qk_norm_rope, rms_norm, silu_mul

    B, T, H = x.shape
    attn = layer.self_attn
    hq, hkv, hd = attn.num_heads, attn.num_kv_heads, attn.head_dim
    ln1 = layer.input_layernorm
    h = rms_norm(x, ln1.weight, ln1.eps, ln1.n_groups)
    qkv = projection(h, proj["qkv"], mask)
    q_end, k_end = hq * hd, (hq + hkv) * hd
    pos = positions.reshape(-1)
    if hd == 128:  # fused QK-norm + RoPE straight from the qkv columns
        flat = qkv.reshape(B * T, -1)
        qn = attn.q_norm.weight if attn.qk_norm else None
        kn = attn.k_norm.weight if attn.qk_norm else None
        q = qk_norm_rope(flat[:, :q_end].unflatten(1, (hq, hd)), qn, attn.eps, pos, cos_sin).reshape(B, T, hq, hd)
        k = qk_norm_rope(flat[:, q_end:k_end].unflatten(1, (hkv, hd)), kn, attn.eps, pos, cos_sin)
        k = k.reshape(B, T, hkv, hd)
        v = qkv[..., k_end:].reshape(B, T, hkv, hd)
    else:
        q = qkv[..., :q_end].reshape(B, T, hq, hd)
        k = qkv[..., q_end:k_end].reshape(B, T, hkv, hd)
        v = qkv[..., k_end:].reshape(B, T, hkv, hd)
        if attn.qk_norm:
            q = R.head_rms_norm(q, attn.q_norm.weight, attn.eps)
            k = R.head_rms_norm(k, attn.k_norm.weight, attn.eps)
        q = R.apply_rope(q.reshape(B * T, hq, hd), pos, cos_sin).reshape(B, T, hq, hd)
        k = R.apply_rope(k.reshape(B * T, hkv, hd), pos, cos_sin).reshape(B, T, hkv, hd)
    if attn_meta is not None and hd == 128:
        from uno_b200.train.attention import block_diffusion_attention

        o = block_diffusion_attention(q, k, v, attn_meta, attn.scale).reshape(B, T, hq * hd)
    else:
        o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                           attn_mask=attn_mask[:, None], scale=attn.scale, enable_gqa=hq != hkv)
        o = o.transpose(1, 2).reshape(B, T, hq * hd)
    x = x + projection(o, proj["o"], mask)
    ln2 = layer.post_attention_layernorm
    h = rms_norm(x, ln2.weight, ln2.eps, ln2.n_groups)
    a = silu_mul(projection(h, proj["gate_up"], mask))
    return x + projection(a, proj["down"], mask)


def uno_hidden_states(model, lora: TrainableLoRA | None, ids: torch.Tensor, positions: torch.Tensor,
                      attn_mask: torch.Tensor, lora_rows: torch.Tensor | None,
                      checkpoint_layers: bool = False, native: list | None = None,
                      attn_meta=None) -> torch.Tensor:
    """Final-norm hidden states ``[B, T, H]`` for the Uno layout.

    ``native`` (from :func:`uno_b200.train.native.build_projections`) runs the
    projections on the tcgen05 GEMMs and, with ``attn_meta``
    (:class:`uno_b200.train.attention.AttentionMeta`, head_dim 128), the
    attention on the block-diffusion kernels; without them every op is a
    torch op.
    """
    dec = model.model
    x = F.embedding(ids, dec.embed_tokens.weight)
    cos_sin = model.cos_sin_cache
    for li, layer in enumerate(dec.layers):
        if native is not None:
            fn, args = _layer_native, (x, layer, native[li], lora_rows, positions, cos_sin, attn_mask, attn_meta)
        else:
            fn, args = _layer, (x, layer, li, lora, lora_rows, positions, cos_sin, attn_mask, model.config)
        if checkpoint_layers and torch.is_grad_enabled():
            x = checkpoint(fn, *args, use_reentrant=False)
        else:
            x = fn(*args)
    norm = dec.norm
    if native is not None:
        from uno_b200.train.native import rms_norm

        return rms_norm(x, norm.weight, norm.eps, norm.n_groups)
    return R.rms_norm(x, norm.weight, norm.eps, norm.n_groups)
