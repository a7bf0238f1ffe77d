"""Plain-PyTorch reference implementations of every fused op.

These are the CPU execution path (fp32) and the numerical
oracles the CUDA kernels are tested against.  Each function reproduces the
reference's own math and rounding order:

* RMSNorm / fused add+RMSNorm: ``layers/layernorm.py:16-40`` (normalise in fp32,
  round, then multiply by the weight in the activation dtype); grouped RMSNorm
  for Llama/K2: ``models/xllm.py:26-84``.
* QK-norm: ``jit_kernel/qk_norm.py:10-87`` (fp32 x * rsqrt(mean x^2 + eps) * w).
* RoPE: ``layers/rotary_embedding.py:8-59`` (NeoX half split in fp32).
* Gated LoRA: ``layers/linear.py:166-307``.
* Attention: the SDPA fallbacks ``layers/attention.py:297-438``.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from uno_b200.layers.meta import ForwardMeta, Mode
from uno_b200.parallel import state as tp


# ----------------------------------------------------------------- norms
def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float, n_groups: int = 1) -> torch.Tensor:
    dtype = x.dtype
    shape = x.shape
    xf = x.float()
    if n_groups > 1:
        xf = xf.reshape(*shape[:-1], n_groups, shape[-1] // n_groups)
    xf = xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)
    return xf.reshape(shape).to(dtype) * weight


def add_rms_norm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float,
                 n_groups: int = 1) -> tuple[torch.Tensor, torch.Tensor]:
    summed = x.float() + residual.float()
    new_residual = summed.to(x.dtype)
    if n_groups > 1:
        return rms_norm(new_residual, weight, eps, n_groups), new_residual
    dtype = x.dtype
    normed = summed * torch.rsqrt(summed.pow(2).mean(dim=-1, keepdim=True) + eps)
    return normed.to(dtype) * weight, new_residual


def silu_and_mul(x: torch.Tensor) -> torch.Tensor:
    gate, up = x.chunk(2, dim=-1)
    return F.silu(gate) * up


# ---------------------------------------------------------------- linear
def _lora_delta_into(y2: torch.Tensor, x2: torch.Tensor, layer, mask: torch.Tensor, row_parallel: bool) -> None:
    for s in layer.lora_slices:
        hidden = F.linear(x2, s.A)
        if row_parallel:
            tp.all_reduce(hidden)
        hidden = hidden * mask.to(hidden.dtype)[:, None]
        y2[:, s.out_start:s.out_end].addmm_(hidden, s.B.t(), beta=1.0, alpha=s.scaling)


def linear(x: torch.Tensor, layer, lora_mask: torch.Tensor | None = None) -> torch.Tensor:
    """Base projection (+ all-reduce for row-parallel) then the gated LoRA delta."""
    row_parallel = layer.tp_dim == 1 and layer.tp_size > 1
    bias = layer.bias
    if row_parallel and layer.tp_rank != 0:
        bias = None
    y = F.linear(x, layer.weight, bias)
    if row_parallel:
        tp.all_reduce(y)
    if lora_mask is not None and layer.has_lora:
        shape = y.shape
        y2 = y.reshape(-1, shape[-1])
        _lora_delta_into(y2, x.reshape(-1, x.shape[-1]), layer, lora_mask.reshape(-1), row_parallel)
        y = y2.reshape(shape)
    return y


def gate_up_silu(x: torch.Tensor, layer, lora_mask: torch.Tensor | None = None) -> torch.Tensor:
    return silu_and_mul(linear(x, layer, lora_mask))


# ------------------------------------------------------ rope / qk-norm
def apply_rope(x: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor) -> torch.Tensor:
    """NeoX rotation of ``x [T, H, D]`` (fp32 math, result in x.dtype)."""
    cs = cos_sin[positions.long()]
    half = cs.shape[-1] // 2
    cos, sin = cs[:, None, :half], cs[:, None, half:]
    x1, x2 = x.float().chunk(2, dim=-1)
    return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1).to(x.dtype)


def head_rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps) * weight.float()
    return xf.to(x.dtype)


def store_kv(k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
             slot_mapping: torch.Tensor) -> None:
    """Scatter ``k, v [T, Hkv, D]`` into caches ``[pages, Hkv, page, D]``; slot -1 is skipped."""
    if k_cache.numel() == 0:
        return
    page = k_cache.shape[2]
    slots = slot_mapping.long()
    keep = slots >= 0
    if not bool(keep.all()):
        k, v, slots = k[keep], v[keep], slots[keep]
    blk, off = slots // page, slots % page
    k_cache[blk, :, off, :] = k.to(k_cache.dtype)
    v_cache[blk, :, off, :] = v.to(v_cache.dtype)


def qkv_rope_store(x: torch.Tensor, layer, lora_mask, positions, cos_sin, q_norm_w, k_norm_w, eps,
                   num_heads: int, num_kv_heads: int, head_dim: int,
                   k_cache: torch.Tensor, v_cache: torch.Tensor, slot_mapping: torch.Tensor) -> torch.Tensor:
    qkv = linear(x, layer, lora_mask)
    q_size, kv_size = num_heads * head_dim, num_kv_heads * head_dim
    q, k, v = qkv.split([q_size, kv_size, kv_size], dim=-1)
    q = q.reshape(-1, num_heads, head_dim)
    k = k.reshape(-1, num_kv_heads, head_dim)
    v = v.reshape(-1, num_kv_heads, head_dim)
    if q_norm_w is not None:
        q = head_rms_norm(q, q_norm_w, eps)
        k = head_rms_norm(k, k_norm_w, eps)
    q = apply_rope(q, positions, cos_sin)
    k = apply_rope(k, positions, cos_sin)
    store_kv(k, v, k_cache, v_cache, slot_mapping)
    return q


# ------------------------------------------------------------- attention
def gather_pages(cache: torch.Tensor, block_table: torch.Tensor, length: int) -> torch.Tensor:
    """``[length, Hkv, D]`` contiguous K or V of one request."""
    page = cache.shape[2]
    n = -(-int(length) // page)
    ids = block_table[:n].long()
    out = cache.index_select(0, ids).permute(0, 2, 1, 3).reshape(n * page, cache.shape[1], cache.shape[3])
    return out[:length]


def _sdpa(q, k, v, scale, mask):
    """q [Tq, Hq, D], k/v [Tk, Hkv, D], bool mask [Tq, Tk] (True = visible)."""
    hq, hkv = q.shape[1], k.shape[1]
    if hq != hkv:
        k = k.repeat_interleave(hq // hkv, dim=1)
        v = v.repeat_interleave(hq // hkv, dim=1)
    out = F.scaled_dot_product_attention(
        q.transpose(0, 1).unsqueeze(0), k.transpose(0, 1).unsqueeze(0), v.transpose(0, 1).unsqueeze(0),
        attn_mask=mask, dropout_p=0.0, scale=scale,
    )
    return out.squeeze(0).transpose(0, 1)


def mask_bits_to_bool(masks: torch.Tensor, n: int) -> torch.Tensor:
    """int64 bitmasks ``[Q]`` -> bool ``[Q, n]``."""
    bits = torch.arange(n, device=masks.device, dtype=torch.int64)
    return ((masks.unsqueeze(-1) >> bits) & 1).bool()


def attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, meta: ForwardMeta,
              scale: float) -> torch.Tensor:
    """Paged attention for every forward mode; K/V of this forward are already stored."""
    T, hq, d = q.shape
    outs = []
    if meta.mode is Mode.PREFILL:
        cq = meta.cu_seqlens_q.tolist()
        ck = meta.cu_seqlens_k.tolist()
        for b in range(len(cq) - 1):
            nq, nk = cq[b + 1] - cq[b], ck[b + 1] - ck[b]
            k = gather_pages(k_cache, meta.block_tables[b], nk)
            v = gather_pages(v_cache, meta.block_tables[b], nk)
            qpos = torch.arange(nq, device=q.device)[:, None] + (nk - nq)
            kpos = torch.arange(nk, device=q.device)[None, :]
            outs.append(_sdpa(q[cq[b]:cq[b + 1]], k, v, scale, kpos <= qpos))
    else:
        Q = meta.seqlen_q
        prefix = meta.prefix_lens.tolist()
        for b in range(len(prefix)):
            nk = prefix[b] + Q
            k = gather_pages(k_cache, meta.block_tables[b], nk)
            v = gather_pages(v_cache, meta.block_tables[b], nk)
            vis = torch.ones(Q, nk, dtype=torch.bool, device=q.device)
            vis[:, prefix[b]:] = mask_bits_to_bool(meta.suffix_mask[b], Q)
            outs.append(_sdpa(q[b * Q:(b + 1) * Q], k, v, scale, vis))
    return torch.cat(outs, dim=0).reshape(T, hq * d)


# ------------------------------------------------------------- embedding
def embedding(ids: torch.Tensor, table: torch.Tensor, vocab_start: int = 0) -> torch.Tensor:
    if tp.tp_size() == 1:
        return F.embedding(ids, table)
    rows = table.shape[0]
    local = ids - vocab_start
    valid = (local >= 0) & (local < rows)
    y = F.embedding(local.clamp(0, rows - 1), table) * valid.unsqueeze(-1).to(table.dtype)
    return tp.all_reduce(y)


def lm_head(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    return F.linear(x, weight)
