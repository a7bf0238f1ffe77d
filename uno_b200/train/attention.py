"""Block-diffusion attention for training on the framework's kernels (CUDA).

Forward and backward of softmax attention under the Uno visibility rule
(:func:`uno_b200.train.layout.visibility`) with grouped KV heads, run by
``train_attn_fwd`` / ``train_attn_bwd`` (``ops/csrc/train_attention.cu``).
The kernels evaluate the rule per element from each token's (segment,
position, noisy) triple; the host only builds the 64 x 64 tile map that lets
them skip empty tiles and drop the per-element test on full ones.
"""

from __future__ import annotations

import torch

TILE = 64


def tile_map(vis: torch.Tensor) -> torch.Tensor:
    """``[B, nt, nt]`` uint8 from a dense ``[B, T, T]`` visibility: 0 empty, 1 partial, 2 full."""
    B, T, _ = vis.shape
    nt = -(-T // TILE)
    pad = nt * TILE - T
    if pad:
        vis = torch.nn.functional.pad(vis, (0, pad, 0, pad), value=False)
    blocks = vis.view(B, nt, TILE, nt, TILE)
    anyv = blocks.any(dim=4).any(dim=2)
    allv = blocks.all(dim=4).all(dim=2)
    return (anyv.to(torch.uint8) + allv.to(torch.uint8)).contiguous()


class AttentionMeta:
    """Per-token metadata of one Uno batch, shared by every layer's attention."""

    def __init__(self, segment, positions, noisy, block_size: int, vis: torch.Tensor | None = None):
        from uno_b200.train.layout import visibility

        self.seg = segment.to(torch.int32).contiguous()
        self.pos = positions.to(torch.int32).contiguous()
        self.noisy = noisy.to(torch.uint8).contiguous()
        self.block = int(block_size)
        if vis is None:
            vis = visibility(segment, positions, noisy, block_size)
        self.tiles = tile_map(vis)


class _BlockDiffusionAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, meta: AttentionMeta, scale: float):
        from uno_b200.ops.cuda import ext

        q, k, v = (t.to(torch.bfloat16).contiguous() for t in (q, k, v))
        B, T, hq, _ = q.shape
        out = torch.empty_like(q)
        lse = torch.empty(B, hq, T, device=q.device, dtype=torch.float32)
        ext().train_attn_fwd(q, k, v, meta.seg, meta.pos, meta.noisy, meta.tiles, meta.block, float(scale), out, lse)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.meta, ctx.scale = meta, float(scale)
        return out

    @staticmethod
    def backward(ctx, dout):
        from uno_b200.ops.cuda import ext

        q, k, v, out, lse = ctx.saved_tensors
        meta = ctx.meta
        dout = dout.to(torch.bfloat16).contiguous()
        delta = torch.empty_like(lse)
        dq = torch.zeros(q.shape, device=q.device, dtype=torch.float32)
        dk = torch.empty_like(k)
        dv = torch.empty_like(v)
        ext().train_attn_bwd(q, k, v, meta.seg, meta.pos, meta.noisy, meta.tiles, meta.block, ctx.scale, out, dout,
                             lse, delta, dq, dk, dv)
        return dq.to(torch.bfloat16), dk, dv, None, None


def block_diffusion_attention(q, k, v, meta: AttentionMeta, scale: float) -> torch.Tensor:
    """``q [B, T, hq, 128]``, ``k``/``v`` ``[B, T, hkv, 128]`` -> ``[B, T, hq, 128]``."""
    return _BlockDiffusionAttention.apply(q, k, v, meta, scale)
