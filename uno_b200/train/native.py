"""Training projections on the framework's tcgen05 GEMMs (CUDA).

A frozen base projection with gated LoRA segments (the reference trains PEFT
LoRA on q,k,v,o,gate,up,down with a token-wise router, ``training/lora.py:
136-179``; its GEMMs are cuBLAS through HF/PEFT):

    y = x W^T + sum_seg  (s * mask * (x A_seg^T)) B_seg^T     (segments tile y's columns)

Forward: ONE ROWSCALE GEMM for the concatenated LoRA hidden ``h = s * mask *
(x A_cat^T)`` and ONE base GEMM whose K dimension is extended by ``h`` against
the block-diagonal ``B_cat`` (the same K-extension the inference kernels use).

Backward (base weights frozen: no weight gradient for W):

    dh  = s * mask * (dy B_cat)              ROWSCALE GEMM against B_cat^T
    dx  = dy W + dh A_cat                    base GEMM against W^T, K-extended by (dh, A_cat^T)
    dB_seg += dy[:, seg]^T h[:, seg]         weight-gradient GEMMs (fp32 accumulate
    dA_cat += dh^T x                         straight into the parameters' .grad)

``W^T`` is a transposed copy of the frozen weight made once (weights never
change during LoRA training), so every GEMM runs K-major operands except the
weight gradients, which use the MN-major tcgen05 form.  LoRA gradients are
accumulated by the backward directly into the fp32 ``.grad`` buffers of the
LoRA parameters (the optimizer's flat gradient), not returned to autograd.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass
class LoraSegment:
    """Columns ``[col0, col0 + width)`` of the output use ``A`` [r, K] and ``B`` [width, r] (fp32 params)."""

    col0: int
    width: int
    A: torch.nn.Parameter
    B: torch.nn.Parameter


@dataclass
class WeightShard:
    """Rows ``[r0, r1)`` of a frozen weight, held by one rank (possibly a peer over NVLink)."""

    r0: int
    r1: int
    W: torch.Tensor   # [r1 - r0, K] bf16
    Wt: torch.Tensor  # [K, r1 - r0] bf16


@dataclass
class ProjectionWeights:
    W: torch.Tensor | None          # [N, K] bf16, frozen (None when sharded)
    Wt: torch.Tensor | None         # [K, N] bf16 copy
    segments: list = field(default_factory=list)
    scale: float = 1.0
    shards: list | None = None      # FSDP: every rank's WeightShard, in row order
    out_features: int = 0
    in_features: int = 0
    # bf16 compute copies of the LoRA factors, rebuilt after every optimizer step
    a_cat: torch.Tensor | None = None   # [S*r, K]
    at_cat: torch.Tensor | None = None  # [K, S*r]
    b_cat: torch.Tensor | None = None   # [N, S*r] block diagonal
    bt_cat: torch.Tensor | None = None  # [S*r, N]
    version: int = -1

    @torch.no_grad()
    def refresh(self, version: int) -> None:
        if not self.segments or self.version == version:
            return
        r = self.segments[0].A.shape[0]
        S = len(self.segments)
        N = self.out_features
        dev = self.segments[0].A.device
        a = torch.cat([seg.A for seg in self.segments], 0).to(torch.bfloat16)
        b = torch.zeros(N, S * r, device=dev, dtype=torch.bfloat16)
        for i, seg in enumerate(self.segments):
            b[seg.col0:seg.col0 + seg.width, i * r:(i + 1) * r] = seg.B.to(torch.bfloat16)
        self.a_cat, self.at_cat = a.contiguous(), a.t().contiguous()
        self.b_cat, self.bt_cat = b, b.t().contiguous()
        self.version = version


def _a_grad_block(segments) -> torch.Tensor:
    """The contiguous fp32 [S*r, K] gradient region of the segments' A factors (one flat buffer)."""
    g0 = segments[0].A.grad
    r, K = g0.shape
    for i, seg in enumerate(segments):
        g = seg.A.grad
        if g is None or g.data_ptr() != g0.data_ptr() + i * r * K * 4:
            raise RuntimeError("LoRA A gradients of one projection must be adjacent in the flat gradient buffer")
    return torch.as_strided(g0, (len(segments) * r, K), (K, 1))


_GATHER_BUF: dict = {}


def _gather_buffer(device, numel: int, name: str) -> torch.Tensor:
    key = (device, name)
    buf = _GATHER_BUF.get(key)
    if buf is None or buf.numel() < numel:
        buf = torch.empty(numel, device=device, dtype=torch.bfloat16)
        _GATHER_BUF[key] = buf
    return buf[:numel]


def gather_rows(proj: "ProjectionWeights", device) -> torch.Tensor:
    """FSDP forward operand: every owner's rows copied into one local ``[N, K]`` weight.

    Each owner block is one contiguous peer-to-local copy (copy engine over NVLink), so the
    GEMM that follows reads local HBM once per tile instead of streaming the weight over NVLink
    for every row tile."""
    N, K = proj.out_features, proj.in_features
    w = _gather_buffer(device, N * K, "w").view(N, K)
    for sh in proj.shards:
        w[sh.r0:sh.r1].copy_(sh.W, non_blocking=True)
    return w


def gather_cols(proj: "ProjectionWeights", device) -> list[torch.Tensor]:
    """FSDP backward operands: every owner's transposed block ``[K, rows]`` as a local copy."""
    K = proj.in_features
    buf = _gather_buffer(device, K * proj.out_features, "wt")
    out, off = [], 0
    for sh in proj.shards:
        n = K * (sh.r1 - sh.r0)
        blk = buf[off:off + n].view(K, sh.r1 - sh.r0)
        blk.copy_(sh.Wt, non_blocking=True)
        out.append(blk)
        off += n
    return out


class _ProjectionFn(torch.autograd.Function):
    # The LoRA factors are passed as extra inputs only so that autograd records
    # the op when ``x`` itself needs no gradient (the first projection sees the
    # frozen embedding); their gradients are accumulated by the backward itself.
    @staticmethod
    def forward(ctx, x, proj: ProjectionWeights, mask, *lora_params):
        from uno_b200.ops import cuda as C

        M = x.shape[0]
        N = proj.out_features
        y = torch.empty(M, N, device=x.device, dtype=torch.bfloat16)
        h = None
        if proj.segments:
            h = torch.empty(M, proj.a_cat.shape[0], device=x.device, dtype=torch.bfloat16)
            C._gemm(x, proj.a_cat, C.EPI_ROWSCALE, c=h, scale=proj.scale, row_mask=mask)
        # FSDP: gather the owners' rows into a local weight first (peer copies), then one GEMM
        W = proj.W if proj.shards is None else gather_rows(proj, x.device)
        C._gemm(x, W, C.EPI_STORE, c=y, a2=h, b2=proj.b_cat if h is not None else None)
        ctx.proj = proj
        ctx.save_for_backward(x, h, mask)
        return y

    @staticmethod
    def backward(ctx, dy):
        from uno_b200.ops import cuda as C

        x, h, mask = ctx.saved_tensors
        proj: ProjectionWeights = ctx.proj
        dy = dy.to(torch.bfloat16).contiguous()
        M, K = x.shape
        n_params = len(ctx.needs_input_grad) - 3
        dx = torch.empty(M, K, device=x.device, dtype=torch.bfloat16) if ctx.needs_input_grad[0] else None
        dh = None
        if proj.segments:
            dh = torch.empty_like(h)
            C._gemm(dy, proj.bt_cat, C.EPI_ROWSCALE, c=dh, scale=proj.scale, row_mask=mask)
        if dx is None:
            pass
        elif proj.shards is None:
            C._gemm(dy, proj.Wt, C.EPI_STORE, c=dx, a2=dh, b2=proj.at_cat if dh is not None else None)
        else:
            # dx = sum over owners of dy[:, rows_j] W_j (local copies of their transposed blocks);
            # the first block also adds dh A_cat
            for j, (sh, wt) in enumerate(zip(proj.shards, gather_cols(proj, x.device))):
                first = j == 0
                C._gemm(dy[:, sh.r0:sh.r1], wt, C.EPI_STORE if first else C.EPI_ADD, c=dx,
                        r=None if first else dx, a2=dh if first else None,
                        b2=proj.at_cat if (first and dh is not None) else None)
        if proj.segments:
            r = proj.segments[0].A.shape[0]
            ext = C.ext()
            for i, seg in enumerate(proj.segments):
                ext.gemm_wgrad(dy[:, seg.col0:seg.col0 + seg.width], h[:, i * r:(i + 1) * r], seg.B.grad, 0)
            ext.gemm_wgrad(dh, x, _a_grad_block(proj.segments), 0)
        return (dx, None, None) + (None,) * n_params


def projection(x: torch.Tensor, proj: ProjectionWeights, mask: torch.Tensor | None) -> torch.Tensor:
    """``x [..., K] -> [..., N]`` through the base + gated-LoRA projection."""
    shape = x.shape
    x2 = x.reshape(-1, shape[-1]).to(torch.bfloat16).contiguous()
    m = (mask.reshape(-1).float().contiguous() if mask is not None
         else torch.ones(x2.shape[0], device=x.device, dtype=torch.float32))
    params = [t for seg in proj.segments for t in (seg.A, seg.B)]
    y = _ProjectionFn.apply(x2, proj, m, *params)
    return y.view(*shape[:-1], y.shape[-1])


def _projection_specs(model, lora):
    """``(layer, name, weight, segments)`` for every projection of the decoder."""

    def seg(li, name, col0, width):
        if lora is None or not lora.has(li, name):
            return None
        key = lora._key(li, name)
        return LoraSegment(col0, width, lora.A[key], lora.B[key])

    for li, layer in enumerate(model.model.layers):
        attn, mlp = layer.self_attn, layer.mlp
        hq, hkv, hd = attn.num_heads, attn.num_kv_heads, attn.head_dim
        inter = mlp.gate_up_proj.weight.shape[0] // 2
        for name, w, segs in (
            ("qkv", attn.qkv_proj.weight, [seg(li, "q_proj", 0, hq * hd), seg(li, "k_proj", hq * hd, hkv * hd),
                                           seg(li, "v_proj", (hq + hkv) * hd, hkv * hd)]),
            ("o", attn.o_proj.weight, [seg(li, "o_proj", 0, attn.o_proj.weight.shape[0])]),
            ("gate_up", mlp.gate_up_proj.weight, [seg(li, "gate_proj", 0, inter), seg(li, "up_proj", inter, inter)]),
            ("down", mlp.down_proj.weight, [seg(li, "down_proj", 0, mlp.down_proj.weight.shape[0])]),
        ):
            yield li, name, w, [s for s in segs if s is not None]


def build_projections(model, lora, group=None, fsdp: bool = False):
    """Per layer: ``qkv``, ``o``, ``gate_up`` and ``down`` projections with their LoRA segments.

    With ``fsdp`` every frozen weight is split by output rows across the ranks
    of ``group`` (:class:`uno_b200.train.fsdp.ShardedWeights`): each rank keeps
    1/world of the rows (and of their transposes); before each projection's
    GEMM the owners' blocks are copied peer-to-local into one reusable buffer
    (:func:`gather_rows`, :func:`gather_cols`).  Returns ``(layers, sharded)``.
    """
    scale = float(lora.scaling) if lora is not None else 1.0
    specs = list(_projection_specs(model, lora))
    sharded = None
    if fsdp:
        from uno_b200.train.fsdp import ShardedWeights

        sharded = ShardedWeights([(f"{li}.{name}", w) for li, name, w, _ in specs], group)
    layers: list[dict[str, ProjectionWeights]] = [dict() for _ in model.model.layers]
    for li, name, w, segs in specs:
        N, K = w.shape
        if sharded is None:
            wb = w.detach().to(torch.bfloat16).contiguous()
            pw = ProjectionWeights(W=wb, Wt=wb.t().contiguous(), segments=segs, scale=scale, out_features=N,
                                   in_features=K)
        else:
            pw = ProjectionWeights(W=None, Wt=None, segments=segs, scale=scale,
                                   shards=sharded.shards(f"{li}.{name}"), out_features=N, in_features=K)
        layers[li][name] = pw
    return layers, sharded


# ------------------------------------------------------------ elementwise ops
class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps: float, groups: int):
        from uno_b200.ops.cuda import ext

        x = x.to(torch.bfloat16).contiguous()
        H = x.shape[-1]
        y = torch.empty_like(x)
        rstd = torch.empty(x.numel() // H * groups, device=x.device, dtype=torch.float32)
        w = weight.detach().to(torch.bfloat16).contiguous()
        ext().rmsnorm_fwd_train(x, w, y, rstd, float(eps), int(groups))
        ctx.save_for_backward(x, w, rstd)
        ctx.groups = int(groups)
        return y

    @staticmethod
    def backward(ctx, dy):
        from uno_b200.ops.cuda import ext

        x, w, rstd = ctx.saved_tensors
        dy = dy.to(torch.bfloat16).contiguous()
        dx = torch.empty_like(x)
        ext().rmsnorm_bwd_train(dy, x, w, rstd, dx, ctx.groups)
        return dx, None, None, None


class _SiluMulFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):
        from uno_b200.ops.cuda import ext

        gu = gu.to(torch.bfloat16).contiguous()
        a = torch.empty(*gu.shape[:-1], gu.shape[-1] // 2, device=gu.device, dtype=torch.bfloat16)
        ext().silu_mul_fwd(gu, a)
        ctx.save_for_backward(gu)
        return a

    @staticmethod
    def backward(ctx, da):
        from uno_b200.ops.cuda import ext

        (gu,) = ctx.saved_tensors
        dgu = torch.empty_like(gu)
        ext().silu_mul_bwd(da.to(torch.bfloat16).contiguous(), gu, dgu)
        return dgu


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float, groups: int = 1) -> torch.Tensor:
    """RMSNorm (fp32 statistics, frozen weight) with a fused backward kernel."""
    return _RMSNormFn.apply(x, weight, eps, groups)


def silu_mul(gu: torch.Tensor) -> torch.Tensor:
    """``silu(gate) * up`` of ``[..., 2I] = [gate | up]`` with a fused backward kernel."""
    return _SiluMulFn.apply(gu)


class _QKNormRopeFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps: float, positions, cos_sin):
        from uno_b200.ops.cuda import ext

        T, H, _ = x.shape
        out = torch.empty(T, H, 128, device=x.device, dtype=torch.bfloat16)
        rstd = torch.empty(T * H, device=x.device, dtype=torch.float32)
        w = weight.detach().to(torch.bfloat16).contiguous() if weight is not None else None
        ext().qk_norm_rope_fwd(x, w, float(eps), positions, cos_sin, out, rstd)
        ctx.save_for_backward(x, rstd, positions, cos_sin)
        ctx.w = w
        return out

    @staticmethod
    def backward(ctx, dy):
        from uno_b200.ops.cuda import ext

        x, rstd, positions, cos_sin = ctx.saved_tensors
        dx = torch.empty_strided(x.shape, x.stride(), device=x.device, dtype=torch.bfloat16)
        ext().qk_norm_rope_bwd(dy.to(torch.bfloat16).contiguous(), x, ctx.w, positions, cos_sin, rstd, dx)
        return dx, None, None, None, None


def qk_norm_rope(x: torch.Tensor, weight: torch.Tensor | None, eps: float, positions: torch.Tensor,
                 cos_sin: torch.Tensor) -> torch.Tensor:
    """Per-head RMSNorm (when ``weight`` is given) + NeoX RoPE of ``x [tokens, heads, 128]``.

    ``x`` may be a column slice of the fused qkv output (token stride > heads * 128); the
    result is contiguous and its backward writes a gradient of ``x``'s layout."""
    return _QKNormRopeFn.apply(x, weight, eps, positions.reshape(-1).long().contiguous(), cos_sin.float().contiguous())
