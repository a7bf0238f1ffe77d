"""CUDA implementations of the fused ops (thin wrappers over ``uno_b200._C``).

Weight preparation for the sm_100a path (:func:`prepare_model`):

* ``gate_up_proj`` rows are interleaved in 64-row groups ``[gate_j | up_j]`` so
  the GEMM epilogue can apply SiLU(gate) * up inside one output tile;
* a gated LoRA layer keeps ``A_cat [R, K]`` and ``B_cat [N, R]`` (B rows in
  the same interleaved order as W).  A skinny split-K GEMM computes the hidden
  ``h = scale * mask * (x A_cat^T)`` (ROWSCALE epilogue), and the base GEMM runs
  its K loop over ``[x | h] . [W | B_cat]^T`` (K extension) with the layer's
  real epilogue (plain, SiLU*up or QK-norm + RoPE + paged KV store), so the
  adapter adds R columns of K and no extra pass over the output.
"""

from __future__ import annotations

import os

import torch

from uno_b200.layers.meta import ForwardMeta, Mode
from uno_b200.parallel import state as tp

_C = None
# Fused tensor-parallel collectives (uno_b200.parallel.symm.FusedTPComm) or None.
_COMM = None


def set_tp_comm(comm) -> None:
    global _COMM
    _COMM = comm


class PendingRS:
    """Marker: row-parallel partials were sent to the owners' receive slots and
    the next (add+)RMSNorm must run the fused reduce-norm-gather kernel."""

    __slots__ = ("T",)

    def __init__(self, T: int):
        self.T = int(T)

EPI_STORE, EPI_SILU, EPI_ROWSCALE, EPI_ADD, EPI_QKROPE = 0, 1, 2, 3, 5
INTERLEAVE = 64


def ext():
    """Import the compiled extension; raise loudly when it is missing."""
    global _C
    if _C is None:
        try:
            from uno_b200 import _C as mod
        except ImportError as e:  # pragma: no cover - depends on the build
            raise RuntimeError(
                "uno_b200._C is not built; run `python setup.py build_ext --inplace` "
                "(CUDA tensors have no fallback path)"
            ) from e
        _C = mod
    return _C


def error_flag(reset: bool = False) -> int:
    return int(ext().error_flag(reset))


def _gemm(a, b, epi, *, c=None, r=None, a2=None, b2=None, scale=0.0, row_mask=None, q_out=None,
          k_cache=None, v_cache=None, slots=None, positions=None, cos_sin=None, q_norm_w=None,
          k_norm_w=None, eps=0.0, hq=0, hkv=0, page=0, bn=0, max_ctas=0, splits=0, rs=None):
    peers, rank, off = ([], 0, 0) if rs is None else rs
    ag_base, ag_rows = _COMM.gather_wait_args(a) if _COMM is not None else (0, 0)
    ext().gemm(a, b, epi, bn, c, r, a2, b2, scale, row_mask, q_out, k_cache, v_cache, slots, positions,
               cos_sin, q_norm_w, k_norm_w, eps, hq, hkv, page, max_ctas, splits, peers, rank, off, ag_base, ag_rows)


def gemm(a: torch.Tensor, b: torch.Tensor, bn: int = 0, splits: int = 0) -> torch.Tensor:
    """Plain ``a @ b.T`` on the tcgen05 GEMM (bf16 out)."""
    out = torch.empty(a.shape[0], b.shape[0], device=a.device, dtype=torch.bfloat16)
    _gemm(a, b, EPI_STORE, c=out, bn=bn, splits=splits)
    return out


# ------------------------------------------------------------ weight prep
def interleave_gate_up(w: torch.Tensor, group: int = INTERLEAVE) -> torch.Tensor:
    """Rows [gate(I); up(I)] -> [g_0..g_63, u_0..u_63, g_64.., u_64.., ...]."""
    two_i = w.shape[0]
    inter = two_i // 2
    if inter % group:
        raise ValueError(f"intermediate size {inter} must be a multiple of {group}")
    gate, up = w[:inter], w[inter:]
    blocks = inter // group
    stacked = torch.stack([gate.reshape(blocks, group, *w.shape[1:]), up.reshape(blocks, group, *w.shape[1:])], dim=1)
    return stacked.reshape(two_i, *w.shape[1:]).contiguous()


@torch.no_grad()
def prepare_linear(layer, interleave: bool = False) -> None:
    if getattr(layer, "_uno_prepared", False):
        return
    if layer.bias is not None:
        raise NotImplementedError("biased linears are not supported on the sm_100a path")
    w = layer.weight.data
    if interleave:
        w = interleave_gate_up(w)
    layer.weight.data = w.contiguous()
    if layer.has_lora:
        if layer.lora_a_cat is None:
            layer.pack_lora()
        b_cat = layer.lora_b_cat
        if interleave:
            b_cat = interleave_gate_up(b_cat)
        layer.lora_a_dev = layer.lora_a_cat.to(w.dtype).contiguous()
        layer.lora_b_dev = b_cat.to(w.dtype).contiguous()
    layer.interleaved = interleave
    layer._uno_prepared = True


def prepare_model(model) -> None:
    for layer in model.model.layers:
        attn, mlp = layer.self_attn, layer.mlp
        prepare_linear(attn.qkv_proj)
        prepare_linear(attn.o_proj)
        prepare_linear(mlp.gate_up_proj, interleave=True)
        prepare_linear(mlp.down_proj)


# ------------------------------------------------------------------ norms
def _rows(x):
    """2-D row view with unit column stride (row stride may be padded)."""
    x2 = x.reshape(-1, x.shape[-1]) if x.dim() != 2 else x
    return x2 if x2.stride(-1) == 1 else x2.contiguous()


def rms_norm(x, weight, eps, n_groups=1):
    x2 = _rows(x)
    y = torch.empty(x2.shape, device=x.device, dtype=x.dtype)
    ext().rms_norm(x2, None, weight, y, float(eps), int(n_groups))
    return y.view(x.shape)


def rms_norm_first(x, weight, eps, n_groups=1, final=False):
    """First norm of the residual stream: returns (normed, residual)."""
    if isinstance(x, PendingRS):
        return _COMM.reduce_norm(x.T, None, weight, eps, n_groups, final)
    return rms_norm(x, weight, eps, n_groups), x


def add_rms_norm(x, residual, weight, eps, n_groups=1, final=False):
    """Returns (normed, new_residual); the residual buffer is updated in place.

    ``final`` marks the last norm of a forward (its output leaves the fused
    tensor-parallel path, so the gather completes before the kernel returns).
    """
    if isinstance(x, PendingRS):
        return _COMM.reduce_norm(x.T, residual, weight, eps, n_groups, final)
    x2 = _rows(x)
    y = torch.empty(x2.shape, device=x.device, dtype=x.dtype)
    res = residual if residual.is_contiguous() else residual.contiguous()
    ext().rms_norm(x2, res, weight, y, float(eps), int(n_groups))
    return y.view(x.shape), res


# ----------------------------------------------------------------- linear
def _row_parallel(layer) -> bool:
    return layer.tp_dim == 1 and layer.tp_size > 1


def lora_hidden(x, layer, lora_mask):
    """``scale * mask * (x A_cat^T)`` [M, R].

    For a row-parallel layer this is the rank's partial hidden (its K shard);
    every rank adds ``h_r . B^T`` to its partial output, and the reduction of
    the outputs sums the partial hiddens as well, so no extra collective runs.
    """
    h = torch.empty(x.shape[0], layer.lora_rank_total, device=x.device, dtype=torch.bfloat16)
    _gemm(x, layer.lora_a_dev, EPI_ROWSCALE, c=h, scale=layer.lora_scaling, row_mask=lora_mask)
    return h


def _lora_ext(x, layer, lora_mask):
    """K-extension operands (a2, b2) for the base GEMM, or (None, None)."""
    if lora_mask is None or not layer.has_lora:
        return None, None
    return lora_hidden(x, layer, lora_mask), layer.lora_b_dev


def linear(x, layer, lora_mask=None):
    x = _rows(x)
    a2, b2 = _lora_ext(x, layer, lora_mask)
    if _COMM is not None and _row_parallel(layer):
        # fused reduce-scatter: partial rows go straight to their owners
        _gemm(x, layer.weight, EPI_STORE, a2=a2, b2=b2, rs=_COMM.rs_args(x.shape[0]))
        return PendingRS(x.shape[0])
    y = torch.empty(x.shape[0], layer.weight.shape[0], device=x.device, dtype=torch.bfloat16)
    _gemm(x, layer.weight, EPI_STORE, c=y, a2=a2, b2=b2)
    if _row_parallel(layer):
        tp.all_reduce(y)
    return y


def gate_up_silu(x, layer, lora_mask=None):
    x = _rows(x)
    a2, b2 = _lora_ext(x, layer, lora_mask)
    inter = layer.weight.shape[0] // 2
    act = torch.empty(x.shape[0], inter, device=x.device, dtype=torch.bfloat16)
    _gemm(x, layer.weight, EPI_SILU, c=act, a2=a2, b2=b2)
    return act


def qkv_rope_store(x, layer, lora_mask, positions, cos_sin, q_norm_w, k_norm_w, eps, num_heads, num_kv_heads,
                   head_dim, k_cache, v_cache, slot_mapping):
    x = _rows(x)
    T = x.shape[0]
    q = torch.empty(T, num_heads, head_dim, device=x.device, dtype=torch.bfloat16)
    page = k_cache.shape[2] if k_cache.numel() else 0
    kc = k_cache if k_cache.numel() else None
    vc = v_cache if v_cache.numel() else None
    slots = slot_mapping if kc is not None else torch.full((T,), -1, dtype=torch.int64, device=x.device)
    if head_dim != 128:
        qkv = linear(x, layer, lora_mask)
        ext().qk_norm_rope_store(qkv, q, k_cache, v_cache, slots, positions, cos_sin, q_norm_w, k_norm_w,
                                 float(eps), num_heads, num_kv_heads, head_dim, page)
        return q
    a2, b2 = _lora_ext(x, layer, lora_mask)
    _gemm(x, layer.weight, EPI_QKROPE, a2=a2, b2=b2, q_out=q, k_cache=kc, v_cache=vc, slots=slots,
          positions=positions, cos_sin=cos_sin, q_norm_w=q_norm_w, k_norm_w=k_norm_w, eps=float(eps),
          hq=num_heads, hkv=num_kv_heads, page=page)
    return q


# -------------------------------------------------------------- attention
_SCRATCH: dict = {}


def _scratch(device, numel: int, name: str) -> torch.Tensor:
    key = (device, name)
    buf = _SCRATCH.get(key)
    if buf is None or buf.numel() < numel:
        buf = torch.empty(max(numel, 1), device=device, dtype=torch.float32)
        _SCRATCH[key] = buf
    return buf[:numel]


def reserve_attention_scratch(device, max_tokens: int, num_heads: int, max_splits: int,
                              num_kv_heads: int = 8) -> None:
    """Pre-size the attention scratch so graph capture never reallocates it."""
    _scratch(device, max_splits * max_tokens * num_heads * 128, "o_part")
    _scratch(device, max_splits * max_tokens * num_heads, "lse")
    _attention_scratch(device, max_tokens * num_kv_heads)


def plan_splits(B: int, hkv: int, qblocks: int, max_kv: int, sms: int = 148):
    ctas = max(1, B * hkv * qblocks)
    want = max(1, -(-2 * sms // ctas))
    max_by_len = max(1, -(-max_kv // 512))
    splits = min(want, max_by_len, 16)
    if splits <= 1:
        return 1, 0
    kps = -(-max_kv // splits)
    kps = -(-kps // 64) * 64
    splits = -(-max_kv // kps)
    return splits, kps


_ATT_IMPL = os.environ.get("UNO_ATTN_IMPL", "mma")


def _attention_scratch(device, rows_needed: int):
    """Partials (two slots per SM), their log-sum-exps and the per-segment arrival counters."""
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    rows = ext().attention_tc_rows() if hasattr(ext(), "attention_tc_rows") else 32
    o_part = _scratch(device, 2 * sms * rows * 128, "att_o_part")
    lse = _scratch(device, 2 * sms * rows, "att_lse")
    key = (device, "att_counters")
    cnt = _SCRATCH.get(key)
    if cnt is None or cnt.numel() < rows_needed:
        cnt = torch.zeros(max(rows_needed, 1), device=device, dtype=torch.int32)
        _SCRATCH[key] = cnt
    return o_part, lse, cnt


def attention(q, k_cache, v_cache, meta: ForwardMeta, scale):
    T, hq, d = q.shape
    o = torch.empty(T, hq * d, device=q.device, dtype=torch.bfloat16)
    hkv = k_cache.shape[1]
    if _ATT_IMPL == "mma":
        return _attention_mma(q, k_cache, v_cache, meta, scale, o)
    o_part, lse, cnt = _attention_scratch(q.device, T * hkv)
    if meta.mode is Mode.PREFILL:
        ext().attention_tc(q, o, k_cache, v_cache, meta.block_tables, None, None, meta.cu_seqlens_q,
                           meta.cu_seqlens_k, 1, meta.batch_size, 0, float(scale), o_part, lse, cnt)
    else:
        ext().attention_tc(q, o, k_cache, v_cache, meta.block_tables, meta.prefix_lens, meta.suffix_mask, None,
                           None, 0, meta.batch_size, meta.seqlen_q, float(scale), o_part, lse, cnt)
    return o


def _attention_mma(q, k_cache, v_cache, meta, scale, o):
    T, hq, d = q.shape
    hkv = k_cache.shape[1]
    if meta.mode is Mode.PREFILL:
        ext().attention(q, o, k_cache, v_cache, meta.block_tables, None, None, meta.cu_seqlens_q,
                        meta.cu_seqlens_k, 1, meta.batch_size, 0, meta.max_seqlen_q, float(scale), 1, 0, None, None)
        return o
    B, Q = meta.batch_size, meta.seqlen_q
    group = hq // hkv
    rows = max(16, -(-Q * group // 16) * 16)
    qpc = max(1, min(256, rows) // group)
    qblocks = -(-Q // qpc)
    max_kv = getattr(meta, "max_kv", 0) or (k_cache.shape[0] * k_cache.shape[2])
    splits, kps = plan_splits(B, hkv, qblocks, max_kv)
    o_part = lse = None
    if splits > 1:
        o_part = _scratch(q.device, splits * T * hq * 128, "o_part")
        lse = _scratch(q.device, splits * T * hq, "lse")
    ext().attention(q, o, k_cache, v_cache, meta.block_tables, meta.prefix_lens, meta.suffix_mask, None, None, 0,
                    B, Q, Q, float(scale), splits, kps, o_part, lse)
    return o


# ------------------------------------------------------------ embeddings
def embedding(ids, table, vocab_start=0):
    if _COMM is not None:
        _COMM.embedding_scatter(ids, table, vocab_start)
        return PendingRS(ids.numel())
    out = torch.empty(ids.numel(), table.shape[1], device=ids.device, dtype=table.dtype)
    ext().embedding(ids.reshape(-1).contiguous(), table, out, int(vocab_start))
    if tp.tp_size() > 1:
        tp.all_reduce(out)
    return out


def lm_head(x, weight):
    return gemm(x.contiguous(), weight)


# --------------------------------------------------------------- sampling
def _n_rows(x):
    return x.shape[0] if x.dim() == 2 else x.shape[0] * x.shape[1]


def argmax(logits):
    """Greedy tokens for 2-D [N, V] or strided 3-D [B, R, V] logits (no copy)."""
    out = torch.empty(_n_rows(logits), device=logits.device, dtype=torch.int64)
    ext().argmax(logits, out)
    return out


def sample_gumbel(logits, inv_temp, seed, offset):
    out = torch.empty(_n_rows(logits), device=logits.device, dtype=torch.int64)
    ext().gumbel_sample(logits, out, float(inv_temp), int(seed), int(offset))
    return out


_STOPS: dict = {}


def cycle_payload(proposal, lookahead, stops: tuple, *, accepted=None, corr=None, target=None):
    """``[B, L+2]`` committed tokens + count of a linear cycle (one kernel; see ``cycle_payload_kernel``)."""
    B, L = proposal.shape
    dev = proposal.device
    key = (dev, stops)
    st = _STOPS.get(key)
    if st is None:
        st = torch.tensor(list(stops), dtype=torch.int64, device=dev)
        _STOPS[key] = st
    out = torch.empty(B, L + 2, dtype=torch.int64, device=dev)
    ext().cycle_payload(proposal.contiguous(), None if accepted is None else accepted.reshape(-1).to(torch.int32),
                        None if target is None else target.reshape(-1).to(torch.int64).contiguous(),
                        None if corr is None else corr.reshape(-1).to(torch.int64).contiguous(),
                        lookahead.reshape(-1).to(torch.int64).contiguous(), st, out)
    return out


def tree_meta(parents, depths, prefix_lens, masks_out, positions_out) -> None:
    """Ancestor-or-self masks and positions (prefix + depth) of draft trees, written in place."""
    ext().tree_meta(parents.contiguous(), depths.to(torch.int64).contiguous(), prefix_lens, masks_out, positions_out)


def fused_verify(clean, draft, spec, inv_temp, seed, offset):
    n = _n_rows(clean)
    acc = torch.empty(n, device=clean.device, dtype=torch.int32)
    corr = torch.empty(n, device=clean.device, dtype=torch.int64)
    ext().fused_verify(clean, draft, spec.reshape(-1).contiguous(), float(inv_temp), int(seed), int(offset), acc,
                       corr)
    return acc, corr


def filtered_sample(logits, inv_temp, top_k, top_p, seed, offset):
    """Top-k / top-p sample of bf16 ``[N, V]`` or strided ``[B, R, V]`` logits (``filtered.cu``).

    Returns ``(tokens [N] int64, params [N, 2] int64)``: per row the key of the
    last kept token, and the row max and kept mass packed as two float32.
    ``top_k == 0`` or ``top_p >= 1`` switches that filter off.
    """
    n = _n_rows(logits)
    tok = torch.empty(n, device=logits.device, dtype=torch.int64)
    params = torch.empty(n, 2, device=logits.device, dtype=torch.int64)
    ext().filtered_sample(logits, float(inv_temp), int(top_k), float(top_p), int(seed), int(offset), tok, params)
    return tok, params


def filtered_verify(clean, draft, draft_params, spec, inv_temp, top_k, top_p, seed, offset):
    """Accept test + residual resample on filtered target / draft distributions (``filtered.cu``)."""
    n = _n_rows(clean)
    acc = torch.empty(n, device=clean.device, dtype=torch.int32)
    corr = torch.empty(n, device=clean.device, dtype=torch.int64)
    ext().filtered_verify(clean, draft, draft_params, spec.reshape(-1).contiguous(), float(inv_temp), int(top_k),
                          float(top_p), int(seed), int(offset), acc, corr)
    return acc, corr


def filtered_keys(logits):
    """Per-token ranking keys of ``filtered.cu`` (value descending, lowest id first) as int64."""
    x = logits.reshape(-1, logits.shape[-1]).contiguous()
    bits = x.view(torch.int16).to(torch.int64) & 0xFFFF
    order = torch.where(bits >= 0x8000, (~bits) & 0xFFFF, bits | 0x8000)
    ids = torch.arange(x.shape[-1], device=x.device, dtype=torch.int64)
    return (order << 32) | (0xFFFFFFFF - ids)


def filtered_kept(logits, params):
    """Boolean keep mask of ``filtered_sample`` params."""
    return filtered_keys(logits) >= params[:, :1]


def unpack_filtered_params(params):
    """``(last-kept key, row max m, kept mass S)`` of ``filtered_sample`` params."""
    packed = params[:, 1].contiguous()
    lo = (packed & 0xFFFFFFFF).to(torch.int32)
    hi = ((packed >> 32) & 0xFFFFFFFF).to(torch.int32)
    return params[:, 0], lo.view(torch.float32), hi.view(torch.float32)


def vp_sample(logits, inv_temp, seed, offset, vocab_start, greedy=False):
    """Sample (or arg-max) from a vocab-parallel logits shard; every rank gets the same global ids."""
    regions, rank, max_rows = _COMM.vp_args()
    out = torch.empty(_n_rows(logits), device=logits.device, dtype=torch.int64)
    ext().vp_sample(logits, out, float(inv_temp), bool(greedy), int(seed), int(offset), regions, rank, max_rows,
                    int(vocab_start))
    return out


def vp_verify(clean, draft, spec, inv_temp, seed, offset, vocab_start):
    """Psi-Spec accept test + residual resample on vocab-parallel shards of the target/draft logits."""
    regions, rank, max_rows = _COMM.vp_args()
    n = _n_rows(clean)
    acc = torch.empty(n, device=clean.device, dtype=torch.int32)
    corr = torch.empty(n, device=clean.device, dtype=torch.int64)
    ext().vp_verify(clean, draft, spec.reshape(-1).contiguous(), float(inv_temp), int(seed), int(offset), acc, corr,
                    regions, rank, max_rows, int(vocab_start))
    return acc, corr


def build_draft_tree(root_tokens, draft_logits, max_nodes, candidate_top_k, temperature, candidates=None):
    """Draft trees on the device; ``candidates`` = precomputed ``(ids, log-probs)`` ``[B, D, K]``."""
    from uno_b200.engine.draft_tree import DraftTreeBatch

    B, D, V = draft_logits.shape
    if candidates is not None:
        ids, lp = (c.reshape(B * D, -1).contiguous() for c in candidates)
        lp = lp.float()
        K = ids.shape[1]
    else:
        K = min(int(candidate_top_k), V)
        rows = draft_logits.reshape(B * D, V)
        ids = torch.empty(B * D, K, device=rows.device, dtype=torch.int64)
        lp = torch.empty(B * D, K, device=rows.device, dtype=torch.float32)
        inv_t = 1.0 / temperature if temperature > 0 else 1.0
        ext().topk_lse(rows, K, inv_t, ids, lp)
    dev = draft_logits.device
    tok = torch.empty(B, max_nodes, device=dev, dtype=torch.int64)
    par = torch.empty_like(tok)
    dep = torch.empty_like(tok)
    mass = torch.empty(B, max_nodes, device=dev, dtype=torch.float32)
    count = torch.empty(B, device=dev, dtype=torch.int32)
    ext().build_tree(root_tokens.contiguous(), ids.view(B, D, K), lp.view(B, D, K), int(max_nodes), tok, par, dep,
                     mass, count)
    return DraftTreeBatch(tok, par, dep, mass)


def walk_tree(tokens, parents, targets, max_depth, pad_token_id):
    B = tokens.shape[0]
    committed = torch.empty(B, max_depth + 2, device=tokens.device, dtype=torch.int64)
    accepted = torch.empty(B, max_depth + 1, device=tokens.device, dtype=torch.int64)
    lengths = torch.empty(B, device=tokens.device, dtype=torch.int64)
    ext().walk_tree(tokens.contiguous(), parents.contiguous(), targets.contiguous(), int(max_depth),
                    int(pad_token_id), committed, accepted, lengths)
    return committed, accepted, lengths


def copy_tree_kv(kv_cache, tables, src, dst, page):
    ext().copy_tree_kv(kv_cache, tables.contiguous(), src.contiguous(), dst.contiguous(), int(page))
