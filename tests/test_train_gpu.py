"""Training on the GPU: native tcgen05 projections vs the torch-op path (same model, same LoRA)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup(seed=0, head_dim=64, hidden=256, heads=4, kv_heads=2, inter=768):
    from uno_b200.models.decoder import build_model
    from uno_b200.train import LoraSettings, TrainableLoRA, build_uno_batch
    from uno_b200.train.optim import ShardedLoraAdamW
    from uno_b200.utils.hf_compat import ModelConfig
    from uno_b200.utils.loader import dummy_init

    cfg = ModelConfig(model_type="qwen3", vocab_size=4096, hidden_size=hidden, intermediate_size=inter,
                      num_hidden_layers=2, num_attention_heads=heads, num_key_value_heads=kv_heads, head_dim=head_dim,
                      max_position_embeddings=2048, mask_token_id=4095, rope_theta=1e6)
    torch.set_default_dtype(torch.bfloat16)
    with torch.device("cuda"):
        model = build_model(cfg)
    torch.set_default_dtype(torch.float32)
    dummy_init(model, seed=seed)
    lora = TrainableLoRA(cfg, LoraSettings(target="all", rank=8, alpha=16), device="cuda", seed=seed)
    with torch.no_grad():
        g = torch.Generator(device="cuda").manual_seed(seed + 1)
        for p in lora.B.values():  # non-zero B so both factors receive gradients
            p.copy_(torch.randn(p.shape, device="cuda", generator=g) * 0.05)
    opt = ShardedLoraAdamW(list(lora.parameters()), lr=1e-3)
    ids = torch.randint(1, 4000, (1, 256), device="cuda", generator=torch.Generator(device="cuda").manual_seed(5))
    labels = ids.clone()
    labels[:, :32] = -100
    pos = torch.arange(256, device="cuda")[None]
    ub = build_uno_batch(ids, labels, pos, block_size=4, mask_token_id=4095,
                         generator=torch.Generator(device="cuda").manual_seed(7))
    return model, lora, opt, ub


def _grads(native: bool, head_dim: int = 64):
    from uno_b200.train.attention import AttentionMeta
    from uno_b200.train.forward import uno_hidden_states
    from uno_b200.train.native import build_projections

    model, lora, opt, ub = _setup(head_dim=head_dim)
    proj = build_projections(model, lora)[0] if native else None
    if proj is not None:
        for layer in proj:
            for p in layer.values():
                p.refresh(0)
    opt.zero_grad()
    vis = ub.attention_mask()
    meta = AttentionMeta(ub.segment, ub.positions, ub.noisy, ub.block_size, vis=vis) if native else None
    h = uno_hidden_states(model, lora, ub.ids, ub.positions, vis, ub.noisy, native=proj, attn_meta=meta)
    w = torch.randn(h.shape, device="cuda", generator=torch.Generator(device="cuda").manual_seed(9))
    (h.float() * w).sum().backward()
    torch.cuda.synchronize()
    out = opt.flat_grad.clone(), h.detach().float()
    opt.close()
    return out


@pytest.mark.parametrize("head_dim", [64, 128])
def test_native_projections_match_torch_path(head_dim):
    """head_dim 128 also runs the block-diffusion attention kernels inside the training forward/backward."""
    from uno_b200.ops import cuda

    g_ref, h_ref = _grads(native=False, head_dim=head_dim)
    g_nat, h_nat = _grads(native=True, head_dim=head_dim)
    assert cuda.error_flag() == 0
    assert ((h_nat - h_ref).norm() / h_ref.norm()).item() < 2e-2
    rel = ((g_nat - g_ref).norm() / g_ref.norm()).item()
    assert g_ref.abs().sum() > 0 and rel < 5e-2, rel


@pytest.mark.parametrize("weights,teacher_ce", [((1.0, 0.0, 0.0), True), ((0.3, 0.5, 0.7), True),
                                                ((0.0, 0.0, 1.0), False), ((0.2, 1.0, 0.0), False)])
def test_loss_kernel_matches_fp32_terms(weights, teacher_ce):
    """The fused TV/KL/CE kernel vs the fp32 torch terms on the same bf16 logits (row losses and d/d logits)."""
    from uno_b200.ops import cuda
    from uno_b200.train.losses import _chunk_terms

    g = torch.Generator(device="cuda").manual_seed(2)
    N, V = 100, 5003  # V not a multiple of 8: the scalar tail runs too
    s = (torch.randn(N, V, device="cuda", generator=g) * 2).bfloat16()
    t = (s.float() + torch.randn(N, V, device="cuda", generator=g)).bfloat16()
    s = torch.nn.functional.pad(s, (0, 5)).contiguous()[:, :V]  # row stride 5008 (16-byte aligned rows)
    t = torch.nn.functional.pad(t, (0, 5)).contiguous()[:, :V]
    tgt = torch.randint(0, V, (N,), device="cuda", generator=g)
    ce_w = torch.rand(N, device="cuda", generator=g) + 0.5
    dist_w = (torch.rand(N, device="cuda", generator=g) > 0.3).float()
    row_loss = torch.empty(N, device="cuda")
    grad = torch.empty(N, V + 5, device="cuda", dtype=torch.bfloat16)[:, :V]
    cuda.ext().uno_loss(s, t, tgt, teacher_ce, ce_w, dist_w, *weights, row_loss, grad)
    y = t.float().argmax(-1) if teacher_ce else tgt
    ref_loss, ref_grad = _chunk_terms(s.float(), t.float(), y, ce_w, dist_w, weights)
    assert cuda.error_flag() == 0
    assert abs(row_loss.sum().item() - ref_loss.item()) <= 1e-3 * abs(ref_loss.item()) + 1e-3
    assert ((grad.float() - ref_grad).norm() / ref_grad.norm()).item() < 1e-2


def test_fused_head_loss_cuda_path_matches_fp32():
    """lm_head GEMM chunks + loss kernel + d h GEMM vs the fp32 path (data-target CE: no arg-max near-ties)."""
    from uno_b200.ops import cuda
    from uno_b200.train.losses import fused_head_loss

    g = torch.Generator(device="cuda").manual_seed(1)
    N, H, V = 300, 256, 4096
    w = (torch.randn(V, H, device="cuda", generator=g) * 0.08).bfloat16()
    s = torch.randn(N, H, device="cuda", generator=g).bfloat16()
    t = (s.float() + 0.3 * torch.randn(N, H, device="cuda", generator=g)).bfloat16()
    dist = torch.rand(N, device="cuda", generator=g) > 0.2
    ce = torch.rand(N, device="cuda", generator=g) > 0.5
    tgt = torch.randint(0, V, (N,), device="cuda", generator=g)
    scale = 1.0 + torch.rand(N, device="cuda", generator=g)
    kw = dict(dist_mask=dist, ce_mask=ce, ce_target=tgt, ce_scale=scale, tv_weight=0.0, kl_weight=0.5,
              ce_weight=1.0, teacher_ce=False, normalizer=int(dist.sum()), chunk=128)
    s1 = s.clone().requires_grad_(True)
    loss = fused_head_loss(s1, t, w, **kw)
    loss.backward()
    s2 = s.float().clone().requires_grad_(True)
    ref = fused_head_loss(s2, t.float(), w.float(), **kw)
    ref.backward()
    assert cuda.error_flag() == 0
    assert abs(loss.item() - ref.item()) <= 1e-2 * abs(ref.item()) + 1e-4
    gerr = ((s1.grad.float() - s2.grad).norm() / s2.grad.norm()).item()
    assert gerr < 3e-2, gerr


@pytest.mark.parametrize("S,block,packed,hq,hkv", [(200, 4, False, 4, 2), (256, 8, True, 8, 2), (96, 16, False, 2, 2)])
def test_block_diffusion_attention_matches_sdpa(S, block, packed, hq, hkv):
    """Forward output and q/k/v gradients of the training attention kernels vs fp32 SDPA with the dense mask."""
    from uno_b200.ops import cuda
    from uno_b200.train import build_uno_batch
    from uno_b200.train.attention import AttentionMeta, block_diffusion_attention

    g = torch.Generator(device="cuda").manual_seed(S + block)
    B = 2
    ids = torch.randint(1, 1000, (B, S), device="cuda", generator=g)
    pos = torch.arange(S, device="cuda").expand(B, S).clone()
    if packed:  # two packed sequences in every row
        pos[:, S // 2 + 8:] -= S // 2 + 8
    ub = build_uno_batch(ids, ids.clone(), pos, block_size=block, mask_token_id=1001, generator=g)
    vis = ub.attention_mask()
    meta = AttentionMeta(ub.segment, ub.positions, ub.noisy, block, vis=vis)
    T = 2 * S
    q = torch.randn(B, T, hq, 128, device="cuda", generator=g).bfloat16().requires_grad_(True)
    k = torch.randn(B, T, hkv, 128, device="cuda", generator=g).bfloat16().requires_grad_(True)
    v = torch.randn(B, T, hkv, 128, device="cuda", generator=g).bfloat16().requires_grad_(True)
    dout = torch.randn(B, T, hq, 128, device="cuda", generator=g).bfloat16()
    scale = 128 ** -0.5
    out = block_diffusion_attention(q, k, v, meta, scale)
    out.backward(dout)
    qf, kf, vf = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    ref = torch.nn.functional.scaled_dot_product_attention(
        qf.transpose(1, 2), kf.transpose(1, 2), vf.transpose(1, 2), attn_mask=vis[:, None], scale=scale,
        enable_gqa=hq != hkv).transpose(1, 2)
    ref.backward(dout.float())
    assert cuda.error_flag() == 0

    def rel(a, b):
        return ((a.float() - b).norm() / b.norm()).item()

    assert rel(out, ref) < 1e-2
    assert rel(q.grad, qf.grad) < 3e-2 and rel(k.grad, kf.grad) < 3e-2 and rel(v.grad, vf.grad) < 3e-2


@pytest.mark.parametrize("groups", [1, 4])
def test_training_rmsnorm_and_silu_kernels_match_torch(groups):
    """Fused RMSNorm / SiLU*up forward and backward vs torch autograd of the fp32-statistics formulation."""
    from uno_b200.ops import reference as R
    from uno_b200.train.native import rms_norm, silu_mul

    g = torch.Generator(device="cuda").manual_seed(groups)
    x = (torch.randn(300, 1024, device="cuda", generator=g) * 2).bfloat16().requires_grad_(True)
    w = (1 + 0.1 * torch.randn(1024, device="cuda", generator=g)).bfloat16()
    dy = torch.randn(300, 1024, device="cuda", generator=g).bfloat16()
    y = rms_norm(x, w, 1e-6, groups)
    y.backward(dy)
    xr = x.detach().float().requires_grad_(True)
    yr = R.rms_norm(xr, w.float(), 1e-6, groups)
    yr.backward(dy.float())
    assert ((y.float() - yr).norm() / yr.norm()).item() < 1e-2
    assert ((x.grad.float() - xr.grad).norm() / xr.grad.norm()).item() < 1e-2

    gu = torch.randn(300, 2 * 768, device="cuda", generator=g).bfloat16().requires_grad_(True)
    da = torch.randn(300, 768, device="cuda", generator=g).bfloat16()
    a = silu_mul(gu)
    a.backward(da)
    gr = gu.detach().float().requires_grad_(True)
    ar = torch.nn.functional.silu(gr[:, :768]) * gr[:, 768:]
    ar.backward(da.float())
    assert ((a.float() - ar).norm() / ar.norm()).item() < 1e-2
    assert ((gu.grad.float() - gr.grad).norm() / gr.grad.norm()).item() < 1e-2


@pytest.mark.parametrize("norm", [True, False])
def test_training_qk_norm_rope_kernel_matches_torch(norm):
    """Fused per-head RMSNorm + NeoX RoPE (forward and backward) on a column slice of a fused qkv output."""
    from uno_b200.layers.rotary import cos_sin_cache
    from uno_b200.ops import reference as R
    from uno_b200.train.native import qk_norm_rope

    g = torch.Generator(device="cuda").manual_seed(7)
    T, H, N = 300, 4, 1024
    qkv = torch.randn(T, N, device="cuda", generator=g).bfloat16().requires_grad_(True)
    w = (1 + 0.1 * torch.randn(128, device="cuda", generator=g)).bfloat16() if norm else None
    pos = torch.randint(0, 2000, (T,), device="cuda", generator=g)
    cs = cos_sin_cache(128, 4096, 1e6, None, device="cuda").float()
    dy = torch.randn(T, H, 128, device="cuda", generator=g).bfloat16()
    x = qkv[:, 128:128 + H * 128].unflatten(1, (H, 128))
    out = qk_norm_rope(x, w, 1e-6, pos, cs)
    out.backward(dy)
    qf = qkv.detach().float().requires_grad_(True)
    xf = qf[:, 128:128 + H * 128].unflatten(1, (H, 128))
    if norm:
        xf = R.head_rms_norm(xf, w.float(), 1e-6)
    ref = R.apply_rope(xf, pos, cs)
    ref.backward(dy.float())
    assert ((out.float() - ref).norm() / ref.norm()).item() < 1e-2
    assert ((qkv.grad.float() - qf.grad).norm() / qf.grad.norm()).item() < 1e-2
    assert qkv.grad[:, :128].abs().max().item() == 0 and qkv.grad[:, 128 + H * 128:].abs().max().item() == 0
