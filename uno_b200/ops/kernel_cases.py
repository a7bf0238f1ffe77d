"""Kernel microbenchmarks at the decode-step shapes (Qwen3-8B, 64 x 8 tokens).

``python -m uno_b200.ops.kernel_cases CASE [--repeat N]`` runs two warm-up
launches of the case, then one launch inside the NVTX range ``capture`` (for
``ncu --nvtx --nvtx-include capture/``), then times a CUDA graph of
``--repeat`` back-to-back launches with CUDA events (per-launch device time,
host launch cost excluded) and prints one JSON line per kernel.  Inputs are
random.  Consecutive launches never find their operands in the L2: GEMM
weights rotate through enough copies to exceed twice the 126 MB L2, the
lm_head weight (1.24 GB) and the decode-attention KV cache (~240 MB) exceed it
alone, and the sampling case alternates two 156 MB logit blocks.

Cases: ``layer-gemms`` (gate_up + SiLU, qkv, o_proj, down, LoRA hidden),
``lm-head``, ``decode-attention`` (and ``decode-attention-vs-fa2``, the same inputs through the
reference's FlashAttention-2 call), ``sampling`` (full-vocab verify and one
vocab-parallel shard), ``filtered`` (top-k / top-p sampling and verify, with
the eager torch nucleus for comparison), ``train-attention`` (block-diffusion
forward / backward).  A case entry marked ``eager`` (a path with host syncs,
which a graph cannot hold) is timed as ``--repeat`` eager calls instead.
"""

from __future__ import annotations

import argparse
import json

import torch


_L2_BYTES = 126 << 20


def _copies(nbytes: int) -> int:
    """Weight copies to rotate through so that consecutive launches never hit the L2."""
    return max(1, -(-2 * _L2_BYTES // max(1, nbytes)))


def _weights(n: int, k: int, scale: float = 0.02) -> list:
    return [torch.randn(n, k, device="cuda").bfloat16() * scale for _ in range(_copies(n * k * 2))]


def _layer_gemms():
    from uno_b200.ops import cuda as C

    M, H, I = 512, 4096, 12288
    x = torch.randn(M, H, device="cuda").bfloat16()
    w_gu = [C.interleave_gate_up(w) for w in _weights(2 * I, H)]
    act = torch.empty(M, I, device="cuda", dtype=torch.bfloat16)
    w_o = _weights(H, H)
    y = torch.empty(M, H, device="cuda", dtype=torch.bfloat16)
    w_qkv = _weights(6144, H)
    qkv = torch.empty(M, 6144, device="cuda", dtype=torch.bfloat16)
    a_i = torch.randn(M, I, device="cuda").bfloat16()
    w_d = _weights(H, I)
    a_l = _weights(192, H)
    h_l = torch.empty(M, 192, device="cuda", dtype=torch.bfloat16)
    mask = torch.ones(M, device="cuda")
    return {
        "gate_up_silu 512x24576x4096": (lambda i: C._gemm(x, w_gu[i % len(w_gu)], C.EPI_SILU, c=act),
                                        2 * M * 2 * I * H, 2 * I * H * 2),
        "qkv (plain store) 512x6144x4096": (lambda i: C._gemm(x, w_qkv[i % len(w_qkv)], C.EPI_STORE, c=qkv),
                                            2 * M * 6144 * H, 6144 * H * 2),
        "o_proj 512x4096x4096": (lambda i: C._gemm(x, w_o[i % len(w_o)], C.EPI_STORE, c=y), 2 * M * H * H,
                                 H * H * 2),
        "down 512x4096x12288": (lambda i: C._gemm(a_i, w_d[i % len(w_d)], C.EPI_STORE, c=y), 2 * M * H * I,
                                H * I * 2),
        "lora_hidden 512x192x4096": (lambda i: C._gemm(x, a_l[i % len(a_l)], C.EPI_ROWSCALE, c=h_l, scale=2.0,
                                                       row_mask=mask), 2 * M * 192 * H, (M + 192) * H * 2),
    }


def _lm_head():
    from uno_b200.ops import cuda as C

    M, H, V = 512, 4096, 151936
    x = torch.randn(M, H, device="cuda").bfloat16()
    w = [torch.randn(V, H, device="cuda").bfloat16() * 0.02]  # 1.24 GB: larger than the L2 by itself
    return {"lm_head 512x151936x4096": (lambda i: C.lm_head(x, w[0]), 2 * M * V * H, V * H * 2)}


def _sampling():
    """Full-vocabulary verify at TP=1 and the vocab-parallel verify of one TP=8 shard (exchange with itself)."""
    from uno_b200.ops import cuda as C

    B, L, V = 64, 8, 151936
    clean = [torch.randn(B, L, V, device="cuda").bfloat16() * 3 for _ in range(2)]  # 2 x 156 MB
    draft = [c + 0.5 for c in clean]
    spec = torch.randint(0, V, (B * (L - 1),), device="cuda")
    Vs = V // 8
    shards = [c[:, :, :Vs].contiguous() for c in clean]
    dshards = [d[:, :, :Vs].contiguous() for d in draft]
    max_rows = B * L
    region = torch.zeros(C.ext().vp_region_bytes(max_rows), dtype=torch.uint8, device="cuda")
    regions = [region.data_ptr()]
    acc = torch.empty(B * (L - 1), dtype=torch.int32, device="cuda")
    corr = torch.empty(B * (L - 1), dtype=torch.int64, device="cuda")
    rows = B * (L - 1)

    def vp(i):
        j = i % 2
        C.ext().vp_verify(shards[j][:, : L - 1], dshards[j][:, 1:], spec, 1.0, 1, i, acc, corr, regions, 0, max_rows,
                          0)

    return {
        f"fused_verify {rows} rows x V={V}": (lambda i: C.fused_verify(clean[i % 2][:, : L - 1], draft[i % 2][:, 1:],
                                                                       spec, 1.0, 1, i), 0, rows * V * 2 * 2),
        f"vp_verify {rows} rows x V/8={Vs} (1 rank)": (vp, 0, rows * Vs * 2 * 2),
    }


def _filtered():
    """Top-p / top-k sampling of the 64 x 7 draft rows of a decode step and the filtered verify.

    Logit rows are a trained-model-like mix: a peaked head of 50 tokens over a
    N(0, 2.5^2) bulk, so the 0.95 nucleus holds thousands of tokens."""
    from uno_b200.engine import sampling as S
    from uno_b200.ops import cuda as C

    B, L, V = 64, 8, 151936
    head = torch.linspace(12, 4, 50, device="cuda")

    def block():
        x = torch.randn(B, L, V, device="cuda") * 2.5
        x[:, :, :50] += head
        return x.bfloat16()

    blocks = [block(), block()]  # 2 x 156 MB
    rows = B * (L - 1)
    drafted = [C.filtered_sample(b[:, 1:], 1.0, 0, 0.95, 1, 0) for b in blocks]
    nbytes = rows * V * 2

    def sample(k, p):
        return lambda i: C.filtered_sample(blocks[i % 2][:, 1:], 1.0, k, p, 1, i)

    def verify(i):
        j = i % 2
        spec, params = drafted[1 - j]
        C.filtered_verify(blocks[j][:, : L - 1], blocks[1 - j][:, 1:], params, spec, 1.0, 0, 0.95, 1, i)

    return {
        f"filtered_sample top-p 0.95, {rows} rows": (sample(0, 0.95), 0, nbytes),
        f"filtered_sample top-k 50, {rows} rows": (sample(50, 1.0), 0, nbytes),
        f"filtered_sample top-k 50 + top-p 0.9, {rows} rows": (sample(50, 0.9), 0, nbytes),
        f"filtered_verify top-p 0.95, {rows} rows": (verify, 0, 2 * nbytes),
        f"torch sparse_top_p 0.95 (eager), {rows} rows": (
            lambda i: S.sparse_top_p(blocks[i % 2][:, 1:].reshape(-1, V), 1.0, 0.95), 0, nbytes, "eager"),
        f"torch topk 50 (eager), {rows} rows": (
            lambda i: torch.topk(blocks[i % 2][:, 1:].reshape(-1, V), 50, dim=-1), 0, nbytes, "eager"),
    }


def _decode_attention_inputs():
    from uno_b200.layers.meta import ForwardMeta, Mode, causal_suffix_masks

    g = torch.Generator().manual_seed(0)
    B, Q, hq, hkv, page = 64, 8, 32, 8, 256
    lens = (torch.randint(128, 1024, (B,), generator=g) + 300).tolist()
    pages = [-(-(n + Q) // page) for n in lens]
    P = sum(pages) + 4
    kc = torch.randn(P, hkv, page, 128, device="cuda").bfloat16()
    vc = torch.randn(P, hkv, page, 128, device="cuda").bfloat16()
    tables = torch.zeros(B, max(pages), dtype=torch.int32)
    used = 0
    for b in range(B):
        tables[b, :pages[b]] = torch.arange(used, used + pages[b])
        used += pages[b]
    q = torch.randn(B * Q, hq, 128, device="cuda").bfloat16()
    meta = ForwardMeta(mode=Mode.BLOCK, positions=None, slot_mapping=None, block_tables=tables.cuda(),
                       prefix_lens=torch.tensor(lens, dtype=torch.int32, device="cuda"),
                       suffix_mask=causal_suffix_masks(Q, "cuda").repeat(B, 1), seqlen_q=Q, max_kv=3328)
    kv_bytes = sum(n + Q for n in lens) * hkv * 128 * 2 * 2
    return B, Q, lens, q, kc, vc, tables, meta, kv_bytes


def _decode_attention():
    from uno_b200.ops import cuda as C

    B, Q, lens, q, kc, vc, _, meta, kv_bytes = _decode_attention_inputs()
    return {f"decode_attention B={B} Q={Q} mean_kv={sum(lens) // B}":
            (lambda i: C.attention(q, kc, vc, meta, 128 ** -0.5), 0, kv_bytes)}


def _decode_attention_vs_fa2():
    """The same decode step through this framework's kernel and through the reference's call,
    ``flash_attn_with_kvcache`` (FlashAttention 2, ``nano_vllm_uno/layers/attention.py:654-668``),
    on identical inputs: the paged cache re-laid out as [pages, page, kv heads, dim] for FA2, whose
    bottom-right causal alignment over ``cache_seqlens = prefix + Q`` is the Q-row causal block mask.
    The largest output difference is printed before the timings."""
    import json

    from flash_attn import flash_attn_with_kvcache

    from uno_b200.ops import cuda as C

    B, Q, lens, q, kc, vc, tables, meta, kv_bytes = _decode_attention_inputs()
    k_fa, v_fa = kc.permute(0, 2, 1, 3).contiguous(), vc.permute(0, 2, 1, 3).contiguous()
    seqlens = torch.tensor([n + Q for n in lens], dtype=torch.int32, device="cuda")
    table = tables.cuda()
    qb = q.view(B, Q, q.shape[1], q.shape[2])

    def fa2(i):
        return flash_attn_with_kvcache(qb, k_fa, v_fa, cache_seqlens=seqlens, block_table=table,
                                       softmax_scale=128 ** -0.5, causal=True)

    ours = C.attention(q, kc, vc, meta, 128 ** -0.5).float()
    ref = fa2(0).reshape(B * Q, q.shape[1], q.shape[2]).float()
    print(json.dumps({"max_abs_diff_vs_fa2": float((ours - ref).abs().max())}))
    return {f"decode_attention (this framework) B={B} Q={Q}": (lambda i: C.attention(q, kc, vc, meta, 128 ** -0.5),
                                                               0, kv_bytes),
            f"flash_attn_with_kvcache (FA2, the reference's call) B={B} Q={Q}": (fa2, 0, kv_bytes)}


def _train_attention():
    """Training attention (block-diffusion mask) of one 4,096-token sequence: 8,192 laid-out tokens,
    32 query / 8 KV heads of 128, diffusion block 8.  Forward and backward are timed separately."""
    from uno_b200.ops import cuda as C
    from uno_b200.train import build_uno_batch
    from uno_b200.train.attention import AttentionMeta

    S, hq, hkv, D = 4096, 32, 8, 128
    g = torch.Generator(device="cuda").manual_seed(0)
    ids = torch.randint(1, 1000, (1, S), device="cuda", generator=g)
    ub = build_uno_batch(ids, ids.clone(), torch.arange(S, device="cuda")[None], block_size=8, mask_token_id=1001,
                         generator=g)
    vis = ub.attention_mask()
    meta = AttentionMeta(ub.segment, ub.positions, ub.noisy, 8, vis=vis)
    pairs = int(vis.sum())
    T = 2 * S
    q = torch.randn(1, T, hq, D, device="cuda").bfloat16()
    k = torch.randn(1, T, hkv, D, device="cuda").bfloat16()
    v = torch.randn(1, T, hkv, D, device="cuda").bfloat16()
    out = torch.empty_like(q)
    lse = torch.empty(1, hq, T, device="cuda")
    dout = torch.randn_like(q)
    delta = torch.empty_like(lse)
    dq = torch.zeros(q.shape, device="cuda")
    dk, dv = torch.empty_like(k), torch.empty_like(v)
    ext = C.ext()
    args = (meta.seg, meta.pos, meta.noisy, meta.tiles, 8, D ** -0.5)

    def fwd(i):
        ext.train_attn_fwd(q, k, v, *args, out, lse)

    def bwd(i):
        ext.train_attn_bwd(q, k, v, *args, out, dout, lse, delta, dq, dk, dv)

    fwd(0)
    return {f"train_attn_fwd T={T} hq={hq} hkv={hkv} visible={pairs / T / T:.3f}": (fwd, 4 * D * pairs * hq, 0),
            f"train_attn_bwd T={T} hq={hq} hkv={hkv}": (bwd, 10 * D * pairs * hq, 0)}


CASES = {"layer-gemms": _layer_gemms, "lm-head": _lm_head, "decode-attention": _decode_attention,
         "decode-attention-vs-fa2": _decode_attention_vs_fa2,
         "sampling": _sampling, "filtered": _filtered, "train-attention": _train_attention}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("case", choices=sorted(CASES))
    ap.add_argument("--repeat", type=int, default=20)
    args = ap.parse_args(argv)
    from uno_b200.ops import cuda as C

    torch.manual_seed(0)
    cases = CASES[args.case]()
    for i in range(2):
        for fn, *_ in cases.values():
            fn(i)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("capture")
    for fn, *_ in cases.values():
        fn(2)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    out = []
    for name, (fn, flops, nbytes, *mode) in cases.items():
        if mode == ["eager"]:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for i in range(args.repeat):
                fn(i)
            b.record()
            torch.cuda.synchronize()
            ms = a.elapsed_time(b) / args.repeat
            rec = {"kernel": name, "us": round(ms * 1e3, 2), "tflops": None, "gbs": round(nbytes / ms / 1e6, 1),
                   "timing": "eager calls (host syncs included)"}
            out.append(rec)
            print(json.dumps(rec))
            continue
        # replay a CUDA graph of back-to-back launches: host launch cost stays off the clock
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(args.repeat):
                fn(i)
        graph.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / args.repeat
        rec = {"kernel": name, "us": round(ms * 1e3, 2), "tflops": round(flops / ms / 1e9, 1) if flops else None,
               "gbs": round(nbytes / ms / 1e6, 1)}
        out.append(rec)
        print(json.dumps(rec))
        del graph
    if C.error_flag() != 0:
        raise SystemExit("a kernel reported an error")
    return out


if __name__ == "__main__":
    main()
