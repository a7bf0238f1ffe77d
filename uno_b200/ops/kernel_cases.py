"""Kernel microbenchmarks at the decode-step shapes (Qwen3-8B, 64 x 8 tokens).

``python -m uno_b200.ops.kernel_cases CASE [--repeat N]`` runs two warm-up
launches of the case, then one launch inside the NVTX range ``capture`` (for
``ncu --nvtx --nvtx-include capture/``), then times a CUDA graph of
``--repeat`` back-to-back launches with CUDA events (per-launch device time,
host launch cost excluded) and prints one JSON line per kernel.  Inputs are random; the
decode-attention KV cache (~240 MB) is larger than the L2.

Cases: ``layer-gemms`` (gate_up + SiLU, qkv, o_proj, down, LoRA hidden), ``decode-attention``.
"""

from __future__ import annotations

import argparse
import json

import torch


def _layer_gemms():
    from uno_b200.ops import cuda as C

    M, H, I = 512, 4096, 12288
    x = torch.randn(M, H, device="cuda").bfloat16()
    w_gu = C.interleave_gate_up(torch.randn(2 * I, H, device="cuda").bfloat16() * 0.02)
    act = torch.empty(M, I, device="cuda", dtype=torch.bfloat16)
    w_o = torch.randn(H, H, device="cuda").bfloat16() * 0.02
    y = torch.empty(M, H, device="cuda", dtype=torch.bfloat16)
    w_qkv = torch.randn(6144, H, device="cuda").bfloat16() * 0.02
    qkv = torch.empty(M, 6144, device="cuda", dtype=torch.bfloat16)
    a_i = torch.randn(M, I, device="cuda").bfloat16()
    w_d = torch.randn(H, I, device="cuda").bfloat16() * 0.02
    a_l = torch.randn(192, H, device="cuda").bfloat16() * 0.02
    h_l = torch.empty(M, 192, device="cuda", dtype=torch.bfloat16)
    mask = torch.ones(M, device="cuda")
    return {
        "gate_up_silu 512x24576x4096": (lambda: C._gemm(x, w_gu, C.EPI_SILU, c=act), 2 * M * 2 * I * H,
                                        2 * I * H * 2),
        "qkv (plain store) 512x6144x4096": (lambda: C._gemm(x, w_qkv, C.EPI_STORE, c=qkv), 2 * M * 6144 * H,
                                            6144 * H * 2),
        "o_proj 512x4096x4096": (lambda: C._gemm(x, w_o, C.EPI_STORE, c=y), 2 * M * H * H, H * H * 2),
        "down 512x4096x12288": (lambda: C._gemm(a_i, w_d, C.EPI_STORE, c=y), 2 * M * H * I, H * I * 2),
        "lora_hidden 512x192x4096": (lambda: C._gemm(x, a_l, C.EPI_ROWSCALE, c=h_l, scale=2.0, row_mask=mask),
                                     2 * M * 192 * H, (M + 192) * H * 2),
    }


def _decode_attention():
    from uno_b200.layers.meta import ForwardMeta, Mode, causal_suffix_masks
    from uno_b200.ops import cuda as C

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
    return {f"decode_attention B={B} Q={Q} mean_kv={sum(lens) // B}":
            (lambda: C.attention(q, kc, vc, meta, 128 ** -0.5), 0, kv_bytes)}


CASES = {"layer-gemms": _layer_gemms, "decode-attention": _decode_attention}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("case", choices=sorted(CASES))
    ap.add_argument("--repeat", type=int, default=20)
    args = ap.parse_args(argv)
    from uno_b200.ops import cuda as C

    torch.manual_seed(0)
    cases = CASES[args.case]()
    for _ in range(2):
        for fn, _, _ in cases.values():
            fn()
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("capture")
    for fn, _, _ in cases.values():
        fn()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    out = []
    for name, (fn, flops, nbytes) in cases.items():
        # replay a CUDA graph of back-to-back launches: host launch cost stays off the clock
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(args.repeat):
                fn()
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
