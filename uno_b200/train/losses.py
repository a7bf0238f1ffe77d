"""Uno losses fused with the LM head, over row chunks.

Objective of ``training/trainer.py:223-287`` and ``training/losses.py:59-183``,
per supervised token (normalised by the number of supervised tokens):

* total variation ``sum_v |p_s - p_t|`` (full vocabulary, exact);
* reverse KL ``sum_v p_s (log p_s - log p_t)``;
* cross entropy of the student against the clean teacher's argmax (or the
  data's next token) on noised positions, weighted by ``1 / p_mask``.

The teacher is the frozen base model on the clean copy (no gradient).
``fused_head_loss`` never materialises the ``[rows, V]`` logits of the whole
batch: rows are processed in chunks, and the loss gradient with respect to
the student logits is formed in closed form inside the same pass --

  d TV / d s  = p_s * (sign(p_s - p_t) - sum_v sign * p_s)
  d KL / d s  = p_s * (log p_s - log p_t - KL_row)
  d CE / d s  = w * (p_s - onehot(y))

-- and immediately projected back to ``d h = d s . W``; only the
``[rows, H]`` gradient is kept for backward.  On CUDA each chunk is two
tcgen05 GEMMs for the logits, one kernel for the three terms and their
gradient (written over the student logits), and one GEMM for ``d h``.
"""

from __future__ import annotations

import torch


def _chunk_terms(s_logits, t_logits, targets, ce_w, dist_w, weights):
    """Loss sum and d loss / d student-logits for one chunk (fp32)."""
    tv_w, kl_w, ce_weight = weights
    ls = torch.log_softmax(s_logits, dim=-1)
    ps = ls.exp()
    grad = torch.zeros_like(s_logits)
    loss = s_logits.new_zeros(())
    if tv_w > 0 or kl_w > 0:
        lt = torch.log_softmax(t_logits, dim=-1)
        dw = dist_w[:, None]
        if tv_w > 0:
            pt = lt.exp()
            sign = torch.sign(ps - pt)
            loss = loss + tv_w * ((ps - pt).abs().sum(-1) * dist_w).sum()
            grad += tv_w * dw * ps * (sign - (sign * ps).sum(-1, keepdim=True))
        if kl_w > 0:
            diff = ls - lt
            kl_row = (ps * diff).sum(-1, keepdim=True)
            loss = loss + kl_w * (kl_row.squeeze(-1) * dist_w).sum()
            grad += kl_w * dw * ps * (diff - kl_row)
    if ce_weight > 0:
        w = ce_w[:, None]
        y = targets.clamp(min=0)
        loss = loss - ce_weight * (ls.gather(1, y[:, None]).squeeze(1) * ce_w).sum()
        g = ps.clone()
        g.scatter_add_(1, y[:, None], -torch.ones_like(y[:, None], dtype=g.dtype))
        grad += ce_weight * w * g
    return loss, grad


def _transposed(weight: torch.Tensor) -> torch.Tensor:
    """A cached ``[H, V]`` copy of the frozen lm_head weight (the K-major operand of ``d h = d s . W``)."""
    cached = getattr(weight, "_uno_transposed", None)
    if cached is None or cached.shape != weight.t().shape:
        cached = weight.detach().t().contiguous()
        weight._uno_transposed = cached
    return cached


def _head_loss_cuda(student_h, teacher_h, w, ce_target, ce_w, dist_w, weights, teacher_ce, chunk):
    """Chunks through the tcgen05 GEMMs and the fused loss kernel (``ops/csrc/train_loss.cu``)."""
    from uno_b200.ops import cuda as C

    rows, H = student_h.shape
    V = w.shape[0]
    wt = _transposed(w)
    tv_w, kl_w, ce_weight = weights
    grad_h = torch.empty(rows, H, dtype=torch.bfloat16, device=student_h.device)
    row_loss = torch.empty(rows, dtype=torch.float32, device=student_h.device)
    s = torch.empty(min(chunk, rows), V, dtype=torch.bfloat16, device=student_h.device)
    t = torch.empty_like(s)
    sh = student_h.to(torch.bfloat16).contiguous()
    th = teacher_h.to(torch.bfloat16).contiguous()
    tgt = ce_target.long().contiguous()
    for r0 in range(0, rows, chunk):
        r1 = min(rows, r0 + chunk)
        n = r1 - r0
        C._gemm(sh[r0:r1], w, C.EPI_STORE, c=s[:n])
        C._gemm(th[r0:r1], w, C.EPI_STORE, c=t[:n])
        # the gradient overwrites the student logits in place
        C.ext().uno_loss(s[:n], t[:n], tgt[r0:r1], bool(teacher_ce), ce_w[r0:r1].contiguous(),
                         dist_w[r0:r1].contiguous(), float(tv_w), float(kl_w), float(ce_weight), row_loss[r0:r1],
                         s[:n])
        C._gemm(s[:n], wt, C.EPI_STORE, c=grad_h[r0:r1])
    return row_loss.sum(), grad_h


class _FusedHeadLoss(torch.autograd.Function):
    @staticmethod
    def forward(ctx, student_h, teacher_h, weight, ce_target, ce_w, dist_w, weights, teacher_ce, normalizer,
                chunk):
        ctx.normalizer = normalizer
        ctx.h_dtype = student_h.dtype
        w = weight
        if student_h.is_cuda and w.dtype == torch.bfloat16 and w.shape[1] % 64 == 0 and w.shape[0] % 64 == 0:
            total, grad_h = _head_loss_cuda(student_h, teacher_h, w, ce_target, ce_w, dist_w, weights, teacher_ce,
                                            chunk)
            ctx.save_for_backward(grad_h)
            return total / normalizer
        rows = student_h.shape[0]
        grad_h = torch.zeros(rows, student_h.shape[1], dtype=torch.float32, device=student_h.device)
        total = torch.zeros((), dtype=torch.float32, device=student_h.device)
        for r0 in range(0, rows, chunk):
            r1 = min(rows, r0 + chunk)
            s = (student_h[r0:r1] @ w.t()).float()
            t = (teacher_h[r0:r1] @ w.t()).float()
            y = t.argmax(-1) if teacher_ce else ce_target[r0:r1]
            loss, g = _chunk_terms(s, t, y, ce_w[r0:r1], dist_w[r0:r1], weights)
            total += loss
            grad_h[r0:r1] = (g.to(w.dtype) @ w).float()
        ctx.save_for_backward(grad_h)
        return total / normalizer

    @staticmethod
    def backward(ctx, grad_out):
        (grad_h,) = ctx.saved_tensors
        g = (grad_h * (grad_out.float() / ctx.normalizer)).to(ctx.h_dtype)
        return g, None, None, None, None, None, None, None, None, None


def fused_head_loss(student_h: torch.Tensor, teacher_h: torch.Tensor, lm_weight: torch.Tensor, *,
                    dist_mask: torch.Tensor, ce_mask: torch.Tensor, ce_target: torch.Tensor | None,
                    ce_scale: torch.Tensor | None, tv_weight: float, kl_weight: float, ce_weight: float,
                    teacher_ce: bool, normalizer: int, chunk: int = 1024) -> torch.Tensor:
    """Combined Uno loss over ``rows = dist_mask | ce_mask``.

    ``student_h``/``teacher_h`` are ``[N, H]`` (the noisy / clean states of
    the same tokens), ``dist_mask``/``ce_mask`` select rows for TV+KL and for
    CE, ``ce_target`` holds data targets (ignored when ``teacher_ce``) and
    ``ce_scale`` the per-row CE weight ``1 / p_mask``.
    """
    rows = dist_mask | ce_mask
    if not bool(rows.any()):
        return student_h.sum() * 0.0
    s_h, t_h = student_h[rows], teacher_h[rows].detach()
    n = s_h.shape[0]
    dev = s_h.device
    dist_w = dist_mask[rows].float()
    ce_w = torch.zeros(n, device=dev) if ce_scale is None else (ce_scale[rows] * ce_mask[rows].float())
    tgt = torch.zeros(n, dtype=torch.long, device=dev) if ce_target is None else ce_target[rows].long()
    return _FusedHeadLoss.apply(s_h, t_h, lm_weight.detach(), tgt, ce_w.float(), dist_w,
                                (float(tv_weight), float(kl_weight), float(ce_weight)), bool(teacher_ce),
                                max(int(normalizer), 1), int(chunk))


def reference_losses(student_logits, teacher_logits, num_tokens):
    """Plain fp32 TV and reverse KL (test oracle)."""
    ls = torch.log_softmax(student_logits.float(), -1)
    lt = torch.log_softmax(teacher_logits.float(), -1)
    tv = (ls.exp() - lt.exp()).abs().sum() / max(num_tokens, 1)
    kl = (ls.exp() * (ls - lt)).sum() / max(num_tokens, 1)
    return tv, kl
