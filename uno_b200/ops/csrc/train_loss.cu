// Uno diffusion loss over full-vocabulary student/teacher logit rows.
//
// Objective of ``training/losses.py:59-183`` / ``training/trainer.py:249-287``
// per supervised token row: total variation sum_v |p_s - p_t|, reverse KL
// sum_v p_s (log p_s - log p_t), and cross entropy of the student against
// the teacher's arg-max (or the data's next token) weighted by 1 / p_mask.
// One CTA per row makes three passes over the two bf16 rows:
//
//   1. online max / sum-exp of both rows (log-normalisers) and the teacher's
//      arg-max (lowest id on ties);
//   2. row sums: TV, sum_v sign(p_s - p_t) p_s, and KL;
//   3. the closed-form gradient with respect to the student logits,
//        tv_w * dw * p_s * (sign - sum sign p_s)
//      + kl_w * dw * p_s * (log p_s - log p_t - KL)
//      + ce * cw * (p_s - onehot(y)),
//      written as bf16 (it may overwrite the student row in place: every
//      element is read and then written by the same thread).
//
// The row's loss contribution goes to row_loss[r]; the caller sums the rows
// and normalises by the supervised-token count.
#include "common.cuh"
#include "sampling_common.cuh"
#include "uno_ops.h"

namespace uno {

constexpr int LOSS_THREADS = 512;

__global__ void __launch_bounds__(LOSS_THREADS)
    uno_loss_kernel(const __nv_bfloat16* __restrict__ s, int64_t lds, const __nv_bfloat16* __restrict__ t, int64_t ldt,
                    int V, const int64_t* __restrict__ target, int teacher_ce, const float* __restrict__ ce_w,
                    const float* __restrict__ dist_w, float tv_w, float kl_w, float ce_weight,
                    float* __restrict__ row_loss, __nv_bfloat16* grad, int64_t ldg) {
  const int r = blockIdx.x;
  const __nv_bfloat16* sr = s + (size_t)r * lds;
  const __nv_bfloat16* tr = t + (size_t)r * ldt;
  __nv_bfloat16* gr = grad + (size_t)r * ldg;
  const int nvec = V / 8;
  const bool need_dist = tv_w > 0.f || kl_w > 0.f;

  // ---- pass 1: log-normalisers and the teacher's arg-max
  MaxSum as{-INFINITY, 0.f}, at{-INFINITY, 0.f};
  ArgBest best{-INFINITY, 0x7fffffff};
  for (int c = threadIdx.x; c < nvec; c += blockDim.x) {
    float a[8], b[8];
    load8(sr + c * 8, a);
    load8(tr + c * 8, b);
    float ma = a[0], mb = b[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) {
      ma = fmaxf(ma, a[i]);
      mb = fmaxf(mb, b[i]);
    }
    float sa = 0.f, sb = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      sa += __expf(a[i] - ma);
      sb += __expf(b[i] - mb);
      best = better(best, ArgBest{b[i], c * 8 + i});
    }
    as = ms_merge(as, MaxSum{ma, sa});
    at = ms_merge(at, MaxSum{mb, sb});
  }
  for (int i = nvec * 8 + threadIdx.x; i < V; i += blockDim.x) {
    const float a = __bfloat162float(sr[i]), b = __bfloat162float(tr[i]);
    as = ms_merge(as, MaxSum{a, 1.f});
    at = ms_merge(at, MaxSum{b, 1.f});
    best = better(best, ArgBest{b, i});
  }
  as = block_maxsum(as);
  at = block_maxsum(at);
  best = block_best(best);
  const float lse_s = as.m + __logf(as.s);
  const float lse_t = at.m + __logf(at.s);
  const int64_t y = teacher_ce ? (int64_t)best.i : target[r];
  const float dw = dist_w[r], cw = ce_w[r];

  // ---- pass 2: row sums
  float tv = 0.f, sgp = 0.f, kl = 0.f;
  if (need_dist) {
    for (int c = threadIdx.x; c < nvec; c += blockDim.x) {
      float a[8], b[8];
      load8(sr + c * 8, a);
      load8(tr + c * 8, b);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float ls = a[i] - lse_s, lt = b[i] - lse_t;
        const float ps = __expf(ls), pt = __expf(lt);
        const float d = ps - pt;
        tv += fabsf(d);
        sgp += d > 0.f ? ps : (d < 0.f ? -ps : 0.f);
        kl += ps * (ls - lt);
      }
    }
    for (int i = nvec * 8 + threadIdx.x; i < V; i += blockDim.x) {
      const float ls = __bfloat162float(sr[i]) - lse_s, lt = __bfloat162float(tr[i]) - lse_t;
      const float ps = __expf(ls), pt = __expf(lt);
      const float d = ps - pt;
      tv += fabsf(d);
      sgp += d > 0.f ? ps : (d < 0.f ? -ps : 0.f);
      kl += ps * (ls - lt);
    }
    tv = block_sum(tv);
    sgp = block_sum(sgp);
    kl = block_sum(kl);
  }
  const float ls_y = (y >= 0 && y < V) ? __bfloat162float(sr[y]) - lse_s : 0.f;
  __syncthreads();  // every thread has read sr[y] before pass 3 may overwrite it in place
  if (threadIdx.x == 0) row_loss[r] = tv_w * dw * tv + kl_w * dw * kl - ce_weight * cw * ls_y;

  // ---- pass 3: gradient with respect to the student logits
  const float gt = tv_w * dw, gk = kl_w * dw, gc = ce_weight * cw;
  for (int c = threadIdx.x; c < nvec; c += blockDim.x) {
    float a[8], b[8], g[8];
    load8(sr + c * 8, a);
    load8(tr + c * 8, b);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float ls = a[i] - lse_s, lt = b[i] - lse_t;
      const float ps = __expf(ls), pt = __expf(lt);
      const float d = ps - pt;
      const float sign = d > 0.f ? 1.f : (d < 0.f ? -1.f : 0.f);
      g[i] = gt * ps * (sign - sgp) + gk * ps * (ls - lt - kl) + gc * (ps - ((int64_t)(c * 8 + i) == y ? 1.f : 0.f));
    }
    uint4 w;
    w.x = pack_bf16x2(g[0], g[1]);
    w.y = pack_bf16x2(g[2], g[3]);
    w.z = pack_bf16x2(g[4], g[5]);
    w.w = pack_bf16x2(g[6], g[7]);
    *reinterpret_cast<uint4*>(gr + c * 8) = w;
  }
  for (int i = nvec * 8 + threadIdx.x; i < V; i += blockDim.x) {
    const float ls = __bfloat162float(sr[i]) - lse_s, lt = __bfloat162float(tr[i]) - lse_t;
    const float ps = __expf(ls), pt = __expf(lt);
    const float d = ps - pt;
    const float sign = d > 0.f ? 1.f : (d < 0.f ? -1.f : 0.f);
    gr[i] = __float2bfloat16(gt * ps * (sign - sgp) + gk * ps * (ls - lt - kl) + gc * (ps - (i == y ? 1.f : 0.f)));
  }
}

void uno_loss_launch(const at::Tensor& s, const at::Tensor& t, const at::Tensor& target, bool teacher_ce,
                     const at::Tensor& ce_w, const at::Tensor& dist_w, double tv_w, double kl_w, double ce_weight,
                     at::Tensor& row_loss, at::Tensor& grad) {
  const at::Tensor* mats[3] = {&s, &t, &grad};
  for (const at::Tensor* x : mats) {
    check_dev(*x, "loss logits");
    TORCH_CHECK(x->scalar_type() == at::kBFloat16 && x->dim() == 2 && x->stride(1) == 1, "bf16 [rows, V] rows");
    TORCH_CHECK(x->stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(x->data_ptr()) % 16 == 0,
                "logit rows must be 16-byte aligned");
  }
  const int rows = s.size(0), V = s.size(1);
  TORCH_CHECK(t.size(0) == rows && t.size(1) == V && grad.size(0) == rows && grad.size(1) == V, "loss shapes");
  TORCH_CHECK(target.scalar_type() == at::kLong && target.numel() >= rows, "targets");
  TORCH_CHECK(ce_w.scalar_type() == at::kFloat && dist_w.scalar_type() == at::kFloat &&
                  row_loss.scalar_type() == at::kFloat && row_loss.numel() >= rows,
              "fp32 row weights / losses");
  if (rows == 0) return;
  uno_loss_kernel<<<rows, LOSS_THREADS, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(s.data_ptr()), s.stride(0),
      reinterpret_cast<const __nv_bfloat16*>(t.data_ptr()), t.stride(0), V, target.data_ptr<int64_t>(),
      teacher_ce ? 1 : 0, ce_w.data_ptr<float>(), dist_w.data_ptr<float>(), (float)tv_w, (float)kl_w,
      (float)ce_weight, row_loss.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(grad.data_ptr()),
      grad.stride(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace uno
