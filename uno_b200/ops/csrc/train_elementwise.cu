// Elementwise training ops with their backward passes, one read of every
// operand per pass (the torch formulation materialises fp32 copies and runs
// several kernels per op):
//
// * rmsnorm_fwd / rmsnorm_bwd  y = x * rstd * w with rstd = 1/sqrt(mean(x^2) + eps)
//   per row (or per group of columns); the weight is frozen, so backward is
//   dx = rstd * (g - xhat * mean(g * xhat)) with g = dy * w, xhat = x * rstd.
//   The reference computes the norm in fp32 (``layers/layernorm.py:16-40``).
// * silu_mul_fwd / silu_mul_bwd  a = silu(gate) * up on [rows, 2I] = [gate | up];
//   backward dgate = da * up * s * (1 + gate * (1 - s)), dup = da * silu(gate)
//   with s = sigmoid(gate) (``layers/activation.py:6-14``).
// * qk_norm_rope_fwd / _bwd  optional per-head RMSNorm (Qwen3 QK-norm,
//   ``jit_kernel/qk_norm.py:10-87``) followed by the NeoX rotation
//   (``layers/rotary_embedding.py:8-59``); backward applies the transposed
//   rotation, then the per-head norm backward.
#include "common.cuh"
#include "sampling_common.cuh"
#include "uno_ops.h"

namespace uno {

constexpr int EW_THREADS = 256;

__device__ __forceinline__ void ld8(const __nv_bfloat16* p, float* v) { load8(p, v); }

__device__ __forceinline__ void st8(__nv_bfloat16* p, const float* v) {
  uint4 w;
  w.x = pack_bf16x2(v[0], v[1]);
  w.y = pack_bf16x2(v[2], v[3]);
  w.z = pack_bf16x2(v[4], v[5]);
  w.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = w;
}

// One CTA per (row, group); the group's columns are processed 8 at a time.
__global__ void __launch_bounds__(EW_THREADS)
    rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                       __nv_bfloat16* __restrict__ y, float* __restrict__ rstd, int H, int groups, float eps) {
  const int row = blockIdx.x, grp = blockIdx.y;
  const int G = H / groups;
  const __nv_bfloat16* xr = x + (size_t)row * H + grp * G;
  float ss = 0.f;
  for (int c = threadIdx.x * 8; c < G; c += blockDim.x * 8) {
    float v[8];
    ld8(xr + c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
  }
  ss = block_sum(ss);
  const float r = rsqrtf(ss / (float)G + eps);
  if (threadIdx.x == 0) rstd[(size_t)row * groups + grp] = r;
  for (int c = threadIdx.x * 8; c < G; c += blockDim.x * 8) {
    float v[8], ww[8];
    ld8(xr + c, v);
    ld8(w + grp * G + c, ww);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = bf16r(v[i] * r) * ww[i];
    st8(y + (size_t)row * H + grp * G + c, v);
  }
}

__global__ void __launch_bounds__(EW_THREADS)
    rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                       const __nv_bfloat16* __restrict__ w, const float* __restrict__ rstd,
                       __nv_bfloat16* __restrict__ dx, int H, int groups) {
  const int row = blockIdx.x, grp = blockIdx.y;
  const int G = H / groups;
  const size_t base = (size_t)row * H + grp * G;
  const float r = rstd[(size_t)row * groups + grp];
  float dot = 0.f;  // sum g * xhat
  for (int c = threadIdx.x * 8; c < G; c += blockDim.x * 8) {
    float d[8], v[8], ww[8];
    ld8(dy + base + c, d);
    ld8(x + base + c, v);
    ld8(w + grp * G + c, ww);
#pragma unroll
    for (int i = 0; i < 8; ++i) dot += d[i] * ww[i] * v[i] * r;
  }
  dot = block_sum(dot) / (float)G;
  for (int c = threadIdx.x * 8; c < G; c += blockDim.x * 8) {
    float d[8], v[8], ww[8], o[8];
    ld8(dy + base + c, d);
    ld8(x + base + c, v);
    ld8(w + grp * G + c, ww);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = r * (d[i] * ww[i] - v[i] * r * dot);
    st8(dx + base + c, o);
  }
}

__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + __expf(-x)); }

// gu [rows, 2I] = [gate | up] -> a [rows, I]
__global__ void silu_mul_fwd_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ a, int64_t rows,
                                    int I) {
  const int64_t per_row = I / 8;
  const int64_t n = rows * per_row;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / per_row, c = (i % per_row) * 8;
    float g[8], u[8];
    ld8(gu + r * 2 * I + c, g);
    ld8(gu + r * 2 * I + I + c, u);
#pragma unroll
    for (int k = 0; k < 8; ++k) g[k] = bf16r(g[k] * sigmoid_f(g[k])) * u[k];
    st8(a + r * I + c, g);
  }
}

__global__ void silu_mul_bwd_kernel(const __nv_bfloat16* __restrict__ da, const __nv_bfloat16* __restrict__ gu,
                                    __nv_bfloat16* __restrict__ dgu, int64_t rows, int I) {
  const int64_t per_row = I / 8;
  const int64_t n = rows * per_row;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / per_row, c = (i % per_row) * 8;
    float g[8], u[8], d[8], dg[8], du[8];
    ld8(gu + r * 2 * I + c, g);
    ld8(gu + r * 2 * I + I + c, u);
    ld8(da + r * I + c, d);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float s = sigmoid_f(g[k]);
      du[k] = d[k] * g[k] * s;
      dg[k] = d[k] * u[k] * s * (1.f + g[k] * (1.f - s));
    }
    st8(dgu + r * 2 * I + c, dg);
    st8(dgu + r * 2 * I + I + c, du);
  }
}

// QK-norm (optional) + NeoX RoPE of one 128-wide head row per warp.  Lane l
// holds elements 4l..4l+3; the rotation partner of element d < 64 is d + 64,
// held by lane l ^ 16.  x rows have a token stride (q / k are column slices of
// the fused qkv output); out is contiguous [tokens, heads, 128].
__global__ void __launch_bounds__(256)
    qk_norm_rope_fwd_kernel(const __nv_bfloat16* __restrict__ x, int64_t ld, int heads, int64_t n_rows,
                            const __nv_bfloat16* __restrict__ w, float eps, const int64_t* __restrict__ pos,
                            const float* __restrict__ cos_sin, __nv_bfloat16* __restrict__ out,
                            float* __restrict__ rstd) {
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;  // token * heads + head
  const int lane = threadIdx.x & 31;
  if (row >= n_rows) return;
  const int64_t t = row / heads;
  const int h = (int)(row % heads);
  const __nv_bfloat16* xr = x + t * ld + h * 128 + lane * 4;
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = __bfloat162float(xr[i]);
  if (w != nullptr) {
    float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
    ss = warp_sum(ss);
    const float r = rsqrtf(ss * (1.f / 128.f) + eps);
    if (lane == 0) rstd[row] = r;
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = bf16r(v[i] * r * __bfloat162float(w[lane * 4 + i]));
  }
  const float* cs = cos_sin + pos[t] * 128;
  const int j0 = (lane & 15) * 4;  // frequency index of element 0 of this lane
  const bool first = lane < 16;
  float o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float partner = __shfl_xor_sync(0xffffffff, v[i], 16);
    const float c = cs[j0 + i], sn = cs[64 + j0 + i];
    o[i] = first ? v[i] * c - partner * sn : v[i] * c + partner * sn;
  }
  __nv_bfloat16* orow = out + row * 128 + lane * 4;
#pragma unroll
  for (int i = 0; i < 4; ++i) orow[i] = __float2bfloat16(o[i]);
}

__global__ void __launch_bounds__(256)
    qk_norm_rope_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x, int64_t ld,
                            int heads, int64_t n_rows, const __nv_bfloat16* __restrict__ w,
                            const int64_t* __restrict__ pos, const float* __restrict__ cos_sin,
                            const float* __restrict__ rstd, __nv_bfloat16* __restrict__ dx) {
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= n_rows) return;
  const int64_t t = row / heads;
  const int h = (int)(row % heads);
  const __nv_bfloat16* dr = dy + row * 128 + lane * 4;
  float d[4], g[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) d[i] = __bfloat162float(dr[i]);
  // transpose of the rotation: first half gets dy1 c + dy2 s, second half dy2 c - dy1 s
  const float* cs = cos_sin + pos[t] * 128;
  const int j0 = (lane & 15) * 4;
  const bool first = lane < 16;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float partner = __shfl_xor_sync(0xffffffff, d[i], 16);
    const float c = cs[j0 + i], sn = cs[64 + j0 + i];
    g[i] = first ? d[i] * c + partner * sn : d[i] * c - partner * sn;
  }
  __nv_bfloat16* orow = dx + t * ld + h * 128 + lane * 4;
  if (w == nullptr) {
#pragma unroll
    for (int i = 0; i < 4; ++i) orow[i] = __float2bfloat16(g[i]);
    return;
  }
  const __nv_bfloat16* xr = x + t * ld + h * 128 + lane * 4;
  const float r = rstd[row];
  float xh[4], dot = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    xh[i] = __bfloat162float(xr[i]) * r;
    g[i] *= __bfloat162float(w[lane * 4 + i]);
    dot += g[i] * xh[i];
  }
  dot = warp_sum(dot) * (1.f / 128.f);
#pragma unroll
  for (int i = 0; i < 4; ++i) orow[i] = __float2bfloat16(r * (g[i] - xh[i] * dot));
}

// ------------------------------------------------------------------- host
static void ew_check(const at::Tensor& t, const char* what) {
  check_dev(t, what);
  TORCH_CHECK(t.scalar_type() == at::kBFloat16 && t.is_contiguous(), what, " must be contiguous bf16");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, what, " must be 16-byte aligned");
}

void rmsnorm_fwd_train(const at::Tensor& x, const at::Tensor& w, at::Tensor& y, at::Tensor& rstd, double eps,
                       int64_t groups) {
  ew_check(x, "x");
  ew_check(w, "weight");
  ew_check(y, "y");
  const int64_t H = x.size(-1), rows = x.numel() / H;
  TORCH_CHECK(groups >= 1 && H % groups == 0 && (H / groups) % 8 == 0, "group width must be a multiple of 8");
  TORCH_CHECK(y.numel() == x.numel() && w.numel() == H, "rmsnorm shapes");
  TORCH_CHECK(rstd.scalar_type() == at::kFloat && rstd.numel() == rows * groups, "rstd [rows, groups] fp32");
  if (rows == 0) return;
  rmsnorm_fwd_kernel<<<dim3((unsigned)rows, (unsigned)groups), EW_THREADS, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), rstd.data_ptr<float>(), (int)H, (int)groups, (float)eps);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rmsnorm_bwd_train(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w, const at::Tensor& rstd,
                       at::Tensor& dx, int64_t groups) {
  ew_check(dy, "dy");
  ew_check(x, "x");
  ew_check(w, "weight");
  ew_check(dx, "dx");
  const int64_t H = x.size(-1), rows = x.numel() / H;
  TORCH_CHECK(dy.numel() == x.numel() && dx.numel() == x.numel() && rstd.numel() == rows * groups, "shapes");
  if (rows == 0) return;
  rmsnorm_bwd_kernel<<<dim3((unsigned)rows, (unsigned)groups), EW_THREADS, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), rstd.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), (int)H, (int)groups);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void silu_mul_fwd(const at::Tensor& gu, at::Tensor& a) {
  ew_check(gu, "gate_up");
  ew_check(a, "act");
  const int64_t I = a.size(-1), rows = a.numel() / I;
  TORCH_CHECK(gu.numel() == 2 * a.numel() && gu.size(-1) == 2 * I && I % 8 == 0, "silu_mul shapes");
  if (rows == 0) return;
  const int64_t n = rows * (I / 8);
  const int grid = (int)std::min<int64_t>((n + 255) / 256, (int64_t)num_sms() * 16);
  silu_mul_fwd_kernel<<<grid, 256, 0, cur_stream()>>>(reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()),
                                                      reinterpret_cast<__nv_bfloat16*>(a.data_ptr()), rows, (int)I);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void silu_mul_bwd(const at::Tensor& da, const at::Tensor& gu, at::Tensor& dgu) {
  ew_check(da, "d act");
  ew_check(gu, "gate_up");
  ew_check(dgu, "d gate_up");
  const int64_t I = da.size(-1), rows = da.numel() / I;
  TORCH_CHECK(gu.numel() == 2 * da.numel() && dgu.numel() == gu.numel() && gu.size(-1) == 2 * I && I % 8 == 0,
              "silu_mul shapes");
  if (rows == 0) return;
  const int64_t n = rows * (I / 8);
  const int grid = (int)std::min<int64_t>((n + 255) / 256, (int64_t)num_sms() * 16);
  silu_mul_bwd_kernel<<<grid, 256, 0, cur_stream()>>>(reinterpret_cast<const __nv_bfloat16*>(da.data_ptr()),
                                                      reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()),
                                                      reinterpret_cast<__nv_bfloat16*>(dgu.data_ptr()), rows, (int)I);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static void qk_check(const at::Tensor& x, int64_t& ld, int& heads, int64_t& rows) {
  check_dev(x, "q/k");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.dim() == 3 && x.size(2) == 128 && x.stride(2) == 1 &&
                  x.stride(1) == 128,
              "q/k must be bf16 [tokens, heads, 128] with contiguous heads");
  TORCH_CHECK(x.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 8 == 0, "q/k row alignment");
  ld = x.stride(0);
  heads = (int)x.size(1);
  rows = x.size(0) * x.size(1);
}

void qk_norm_rope_fwd(const at::Tensor& x, c10::optional<at::Tensor> w, double eps, const at::Tensor& pos,
                      const at::Tensor& cos_sin, at::Tensor& out, at::Tensor& rstd) {
  int64_t ld, rows;
  int heads;
  qk_check(x, ld, heads, rows);
  TORCH_CHECK(out.is_contiguous() && out.numel() == rows * 128 && out.scalar_type() == at::kBFloat16, "out");
  TORCH_CHECK(pos.scalar_type() == at::kLong && pos.numel() == x.size(0), "positions");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.size(-1) == 128, "cos_sin [max_pos, 128] fp32");
  TORCH_CHECK(rstd.scalar_type() == at::kFloat && rstd.numel() >= rows, "rstd");
  if (rows == 0) return;
  const __nv_bfloat16* wp = (w.has_value() && w->defined()) ? reinterpret_cast<const __nv_bfloat16*>(w->data_ptr())
                                                            : nullptr;
  qk_norm_rope_fwd_kernel<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), ld, heads, rows, wp, (float)eps, pos.data_ptr<int64_t>(),
      cos_sin.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), rstd.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void qk_norm_rope_bwd(const at::Tensor& dy, const at::Tensor& x, c10::optional<at::Tensor> w, const at::Tensor& pos,
                      const at::Tensor& cos_sin, const at::Tensor& rstd, at::Tensor& dx) {
  int64_t ld, rows;
  int heads;
  qk_check(x, ld, heads, rows);
  TORCH_CHECK(dy.is_contiguous() && dy.numel() == rows * 128 && dy.scalar_type() == at::kBFloat16, "dy");
  TORCH_CHECK(dx.sizes() == x.sizes() && dx.strides() == x.strides() && dx.scalar_type() == at::kBFloat16,
              "dx must have the layout of x");
  if (rows == 0) return;
  const __nv_bfloat16* wp = (w.has_value() && w->defined()) ? reinterpret_cast<const __nv_bfloat16*>(w->data_ptr())
                                                            : nullptr;
  qk_norm_rope_bwd_kernel<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), ld,
      heads, rows, wp, pos.data_ptr<int64_t>(), cos_sin.data_ptr<float>(), rstd.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace uno
