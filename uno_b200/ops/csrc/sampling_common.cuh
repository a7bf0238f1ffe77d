// Shared pieces of the sampling kernels: row addressing of [rows, V] and
// [groups, rows_per_group, V] logit views, arg-max reductions, vectorised bf16
// loads and Philox-keyed Gumbel noise.
#pragma once
#include "common.cuh"
#include "uno_ops.h"

namespace uno {

constexpr int SAMPLE_THREADS = 512;

// Logit rows may be a strided [groups, rows_per_group, V] view (for example the
// draft rows 1..L-1 of every request in a [B, L, V] block): row r lives at
// (r / rpg) * gstride + (r % rpg) * ld elements from the base pointer.
struct RowMap {
  int rpg;
  int64_t gstride, ld;
  __device__ __forceinline__ int64_t off(int r) const { return (int64_t)(r / rpg) * gstride + (int64_t)(r % rpg) * ld; }
};

struct ArgBest {
  float v;
  int i;
};

__device__ __forceinline__ ArgBest better(ArgBest a, ArgBest b) {
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}

__device__ __forceinline__ ArgBest warp_best(ArgBest a) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ArgBest b{__shfl_xor_sync(0xffffffff, a.v, o), __shfl_xor_sync(0xffffffff, a.i, o)};
    a = better(a, b);
  }
  return a;
}

static __device__ ArgBest block_best(ArgBest a) {
  __shared__ float sv[32];
  __shared__ int si[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  a = warp_best(a);
  __syncthreads();
  if (lane == 0) {
    sv[warp] = a.v;
    si[warp] = a.i;
  }
  __syncthreads();
  if (warp == 0) {
    ArgBest b{-INFINITY, 0x7fffffff};
    if (lane < (int)(blockDim.x >> 5)) b = ArgBest{sv[lane], si[lane]};
    b = warp_best(b);
    if (lane == 0) {
      sv[0] = b.v;
      si[0] = b.i;
    }
  }
  __syncthreads();
  return ArgBest{sv[0], si[0]};
}

static __device__ float block_sum(float v) {
  __shared__ float s[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) s[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float t = lane < (int)(blockDim.x >> 5) ? s[lane] : 0.f;
    t = warp_sum(t);
    if (lane == 0) s[0] = t;
  }
  __syncthreads();
  return s[0];
}

static __device__ float block_max(float v) {
  __shared__ float s[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) s[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float t = lane < (int)(blockDim.x >> 5) ? s[lane] : -INFINITY;
    t = warp_max(t);
    if (lane == 0) s[0] = t;
  }
  __syncthreads();
  return s[0];
}

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* v) {
  uint4 w = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// Gumbel noise -log(E), E = -log(U), for 8 consecutive entries starting at v0 (v0 % 4 == 0).
__device__ __forceinline__ void gumbel8(uint32_t seed, uint32_t offset, uint32_t row, uint32_t stream, int v0,
                                        float* g) {
  Philox4 a = philox4x32_10((uint32_t)(v0 >> 2), row, stream, 0u, seed, offset);
  Philox4 b = philox4x32_10((uint32_t)(v0 >> 2) + 1u, row, stream, 0u, seed, offset);
  const uint32_t bits[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) g[i] = -__logf(-__logf(u01(bits[i])));
}

__device__ __forceinline__ float gumbel1(uint32_t seed, uint32_t offset, uint32_t row, uint32_t stream, int v) {
  Philox4 a = philox4x32_10((uint32_t)(v >> 2), row, stream, 0u, seed, offset);
  const uint32_t bits[4] = {a.x, a.y, a.z, a.w};
  return -__logf(-__logf(u01(bits[v & 3])));
}

struct MaxSum {
  float m, s;
};

__device__ __forceinline__ MaxSum ms_merge(MaxSum a, MaxSum b) {
  const float m = fmaxf(a.m, b.m);
  if (m == -INFINITY) return {m, 0.f};
  return {m, a.s * __expf(a.m - m) + b.s * __expf(b.m - m)};
}

static __device__ MaxSum block_maxsum(MaxSum v) {
  __shared__ float sm[32], ss[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    MaxSum w{__shfl_xor_sync(0xffffffff, v.m, o), __shfl_xor_sync(0xffffffff, v.s, o)};
    v = ms_merge(v, w);
  }
  __syncthreads();
  if (lane == 0) {
    sm[warp] = v.m;
    ss[warp] = v.s;
  }
  __syncthreads();
  if (warp == 0) {
    MaxSum w{-INFINITY, 0.f};
    if (lane < (int)(blockDim.x >> 5)) w = MaxSum{sm[lane], ss[lane]};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      MaxSum u{__shfl_xor_sync(0xffffffff, w.m, o), __shfl_xor_sync(0xffffffff, w.s, o)};
      w = ms_merge(w, u);
    }
    if (lane == 0) {
      sm[0] = w.m;
      ss[0] = w.s;
    }
  }
  __syncthreads();
  return {sm[0], ss[0]};
}

// Softmax statistics of two rows in ONE pass: (max, sum exp(x * inv_temp - max))
// of each, merged online per 8-wide vector and then across the block.
static __device__ void row_stats2(const __nv_bfloat16* c, const __nv_bfloat16* d, int n, float inv_temp, float& cm,
                                  float& cs, float& dm, float& ds) {
  MaxSum a{-INFINITY, 0.f}, b{-INFINITY, 0.f};
  const int nvec = n / 8;
  for (int k = threadIdx.x; k < nvec; k += blockDim.x) {
    float x[8], y[8];
    load8(c + k * 8, x);
    load8(d + k * 8, y);
    float mx = x[0] * inv_temp, my = y[0] * inv_temp;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      x[i] *= inv_temp;
      y[i] *= inv_temp;
      mx = fmaxf(mx, x[i]);
      my = fmaxf(my, y[i]);
    }
    float sx = 0.f, sy = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      sx += __expf(x[i] - mx);
      sy += __expf(y[i] - my);
    }
    a = ms_merge(a, MaxSum{mx, sx});
    b = ms_merge(b, MaxSum{my, sy});
  }
  for (int i = nvec * 8 + threadIdx.x; i < n; i += blockDim.x) {
    a = ms_merge(a, MaxSum{__bfloat162float(c[i]) * inv_temp, 1.f});
    b = ms_merge(b, MaxSum{__bfloat162float(d[i]) * inv_temp, 1.f});
  }
  a = block_maxsum(a);
  b = block_maxsum(b);
  cm = a.m;
  cs = a.s;
  dm = b.m;
  ds = b.s;
}

// ------------------------------------------------------------------- host
// 2-D [rows, V] or 3-D [groups, rpg, V] logits with unit stride along V.
static inline RowMap row_map(const at::Tensor& x, int& rows, int& V) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16, "logits must be bfloat16");
  TORCH_CHECK(x.stride(-1) == 1, "logits must be contiguous along the vocabulary");
  RowMap m{};
  if (x.dim() == 2) {
    rows = x.size(0);
    V = x.size(1);
    m.rpg = std::max<int>(1, rows);
    m.gstride = 0;
    m.ld = x.stride(0);
  } else {
    TORCH_CHECK(x.dim() == 3, "logits must be 2-D or 3-D");
    rows = x.size(0) * x.size(1);
    V = x.size(2);
    m.rpg = std::max<int>(1, x.size(1));
    m.gstride = x.stride(0);
    m.ld = x.stride(1);
  }
  TORCH_CHECK(m.ld % 8 == 0 && m.gstride % 8 == 0, "logit row strides must be multiples of 8 elements");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0, "logits must be 16-byte aligned");
  return m;
}

}  // namespace uno
