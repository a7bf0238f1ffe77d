// Bandwidth-bound fused kernels: (add+)RMSNorm (plain and grouped), embedding
// gather, SiLU*up, standalone QK-norm/RoPE/KV-store (for head sizes the GEMM
// epilogue does not cover) and the paged KV scatter.
//
// Rounding follows the reference (``layers/layernorm.py:16-40``): the residual
// sum is rounded to the activation dtype, the normalised value is rounded
// before it is multiplied by the (bf16) weight, and that product is rounded
// again.  Grouped RMSNorm (``models/xllm.py:26-84``) normalises the rounded
// residual per group.
#include "common.cuh"
#include "uno_ops.h"

namespace uno {

// One CTA per row; each thread owns 8 consecutive elements (one 16-byte vector).
template <bool ADD>
__global__ void rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, __nv_bfloat16* __restrict__ residual,
                               const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ y, int H,
                               int groups, float eps) {
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const int nvec = H / 8;
  __shared__ float red[1024 + 32];
  pdl_wait();
  float v[8];
  bool active = tid < nvec;
  if (active) {
    uint4 raw = reinterpret_cast<const uint4*>(x + (size_t)row * ldx)[tid];
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __bfloat1622float2(h2[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
    if (ADD) {
      uint4 rr = reinterpret_cast<const uint4*>(residual + (size_t)row * H)[tid];
      const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&rr);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float2 f = __bfloat1622float2(r2[i]);
        v[2 * i] += f.x;
        v[2 * i + 1] += f.y;
      }
      uint4 out;
      out.x = pack_bf16x2(v[0], v[1]);
      out.y = pack_bf16x2(v[2], v[3]);
      out.z = pack_bf16x2(v[4], v[5]);
      out.w = pack_bf16x2(v[6], v[7]);
      reinterpret_cast<uint4*>(residual + (size_t)row * H)[tid] = out;
      if (groups > 1) {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = bf16r(v[i]);
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.f;
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
  float inv;
  if (groups == 1) {
    ss = warp_sum(ss);
    const int warp = tid >> 5, lane = tid & 31;
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (warp == 0) {
      float t = lane < (blockDim.x >> 5) ? red[lane] : 0.f;
      t = warp_sum(t);
      if (lane == 0) red[32] = t;
    }
    __syncthreads();
    inv = rsqrtf(red[32] / H + eps);
  } else {
    // threads of one group are contiguous: gsize/8 threads per group
    const int per = (H / groups) / 8;
    red[tid] = ss;
    __syncthreads();
    const int g0 = (tid / per) * per;
    float t = 0.f;
    for (int i = 0; i < per; ++i) t += red[g0 + i];
    inv = rsqrtf(t / (H / groups) + eps);
  }
  if (!active) return;
  uint4 wr = reinterpret_cast<const uint4*>(w)[tid];
  const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&wr);
  float o[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(w2[i]);
    o[2 * i] = bf16r(bf16r(v[2 * i] * inv) * f.x);
    o[2 * i + 1] = bf16r(bf16r(v[2 * i + 1] * inv) * f.y);
  }
  uint4 out;
  out.x = pack_bf16x2(o[0], o[1]);
  out.y = pack_bf16x2(o[2], o[3]);
  out.z = pack_bf16x2(o[4], o[5]);
  out.w = pack_bf16x2(o[6], o[7]);
  reinterpret_cast<uint4*>(y + (size_t)row * H)[tid] = out;
}

void rmsnorm_launch(const at::Tensor& x, const c10::optional<at::Tensor>& residual, const at::Tensor& w,
                    at::Tensor& y, double eps, int groups) {
  check_dev(x, "x");
  check_dev(w, "weight");
  check_dev(y, "y");
  if (residual.has_value()) check_dev(*residual, "residual");
  const int H = x.size(-1);
  const int rows = x.numel() / H;
  TORCH_CHECK(H % 8 == 0 && H / 8 <= 1024, "hidden size must be a multiple of 8 and <= 8192");
  TORCH_CHECK(groups >= 1 && H % groups == 0 && (H / groups) % 8 == 0, "bad RMSNorm group count");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && x.stride(0) % 8 == 0, "x must be [rows, H] with 16-byte rows");
  TORCH_CHECK(y.is_contiguous() && (!residual.has_value() || residual->is_contiguous()), "y/residual contiguous");
  if (rows == 0) return;
  int threads = ((H / 8 + 31) / 32) * 32;
  if (residual.has_value()) {
    launch_pdl(rmsnorm_kernel<true>, dim3(rows), dim3(threads), 0, cur_stream(),
               reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), (int64_t)x.stride(0),
               reinterpret_cast<__nv_bfloat16*>(residual->data_ptr()),
               reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), reinterpret_cast<__nv_bfloat16*>(y.data_ptr()),
               H, (int)groups, (float)eps);
  } else {
    launch_pdl(rmsnorm_kernel<false>, dim3(rows), dim3(threads), 0, cur_stream(),
               reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), (int64_t)x.stride(0),
               static_cast<__nv_bfloat16*>(nullptr), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
               reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), H, (int)groups, (float)eps);
  }
}

// Vocab-parallel embedding gather: rows outside [start, start + rows) are zero.
__global__ void embedding_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                                 __nv_bfloat16* __restrict__ out, int T, int H, int64_t start, int64_t rows) {
  const int t = blockIdx.x;
  pdl_wait();
  const int64_t id = ids[t] - start;
  const bool ok = id >= 0 && id < rows;
  const uint4* src = reinterpret_cast<const uint4*>(table + (ok ? id : 0) * (int64_t)H);
  uint4* dst = reinterpret_cast<uint4*>(out + (size_t)t * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = ok ? src[i] : make_uint4(0, 0, 0, 0);
}

void embedding_launch(const at::Tensor& ids, const at::Tensor& table, at::Tensor& out, int64_t start) {
  check_dev(ids, "ids");
  check_dev(table, "table");
  check_dev(out, "out");
  const int T = ids.numel(), H = table.size(1);
  if (T == 0) return;
  launch_pdl(embedding_kernel, dim3(T), dim3(256), 0, cur_stream(), ids.data_ptr<int64_t>(),
             reinterpret_cast<const __nv_bfloat16*>(table.data_ptr()),
             reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), T, H, (int64_t)start, (int64_t)table.size(0));
}

// out[t, i] = silu(x[t, i]) * x[t, I + i]
__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ out, int T, int I) {
  const int64_t n = (int64_t)T * I;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < n; idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = idx / I, i = idx % I;
    const float g = __bfloat162float(x[t * 2 * I + i]);
    const float u = __bfloat162float(x[t * 2 * I + I + i]);
    out[idx] = __float2bfloat16(g / (1.f + __expf(-g)) * u);
  }
}

void silu_mul_launch(const at::Tensor& x, at::Tensor& out) {
  check_dev(x, "x");
  check_dev(out, "out");
  const int I = out.size(-1);
  const int T = out.numel() / I;
  if (T == 0) return;
  silu_mul_kernel<<<std::min<int64_t>(((int64_t)T * I + 255) / 256, 148 * 16), 256, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), T, I);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// qkv [T, (hq + 2 hkv) * D] -> q [T, hq, D]; k, v -> paged caches.  One warp per
// (token, head); D <= 256, each lane holds D/32 elements (pairs i, i+D/2 split
// across lanes l and l + 16 when D/32 == 2 ... handled generically via smem).
__global__ void qk_norm_rope_store_kernel(const __nv_bfloat16* __restrict__ qkv, __nv_bfloat16* __restrict__ q_out,
                                          __nv_bfloat16* __restrict__ k_cache, __nv_bfloat16* __restrict__ v_cache,
                                          const int64_t* __restrict__ slots, const int64_t* __restrict__ positions,
                                          const float* __restrict__ cos_sin, const __nv_bfloat16* __restrict__ qw,
                                          const __nv_bfloat16* __restrict__ kw, float eps, int T, int hq, int hkv,
                                          int D, int page) {
  extern __shared__ float buf[];  // [warps][D]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int heads = hq + 2 * hkv;
  const int64_t item = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
  if (item >= (int64_t)T * heads) return;
  const int t = item / heads, head = item % heads;
  float* v = buf + warp * D;
  const __nv_bfloat16* src = qkv + (size_t)t * heads * D + head * D;
  for (int i = lane; i < D; i += 32) v[i] = __bfloat162float(src[i]);
  __syncwarp();
  const int64_t slot = slots[t];
  if (head < hq + hkv) {
    const __nv_bfloat16* w = head < hq ? qw : kw;
    if (w != nullptr) {
      float ss = 0.f;
      for (int i = lane; i < D; i += 32) ss += v[i] * v[i];
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss / D + eps);
      for (int i = lane; i < D; i += 32) v[i] = bf16r(v[i] * inv * __bfloat162float(w[i]));
      __syncwarp();
    }
    const float* cs = cos_sin + (size_t)positions[t] * D;
    const int half = D / 2;
    float outv[8];
    int n = 0;
    for (int i = lane; i < half; i += 32) {
      const float c = cs[i], s = cs[half + i];
      const float x1 = v[i], x2 = v[half + i];
      outv[n++] = x1 * c - x2 * s;
      outv[n++] = x2 * c + x1 * s;
    }
    __syncwarp();
    n = 0;
    for (int i = lane; i < half; i += 32) {
      v[i] = outv[n++];
      v[half + i] = outv[n++];
    }
    __syncwarp();
    __nv_bfloat16* dst;
    if (head < hq) {
      dst = q_out + ((size_t)t * hq + head) * D;
    } else {
      if (slot < 0) return;
      dst = k_cache + (((size_t)(slot / page) * hkv + (head - hq)) * page + slot % page) * D;
    }
    for (int i = lane; i < D; i += 32) dst[i] = __float2bfloat16(v[i]);
    return;
  }
  if (slot < 0) return;
  __nv_bfloat16* dst = v_cache + (((size_t)(slot / page) * hkv + (head - hq - hkv)) * page + slot % page) * D;
  for (int i = lane; i < D; i += 32) dst[i] = __float2bfloat16(v[i]);
}

void qk_norm_rope_store_launch(const at::Tensor& qkv, at::Tensor& q_out, at::Tensor& k_cache, at::Tensor& v_cache,
                               const at::Tensor& slots, const at::Tensor& positions, const at::Tensor& cos_sin,
                               const c10::optional<at::Tensor>& qw, const c10::optional<at::Tensor>& kw, double eps,
                               int hq, int hkv, int D, int page) {
  check_dev(qkv, "qkv");
  check_dev(q_out, "q_out");
  check_dev(slots, "slots");
  check_dev(positions, "positions");
  check_dev(cos_sin, "cos_sin");
  if (k_cache.numel()) check_dev(k_cache, "k_cache");
  if (v_cache.numel()) check_dev(v_cache, "v_cache");
  const int T = qkv.size(0);
  if (T == 0) return;
  TORCH_CHECK(D % 2 == 0 && D <= 256, "unsupported head dim");
  const int warps = 8;
  const int64_t items = (int64_t)T * (hq + 2 * hkv);
  qk_norm_rope_store_kernel<<<(items + warps - 1) / warps, warps * 32, warps * D * sizeof(float), cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr()),
      k_cache.numel() ? reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr()) : nullptr,
      v_cache.numel() ? reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr()) : nullptr, slots.data_ptr<int64_t>(),
      positions.data_ptr<int64_t>(), cos_sin.data_ptr<float>(),
      qw.has_value() ? reinterpret_cast<const __nv_bfloat16*>(qw->data_ptr()) : nullptr,
      kw.has_value() ? reinterpret_cast<const __nv_bfloat16*>(kw->data_ptr()) : nullptr, (float)eps, T, hq, hkv, D,
      page);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// In-place compaction of accepted tree paths: for request b and path slot j,
// copy K/V (all layers, all kv heads) from logical src[b, j] to dst[b, j].
// One CTA per (layer * 2 + k/v, request): all reads land in shared memory
// before any write so overlapping moves are safe.
__global__ void copy_tree_kv_kernel(__nv_bfloat16* __restrict__ cache, const int64_t* __restrict__ tables,
                                    int table_stride, const int64_t* __restrict__ src, const int64_t* __restrict__ dst,
                                    int P, int pages, int hkv, int page, int D) {
  extern __shared__ uint4 stage[];  // [P][hkv * D / 8]
  const int lk = blockIdx.x, b = blockIdx.y;
  __nv_bfloat16* base = cache + (size_t)lk * pages * hkv * page * D;
  const int per = hkv * D / 8;  // uint4 per position (all heads)
  const int64_t* s = src + (size_t)b * P;
  const int64_t* d = dst + (size_t)b * P;
  const int64_t* tb = tables + (size_t)b * table_stride;
  for (int idx = threadIdx.x; idx < P * per; idx += blockDim.x) {
    const int j = idx / per, e = idx % per;
    const int64_t pos = s[j];
    if (pos < 0 || pos == d[j]) continue;
    const int head = e / (D / 8), c = e % (D / 8);
    const int64_t pg = tb[pos / page];
    stage[idx] = reinterpret_cast<const uint4*>(base + ((pg * hkv + head) * page + pos % page) * D)[c];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < P * per; idx += blockDim.x) {
    const int j = idx / per, e = idx % per;
    const int64_t pos = d[j];
    if (s[j] < 0 || s[j] == pos) continue;
    const int head = e / (D / 8), c = e % (D / 8);
    const int64_t pg = tb[pos / page];
    reinterpret_cast<uint4*>(base + ((pg * hkv + head) * page + pos % page) * D)[c] = stage[idx];
  }
}

void copy_tree_kv_launch(at::Tensor& cache, const at::Tensor& tables, const at::Tensor& src, const at::Tensor& dst,
                         int page) {
  check_dev(cache, "cache");
  check_dev(tables, "tables");
  check_dev(src, "src");
  check_dev(dst, "dst");
  // cache [layers, 2, pages, hkv, page, D]
  const int layers2 = cache.size(0) * cache.size(1);
  const int pages = cache.size(2), hkv = cache.size(3), D = cache.size(5);
  const int B = src.size(0), P = src.size(1);
  if (B == 0 || P == 0) return;
  const size_t smem = (size_t)P * hkv * D * 2;
  TORCH_CHECK(smem <= 200 * 1024, "tree path too long for the compaction kernel");
  if (smem > 48 * 1024)
    C10_CUDA_CHECK(cudaFuncSetAttribute(copy_tree_kv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  copy_tree_kv_kernel<<<dim3(layers2, B), 256, smem, cur_stream()>>>(
      reinterpret_cast<__nv_bfloat16*>(cache.data_ptr()), tables.data_ptr<int64_t>(), tables.stride(0),
      src.data_ptr<int64_t>(), dst.data_ptr<int64_t>(), P, pages, hkv, page, D);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace uno
