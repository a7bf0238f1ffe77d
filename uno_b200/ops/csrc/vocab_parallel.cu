// Vocab-parallel sampling and Psi-Spec verification over NVLink peer memory.
//
// Under tensor parallelism the lm_head leaves every rank with a [rows, V/tp]
// shard of the logits.  Instead of all-gathering [rows, V] (the reference
// gathers the full logits, ``nano_vllm_uno/layers/embed_head.py:55-66``, then
// samples, ``nano_vllm_uno/layers/sampler.py:14-133`` and verifies,
// ``nano_vllm_uno/engine/fused_verify_kernel.py:8-98``), each kernel here
// reduces its shard to a few numbers per row, stores them straight into every
// peer's exchange slots, and combines the tp partials it receives:
//
// * vp_sample_kernel  Gumbel-max sample (or arg-max when greedy): partial =
//                     (best score, global id), 8 bytes per row and rank;
// * vp_verify_kernel  accept test min(1, p(s)/q(s)) + residual resample:
//                     phase A exchanges (max, sum of exp) of both rows and the
//                     spec token's logits (owned by one rank); every rank then
//                     takes the same accept decision; rejected rows run phase B,
//                     a Gumbel-max over log(max(p - q, 0)) of the shard, whose
//                     (score, id) partials are exchanged like a sample.
//
// The Philox noise of vocabulary entry v is keyed by the GLOBAL id, so a
// vocab-parallel sample equals the single-GPU sample of the same logits; the
// verify statistics differ from single-GPU only by summation order.
//
// Exchange region (byte offsets inside every rank's symmetric workspace):
//   +0    u64 epoch (calls completed on this rank), +8 u32 CTA counter
//   +64   u64 flag_a[8][max_rows], flag_b[8][max_rows]   (value = epoch + 1)
//   then  float slot_a[2][8][max_rows][8]   (parity = epoch & 1)
//   then  u64   slot_b[2][8][max_rows]
// A rank writes call k's partials for row r into slot[k & 1][rank][r] of every
// peer, then releases flag[rank][r] = k + 1.  Two parities suffice: a rank can
// only start call k + 2 after every peer has published call k + 1, i.e. after
// every peer finished reading call k.
//
// Every CTA publishes all its rows before it waits for any, and the grid is at
// most one CTA per SM, so a wait only depends on the peer's CTA of the same
// index having started.  Waits are bounded (error code 4) and skip once any
// error is recorded.
#include "common.cuh"
#include "sampling_common.cuh"
#include "uno_ops.h"

namespace uno {

constexpr int VP_MAX_TP = 8;

struct VpRegion {
  uint8_t* base;
  int max_rows;
  __device__ __forceinline__ unsigned long long* epoch() const { return reinterpret_cast<unsigned long long*>(base); }
  __device__ __forceinline__ unsigned int* count() const { return reinterpret_cast<unsigned int*>(base + 8); }
  __device__ __forceinline__ unsigned long long* flag_a(int src, int r) const {
    return reinterpret_cast<unsigned long long*>(base + 64) + (size_t)src * max_rows + r;
  }
  __device__ __forceinline__ unsigned long long* flag_b(int src, int r) const {
    return reinterpret_cast<unsigned long long*>(base + 64) + (size_t)(VP_MAX_TP + src) * max_rows + r;
  }
  __device__ __forceinline__ float* slot_a(int par, int src, int r) const {
    float* s = reinterpret_cast<float*>(base + 64 + 16 * VP_MAX_TP * (size_t)max_rows);
    return s + (((size_t)par * VP_MAX_TP + src) * max_rows + r) * 8;
  }
  __device__ __forceinline__ unsigned long long* slot_b(int par, int src, int r) const {
    unsigned long long* s =
        reinterpret_cast<unsigned long long*>(base + 64 + 80 * VP_MAX_TP * (size_t)max_rows);
    return s + ((size_t)par * VP_MAX_TP + src) * max_rows + r;
  }
};

int64_t vp_region_bytes(int64_t max_rows) { return 64 + 96 * VP_MAX_TP * max_rows; }

struct VpParams {
  uint8_t* peers[VP_MAX_TP];  // exchange region of every rank (own included)
  int tp, rank, max_rows;
  int vstart;  // first global vocabulary id of this rank's shard
  int* err;
};

__device__ __forceinline__ void st_release_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ float ld_relaxed_f32(const float* p) {
  float v;
  asm volatile("ld.relaxed.sys.global.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
  return v;
}

__device__ bool vp_wait(const unsigned long long* flag, unsigned long long target, int* err) {
  if (ld_acquire_sys_u64(flag) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  while (ld_acquire_sys_u64(flag) < target) {
    if (*reinterpret_cast<volatile int*>(err) != 0) return false;
    if (globaltimer_ns() - t0 > 5000000000ull) {
      set_error(err, 4);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ unsigned long long pack_best(ArgBest b) {
  return ((unsigned long long)__float_as_uint(b.v) << 32) | (unsigned int)b.i;
}

__device__ __forceinline__ ArgBest unpack_best(unsigned long long w) {
  return ArgBest{__uint_as_float((unsigned int)(w >> 32)), (int)(unsigned int)(w & 0xffffffffu)};
}

// Thread 0: send one 8-byte partial of row r to every rank.
__device__ __forceinline__ void vp_send_b(const VpParams& p, int par, int r, unsigned long long w,
                                          unsigned long long target) {
  for (int j = 0; j < p.tp; ++j) {
    VpRegion peer{p.peers[j], p.max_rows};
    *reinterpret_cast<volatile unsigned long long*>(peer.slot_b(par, p.rank, r)) = w;
    st_release_u64(peer.flag_b(p.rank, r), target);
  }
}

// Warp 0: best of the tp partials of row r (lowest global id wins ties).
__device__ __forceinline__ ArgBest vp_gather_b(const VpParams& p, const VpRegion& own, int par, int r,
                                               unsigned long long target) {
  const int lane = threadIdx.x & 31;
  ArgBest b{-INFINITY, 0x7fffffff};
  if (lane < p.tp && vp_wait(own.flag_b(lane, r), target, p.err))
    b = unpack_best(ld_relaxed_u64(own.slot_b(par, lane, r)));
  return warp_best(b);
}

// The last CTA to finish advances this rank's exchange epoch.
__device__ __forceinline__ void vp_finish(const VpRegion& own, unsigned long long epoch) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned int prev = atomicAdd(own.count(), 1u);
    if (prev == gridDim.x - 1) {
      *own.count() = 0;
      *reinterpret_cast<volatile unsigned long long*>(own.epoch()) = epoch + 1;
      __threadfence();
    }
  }
}

// Shard-local best of (x / T + Gumbel) (or of x when greedy), global ids.
__device__ ArgBest shard_best(const __nv_bfloat16* row, int Vs, int vstart, float inv_temp, bool greedy,
                              uint32_t seed, uint32_t offset, int r) {
  ArgBest best{-INFINITY, 0x7fffffff};
  const int nvec = Vs / 8;
  for (int c = threadIdx.x; c < nvec; c += blockDim.x) {
    float v[8], g[8];
    load8(row + c * 8, v);
    if (greedy) {
#pragma unroll
      for (int i = 0; i < 8; ++i) best = better(best, ArgBest{v[i], vstart + c * 8 + i});
    } else {
      gumbel8(seed, offset, r, 1u, vstart + c * 8, g);
#pragma unroll
      for (int i = 0; i < 8; ++i) best = better(best, ArgBest{v[i] * inv_temp + g[i], vstart + c * 8 + i});
    }
  }
  for (int i = nvec * 8 + threadIdx.x; i < Vs; i += blockDim.x) {
    const float x = __bfloat162float(row[i]);
    const float s = greedy ? x : x * inv_temp + gumbel1(seed, offset, r, 1u, vstart + i);
    best = better(best, ArgBest{s, vstart + i});
  }
  return block_best(best);
}

__global__ void __launch_bounds__(SAMPLE_THREADS)
    vp_sample_kernel(const __nv_bfloat16* __restrict__ x, RowMap rm, int rows, int Vs, float inv_temp, int greedy,
                     uint32_t seed, uint32_t offset, VpParams p, int64_t* __restrict__ out) {
  const VpRegion own{p.peers[p.rank], p.max_rows};
  const unsigned long long epoch = *reinterpret_cast<volatile unsigned long long*>(own.epoch());
  const unsigned long long target = epoch + 1;
  const int par = (int)(epoch & 1);
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const ArgBest b = shard_best(x + rm.off(r), Vs, p.vstart, inv_temp, greedy != 0, seed, offset, r);
    if (threadIdx.x == 0) vp_send_b(p, par, r, pack_best(b), target);
  }
  if (threadIdx.x < 32) {
    for (int r = blockIdx.x; r < rows; r += gridDim.x) {
      const ArgBest b = vp_gather_b(p, own, par, r, target);
      if (threadIdx.x == 0) out[r] = b.i == 0x7fffffff ? 0 : b.i;
    }
  }
  vp_finish(own, epoch);
}

__global__ void __launch_bounds__(SAMPLE_THREADS)
    vp_verify_kernel(const __nv_bfloat16* __restrict__ clean, RowMap cmap, const __nv_bfloat16* __restrict__ draft,
                     RowMap dmap, const int64_t* __restrict__ spec, int rows, int Vs, float inv_temp, uint32_t seed,
                     uint32_t offset, VpParams p, int32_t* __restrict__ accepted, int64_t* __restrict__ corr) {
  const VpRegion own{p.peers[p.rank], p.max_rows};
  const unsigned long long epoch = *reinterpret_cast<volatile unsigned long long*>(own.epoch());
  const unsigned long long target = epoch + 1;
  const int par = (int)(epoch & 1);
  const int nvec = Vs / 8;
  __shared__ float stats[VP_MAX_TP][8];

  // phase A: shard statistics of both rows (+ spec logits when owned)
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const __nv_bfloat16* c = clean + cmap.off(r);
    const __nv_bfloat16* d = draft + dmap.off(r);
    float cm, cs, dm, ds;
    row_stats2(c, d, Vs, inv_temp, cm, cs, dm, ds);
    if (threadIdx.x == 0) {
      const int64_t s = spec[r] - p.vstart;
      const bool mine = s >= 0 && s < Vs;
      const float4 lo = make_float4(cm, cs, dm, ds);
      const float4 hi = make_float4(mine ? __bfloat162float(c[s]) * inv_temp : 0.f,
                                    mine ? __bfloat162float(d[s]) * inv_temp : 0.f, mine ? 1.f : 0.f, 0.f);
      for (int j = 0; j < p.tp; ++j) {
        VpRegion peer{p.peers[j], p.max_rows};
        volatile float4* dst = reinterpret_cast<volatile float4*>(peer.slot_a(par, p.rank, r));
        dst[0].x = lo.x; dst[0].y = lo.y; dst[0].z = lo.z; dst[0].w = lo.w;
        dst[1].x = hi.x; dst[1].y = hi.y; dst[1].z = hi.z; dst[1].w = hi.w;
        st_release_u64(peer.flag_a(p.rank, r), target);
      }
    }
  }

  // phase B: global statistics, the accept test, local residual samples of rejected rows
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    if (threadIdx.x < p.tp) {
      const bool ok = vp_wait(own.flag_a(threadIdx.x, r), target, p.err);
      const float* src = own.slot_a(par, threadIdx.x, r);
#pragma unroll
      for (int i = 0; i < 8; ++i) stats[threadIdx.x][i] = ok ? ld_relaxed_f32(src + i) : 0.f;
      if (!ok) stats[threadIdx.x][0] = stats[threadIdx.x][2] = -INFINITY;
    }
    __syncthreads();
    float cm = -INFINITY, dm = -INFINITY;
    for (int j = 0; j < p.tp; ++j) {
      cm = fmaxf(cm, stats[j][0]);
      dm = fmaxf(dm, stats[j][2]);
    }
    float cs = 0.f, ds = 0.f, c_s = -INFINITY, d_s = -INFINITY;
    for (int j = 0; j < p.tp; ++j) {
      if (stats[j][0] > -INFINITY) cs += stats[j][1] * __expf(stats[j][0] - cm);
      if (stats[j][2] > -INFINITY) ds += stats[j][3] * __expf(stats[j][2] - dm);
      if (stats[j][6] != 0.f) {
        c_s = stats[j][4];
        d_s = stats[j][5];
      }
    }
    __syncthreads();  // stats is rewritten by the next row
    const float ps = __expf(c_s - cm) / cs;
    const float qs = __expf(d_s - dm) / ds;
    const float ratio = qs > 0.f ? ps / qs : 0.f;
    Philox4 ur = philox4x32_10(0u, (uint32_t)r, 2u, 0u, seed, offset);
    const float u = u01(ur.x);
    if (ratio >= 1.f || u < ratio) {
      if (threadIdx.x == 0) {
        accepted[r] = 1;
        corr[r] = 0;
      }
      continue;
    }
    const __nv_bfloat16* c = clean + cmap.off(r);
    const __nv_bfloat16* d = draft + dmap.off(r);
    const float cinv = 1.f / cs, dinv = 1.f / ds;
    ArgBest best{-INFINITY, 0x7fffffff};
    for (int k = threadIdx.x; k < nvec; k += blockDim.x) {
      float a[8], b[8], g[8];
      load8(c + k * 8, a);
      load8(d + k * 8, b);
      gumbel8(seed, offset, r, 3u, p.vstart + k * 8, g);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float res = __expf(a[i] * inv_temp - cm) * cinv - __expf(b[i] * inv_temp - dm) * dinv;
        if (res > 0.f) best = better(best, ArgBest{__logf(res) + g[i], p.vstart + k * 8 + i});
      }
    }
    for (int i = nvec * 8 + threadIdx.x; i < Vs; i += blockDim.x) {
      const float res = __expf(__bfloat162float(c[i]) * inv_temp - cm) * cinv -
                        __expf(__bfloat162float(d[i]) * inv_temp - dm) * dinv;
      if (res > 0.f) best = better(best, ArgBest{__logf(res) + gumbel1(seed, offset, r, 3u, p.vstart + i),
                                                 p.vstart + i});
    }
    best = block_best(best);
    if (threadIdx.x == 0) {
      accepted[r] = 0;
      vp_send_b(p, par, r, pack_best(best), target);
    }
  }
  __syncthreads();

  // phase C: residual samples of rejected rows
  if (threadIdx.x < 32) {
    for (int r = blockIdx.x; r < rows; r += gridDim.x) {
      if (*reinterpret_cast<volatile int32_t*>(accepted + r)) continue;
      const ArgBest b = vp_gather_b(p, own, par, r, target);
      if (threadIdx.x == 0) corr[r] = b.i == 0x7fffffff ? spec[r] : b.i;
    }
  }
  vp_finish(own, epoch);
}

// ------------------------------------------------------------------- host
static VpParams vp_params(const std::vector<int64_t>& regions, int64_t rank, int64_t max_rows, int64_t vstart,
                          int rows) {
  VpParams p{};
  const int tp = (int)regions.size();
  TORCH_CHECK(tp >= 1 && tp <= VP_MAX_TP, "vocab-parallel exchange supports 1..8 ranks");
  TORCH_CHECK(rank >= 0 && rank < tp, "bad rank");
  TORCH_CHECK(rows <= max_rows, "more logit rows (", rows, ") than the exchange region holds (", max_rows, ")");
  TORCH_CHECK(vstart % 4 == 0, "vocabulary shard must start at a multiple of 4");
  for (int j = 0; j < tp; ++j) {
    p.peers[j] = reinterpret_cast<uint8_t*>(regions[j]);
    TORCH_CHECK(regions[j] % 16 == 0, "exchange region must be 16-byte aligned");
  }
  p.tp = tp;
  p.rank = (int)rank;
  p.max_rows = (int)max_rows;
  p.vstart = (int)vstart;
  p.err = device_error_flag();
  return p;
}

void vp_sample_launch(const at::Tensor& x, at::Tensor& out, double inv_temp, bool greedy, int64_t seed,
                      int64_t offset, const std::vector<int64_t>& regions, int64_t rank, int64_t max_rows,
                      int64_t vstart) {
  check_dev(x, "logits shard");
  check_dev(out, "out");
  int rows, Vs;
  RowMap m = row_map(x, rows, Vs);
  TORCH_CHECK(out.numel() == rows && out.scalar_type() == at::kLong, "sample output");
  if (rows == 0) return;
  VpParams p = vp_params(regions, rank, max_rows, vstart, rows);
  const int grid = std::min(rows, num_sms());
  vp_sample_kernel<<<grid, SAMPLE_THREADS, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), m, rows, Vs, (float)inv_temp, greedy ? 1 : 0,
      (uint32_t)seed, (uint32_t)offset, p, out.data_ptr<int64_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void vp_verify_launch(const at::Tensor& clean, const at::Tensor& draft, const at::Tensor& spec, double inv_temp,
                      int64_t seed, int64_t offset, at::Tensor& accepted, at::Tensor& corr,
                      const std::vector<int64_t>& regions, int64_t rank, int64_t max_rows, int64_t vstart) {
  check_dev(clean, "clean shard");
  check_dev(draft, "draft shard");
  check_dev(spec, "spec");
  check_dev(accepted, "accepted");
  check_dev(corr, "corr");
  int rows, Vs, rows2, Vs2;
  RowMap cm = row_map(clean, rows, Vs);
  RowMap dm = row_map(draft, rows2, Vs2);
  TORCH_CHECK(rows == rows2 && Vs == Vs2 && spec.numel() == rows, "verify shapes");
  TORCH_CHECK(accepted.numel() == rows && accepted.scalar_type() == at::kInt, "accepted output");
  TORCH_CHECK(corr.numel() == rows && corr.scalar_type() == at::kLong, "corr output");
  if (rows == 0) return;
  VpParams p = vp_params(regions, rank, max_rows, vstart, rows);
  const int grid = std::min(rows, num_sms());
  vp_verify_kernel<<<grid, SAMPLE_THREADS, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(clean.data_ptr()), cm,
      reinterpret_cast<const __nv_bfloat16*>(draft.data_ptr()), dm, spec.data_ptr<int64_t>(), rows, Vs,
      (float)inv_temp, (uint32_t)seed, (uint32_t)offset, p, accepted.data_ptr<int32_t>(), corr.data_ptr<int64_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace uno
