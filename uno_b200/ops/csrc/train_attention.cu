// Block-diffusion attention for Uno training, forward and backward.
//
// Layout (``uno_b200/train/layout.py``): every packed sequence contributes a
// noisy copy followed by a clean copy.  Query q may attend key k iff both are
// in the same packed sequence and
//   noisy q, noisy k : same diffusion block (pos_k / bs == pos_q / bs)
//   noisy q, clean k : pos_k < (pos_q / bs) * bs       (clean prefix before q's block)
//   clean q, clean k : pos_k <= pos_q                   (causal)
//   clean q, noisy k : never
// (the reference gets this mask from the checkpoint's remote code and runs
// flex-attention, ``training/train.py:136-143``).  The rule is evaluated per
// element from (segment, position, noisy) of the query and the key; a
// host-built map of 64 x 64 tiles says which tiles are empty (skipped), full
// (no per-element test) or partial.
//
// Forward: one CTA per (64-query tile, query head, batch row), 4 warps of 16
// queries; S = Q K^T and O += P V on mma.sync m16n8k16 (bf16 in, fp32
// accumulate), online softmax in the log2 domain, K/V tiles double-buffered
// with cp.async, three CTAs per SM.  Outputs O and the per-row log2-sum-exp
// (for backward).
//
// Backward: one CTA per (64-key tile, KV head, batch row) looping over the
// query heads of its group and the query tiles that see it (FlashAttention-2
// order): recompute P^T = exp2(K Q^T * c - lse), dV += P^T dO,
// dP^T = V dO^T, dS^T = P^T (dP^T - D) with D = rowsum(dO * O), dK += dS^T Q;
// dQ += dS K goes through shared memory and fp32 atomics.  dK and dV are
// written once per CTA (no atomics: the CTA owns its keys for all heads of
// the group).
#include "common.cuh"
#include "uno_ops.h"

namespace uno {

constexpr int TA_D = 128;             // head dim
constexpr int TA_B = 64;              // query / key tile
constexpr int TA_PITCH = TA_D + 8;    // smem row pitch (elements): conflict-free ldmatrix
constexpr int TA_TILE_BYTES = TA_B * TA_PITCH * 2;
constexpr int TA_DS_PITCH = TA_B + 8;

struct TAParams {
  const __nv_bfloat16 *q, *k, *v, *o, *dout;
  __nv_bfloat16 *out, *dk, *dv;
  float *lse, *dq, *delta;
  const int *seg, *pos;
  const uint8_t* noisy;
  const uint8_t* tiles;  // [B][nt][nt]: 0 empty, 1 partial, 2 full
  int B, T, hq, hkv, nt, block;
  float scale_log2;      // softmax scale * log2(e)
  float scale;
};

__device__ __forceinline__ void ta_ldsm(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ta_ldsm_t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ta_mma(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;  // zero-fill rows past the sequence end
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) { return pack_bf16x2(lo, hi); }

// Copy rows [row0, row0 + 64) of head `head` of a [B, T, H, D] tensor into a padded smem tile.
__device__ __forceinline__ void ta_load_tile(uint32_t smem, const __nv_bfloat16* base, int b, int row0, int head,
                                             int H, int T) {
  for (int i = threadIdx.x; i < TA_B * 16; i += blockDim.x) {
    const int r = i >> 4, c = i & 15;
    const int t = row0 + r;
    const bool ok = t < T;
    const __nv_bfloat16* src = base + (((size_t)b * T + (ok ? t : 0)) * H + head) * TA_D + c * 8;
    cp_async16(smem + (uint32_t)(r * TA_PITCH + c * 8) * 2, src, ok);
  }
}

struct TokMeta {
  int seg, pos, noisy;
};

__device__ __forceinline__ bool ta_visible(TokMeta q, TokMeta k, int bs) {
  if (q.seg != k.seg) return false;
  const int bq = q.pos / bs;
  if (q.noisy) return k.noisy ? (k.pos / bs == bq) : (k.pos < bq * bs);
  return !k.noisy && k.pos <= q.pos;
}

__device__ __forceinline__ TokMeta ta_meta(const TAParams& p, int b, int t) {
  if (t >= p.T) return {-1 - t, 0, 0};  // padding: a segment of its own
  const size_t i = (size_t)b * p.T + t;
  return {p.seg[i], p.pos[i], (int)p.noisy[i]};
}

// ------------------------------------------------------------------ forward
__global__ void __launch_bounds__(128, 3) train_attn_fwd_kernel(TAParams p) {
  extern __shared__ __align__(128) uint8_t ta_smem[];
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (p.hq / p.hkv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;
  // K and V stages 0/1; the Q tile is staged in V stage 1 and moved to registers
  // before that stage is first loaded (4 tiles: three CTAs fit on an SM)
  uint8_t* sK = ta_smem;                   // 2 stages
  uint8_t* sV = sK + 2 * TA_TILE_BYTES;    // 2 stages
  uint8_t* sQ = sV + TA_TILE_BYTES;
  int* sKm = reinterpret_cast<int*>(sV + 2 * TA_TILE_BYTES);  // [2][3][64] key meta
  int* sList = sKm + 2 * 3 * TA_B;                             // visible key tiles (<= nt)
  __shared__ int s_count;

  const uint8_t* trow = p.tiles + ((size_t)b * p.nt + qt) * p.nt;
  if (threadIdx.x == 0) {
    int n = 0;
    for (int j = 0; j < p.nt; ++j)
      if (trow[j]) sList[n++] = j;
    s_count = n;
  }
  const uint32_t qs = smem_u32(sQ), ks = smem_u32(sK), vs = smem_u32(sV);
  ta_load_tile(qs, p.q, b, qt * TA_B, h, p.hq, p.T);
  cp_async_commit();
  __syncthreads();
  const int n_tiles = s_count;

  auto load_kv = [&](int idx, int stage) {
    const int j = sList[idx];
    ta_load_tile(ks + stage * TA_TILE_BYTES, p.k, b, j * TA_B, kvh, p.hkv, p.T);
    ta_load_tile(vs + stage * TA_TILE_BYTES, p.v, b, j * TA_B, kvh, p.hkv, p.T);
    for (int i = threadIdx.x; i < TA_B; i += blockDim.x) {
      const TokMeta m = ta_meta(p, b, j * TA_B + i);
      sKm[(stage * 3 + 0) * TA_B + i] = m.seg;
      sKm[(stage * 3 + 1) * TA_B + i] = m.pos;
      sKm[(stage * 3 + 2) * TA_B + i] = m.noisy;
    }
  };
  if (n_tiles > 0) load_kv(0, 0);
  cp_async_commit();

  const int qrow0 = qt * TA_B + warp * 16;
  const TokMeta qm0 = ta_meta(p, b, qrow0 + g), qm1 = ta_meta(p, b, qrow0 + g + 8);
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  uint32_t qa[8][4];
  cp_async_wait<1>();
  __syncthreads();
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const int r = warp * 16 + (lane & 15), c = kk * 16 + (lane >> 4) * 8;
    ta_ldsm(qs + (uint32_t)(r * TA_PITCH + c) * 2, qa[kk]);
  }
  __syncthreads();  // every warp holds its Q fragments before V stage 1 is overwritten

  for (int it = 0; it < n_tiles; ++it) {
    const int stage = it & 1;
    if (it + 1 < n_tiles) load_kv(it + 1, stage ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const int j = sList[it];
    const bool full = trow[j] == 2;
    const uint32_t kb = ks + stage * TA_TILE_BYTES, vb = vs + stage * TA_TILE_BYTES;
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {  // two 8-key n-tiles per ldmatrix.x4
        uint32_t bf[4];
        const int r = np * 16 + (lane & 7) + (lane >> 4) * 8, c = kk * 16 + ((lane >> 3) & 1) * 8;
        ta_ldsm(kb + (uint32_t)(r * TA_PITCH + c) * 2, bf);
        ta_mma(s[2 * np], qa[kk], bf[0], bf[1]);
        ta_mma(s[2 * np + 1], qa[kk], bf[2], bf[3]);
      }
    }
    // scale, mask, online softmax (rows g and g + 8 of this warp)
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = n * 8 + 2 * tq + (e & 1);
        float x = s[n][e] * p.scale_log2;
        if (!full) {
          const TokMeta km{sKm[(stage * 3 + 0) * TA_B + col], sKm[(stage * 3 + 1) * TA_B + col],
                           sKm[(stage * 3 + 2) * TA_B + col]};
          if (!ta_visible(e < 2 ? qm0 : qm1, km, p.block)) x = -INFINITY;
        }
        s[n][e] = x;
      }
      mx0 = fmaxf(mx0, fmaxf(s[n][0], s[n][1]));
      mx1 = fmaxf(mx1, fmaxf(s[n][2], s[n][3]));
    }
#pragma unroll
    for (int o2 = 1; o2 <= 2; o2 <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffff, mx0, o2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffff, mx1, o2));
    }
    const float base0 = mx0 == -INFINITY ? 0.f : mx0, base1 = mx1 == -INFINITY ? 0.f : mx1;
    const float c0 = exp2f(m0 - base0), c1 = exp2f(m1 - base1);  // m == -inf -> 0
    m0 = mx0;
    m1 = mx1;
    float rs0 = 0.f, rs1 = 0.f;
    uint32_t pa[4][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const float p0 = exp2f(s[n][0] - base0), p1 = exp2f(s[n][1] - base0);
      const float p2 = exp2f(s[n][2] - base1), p3 = exp2f(s[n][3] - base1);
      rs0 += p0 + p1;
      rs1 += p2 + p3;
      // C layout of two adjacent n-tiles = A layout of one 16-deep k step
      pa[n >> 1][(n & 1) * 2 + 0] = pack2(p0, p1);
      pa[n >> 1][(n & 1) * 2 + 1] = pack2(p2, p3);
    }
    l0 = l0 * c0 + rs0;
    l1 = l1 * c1 + rs1;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      o[i][0] *= c0;
      o[i][1] *= c0;
      o[i][2] *= c1;
      o[i][3] *= c1;
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int np = 0; np < 8; ++np) {  // two 8-wide d tiles per ldmatrix.x4.trans
        uint32_t bf[4];
        const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, c = np * 16 + (lane >> 4) * 8;
        ta_ldsm_t(vb + (uint32_t)(r * TA_PITCH + c) * 2, bf);
        ta_mma(o[2 * np], pa[kk], bf[0], bf[1]);
        ta_mma(o[2 * np + 1], pa[kk], bf[2], bf[3]);
      }
    }
    __syncthreads();  // this stage is reloaded two iterations later
  }
  cp_async_wait<0>();
  // row sums across the 4 threads of a row
#pragma unroll
  for (int o2 = 1; o2 <= 2; o2 <<= 1) {
    l0 += __shfl_xor_sync(0xffffffff, l0, o2);
    l1 += __shfl_xor_sync(0xffffffff, l1, o2);
  }
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  const int r0 = qrow0 + g, r1 = r0 + 8;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int col = i * 8 + 2 * tq;
    if (r0 < p.T)
      *reinterpret_cast<uint32_t*>(p.out + (((size_t)b * p.T + r0) * p.hq + h) * TA_D + col) =
          pack2(o[i][0] * inv0, o[i][1] * inv0);
    if (r1 < p.T)
      *reinterpret_cast<uint32_t*>(p.out + (((size_t)b * p.T + r1) * p.hq + h) * TA_D + col) =
          pack2(o[i][2] * inv1, o[i][3] * inv1);
  }
  if (tq == 0) {
    if (r0 < p.T) p.lse[((size_t)b * p.hq + h) * p.T + r0] = l0 > 0.f ? m0 + __log2f(l0) : INFINITY;
    if (r1 < p.T) p.lse[((size_t)b * p.hq + h) * p.T + r1] = l1 > 0.f ? m1 + __log2f(l1) : INFINITY;
  }
}

// D = rowsum(dO * O) per (row, head): one warp per row-head.
__global__ void train_attn_delta_kernel(TAParams p) {
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t n = (int64_t)p.B * p.T * p.hq;
  if (w >= n) return;
  const int h = (int)(w % p.hq);
  const int64_t bt = w / p.hq;
  const __nv_bfloat16* a = p.o + w * TA_D + lane * 4;
  const __nv_bfloat16* d = p.dout + w * TA_D + lane * 4;
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) acc += __bfloat162float(a[i]) * __bfloat162float(d[i]);
  acc = warp_sum(acc);
  if (lane == 0) {
    const int64_t b = bt / p.T, t = bt % p.T;
    p.delta[(b * p.hq + h) * p.T + t] = acc;
  }
}

// ----------------------------------------------------------------- backward
__global__ void __launch_bounds__(128) train_attn_bwd_kernel(TAParams p) {
  extern __shared__ __align__(128) uint8_t ta_smem[];
  const int kt = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int group = p.hq / p.hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;
  uint8_t* sK = ta_smem;
  uint8_t* sV = sK + TA_TILE_BYTES;
  uint8_t* sQ = sV + TA_TILE_BYTES;
  uint8_t* sO = sQ + TA_TILE_BYTES;  // dO
  uint8_t* sDS = sO + TA_TILE_BYTES; // dS^T bf16 [64 keys][64 + 8]
  float* sL = reinterpret_cast<float*>(sDS + TA_B * TA_DS_PITCH * 2);  // lse2 [64]
  float* sD = sL + TA_B;                                                // delta [64]
  int* sQm = reinterpret_cast<int*>(sD + TA_B);                         // [3][64] query meta
  const uint32_t ks = smem_u32(sK), vs = smem_u32(sV), qs = smem_u32(sQ), os = smem_u32(sO), ds = smem_u32(sDS);

  ta_load_tile(ks, p.k, b, kt * TA_B, kvh, p.hkv, p.T);
  ta_load_tile(vs, p.v, b, kt * TA_B, kvh, p.hkv, p.T);
  cp_async_commit();
  const int krow0 = kt * TA_B + warp * 16;
  const TokMeta km0 = ta_meta(p, b, krow0 + g), km1 = ta_meta(p, b, krow0 + g + 8);

  float dk[16][4], dv[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[i][e] = dv[i][e] = 0.f;

  for (int hh = 0; hh < group; ++hh) {
    const int h = kvh * group + hh;
    for (int qt = 0; qt < p.nt; ++qt) {
      const uint8_t tile = p.tiles[((size_t)b * p.nt + qt) * p.nt + kt];
      if (!tile) continue;
      const bool full = tile == 2;
      __syncthreads();  // previous tile's smem readers are done
      ta_load_tile(qs, p.q, b, qt * TA_B, h, p.hq, p.T);
      ta_load_tile(os, p.dout, b, qt * TA_B, h, p.hq, p.T);
      cp_async_commit();
      for (int i = threadIdx.x; i < TA_B; i += blockDim.x) {
        const int t = qt * TA_B + i;
        const bool ok = t < p.T;
        sL[i] = ok ? p.lse[((size_t)b * p.hq + h) * p.T + t] : INFINITY;
        sD[i] = ok ? p.delta[((size_t)b * p.hq + h) * p.T + t] : 0.f;
        const TokMeta m = ta_meta(p, b, t);
        sQm[i] = m.seg;
        sQm[TA_B + i] = m.pos;
        sQm[2 * TA_B + i] = m.noisy;
      }
      cp_async_wait<0>();
      __syncthreads();

      // S^T = K Q^T (16 keys x 64 queries per warp)
      float s[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t a[4];
        ta_ldsm(ks + (uint32_t)((warp * 16 + (lane & 15)) * TA_PITCH + kk * 16 + (lane >> 4) * 8) * 2, a);
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t bf[4];
          const int r = np * 16 + (lane & 7) + (lane >> 4) * 8, c = kk * 16 + ((lane >> 3) & 1) * 8;
          ta_ldsm(qs + (uint32_t)(r * TA_PITCH + c) * 2, bf);
          ta_mma(s[2 * np], a, bf[0], bf[1]);
          ta_mma(s[2 * np + 1], a, bf[2], bf[3]);
        }
      }
      // P^T = exp2(S^T c - lse2[q]) with the mask
#pragma unroll
      for (int n = 0; n < 8; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int col = n * 8 + 2 * tq + (e & 1);
          float pv = exp2f(s[n][e] * p.scale_log2 - sL[col]);
          if (!full) {
            const TokMeta qm{sQm[col], sQm[TA_B + col], sQm[2 * TA_B + col]};
            if (!ta_visible(qm, e < 2 ? km0 : km1, p.block)) pv = 0.f;
          }
          s[n][e] = pv;
        }
      }
      // dV += P^T dO
      uint32_t pa[4][4];
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        pa[n >> 1][(n & 1) * 2 + 0] = pack2(s[n][0], s[n][1]);
        pa[n >> 1][(n & 1) * 2 + 1] = pack2(s[n][2], s[n][3]);
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
        for (int np = 0; np < 8; ++np) {
          uint32_t bf[4];
          const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, c = np * 16 + (lane >> 4) * 8;
          ta_ldsm_t(os + (uint32_t)(r * TA_PITCH + c) * 2, bf);
          ta_mma(dv[2 * np], pa[kk], bf[0], bf[1]);
          ta_mma(dv[2 * np + 1], pa[kk], bf[2], bf[3]);
        }
      }
      // dP^T = V dO^T
      float dp[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n) dp[n][0] = dp[n][1] = dp[n][2] = dp[n][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t a[4];
        ta_ldsm(vs + (uint32_t)((warp * 16 + (lane & 15)) * TA_PITCH + kk * 16 + (lane >> 4) * 8) * 2, a);
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t bf[4];
          const int r = np * 16 + (lane & 7) + (lane >> 4) * 8, c = kk * 16 + ((lane >> 3) & 1) * 8;
          ta_ldsm(os + (uint32_t)(r * TA_PITCH + c) * 2, bf);
          ta_mma(dp[2 * np], a, bf[0], bf[1]);
          ta_mma(dp[2 * np + 1], a, bf[2], bf[3]);
        }
      }
      // dS^T = P^T (dP^T - D[q]); stage it for dQ and use it for dK
      uint32_t da[4][4];
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const int col = n * 8 + 2 * tq;
        const float d0 = s[n][0] * (dp[n][0] - sD[col]), d1 = s[n][1] * (dp[n][1] - sD[col + 1]);
        const float d2 = s[n][2] * (dp[n][2] - sD[col]), d3 = s[n][3] * (dp[n][3] - sD[col + 1]);
        const uint32_t w01 = pack2(d0, d1), w23 = pack2(d2, d3);
        da[n >> 1][(n & 1) * 2 + 0] = w01;
        da[n >> 1][(n & 1) * 2 + 1] = w23;
        const int krow = warp * 16 + g;
        *reinterpret_cast<uint32_t*>(sDS + (krow * TA_DS_PITCH + col) * 2) = w01;
        *reinterpret_cast<uint32_t*>(sDS + ((krow + 8) * TA_DS_PITCH + col) * 2) = w23;
      }
      // dK += dS^T Q
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
        for (int np = 0; np < 8; ++np) {
          uint32_t bf[4];
          const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, c = np * 16 + (lane >> 4) * 8;
          ta_ldsm_t(qs + (uint32_t)(r * TA_PITCH + c) * 2, bf);
          ta_mma(dk[2 * np], da[kk], bf[0], bf[1]);
          ta_mma(dk[2 * np + 1], da[kk], bf[2], bf[3]);
        }
      }
      __syncthreads();  // dS^T staged by every warp
      // dQ[q rows of this warp] += dS K  (A = dS from its transposed staging, B = K rows)
      float dq[16][4];
#pragma unroll
      for (int i = 0; i < 16; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t a[4];
        {
          const int mi = lane >> 3;  // matrix: (q +0/+8) x (key +0/+8)
          const int krow = kk * 16 + (mi >> 1) * 8 + (lane & 7);
          const int qcol = warp * 16 + (mi & 1) * 8;
          ta_ldsm_t(ds + (uint32_t)(krow * TA_DS_PITCH + qcol) * 2, a);
        }
#pragma unroll
        for (int np = 0; np < 8; ++np) {
          uint32_t bf[4];
          const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, c = np * 16 + (lane >> 4) * 8;
          ta_ldsm_t(ks + (uint32_t)(r * TA_PITCH + c) * 2, bf);
          ta_mma(dq[2 * np], a, bf[0], bf[1]);
          ta_mma(dq[2 * np + 1], a, bf[2], bf[3]);
        }
      }
      const int q0 = qt * TA_B + warp * 16 + g, q1 = q0 + 8;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int col = i * 8 + 2 * tq;
        if (q0 < p.T) {
          float* d = p.dq + (((size_t)b * p.T + q0) * p.hq + h) * TA_D + col;
          atomicAdd(d, dq[i][0] * p.scale);
          atomicAdd(d + 1, dq[i][1] * p.scale);
        }
        if (q1 < p.T) {
          float* d = p.dq + (((size_t)b * p.T + q1) * p.hq + h) * TA_D + col;
          atomicAdd(d, dq[i][2] * p.scale);
          atomicAdd(d + 1, dq[i][3] * p.scale);
        }
      }
    }
  }
  cp_async_wait<0>();
  const int r0 = krow0 + g, r1 = r0 + 8;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int col = i * 8 + 2 * tq;
    if (r0 < p.T) {
      const size_t o = (((size_t)b * p.T + r0) * p.hkv + kvh) * TA_D + col;
      *reinterpret_cast<uint32_t*>(p.dk + o) = pack2(dk[i][0] * p.scale, dk[i][1] * p.scale);
      *reinterpret_cast<uint32_t*>(p.dv + o) = pack2(dv[i][0], dv[i][1]);
    }
    if (r1 < p.T) {
      const size_t o = (((size_t)b * p.T + r1) * p.hkv + kvh) * TA_D + col;
      *reinterpret_cast<uint32_t*>(p.dk + o) = pack2(dk[i][2] * p.scale, dk[i][3] * p.scale);
      *reinterpret_cast<uint32_t*>(p.dv + o) = pack2(dv[i][2], dv[i][3]);
    }
  }
}

// ------------------------------------------------------------------- host
static TAParams ta_params(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& seg,
                          const at::Tensor& pos, const at::Tensor& noisy, const at::Tensor& tiles, int64_t block,
                          double scale) {
  const at::Tensor* ops[3] = {&q, &k, &v};
  for (const at::Tensor* t : ops) {
    check_dev(*t, "attention operand");
    TORCH_CHECK(t->scalar_type() == at::kBFloat16 && t->is_contiguous() && t->dim() == 4 && t->size(3) == TA_D,
                "q/k/v must be contiguous bf16 [B, T, heads, 128]");
  }
  TORCH_CHECK(seg.scalar_type() == at::kInt && pos.scalar_type() == at::kInt && noisy.scalar_type() == at::kByte &&
                  tiles.scalar_type() == at::kByte && seg.is_contiguous() && pos.is_contiguous() &&
                  noisy.is_contiguous() && tiles.is_contiguous(),
              "metadata: int32 segment/position, uint8 noisy flags and tile map");
  TAParams p{};
  p.B = q.size(0);
  p.T = q.size(1);
  p.hq = q.size(2);
  p.hkv = k.size(2);
  TORCH_CHECK(k.size(0) == p.B && k.size(1) == p.T && v.sizes() == k.sizes() && p.hq % p.hkv == 0, "shapes");
  p.nt = (p.T + TA_B - 1) / TA_B;
  TORCH_CHECK(seg.numel() == (int64_t)p.B * p.T && pos.numel() == seg.numel() && noisy.numel() == seg.numel(),
              "metadata size");
  TORCH_CHECK(tiles.numel() == (int64_t)p.B * p.nt * p.nt, "tile map size");
  TORCH_CHECK(block >= 1, "block size");
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.k = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
  p.v = reinterpret_cast<const __nv_bfloat16*>(v.data_ptr());
  p.seg = seg.data_ptr<int>();
  p.pos = pos.data_ptr<int>();
  p.noisy = noisy.data_ptr<uint8_t>();
  p.tiles = tiles.data_ptr<uint8_t>();
  p.block = (int)block;
  p.scale = (float)scale;
  p.scale_log2 = (float)(scale * 1.4426950408889634);
  return p;
}

void train_attn_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& seg,
                    const at::Tensor& pos, const at::Tensor& noisy, const at::Tensor& tiles, int64_t block,
                    double scale, at::Tensor& out, at::Tensor& lse) {
  TAParams p = ta_params(q, k, v, seg, pos, noisy, tiles, block, scale);
  TORCH_CHECK(out.sizes() == q.sizes() && out.is_contiguous() && out.scalar_type() == at::kBFloat16, "out");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.numel() == (int64_t)p.B * p.hq * p.T, "lse [B, hq, T] fp32");
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.lse = lse.data_ptr<float>();
  const int smem = 4 * TA_TILE_BYTES + 2 * 3 * TA_B * 4 + p.nt * 4;
  static PerDeviceOnce smem_opt_in;
  smem_opt_in([] {
    C10_CUDA_CHECK(cudaFuncSetAttribute(train_attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        4 * TA_TILE_BYTES + 2 * 3 * TA_B * 4 + 4096 * 4));
  });
  TORCH_CHECK(p.nt <= 4096, "sequence too long for the tile list");
  train_attn_fwd_kernel<<<dim3(p.nt, p.hq, p.B), 128, smem, cur_stream()>>>(p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void train_attn_bwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& seg,
                    const at::Tensor& pos, const at::Tensor& noisy, const at::Tensor& tiles, int64_t block,
                    double scale, const at::Tensor& out, const at::Tensor& dout, const at::Tensor& lse,
                    at::Tensor& delta, at::Tensor& dq, at::Tensor& dk, at::Tensor& dv) {
  TAParams p = ta_params(q, k, v, seg, pos, noisy, tiles, block, scale);
  TORCH_CHECK(out.sizes() == q.sizes() && dout.sizes() == q.sizes() && out.is_contiguous() && dout.is_contiguous() &&
                  dout.scalar_type() == at::kBFloat16,
              "out / dout");
  TORCH_CHECK(dq.scalar_type() == at::kFloat && dq.sizes() == q.sizes() && dq.is_contiguous(), "dq fp32 like q");
  TORCH_CHECK(dk.sizes() == k.sizes() && dv.sizes() == k.sizes() && dk.scalar_type() == at::kBFloat16 &&
                  dv.scalar_type() == at::kBFloat16 && dk.is_contiguous() && dv.is_contiguous(),
              "dk / dv bf16 like k");
  TORCH_CHECK(lse.numel() == (int64_t)p.B * p.hq * p.T && delta.numel() == lse.numel(), "lse / delta");
  p.o = reinterpret_cast<const __nv_bfloat16*>(out.data_ptr());
  p.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  p.lse = lse.data_ptr<float>();
  p.delta = delta.data_ptr<float>();
  p.dq = dq.data_ptr<float>();
  p.dk = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
  p.dv = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
  const int64_t rows = (int64_t)p.B * p.T * p.hq;
  train_attn_delta_kernel<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, cur_stream()>>>(p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  const int smem = 4 * TA_TILE_BYTES + TA_B * TA_DS_PITCH * 2 + 2 * TA_B * 4 + 3 * TA_B * 4;
  static PerDeviceOnce smem_opt_in;
  smem_opt_in([smem] {
    C10_CUDA_CHECK(
        cudaFuncSetAttribute(train_attn_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  });
  train_attn_bwd_kernel<<<dim3(p.nt, p.hkv, p.B), 128, smem, cur_stream()>>>(p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace uno
