// Persistent warp-specialised bf16 GEMM for sm_100a with fused epilogues.
//
//   D[M, N] = A[M, K] . B[N, K]^T     (A = activations, B = weights, both K-major)
//
// Per CTA (one per SM, persistent over work units = output tile x K split):
//   warp 0      TMA producer: 128x64 A tile + BNx64 B tile per stage (128-byte
//               swizzle) into a STAGES-deep shared-memory ring;
//   warp 1      allocates TMEM and issues tcgen05.mma (M=128, N=BN, K=16) from
//               one elected thread into a double-buffered fp32 TMEM accumulator;
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time from their TMEM lane
//               quarter, apply the fused epilogue, and move every global
//               load/store through a per-warp shared-memory staging tile so
//               that rows are read and written as contiguous segments.
// The accumulator double buffer lets the epilogue of tile i overlap the main
// loop of tile i+1.  Tiles are visited M-fastest so CTAs that run at the same
// time share weight tiles through L2.
//
// Split-K: when there are too few output tiles to fill the SMs, each tile's K
// range is split across CTAs.  Every split writes its fp32 partial to a global
// workspace; the last split to finish (per-tile arrival counter) sums the
// partials and runs the fused epilogue, then resets the counter so the next
// launch (or CUDA-graph replay) starts from zero.  Launches that share the
// workspace must not overlap on the GPU (one stream).
//
// K extension: a second operand pair (A2 [M, K2], B2 [N, K2]) continues the
// same K loop after the first, so D = A.B^T + A2.B2^T in one accumulator.  The
// gated LoRA uses it: A2 = scale * mask * (x . A_lora^T) (computed by a skinny
// ROWSCALE GEMM) and B2 = B_lora, so the adapter costs R extra K columns and
// no extra pass over the output.
//
// Epilogues (EPI template argument):
//   STORE      C = bf16(acc)
//   SILU       gate/up rows interleaved in 64-row groups: out = silu(g) * u
//   ROWSCALE   C = bf16(scale * row_mask[row] * acc)   (LoRA hidden)
//   ADD        C = bf16(acc + R)          (R may alias C)
//   QKROPE     per 128-wide head: bf16 round, optional per-head RMSNorm,
//              NeoX RoPE; q heads -> Qout, k/v heads -> paged KV cache slots
// Every mbarrier wait is bounded (common.cuh); on timeout the kernel flags the
// error word, lets in-flight copies land and unwinds, freeing its TMEM.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "uno_ops.h"

namespace uno {

// EPI_WGRAD: weight-gradient form.  Both operands are MN-major (A is [K, M]
// and B is [K, N], row-major, reduced over their rows: C = A^T B) and the
// epilogue accumulates into an fp32 matrix (C32 += A^T B).  Used for LoRA
// gradients, where the reduction runs over the tokens.
enum Epi : int { EPI_STORE = 0, EPI_SILU = 1, EPI_ROWSCALE = 2, EPI_ADD = 3, EPI_QKROPE = 5, EPI_WGRAD = 6 };

template <int EPI>
constexpr bool is_qkrope() {
  return EPI == EPI_QKROPE;
}

template <int EPI>
constexpr bool mn_major() {
  return EPI == EPI_WGRAD;
}

template <int BN, int EPI>
struct GemmCfg {
  static constexpr int BM = 128, BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int EPI_COLS = is_qkrope<EPI>() ? 128 : 32;
  static constexpr int PITCH = EPI_COLS * 2 + 16;          // staging row pitch (bytes)
  static constexpr int EPI_BYTES = 4 * 32 * PITCH;         // 4 epilogue warps x 32 rows
  static constexpr int RING = 200 * 1024 - EPI_BYTES;
  static constexpr int STAGES = RING / STAGE_BYTES > 8 ? 8 : RING / STAGE_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM = STAGES * STAGE_BYTES + EPI_BYTES + 1024 /*align*/ + 256 /*barriers*/;
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }

__device__ __forceinline__ uint64_t shfl64(uint64_t v, int src) {
  uint32_t lo = __shfl_sync(0xffffffff, (uint32_t)v, src);
  uint32_t hi = __shfl_sync(0xffffffff, (uint32_t)(v >> 32), src);
  return ((uint64_t)hi << 32) | lo;
}

// ---- per-warp staging tile [32 rows][COLS bf16] with padded rows ----------
template <int COLS>
struct Stage {
  static constexpr int PITCH = COLS * 2 + 16;
  static constexpr int PPR = COLS / 8;  // 16-byte pieces per row

  // This thread (row = lane) writes n (multiple of 8) values at column c0.
  __device__ static void row_write(uint8_t* buf, int lane, int c0, const float* v, int n) {
#pragma unroll
    for (int j = 0; j < n / 8; ++j) {
      uint4 w;
      w.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
      w.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
      w.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
      w.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
      *reinterpret_cast<uint4*>(buf + lane * PITCH + c0 * 2 + j * 16) = w;
    }
  }

  __device__ static void row_read(const uint8_t* buf, int lane, int c0, float* v, int n) {
#pragma unroll
    for (int j = 0; j < n / 8; ++j) {
      uint4 w = *reinterpret_cast<const uint4*>(buf + lane * PITCH + c0 * 2 + j * 16);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float2 f = __bfloat1622float2(h[i]);
        v[8 * j + 2 * i] = f.x;
        v[8 * j + 2 * i + 1] = f.y;
      }
    }
  }

  // Each lane supplies the global address of its own row (0 = skip); the warp
  // copies the staged rows out with contiguous 16-byte pieces per row.
  __device__ static void store(const uint8_t* buf, int lane, uint64_t my_dst, int valid_cols) {
#pragma unroll
    for (int k = 0; k < PPR; ++k) {
      const int pc = k * 32 + lane;
      const int r = pc / PPR, c = pc % PPR;
      const uint64_t d = shfl64(my_dst, r);
      if (d != 0 && c * 8 < valid_cols)
        *reinterpret_cast<uint4*>(d + c * 16) = *reinterpret_cast<const uint4*>(buf + r * PITCH + c * 16);
    }
  }

  __device__ static void load(uint8_t* buf, int lane, uint64_t my_src, int valid_cols) {
#pragma unroll
    for (int k = 0; k < PPR; ++k) {
      const int pc = k * 32 + lane;
      const int r = pc / PPR, c = pc % PPR;
      const uint64_t s = shfl64(my_src, r);
      uint4 w = make_uint4(0, 0, 0, 0);
      if (s != 0 && c * 8 < valid_cols) w = *reinterpret_cast<const uint4*>(s + c * 16);
      *reinterpret_cast<uint4*>(buf + r * PITCH + c * 16) = w;
    }
  }
};

// Accumulator source: TMEM (single split) or the sum of split-K partials.
struct AccSrc {
  uint32_t taddr;      // this warp's TMEM lane quarter + accumulator buffer
  const float* parts;  // first split partial of this tile (split mode), else null
  int splits;
  int bn;
  int row_in_tile;

  __device__ __forceinline__ void load32(int c, float* v) const {
    if (parts == nullptr) {
      tmem_ld32(taddr + c, v);
      return;
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = 0.f;
    for (int s = 0; s < splits; ++s) {
      const float* base = parts + (size_t)s * 128 * bn;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 f = *reinterpret_cast<const float4*>(base + ((size_t)(c / 4 + q) * 128 + row_in_tile) * 4);
        v[4 * q] += f.x;
        v[4 * q + 1] += f.y;
        v[4 * q + 2] += f.z;
        v[4 * q + 3] += f.w;
      }
    }
  }
};

// One 128-wide head of the QK-norm / RoPE / KV-store epilogue.
__device__ __forceinline__ void qkrope_head(const GemmParams& p, const AccSrc& src, uint8_t* buf, int lane, int row,
                                            bool row_ok, int cbase, int col0) {
  using S = Stage<128>;
  float v[128];
#pragma unroll
  for (int c = 0; c < 4; ++c) src.load32(cbase + c * 32, v + c * 32);
#pragma unroll
  for (int i = 0; i < 128; ++i) v[i] = bf16r(v[i]);
  const int head = col0 / 128;
  const int hq = p.num_q_heads, hkv = p.num_kv_heads;
  uint64_t dst = 0;
  if (row_ok) {
    const int64_t slot = p.slots[row];
    if (head < hq) {
      dst = (uint64_t)(p.q_out + ((size_t)row * hq + head) * 128);
    } else if (slot >= 0) {
      const bool is_k = head < hq + hkv;
      const int kvh = is_k ? head - hq : head - hq - hkv;
      __nv_bfloat16* cache = is_k ? p.k_cache : p.v_cache;
      dst = (uint64_t)(cache + (((size_t)(slot / p.page_size) * hkv + kvh) * p.page_size + slot % p.page_size) * 128);
    }
    if (head < hq + hkv) {
      const __nv_bfloat16* w = head < hq ? p.q_norm_w : p.k_norm_w;
      if (w != nullptr) {
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < 128; ++i) ss += v[i] * v[i];
        const float inv = rsqrtf(ss * (1.0f / 128.0f) + p.eps);
        const uint4* w4 = reinterpret_cast<const uint4*>(w);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const uint4 ww = __ldg(w4 + j);
          const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&ww);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(h2[e]);
            v[8 * j + 2 * e] = bf16r(v[8 * j + 2 * e] * inv * f.x);
            v[8 * j + 2 * e + 1] = bf16r(v[8 * j + 2 * e + 1] * inv * f.y);
          }
        }
      }
      // NeoX rotation with the [cos | sin] row of this position (float4 loads)
      const float4* cs4 = reinterpret_cast<const float4*>(p.cos_sin + (size_t)p.positions[row] * 128);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float4 c = __ldg(cs4 + j), sn = __ldg(cs4 + 16 + j);
        const float cc[4] = {c.x, c.y, c.z, c.w}, ss4[4] = {sn.x, sn.y, sn.z, sn.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = 4 * j + e;
          const float x1 = v[i], x2 = v[64 + i];
          v[i] = x1 * cc[e] - x2 * ss4[e];
          v[64 + i] = x2 * cc[e] + x1 * ss4[e];
        }
      }
    }
  }
  S::row_write(buf, lane, 0, v, 128);
  __syncwarp();
  S::store(buf, lane, dst, 128);
  __syncwarp();
}

template <int BN, int EPI>
__device__ __forceinline__ void run_epilogue(const GemmParams& p, const AccSrc& src, uint8_t* buf, int lane, int row,
                                             int n_blk) {
  const bool row_ok = row < p.M;
  const int n0 = n_blk * BN;
  if constexpr (is_qkrope<EPI>()) {
#pragma unroll 1
    for (int h = 0; h < BN / 128; ++h) {
      if (n0 + h * 128 >= p.N) break;
      qkrope_head(p, src, buf, lane, row, row_ok, h * 128, n0 + h * 128);
    }
  } else if constexpr (EPI == EPI_WGRAD) {
    // every lane takes part in the (warp-collective) TMEM loads; only the
    // stores of rows inside the matrix happen
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      const int col = n0 + c;
      if (col >= p.N) break;
      float v[32];
      src.load32(c, v);
      if (!row_ok) continue;
      float* dst = p.C32 + (size_t)row * p.ldc32 + col;
      if (col + 32 <= p.N) {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          float4 o = reinterpret_cast<float4*>(dst)[q];
          o.x += v[4 * q];
          o.y += v[4 * q + 1];
          o.z += v[4 * q + 2];
          o.w += v[4 * q + 3];
          reinterpret_cast<float4*>(dst)[q] = o;
        }
      } else {
        for (int i = 0; i < p.N - col; ++i) dst[i] += v[i];
      }
    }
  } else if constexpr (EPI == EPI_SILU) {
    using S = Stage<32>;
    // Tile columns hold [gate 64 | up 64] pairs; output column block n_blk*BN/2.
#pragma unroll 1
    for (int pr = 0; pr < BN / 128; ++pr) {
#pragma unroll 1
      for (int c = 0; c < 64; c += 32) {
        const int gcol = n0 + pr * 128 + c;
        if (gcol >= p.N) break;
        float g[32], u[32];
        src.load32(pr * 128 + c, g);
        src.load32(pr * 128 + 64 + c, u);
#pragma unroll
        for (int i = 0; i < 32; ++i) g[i] = silu_f(bf16r(g[i])) * bf16r(u[i]);
        const int ocol = (n0 >> 1) + pr * 64 + c;
        S::row_write(buf, lane, 0, g, 32);
        __syncwarp();
        S::store(buf, lane, row_ok ? (uint64_t)(p.C + (size_t)row * p.ldc + ocol) : 0ull, 32);
        __syncwarp();
      }
    }
  } else {
    using S = Stage<32>;
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      const int col = n0 + c;
      if (col >= p.N) break;
      const int valid = min(32, p.N - col);
      float v[32];
      src.load32(c, v);
      uint64_t dst = 0;
      if constexpr (EPI == EPI_ADD) {
        float r[32];
        S::load(buf, lane, row_ok ? (uint64_t)(p.R + (size_t)row * p.ldr + col) : 0ull, valid);
        __syncwarp();
        S::row_read(buf, lane, 0, r, 32);
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] += r[i];
      }
      const int vcols = valid;
      if constexpr (EPI == EPI_ROWSCALE) {
        const float sc = row_ok ? p.lora_scale * p.row_mask[row] : 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] *= sc;
      }
      if (row_ok) {
        if (EPI == EPI_STORE && p.rs_enable) {
          // reduce-scatter send: partial row -> owner's receive slot (NVLink P2P store)
          const int owner = row / p.rs_R, lr = row - owner * p.rs_R;
          dst = (uint64_t)(p.rs_peers[owner] + p.rs_recv_off +
                           (((size_t)p.rs_rank * p.rs_R + lr) * p.N + col) * 2);
        } else {
          dst = (uint64_t)(p.C + (size_t)row * p.ldc + col);
        }
      }
      S::row_write(buf, lane, 0, v, 32);
      __syncwarp();
      S::store(buf, lane, dst, vcols);
      __syncwarp();
    }
  }
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

template <int BN, int EPI>
__global__ void __launch_bounds__(192, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2, GemmParams p) {
  using Cfg = GemmCfg<BN, EPI>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint8_t* sEpi = smem + STAGES * Cfg::STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sEpi + Cfg::EPI_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = abort_flag + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (p.K2 > 0) {
      tma_prefetch_desc(&tmA2);
      tma_prefetch_desc(&tmB2);
    }
  }
  if (warp == 1) tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();     // the previous kernel's outputs (A operand, residual, split-K counters) are complete
  pdl_trigger();  // the next kernel may start its own set-up as SMs drain

  const int num_tiles = p.num_m * p.num_n;
  const int splits = p.splits;
  const int num_units = num_tiles * splits;
  const int kb_main = (p.K + Cfg::BK - 1) / Cfg::BK;
  const int k_blocks = kb_main + (p.K2 + Cfg::BK - 1) / Cfg::BK;
  const int kb_per = (k_blocks + splits - 1) / splits;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_phase[STAGES];
      bool issued[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) issued[s] = false;
      const unsigned long long ag_target =
          p.ag_base ? 2ull * *reinterpret_cast<const volatile unsigned long long*>(p.ag_base + COMM_EPOCH_OFF) : 0;
      for (int u = blockIdx.x; u < num_units && !*abort_flag; u += gridDim.x) {
        const int tile = u % num_tiles, ks = u / num_tiles;
        const int m_blk = tile % p.num_m, n_blk = tile / p.num_m;
        const int kb0 = ks * kb_per, kb1 = min(k_blocks, kb0 + kb_per);
        if (p.ag_base && !wait_row_owners(reinterpret_cast<const unsigned long long*>(p.ag_base + COMM_DONE_OFF),
                                          m_blk * Cfg::BM, min(p.M, (m_blk + 1) * Cfg::BM), p.ag_R, ag_target,
                                          p.err)) {
          *abort_flag = 1;
          break;
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err)) {
            *abort_flag = 1;
            break;
          }
          if constexpr (mn_major<EPI>()) {
            // [K rows][64 MN] boxes: BM / 64 for A, BN / 64 for B, 8 KB apart.  A
            // box that would start past the matrix edge is not issued (its
            // smem only feeds output rows / columns that are never stored).
            const int na = min(Cfg::BM / 64, (p.M - m_blk * Cfg::BM + 63) / 64);
            const int nb = min(BN / 64, (p.N - n_blk * BN + 63) / 64);
            mbar_arrive_expect_tx(&full[stage], (uint32_t)(na + nb) * 8192u);
            for (int h = 0; h < na; ++h)
              tma_load_2d(sA + stage * Cfg::A_BYTES + h * 8192, &tmA, &full[stage], m_blk * Cfg::BM + h * 64,
                          kb * Cfg::BK);
            for (int h = 0; h < nb; ++h)
              tma_load_2d(sB + stage * Cfg::B_BYTES + h * 8192, &tmB, &full[stage], n_blk * BN + h * 64,
                          kb * Cfg::BK);
          } else if (kb < kb_main) {
            mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
            tma_load_2d(sA + stage * Cfg::A_BYTES, &tmA, &full[stage], kb * Cfg::BK, m_blk * Cfg::BM);
            tma_load_2d(sB + stage * Cfg::B_BYTES, &tmB, &full[stage], kb * Cfg::BK, n_blk * BN);
          } else {
            mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
            const int k2 = (kb - kb_main) * Cfg::BK;
            tma_load_2d(sA + stage * Cfg::A_BYTES, &tmA2, &full[stage], k2, m_blk * Cfg::BM);
            tma_load_2d(sB + stage * Cfg::B_BYTES, &tmB2, &full[stage], k2, n_blk * BN);
          }
#pragma unroll
          for (int s = 0; s < STAGES; ++s)
            if (s == stage) {
              issued[s] = true;
              issued_phase[s] = phase;
            }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (*abort_flag) {  // let in-flight copies land before the CTA exits
#pragma unroll
        for (int s = 0; s < STAGES; ++s)
          if (issued[s]) mbar_wait(&full[s], issued_phase[s], p.err);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(128, BN) | (mn_major<EPI>() ? (1u << 15) | (1u << 16) : 0u);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int u = blockIdx.x; u < num_units && !*abort_flag; u += gridDim.x) {
        const int ks = u / num_tiles;
        const int kb0 = ks * kb_per, kb1 = min(k_blocks, kb0 + kb_per);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, p.err)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if constexpr (mn_major<EPI>()) {
            const uint64_t adesc = smem_desc_mn_sw128(sA + stage * Cfg::A_BYTES);
            const uint64_t bdesc = smem_desc_mn_sw128(sB + stage * Cfg::B_BYTES);
#pragma unroll
            for (int k = 0; k < Cfg::BK / 16; ++k) {
              // advance 16 K rows = 2048 bytes (two 8-row groups)
              tc_mma_bf16(d, adesc + (uint64_t)(k * 128), bdesc + (uint64_t)(k * 128), idesc, (kb > kb0 || k > 0));
            }
          } else {
            const uint64_t adesc = smem_desc_sw128(sA + stage * Cfg::A_BYTES);
            const uint64_t bdesc = smem_desc_sw128(sB + stage * Cfg::B_BYTES);
#pragma unroll
            for (int k = 0; k < Cfg::BK / 16; ++k) {
              // advance 16 bf16 = 32 bytes along K inside the swizzle atom
              tc_mma_bf16(d, adesc + (uint64_t)(k * 2), bdesc + (uint64_t)(k * 2), idesc, (kb > kb0 || k > 0));
            }
          }
          tc_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
        tc_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = quarter * 32 + lane;
    uint8_t* buf = sEpi + (warp - 2) * 32 * Cfg::PITCH;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = blockIdx.x; u < num_units; u += gridDim.x) {
      const int tile = u % num_tiles, ks = u / num_tiles;
      const int m_blk = tile % p.num_m, n_blk = tile / p.num_m;
      bool ok = true;
      if (lane == 0) ok = mbar_wait(&tfull[acc], acc_phase, p.err);
      ok = __shfl_sync(0xffffffff, ok, 0);
      if (!ok || *abort_flag) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
      const int row = m_blk * 128 + row_in_tile;
      if (splits == 1) {
        AccSrc src{taddr, nullptr, 1, BN, row_in_tile};
        run_epilogue<BN, EPI>(p, src, buf, lane, row, n_blk);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
      } else {
        // write this split's fp32 partial ([BN/4][128 rows][4] layout: coalesced per warp)
        float* mine = p.ws + ((size_t)tile * splits + ks) * 128 * BN;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          float v[32];
          tmem_ld32(taddr + c, v);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<float4*>(mine + ((size_t)(c / 4 + q) * 128 + row_in_tile) * 4) =
                make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
        __threadfence();
        epi_bar();
        if (threadIdx.x == 64) {
          const int old = atomicAdd(p.counters + tile, 1);
          *last_flag = (old == splits - 1);
        }
        epi_bar();
        if (*last_flag) {
          __threadfence();
          AccSrc src{0u, p.ws + (size_t)tile * splits * 128 * BN, splits, BN, row_in_tile};
          run_epilogue<BN, EPI>(p, src, buf, lane, row, n_blk);
          epi_bar();
          if (threadIdx.x == 64) p.counters[tile] = 0;  // ready for the next launch
        }
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }
  if (EPI == EPI_STORE && p.rs_enable) __threadfence_system();  // peer stores visible before the reduce
  __syncwarp();  // the single-lane producer / MMA roles rejoin their warps before the CTA barrier
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ------------------------------------------------------------ CTA-pair kernel
// Two CTAs of a cluster compute one 256 x 256 output tile with
// tcgen05.mma.cta_group::2 (M = 256): each CTA stages its own 128 rows of A and
// half (128 rows) of the B tile, so every SM streams 32 KB per 64-deep k-block
// instead of 48 KB for the same tensor work.  The leader CTA (cluster rank 0)
// owns the stage-full and accumulator-empty barriers and issues every MMA; the
// peer's TMA loads report their bytes to the leader's barrier (cta_group::2
// load form), and MMA completion is committed to both CTAs' barriers.  Each CTA
// runs the epilogue on its own 128 accumulator rows.
template <int EPI>
__global__ void __launch_bounds__(192, 1)
    gemm_bf16_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2,
                          GemmParams p) {
  constexpr int BN = 256;
  using Cfg = GemmCfg<128, EPI>;  // per-CTA stage = 128x64 A + 128x64 B
  constexpr int STAGES = Cfg::STAGES;
  constexpr int TMEM_COLS = 2 * BN;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint8_t* sEpi = smem + STAGES * Cfg::STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sEpi + Cfg::EPI_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = abort_flag + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);  // 4 epilogue warps in each CTA of the pair
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (p.K2 > 0) {
      tma_prefetch_desc(&tmA2);
      tma_prefetch_desc(&tmB2);
    }
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, TMEM_COLS);
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers exist before any remote use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();
  pdl_trigger();

  const int num_m2 = (p.M + 255) / 256;
  const int num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m2 * num_n;
  const int splits = p.splits;
  const int num_units = num_tiles * splits;
  const int kb_main = (p.K + Cfg::BK - 1) / Cfg::BK;
  const int k_blocks = kb_main + (p.K2 + Cfg::BK - 1) / Cfg::BK;
  const int kb_per = (k_blocks + splits - 1) / splits;
  const int cid = (int)cluster_id_x(), ncl = (int)num_clusters_x();

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_phase[STAGES];
      bool issued[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) issued[s] = false;
      const unsigned long long ag_target =
          p.ag_base ? 2ull * *reinterpret_cast<const volatile unsigned long long*>(p.ag_base + COMM_EPOCH_OFF) : 0;
      for (int u = cid; u < num_units && !*abort_flag; u += ncl) {
        const int tile = u % num_tiles, ks = u / num_tiles;
        const int m2 = tile % num_m2, n_blk = tile / num_m2;
        const int kb0 = ks * kb_per, kb1 = min(k_blocks, kb0 + kb_per);
        const int arow = m2 * 256 + (int)rank * 128;
        const int brow = n_blk * BN + (int)rank * 128;
        if (p.ag_base && arow < p.M &&
            !wait_row_owners(reinterpret_cast<const unsigned long long*>(p.ag_base + COMM_DONE_OFF), arow,
                             min(p.M, arow + 128), p.ag_R, ag_target, p.err)) {
          *abort_flag = 1;
          break;
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err)) {
            *abort_flag = 1;
            break;
          }
          const uint32_t lead_full = mapa_shared(smem_u32(&full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::STAGE_BYTES);
          if (kb < kb_main) {
            tma_load_2d_pair(sA + stage * Cfg::A_BYTES, &tmA, lead_full, kb * Cfg::BK, arow);
            tma_load_2d_pair(sB + stage * Cfg::B_BYTES, &tmB, lead_full, kb * Cfg::BK, brow);
          } else {
            const int k2 = (kb - kb_main) * Cfg::BK;
            tma_load_2d_pair(sA + stage * Cfg::A_BYTES, &tmA2, lead_full, k2, arow);
            tma_load_2d_pair(sB + stage * Cfg::B_BYTES, &tmB2, lead_full, k2, brow);
          }
#pragma unroll
          for (int s = 0; s < STAGES; ++s)
            if (s == stage) {
              issued[s] = true;
              issued_phase[s] = phase;
            }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (*abort_flag && leader) {  // let in-flight copies land before the CTA exits
#pragma unroll
        for (int s = 0; s < STAGES; ++s)
          if (issued[s]) mbar_wait(&full[s], issued_phase[s], p.err);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = idesc_bf16(256, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int u = cid; u < num_units && !*abort_flag; u += ncl) {
        const int ks = u / num_tiles;
        const int kb0 = ks * kb_per, kb1 = min(k_blocks, kb0 + kb_per);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, p.err)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = smem_desc_sw128(sA + stage * Cfg::A_BYTES);
          const uint64_t bdesc = smem_desc_sw128(sB + stage * Cfg::B_BYTES);
#pragma unroll
          for (int k = 0; k < Cfg::BK / 16; ++k)
            tc_mma_bf16_pair(d, adesc + (uint64_t)(k * 2), bdesc + (uint64_t)(k * 2), idesc, (kb > kb0 || k > 0));
          const uint32_t e_addr = smem_u32(&empty[stage]);
          tc_commit_pair(mapa_shared(e_addr, 0));
          tc_commit_pair(mapa_shared(e_addr, 1));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
        const uint32_t f_addr = smem_u32(&tfull[acc]);
        tc_commit_pair(mapa_shared(f_addr, 0));
        tc_commit_pair(mapa_shared(f_addr, 1));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    uint8_t* buf = sEpi + (warp - 2) * 32 * Cfg::PITCH;
    const int num_m128 = num_m2 * 2;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = cid; u < num_units; u += ncl) {
      const int tile = u % num_tiles, ks = u / num_tiles;
      const int m2 = tile % num_m2, n_blk = tile / num_m2;
      const int m_blk = m2 * 2 + (int)rank;  // this CTA's 128-row block
      const int ctile = m_blk + num_m128 * n_blk;
      bool ok = true;
      if (lane == 0) ok = mbar_wait(&tfull[acc], acc_phase, p.err);
      ok = __shfl_sync(0xffffffff, ok, 0);
      if (!ok || *abort_flag) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
      const int row = m_blk * 128 + row_in_tile;
      const uint32_t lead_tempty = mapa_shared(smem_u32(&tempty[acc]), 0);
      if (splits == 1) {
        AccSrc src{taddr, nullptr, 1, BN, row_in_tile};
        run_epilogue<BN, EPI>(p, src, buf, lane, row, n_blk);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(lead_tempty);
      } else {
        float* mine = p.ws + ((size_t)ctile * splits + ks) * 128 * BN;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          float v[32];
          tmem_ld32(taddr + c, v);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<float4*>(mine + ((size_t)(c / 4 + q) * 128 + row_in_tile) * 4) =
                make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(lead_tempty);
        __threadfence();
        epi_bar();
        if (threadIdx.x == 64) {
          const int old = atomicAdd(p.counters + ctile, 1);
          *last_flag = (old == splits - 1);
        }
        epi_bar();
        if (*last_flag) {
          __threadfence();
          AccSrc src{0u, p.ws + (size_t)ctile * splits * 128 * BN, splits, BN, row_in_tile};
          run_epilogue<BN, EPI>(p, src, buf, lane, row, n_blk);
          epi_bar();
          if (threadIdx.x == 64) p.counters[ctile] = 0;
        }
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }
  if (EPI == EPI_STORE && p.rs_enable) __threadfence_system();
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the peer is done with the leader's barriers and TMEM
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  TORCH_CHECK(fn != nullptr, "cuTensorMapEncodeTiled unavailable");
  return fn;
}

// 2-D bf16 tensor map over a row-major [rows, cols] matrix with row stride
// `ld` elements; box = [64 cols, box_rows rows], 128-byte swizzle.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() { return get_encode(); }

CUtensorMap make_tmap_bf16(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(ptr) % 16 == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
  return m;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("UNO_PDL");
    return e == nullptr || e[0] != '0';
  }();
  return on;
}

int num_sms() {
  static std::atomic<int> counts[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  int n = counts[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    counts[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

template <int BN, int EPI>
static void launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ta2, const CUtensorMap& tb2,
                   GemmParams& p, cudaStream_t stream, int max_ctas) {
  using Cfg = GemmCfg<BN, EPI>;
  static PerDeviceOnce smem_opt_in;
  smem_opt_in([] {
    C10_CUDA_CHECK(
        cudaFuncSetAttribute(gemm_bf16_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
  });
  const int units = p.num_m * p.num_n * p.splits;
  const int grid = std::min(units, max_ctas > 0 ? max_ctas : num_sms());
  launch_pdl(gemm_bf16_kernel<BN, EPI>, dim3(grid), dim3(192), Cfg::SMEM, stream, ta, tb, ta2, tb2, p);
}

template <int EPI>
static void launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ta2, const CUtensorMap& tb2,
                        GemmParams& p, cudaStream_t stream, int max_ctas) {
  using Cfg = GemmCfg<128, EPI>;
  static PerDeviceOnce smem_opt_in;
  smem_opt_in([] {
    C10_CUDA_CHECK(
        cudaFuncSetAttribute(gemm_bf16_pair_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
  });
  const int units = ((p.M + 255) / 256) * ((p.N + 255) / 256) * p.splits;
  const int pairs = std::max(1, std::min(units, (max_ctas > 0 ? max_ctas : num_sms()) / 2));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(192, 1, 1);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, gemm_bf16_pair_kernel<EPI>, ta, tb, ta2, tb2, p));
}

static bool pair_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("UNO_GEMM_PAIR");
    v = (e == nullptr || e[0] != '0') ? 1 : 0;
  }
  return v == 1;
}

int pick_bn(int M, int N, int forced) {
  if (forced) return forced;
  if (N <= 256) return 32;  // skinny outputs (LoRA hidden): many small tiles, cheap split-K reduction
  return 256;
}

// K splits for a (M, N, K) problem with tile width bn: only when the output
// tiles leave most SMs idle and each split keeps a long enough K loop.
int pick_splits(int M, int N, int K, int bn, int forced) {
  if (forced > 0) return forced;
  const int sms = num_sms();
  const int tiles = ((M + 127) / 128) * ((N + bn - 1) / bn);
  const int kb = (K + 63) / 64;
  if (tiles * 5 >= sms * 3 || kb < 16) return 1;
  // Few tiles: up to 8 splits of >= 4 k-blocks for skinny outputs, else 4.
  const int cap = bn <= 64 ? 8 : 4;
  int s = std::min({cap, std::max(1, sms / tiles), kb / (bn <= 64 ? 4 : 8)});
  return std::max(1, s);
}

// Tile width and K splits for one GEMM.  A single row of 128-row tiles
// (M <= 128: small-batch decode, tree verification) is bound by streaming
// the weights, so it takes narrow tiles -- 64 columns when K <= 4096 and the
// epilogue allows, else 128 -- and enough K splits for about 128 CTAs.
void pick_tile(int M, int N, int K, int epi, int forced_bn, int forced_splits, int* bn, int* splits) {
  const bool wide_epi = (epi == EPI_SILU || epi == EPI_QKROPE);  // head / gate-up aligned tiles
  // More rows: 128x128 single-SM tiles without a K split while they fit in
  // one wave of SMs (the partial-sum reduction costs more than it saves
  // there); K splits only when those tiles are few; CTA pairs with 256x256
  // tiles for the large GEMMs.
  const int sms = num_sms();
  const int t128 = ((M + 127) / 128) * ((N + 127) / 128);
  const bool narrow_rows = M <= 128 && N > 256;
  const bool mid = M > 128 && N > 256 && t128 <= sms;
  // ... except a long K loop (down_proj, K = 12288), where two K splits of
  // CTA-pair 256x256 tiles beat one wave of 128x128 tiles (64 -> 53 us at
  // 512 x 4096 x 12288)
  const bool mid_long_k = mid && K >= 6144 && M >= 256 && pair_enabled();
  int tile;
  if (forced_bn) {
    tile = forced_bn;
  } else if (narrow_rows) {
    tile = (!wide_epi && K <= 4096) ? 64 : 128;
  } else if (mid_long_k) {
    tile = 256;
  } else if (mid) {
    tile = 128;
  } else {
    tile = pick_bn(M, N, 0);
  }
  if (wide_epi && tile < 128) tile = 128;
  int s;
  const int kb = (K + 63) / 64;
  if (forced_splits > 0) {
    s = forced_splits;
  } else if (!forced_bn && narrow_rows) {
    const int tiles = (N + tile - 1) / tile;
    s = std::max(1, std::min({4, (128 + tiles / 2) / tiles, kb / 16}));
  } else if (!forced_bn && mid_long_k) {
    s = 2;
  } else if (!forced_bn && mid) {
    s = t128 * 2 >= sms ? 1 : std::max(1, std::min({4, (128 + t128 / 2) / t128, kb / 16}));
  } else {
    s = pick_splits(M, N, K, tile, 0);
  }
  *bn = tile;
  *splits = s;
}

template <int EPI>
static void dispatch_bn(int bn, const void* a, int64_t lda, const void* b, int64_t ldb, const void* a2, int64_t lda2,
                        const void* b2, int64_t ldb2, GemmParams& p, cudaStream_t stream, int max_ctas) {
  CUtensorMap ta = make_tmap_bf16(a, p.M, p.K, lda, 128);
  CUtensorMap ta2 = p.K2 > 0 ? make_tmap_bf16(a2, p.M, p.K2, lda2, 128) : ta;
  p.num_m = (p.M + 127) / 128;
  p.num_n = (p.N + bn - 1) / bn;
  if (bn == 256 && p.M >= 256 && pair_enabled()) {
    // CTA-pair path: 128-row boxes for both operands (each CTA stages half of B)
    CUtensorMap tb = make_tmap_bf16(b, p.N, p.K, ldb, 128);
    CUtensorMap tb2 = p.K2 > 0 ? make_tmap_bf16(b2, p.N, p.K2, ldb2, 128) : tb;
    p.num_m = ((p.M + 255) / 256) * 2;
    launch_pair<EPI>(ta, tb, ta2, tb2, p, stream, max_ctas);
  } else if (bn == 256) {
    CUtensorMap tb = make_tmap_bf16(b, p.N, p.K, ldb, 256);
    CUtensorMap tb2 = p.K2 > 0 ? make_tmap_bf16(b2, p.N, p.K2, ldb2, 256) : tb;
    launch<256, EPI>(ta, tb, ta2, tb2, p, stream, max_ctas);
  } else if (bn == 128) {
    CUtensorMap tb = make_tmap_bf16(b, p.N, p.K, ldb, 128);
    CUtensorMap tb2 = p.K2 > 0 ? make_tmap_bf16(b2, p.N, p.K2, ldb2, 128) : tb;
    launch<128, EPI>(ta, tb, ta2, tb2, p, stream, max_ctas);
  } else {
    if constexpr (EPI == EPI_SILU || is_qkrope<EPI>()) {
      TORCH_CHECK(false, "this epilogue needs a 128 or 256 column tile");
    } else if (bn == 64) {
      CUtensorMap tb = make_tmap_bf16(b, p.N, p.K, ldb, 64);
      CUtensorMap tb2 = p.K2 > 0 ? make_tmap_bf16(b2, p.N, p.K2, ldb2, 64) : tb;
      launch<64, EPI>(ta, tb, ta2, tb2, p, stream, max_ctas);
    } else {
      TORCH_CHECK(bn == 32, "unsupported tile width ", bn);
      CUtensorMap tb = make_tmap_bf16(b, p.N, p.K, ldb, 32);
      CUtensorMap tb2 = p.K2 > 0 ? make_tmap_bf16(b2, p.N, p.K2, ldb2, 32) : tb;
      launch<32, EPI>(ta, tb, ta2, tb2, p, stream, max_ctas);
    }
  }
}

// C32[M, N] += A^T B for row-major A [K, M] and B [K, N] (weight gradients).
void gemm_wgrad_dispatch(const void* a, int64_t lda, const void* b, int64_t ldb, GemmParams& p, int bn,
                         cudaStream_t stream) {
  TORCH_CHECK(p.K2 == 0, "the weight-gradient GEMM has no K extension");
  CUtensorMap ta = make_tmap_bf16(a, p.K, p.M, lda, 64);
  CUtensorMap tb = make_tmap_bf16(b, p.K, p.N, ldb, 64);
  p.num_m = (p.M + 127) / 128;
  p.num_n = (p.N + bn - 1) / bn;
  if (bn == 64)
    launch<64, EPI_WGRAD>(ta, tb, ta, tb, p, stream, 0);
  else if (bn == 128)
    launch<128, EPI_WGRAD>(ta, tb, ta, tb, p, stream, 0);
  else
    TORCH_CHECK(false, "weight-gradient GEMM tiles are 64 or 128 columns wide");
}

void gemm_dispatch(int epi, int bn, const void* a, int64_t lda, const void* b, int64_t ldb, const void* a2,
                   int64_t lda2, const void* b2, int64_t ldb2, GemmParams& p, cudaStream_t stream, int max_ctas) {
  TORCH_CHECK(p.K2 == 0 || p.K % 64 == 0, "the K extension needs the main K to be a multiple of 64");
  switch (epi) {
    case EPI_STORE: dispatch_bn<EPI_STORE>(bn, a, lda, b, ldb, a2, lda2, b2, ldb2, p, stream, max_ctas); break;
    case EPI_SILU: dispatch_bn<EPI_SILU>(bn, a, lda, b, ldb, a2, lda2, b2, ldb2, p, stream, max_ctas); break;
    case EPI_ROWSCALE: dispatch_bn<EPI_ROWSCALE>(bn, a, lda, b, ldb, a2, lda2, b2, ldb2, p, stream, max_ctas); break;
    case EPI_ADD: dispatch_bn<EPI_ADD>(bn, a, lda, b, ldb, a2, lda2, b2, ldb2, p, stream, max_ctas); break;
    case EPI_QKROPE: dispatch_bn<EPI_QKROPE>(bn, a, lda, b, ldb, a2, lda2, b2, ldb2, p, stream, max_ctas); break;
    default: TORCH_CHECK(false, "unknown epilogue ", epi);
  }
}

}  // namespace uno
