// Persistent warp-specialised bf16 GEMM for sm_100a with fused epilogues.
//
//   D[M, N] = A[M, K] . B[N, K]^T     (A = activations, B = weights, both K-major)
//
// Per CTA (one per SM, persistent over output tiles of 128 x BN):
//   warp 0      TMA producer: 128x64 A tile + BNx64 B tile per stage (128-byte
//               swizzle) into a STAGES-deep shared-memory ring;
//   warp 1      allocates TMEM and issues tcgen05.mma (M=128, N=BN, K=16) from
//               one elected thread into a double-buffered fp32 TMEM accumulator;
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time from their TMEM lane
//               quarter, apply the fused epilogue, store to global memory.
// The accumulator double buffer lets the epilogue of tile i overlap the
// main loop of tile i+1.  Tiles are visited M-fastest so the CTAs that run
// concurrently share weight tiles through L2.
//
// Epilogues (EPI template argument):
//   STORE      C = bf16(acc)
//   SILU       gate/up rows interleaved in 64-row groups: out = silu(g) * u
//   LORA_SPLIT columns < n_base -> C (raw), columns >= n_base -> H = bf16(scale*mask[row]*acc)
//   ADD        C = bf16(acc + R)          (R may alias C)
//   ADD_SILU   as SILU with g, u = bf16(acc + R)
//   QKROPE     per 128-wide head: [+R], bf16 round, optional per-head RMSNorm,
//              NeoX RoPE; q heads -> Qout, k/v heads -> paged KV cache slots
//   ADD_QKROPE QKROPE with the residual add
// Every mbarrier wait is bounded (common.cuh); on timeout the kernel flags the
// error word and unwinds, freeing its TMEM.
#include <cudaTypedefs.h>

#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "uno_ops.h"

namespace uno {

enum Epi : int { EPI_STORE = 0, EPI_SILU = 1, EPI_LORA_SPLIT = 2, EPI_ADD = 3, EPI_ADD_SILU = 4, EPI_QKROPE = 5, EPI_ADD_QKROPE = 6 };


template <int BN>
struct GemmCfg {
  static constexpr int BM = 128, BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (196 * 1024) / STAGE_BYTES > 8 ? 8 : (196 * 1024) / STAGE_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }

__device__ __forceinline__ void store32_bf16(__nv_bfloat16* dst, const float* v, int valid_cols) {
  // valid_cols is a multiple of 8 (checked on host); write 16-byte granules.
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    if (g * 8 < valid_cols) {
      uint4 w;
      w.x = pack_bf16x2(v[g * 8 + 0], v[g * 8 + 1]);
      w.y = pack_bf16x2(v[g * 8 + 2], v[g * 8 + 3]);
      w.z = pack_bf16x2(v[g * 8 + 4], v[g * 8 + 5]);
      w.w = pack_bf16x2(v[g * 8 + 6], v[g * 8 + 7]);
      *reinterpret_cast<uint4*>(dst + g * 8) = w;
    }
  }
}

__device__ __forceinline__ void load32_bf16(const __nv_bfloat16* src, float* v, int valid_cols) {
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    if (g * 8 < valid_cols) {
      uint4 w = *reinterpret_cast<const uint4*>(src + g * 8);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float2 f = __bfloat1622float2(h[i]);
        v[g * 8 + 2 * i] = f.x;
        v[g * 8 + 2 * i + 1] = f.y;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[g * 8 + i] = 0.f;
    }
  }
}

// One 128-wide head of the QK-norm / RoPE / KV-store epilogue.
template <bool ADD>
__device__ __forceinline__ void qkrope_head(const GemmParams& p, uint32_t taddr, int row, bool row_ok, int col0) {
  float v[128];
#pragma unroll
  for (int c = 0; c < 4; ++c) tmem_ld32(taddr + c * 32, v + c * 32);
  if (!row_ok) return;
  if (ADD) {
    float r[32];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      load32_bf16(p.R + (size_t)row * p.ldr + col0 + c * 32, r, 32);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[c * 32 + i] += r[i];
    }
  }
#pragma unroll
  for (int i = 0; i < 128; ++i) v[i] = bf16r(v[i]);
  const int head = col0 / 128;
  const int hq = p.num_q_heads, hkv = p.num_kv_heads;
  const int64_t slot = p.slots[row];
  if (head < hq + hkv) {
    const __nv_bfloat16* w = head < hq ? p.q_norm_w : p.k_norm_w;
    if (w != nullptr) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 128; ++i) ss += v[i] * v[i];
      const float inv = rsqrtf(ss * (1.0f / 128.0f) + p.eps);
#pragma unroll
      for (int i = 0; i < 128; ++i) v[i] = bf16r(v[i] * inv * __bfloat162float(w[i]));
    }
    const float* cs = p.cos_sin + (size_t)p.positions[row] * 128;
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      const float c = cs[i], s = cs[64 + i];
      const float x1 = v[i], x2 = v[64 + i];
      v[i] = x1 * c - x2 * s;
      v[64 + i] = x2 * c + x1 * s;
    }
    if (head < hq) {
      __nv_bfloat16* dst = p.q_out + ((size_t)row * hq + head) * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) store32_bf16(dst + c * 32, v + c * 32, 32);
      return;
    }
    if (slot < 0) return;
    const int kvh = head - hq;
    __nv_bfloat16* dst = p.k_cache + (((size_t)(slot / p.page_size) * hkv + kvh) * p.page_size + slot % p.page_size) * 128;
#pragma unroll
    for (int c = 0; c < 4; ++c) store32_bf16(dst + c * 32, v + c * 32, 32);
    return;
  }
  if (slot < 0) return;
  const int kvh = head - hq - hkv;
  __nv_bfloat16* dst = p.v_cache + (((size_t)(slot / p.page_size) * hkv + kvh) * p.page_size + slot % p.page_size) * 128;
#pragma unroll
  for (int c = 0; c < 4; ++c) store32_bf16(dst + c * 32, v + c * 32, 32);
}

template <int BN, int EPI>
__device__ __forceinline__ void run_epilogue(const GemmParams& p, uint32_t taddr, int row, int n_blk) {
  const bool row_ok = row < p.M;
  const int n0 = n_blk * BN;
  if constexpr (EPI == EPI_QKROPE || EPI == EPI_ADD_QKROPE) {
#pragma unroll 1
    for (int h = 0; h < BN / 128; ++h) qkrope_head<EPI == EPI_ADD_QKROPE>(p, taddr + h * 128, row, row_ok, n0 + h * 128);
  } else if constexpr (EPI == EPI_SILU || EPI == EPI_ADD_SILU) {
    // Tile columns hold [gate 64 | up 64] pairs; output column block n_blk*BN/2.
#pragma unroll 1
    for (int pr = 0; pr < BN / 128; ++pr) {
#pragma unroll 1
      for (int c = 0; c < 64; c += 32) {
        float g[32], u[32];
        tmem_ld32(taddr + pr * 128 + c, g);
        tmem_ld32(taddr + pr * 128 + 64 + c, u);
        const int gcol = n0 + pr * 128 + c;
        if (!row_ok || gcol >= p.N) continue;
        if constexpr (EPI == EPI_ADD_SILU) {
          float r[32];
          load32_bf16(p.R + (size_t)row * p.ldr + gcol, r, 32);
#pragma unroll
          for (int i = 0; i < 32; ++i) g[i] += r[i];
          load32_bf16(p.R + (size_t)row * p.ldr + gcol + 64, r, 32);
#pragma unroll
          for (int i = 0; i < 32; ++i) u[i] += r[i];
        }
        float o[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float gg = bf16r(g[i]), uu = bf16r(u[i]);
          o[i] = silu_f(gg) * uu;
        }
        const int ocol = (n0 >> 1) + pr * 64 + c;
        store32_bf16(p.C + (size_t)row * p.ldc + ocol, o, 32);
      }
    }
  } else {
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      float v[32];
      tmem_ld32(taddr + c, v);
      const int col = n0 + c;
      if (!row_ok || col >= p.N) continue;
      const int valid = min(32, p.N - col);
      if constexpr (EPI == EPI_STORE) {
        store32_bf16(p.C + (size_t)row * p.ldc + col, v, valid);
      } else if constexpr (EPI == EPI_ADD) {
        float r[32];
        load32_bf16(p.R + (size_t)row * p.ldr + col, r, valid);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] += r[i];
        store32_bf16(p.C + (size_t)row * p.ldc + col, v, valid);
      } else if constexpr (EPI == EPI_LORA_SPLIT) {
        if (col < p.n_base) {
          store32_bf16(p.C + (size_t)row * p.ldc + col, v, min(valid, p.n_base - col));
        } else {
          const float s = p.lora_scale * p.row_mask[row];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] *= s;
          store32_bf16(p.H + (size_t)row * p.ldh + (col - p.n_base), v, valid);
        }
      }
    }
  }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(192, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmParams p) {
  using Cfg = GemmCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

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
  }
  if (warp == 1) tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_tiles = p.num_m * p.num_n;
  const int k_blocks = (p.K + Cfg::BK - 1) / Cfg::BK;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
        const int m_blk = tile % p.num_m, n_blk = tile / p.num_m;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err)) { *abort_flag = 1; break; }
          mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
          tma_load_2d(sA + stage * Cfg::A_BYTES, &tmA, &full[stage], kb * Cfg::BK, m_blk * Cfg::BM);
          tma_load_2d(sB + stage * Cfg::B_BYTES, &tmB, &full[stage], kb * Cfg::BK, n_blk * BN);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // Drain: make sure every issued load has landed before the CTA may exit.
      for (int s = 0; s < STAGES; ++s) {
        // A stage whose load is in flight completes its `full` phase; waiting
        // for the MMA's release of each stage covers all of them.
        (void)s;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(128, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, p.err)) { *abort_flag = 1; break; }
        tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err)) { ok = false; break; }
          tc_fence_after();
          const uint64_t adesc = smem_desc_sw128(sA + stage * Cfg::A_BYTES);
          const uint64_t bdesc = smem_desc_sw128(sB + stage * Cfg::B_BYTES);
#pragma unroll
          for (int k = 0; k < Cfg::BK / 16; ++k) {
            // advance 16 bf16 = 32 bytes along K inside the swizzle atom
            tc_mma_bf16(d, adesc + (uint64_t)(k * 2), bdesc + (uint64_t)(k * 2), idesc, (kb | k) != 0);
          }
          tc_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) { *abort_flag = 1; break; }
        tc_commit(&tfull[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
    }
  } else {
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int m_blk = tile % p.num_m, n_blk = tile / p.num_m;
      bool ok = true;
      if (lane == 0) ok = mbar_wait(&tfull[acc], acc_phase, p.err);
      ok = __shfl_sync(0xffffffff, ok, 0);
      if (!ok || *abort_flag) { *abort_flag = 1; break; }
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
      run_epilogue<BN, EPI>(p, taddr, m_blk * 128 + row_in_tile, n_blk);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
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

static int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

template <int BN, int EPI>
static void launch(const CUtensorMap& ta, const CUtensorMap& tb, GemmParams& p, cudaStream_t stream, int max_ctas) {
  using Cfg = GemmCfg<BN>;
  static bool configured = false;
  if (!configured) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(gemm_bf16_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    configured = true;
  }
  p.num_m = (p.M + 127) / 128;
  p.num_n = (p.N + BN - 1) / BN;
  int tiles = p.num_m * p.num_n;
  int grid = std::min(tiles, max_ctas > 0 ? max_ctas : num_sms());
  gemm_bf16_kernel<BN, EPI><<<grid, 192, Cfg::SMEM, stream>>>(ta, tb, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

int pick_bn(int M, int N, int forced) {
  if (forced) return forced;
  const int sms = num_sms();
  const int num_m = (M + 127) / 128;
  // Largest tile whose wave count keeps most SMs busy.
  for (int bn : {256, 128}) {
    int tiles = num_m * ((N + bn - 1) / bn);
    if (tiles >= (sms * 3) / 4) return bn;
  }
  return 64;
}

template <int EPI>
static void dispatch_bn(int bn, const void* a, int64_t lda, const void* b, int64_t ldb, GemmParams& p,
                        cudaStream_t stream, int max_ctas) {
  CUtensorMap ta = make_tmap_bf16(a, p.M, p.K, lda, 128);
  if (bn == 256) {
    CUtensorMap tb = make_tmap_bf16(b, p.N, p.K, ldb, 256);
    launch<256, EPI>(ta, tb, p, stream, max_ctas);
  } else if (bn == 128) {
    CUtensorMap tb = make_tmap_bf16(b, p.N, p.K, ldb, 128);
    launch<128, EPI>(ta, tb, p, stream, max_ctas);
  } else {
    if constexpr (EPI == EPI_SILU || EPI == EPI_ADD_SILU || EPI == EPI_QKROPE || EPI == EPI_ADD_QKROPE) {
      TORCH_CHECK(false, "this epilogue needs a 128 or 256 column tile");
    } else {
      CUtensorMap tb = make_tmap_bf16(b, p.N, p.K, ldb, 64);
      launch<64, EPI>(ta, tb, p, stream, max_ctas);
    }
  }
}

void gemm_dispatch(int epi, int bn, const void* a, int64_t lda, const void* b, int64_t ldb, GemmParams& p,
                   cudaStream_t stream, int max_ctas) {
  switch (epi) {
    case EPI_STORE: dispatch_bn<EPI_STORE>(bn, a, lda, b, ldb, p, stream, max_ctas); break;
    case EPI_SILU: dispatch_bn<EPI_SILU>(bn, a, lda, b, ldb, p, stream, max_ctas); break;
    case EPI_LORA_SPLIT: dispatch_bn<EPI_LORA_SPLIT>(bn, a, lda, b, ldb, p, stream, max_ctas); break;
    case EPI_ADD: dispatch_bn<EPI_ADD>(bn, a, lda, b, ldb, p, stream, max_ctas); break;
    case EPI_ADD_SILU: dispatch_bn<EPI_ADD_SILU>(bn, a, lda, b, ldb, p, stream, max_ctas); break;
    case EPI_QKROPE: dispatch_bn<EPI_QKROPE>(bn, a, lda, b, ldb, p, stream, max_ctas); break;
    case EPI_ADD_QKROPE: dispatch_bn<EPI_ADD_QKROPE>(bn, a, lda, b, ldb, p, stream, max_ctas); break;
    default: TORCH_CHECK(false, "unknown epilogue ", epi);
  }
}

}  // namespace uno
