// Paged attention for prefill, linear-block decode and tree verification.
//
// One kernel serves every mode through a single visibility rule:
//   * decode / tree (MODE_SUFFIX): request b has prefix_lens[b] cached keys that
//     every query sees; query i additionally sees its forward's own key j
//     (logical position prefix + j) iff bit j of suffix_mask[b, i] is set
//     (causal block: (2 << i) - 1; tree: ancestor-or-self mask);
//   * prefill (MODE_CAUSAL): query i of a request with nq new and nk total keys
//     sees keys 0 .. nk - nq + i.
// K/V live in the paged cache [pages, kv_heads, page, 128] (bf16); they are
// stored by the QKV epilogue before this kernel runs.
//
// CTA = (query block, request, kv head, key split).  Rows are (query, head in
// GQA group) pairs so one K/V tile feeds every query head of the group.
// Warp 0 streams 64-key K and V tiles with TMA (128-byte swizzle, two 64-dim
// boxes each) through a 3-stage mbarrier ring; warps 1..NW each own 16 rows
// and run S = Q K^T and O += P V on the tensor cores (mma.sync m16n8k16 bf16)
// with an online softmax in registers.  Decode attention streams the KV cache
// once per (request, kv head), so the kernel is bound by HBM bandwidth; key
// splits (flash-decoding) give long contexts enough CTAs, and a combine kernel
// merges the partial (O, log-sum-exp) pairs.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "uno_ops.h"

namespace uno {

constexpr int ATT_D = 128;
constexpr int ATT_BK = 64;           // keys per tile
constexpr int ATT_STAGES = 3;
constexpr int ATT_TILE_BYTES = ATT_BK * ATT_D * 2;  // 16 KB (K or V)

enum AttMode : int { MODE_SUFFIX = 0, MODE_CAUSAL = 1 };

struct AttnParams {
  const __nv_bfloat16* q;      // [T, Hq, 128]
  __nv_bfloat16* o;            // [T, Hq, 128]
  float* o_part;               // [splits, T, Hq, 128] (split mode)
  float* lse_part;             // [splits, T, Hq]
  const int* block_tables;     // [B, max_pages]
  int bt_stride;
  const int* prefix_lens;      // [B] (suffix mode)
  const int64_t* suffix_mask;  // [B, Q] (suffix mode)
  const int* cu_q;             // [B+1] (causal mode)
  const int* cu_k;             // [B+1] (causal mode)
  int Q;                       // queries per request (suffix mode)
  int hq, hkv, group, page;
  int rows_per_cta;            // 16 * compute warps
  int queries_per_cta;         // rows_per_cta / group
  int keys_per_split;          // multiple of ATT_BK (0 = no split)
  int num_splits;
  int T;
  float scale_log2;            // softmax scale * log2(e)
  int mode;
  int* err;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16_16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Byte offset of (key, 16-byte chunk c in 0..15) inside a swizzled 64x128 tile.
__device__ __forceinline__ uint32_t tile_off(int key, int c) {
  return (uint32_t)((c >> 3) * (ATT_BK * 128) + key * 128 + (((c & 7) ^ (key & 7)) << 4));
}

template <int NWR, int KS>
__global__ void __launch_bounds__(32 * (NWR * KS + 1), 1)
    paged_attention_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                           AttnParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = smem + ATT_STAGES * ATT_TILE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * ATT_STAGES * ATT_TILE_BYTES);
  uint64_t* empty = full + ATT_STAGES;

  const int qblk = blockIdx.x, b = blockIdx.y;
  const int h = blockIdx.z % p.hkv, split = blockIdx.z / p.hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int n_compute = NWR * KS;
  constexpr int KPW = ATT_BK / KS;  // keys of each tile handled by one warp
  constexpr int NT = KPW / 8;       // 8-key n-tiles per warp

  // ---- geometry of this request
  int q_begin, nq, kv_len, prefix;
  if (p.mode == MODE_SUFFIX) {
    prefix = p.prefix_lens[b];
    nq = p.Q;
    q_begin = b * p.Q;
    kv_len = prefix + p.Q;
  } else {
    q_begin = p.cu_q[b];
    nq = p.cu_q[b + 1] - q_begin;
    kv_len = p.cu_k[b + 1] - p.cu_k[b];
    prefix = kv_len - nq;
  }
  const int i0 = qblk * p.queries_per_cta;  // first query of this CTA
  if (i0 >= nq) return;
  const int i1 = min(nq, i0 + p.queries_per_cta);
  // keys this CTA may need: up to the last visible key of its last query
  int k_hi = (p.mode == MODE_CAUSAL) ? min(kv_len, prefix + i1) : kv_len;
  int k_lo = 0;
  if (p.num_splits > 1) {
    k_lo = split * p.keys_per_split;
    k_hi = min(k_hi, k_lo + p.keys_per_split);
  }
  const int n_tiles = k_hi > k_lo ? (k_hi - k_lo + ATT_BK - 1) / ATT_BK : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ATT_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], n_compute);
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_wait();     // q and the KV cache writes of the previous kernel are complete
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0 && n_tiles > 0) {
      int stage = 0;
      uint32_t phase = 0;
      const int* bt = p.block_tables + (size_t)b * p.bt_stride;
      int issued_phase[ATT_STAGES];
      bool issued[ATT_STAGES];
      for (int s = 0; s < ATT_STAGES; ++s) issued[s] = false;
      bool ok = true;
      for (int t = 0; t < n_tiles; ++t) {
        if (!mbar_wait(&empty[stage], phase ^ 1, p.err)) { ok = false; break; }
        const int k0 = k_lo + t * ATT_BK;
        const int page_id = bt[k0 / p.page];
        const int row = (page_id * p.hkv + h) * p.page + (k0 % p.page);
        mbar_arrive_expect_tx(&full[stage], 2 * ATT_TILE_BYTES);
        tma_load_2d(sK + stage * ATT_TILE_BYTES, &tmK, &full[stage], 0, row);
        tma_load_2d(sK + stage * ATT_TILE_BYTES + ATT_TILE_BYTES / 2, &tmK, &full[stage], 64, row);
        tma_load_2d(sV + stage * ATT_TILE_BYTES, &tmV, &full[stage], 0, row);
        tma_load_2d(sV + stage * ATT_TILE_BYTES + ATT_TILE_BYTES / 2, &tmV, &full[stage], 64, row);
        issued[stage] = true;
        issued_phase[stage] = phase;
        if (++stage == ATT_STAGES) { stage = 0; phase ^= 1; }
      }
      if (!ok) {  // let in-flight copies land before the CTA exits
        for (int s = 0; s < ATT_STAGES; ++s)
          if (issued[s]) mbar_wait(&full[s], issued_phase[s], p.err);
      }
    }
    return;
  }

  // ---- compute warps: 16 rows x KPW keys of every tile each
  const int cw = warp - 1;
  const int rg = cw % NWR, kss = cw / NWR;
  const int g = lane >> 2, tq = lane & 3;
  const int row_base = rg * 16;  // row index within CTA
  const int kofs = kss * KPW;    // first key of this warp inside a tile
  // rows g and g+8 of this warp
  int qi[2], qh[2];
  bool row_valid[2];
  int64_t smask[2];
  int qlimit[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int rr = row_base + g + r * 8;
    const int i = i0 + rr / p.group;
    qi[r] = i;
    qh[r] = h * p.group + rr % p.group;
    row_valid[r] = (rr < p.rows_per_cta) && (i < i1);
    smask[r] = (p.mode == MODE_SUFFIX && row_valid[r]) ? p.suffix_mask[(size_t)b * p.Q + i] : 0;
    qlimit[r] = prefix + i;  // causal: last visible key
  }
  // Q fragments (A operand) for 8 k-steps of 16 dims
  uint32_t qa[8][4];
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
    for (int part = 0; part < 4; ++part) {
      const int r = part & 1;  // a0,a2 -> row g ; a1,a3 -> row g+8
      const int col = ks * 16 + tq * 2 + (part >> 1) * 8;
      uint32_t v = 0;
      if (row_valid[r]) {
        const __nv_bfloat16* src = p.q + ((size_t)(q_begin + qi[r]) * p.hq + qh[r]) * ATT_D + col;
        v = *reinterpret_cast<const uint32_t*>(src);
      }
      qa[ks][part] = v;
    }
  }
  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};

  int stage = 0;
  uint32_t phase = 0;
  const uint32_t sK_base = smem_u32(sK), sV_base = smem_u32(sV);
  for (int t = 0; t < n_tiles; ++t) {
    bool ok = true;
    if (lane == 0) ok = mbar_wait(&full[stage], phase, p.err);
    ok = __shfl_sync(0xffffffff, ok, 0);
    if (!ok) break;
    const uint32_t kb = sK_base + stage * ATT_TILE_BYTES;
    const uint32_t vb = sV_base + stage * ATT_TILE_BYTES;
    const int k0 = k_lo + t * ATT_BK;
    // ---- S = Q K^T  (16 rows x KPW keys)
    float s[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int np = 0; np < NT / 2; ++np) {
        // matrices: (keys np*16+0..7, chunk 2ks), (same keys, chunk 2ks+1),
        //           (keys np*16+8..15, chunk 2ks), (.., chunk 2ks+1)
        const int mtx = lane >> 3, r8 = lane & 7;
        const int key = kofs + np * 16 + (mtx >> 1) * 8 + r8;
        const int chunk = ks * 2 + (mtx & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kb + tile_off(key, chunk), b0, b1, b2, b3);
        mma_bf16_16816(s[np * 2], qa[ks], b0, b1);
        mma_bf16_16816(s[np * 2 + 1], qa[ks], b2, b3);
      }
    }
    // ---- mask + online softmax
    float mx[2] = {-INFINITY, -INFINITY};
    // tiles every row sees in full (prefix keys, or causal keys below every row's limit) skip the mask
    const bool tile_visible = row_valid[0] && row_valid[1] && k0 + ATT_BK <= k_hi &&
                              (p.mode == MODE_SUFFIX ? k0 + ATT_BK <= prefix
                                                     : k0 + ATT_BK - 1 <= min(qlimit[0], qlimit[1]));
    if (__all_sync(0xffffffff, tile_visible)) {
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          s[n][e] *= p.scale_log2;
          mx[e >> 1] = fmaxf(mx[e >> 1], s[n][e]);
        }
    } else {
#pragma unroll
      for (int n = 0; n < NT; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = e >> 1;
          const int key = k0 + kofs + n * 8 + tq * 2 + (e & 1);
          bool vis = row_valid[r] && key < k_hi;
          if (vis) {
            if (p.mode == MODE_SUFFIX) {
              const int j = key - prefix;
              vis = (j < 0) || ((smask[r] >> j) & 1);
            } else {
              vis = key <= qlimit[r];
            }
          }
          const float v = vis ? s[n][e] * p.scale_log2 : -INFINITY;
          s[n][e] = v;
          mx[r] = fmaxf(mx[r], v);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffff, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffff, mx[r], 2));
    }
    // Lazy rescale: the running max only moves when a score exceeds it by
    // more than 2^8 (so exp2 arguments stay <= 8, far inside fp32/bf16
    // range); after the first tiles the O rescale below is rarely taken.
    const bool raise = (mx[0] > m_run[0] + 8.f) || (mx[1] > m_run[1] + 8.f);
    if (__any_sync(0xffffffff, raise)) {
      float corr[2];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const float m_new = fmaxf(m_run[r], mx[r]);
        corr[r] = (m_run[r] == -INFINITY) ? 0.f : exp2f(m_run[r] - m_new);
        m_run[r] = m_new;
        l_run[r] *= corr[r];
      }
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        o[n][0] *= corr[0];
        o[n][1] *= corr[0];
        o[n][2] *= corr[1];
        o[n][3] *= corr[1];
      }
    }
    float rs[2] = {0.f, 0.f};
    uint32_t pa[NT / 2][4];  // P as A fragments for the k-steps of 16 keys
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      float e4[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = e >> 1;
        const float v = (s[n][e] == -INFINITY) ? 0.f : exp2f(s[n][e] - m_run[r]);
        e4[e] = v;
        rs[r] += v;
      }
      // C fragment of n-tile n -> A fragment halves of k-step n/2
      const int ks = n >> 1, hi = n & 1;
      pa[ks][hi * 2 + 0] = pack_bf16x2(e4[0], e4[1]);
      pa[ks][hi * 2 + 1] = pack_bf16x2(e4[2], e4[3]);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) l_run[r] += rs[r];
    // ---- O += P V
#pragma unroll
    for (int ks = 0; ks < NT / 2; ++ks) {
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        // matrices: (keys ks*16+0..7, dim chunk 2dp), (keys +8..15, chunk 2dp),
        //           (keys 0..7, chunk 2dp+1), (keys 8..15, chunk 2dp+1) -- transposed
        const int mtx = lane >> 3, r8 = lane & 7;
        const int key = kofs + ks * 16 + (mtx & 1) * 8 + r8;
        const int chunk = dp * 2 + (mtx >> 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vb + tile_off(key, chunk), b0, b1, b2, b3);
        mma_bf16_16816(o[dp * 2], pa[ks], b0, b1);
        mma_bf16_16816(o[dp * 2 + 1], pa[ks], b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    if (++stage == ATT_STAGES) { stage = 0; phase ^= 1; }
  }

  // ---- finalize rows
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_run[r] += __shfl_xor_sync(0xffffffff, l_run[r], 1);
    l_run[r] += __shfl_xor_sync(0xffffffff, l_run[r], 2);
  }
  if constexpr (KS > 1) {
    // Merge the KS key-split partial states of each row group through shared
    // memory (the K/V ring is idle now: every issued tile was consumed).
    constexpr int PER_THREAD = 68;  // m[2], l[2], o[16][4]
    float* part = reinterpret_cast<float*>(smem) + (size_t)(cw * 32 + lane) * PER_THREAD;
    asm volatile("bar.sync 1, %0;" ::"r"(n_compute * 32) : "memory");
    if (kss > 0) {
      part[0] = m_run[0];
      part[1] = m_run[1];
      part[2] = l_run[0];
      part[3] = l_run[1];
#pragma unroll
      for (int n = 0; n < 16; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) part[4 + n * 4 + e] = o[n][e];
    }
    asm volatile("bar.sync 1, %0;" ::"r"(n_compute * 32) : "memory");
    if (kss > 0) return;
#pragma unroll
    for (int k = 1; k < KS; ++k) {
      const float* q = reinterpret_cast<const float*>(smem) + (size_t)(((k * NWR + rg) * 32) + lane) * PER_THREAD;
      float cm[2], co[2];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const float mo = q[r];
        const float mn = fmaxf(m_run[r], mo);
        cm[r] = (m_run[r] == -INFINITY) ? 0.f : exp2f(m_run[r] - mn);
        co[r] = (mo == -INFINITY) ? 0.f : exp2f(mo - mn);
        l_run[r] = l_run[r] * cm[r] + q[2 + r] * co[r];
        m_run[r] = mn;
      }
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        o[n][0] = o[n][0] * cm[0] + q[4 + n * 4 + 0] * co[0];
        o[n][1] = o[n][1] * cm[0] + q[4 + n * 4 + 1] * co[0];
        o[n][2] = o[n][2] * cm[1] + q[4 + n * 4 + 2] * co[1];
        o[n][3] = o[n][3] * cm[1] + q[4 + n * 4 + 3] * co[1];
      }
    }
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    if (!row_valid[r]) continue;
    const size_t tok = (size_t)(q_begin + qi[r]);
    const size_t orow = tok * p.hq + qh[r];
    const float inv = l_run[r] > 0.f ? 1.f / l_run[r] : 0.f;
    if (p.num_splits > 1) {
      float* dst = p.o_part + ((size_t)split * p.T * p.hq + orow) * ATT_D;
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        const int col = n * 8 + tq * 2;
        *reinterpret_cast<float2*>(dst + col) = make_float2(o[n][r * 2] * inv, o[n][r * 2 + 1] * inv);
      }
      if (tq == 0) {
        // log2-domain LSE of this split (-inf when the split saw no key)
        p.lse_part[(size_t)split * p.T * p.hq + orow] = l_run[r] > 0.f ? m_run[r] + log2f(l_run[r]) : -INFINITY;
      }
    } else {
      __nv_bfloat16* dst = p.o + orow * ATT_D;
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        const int col = n * 8 + tq * 2;
        *reinterpret_cast<uint32_t*>(dst + col) = pack_bf16x2(o[n][r * 2] * inv, o[n][r * 2 + 1] * inv);
      }
    }
  }
  // Return the ring slots of any tile skipped after an error so the producer drains.
}

// Merge split partials: one warp per (token, head); 4 dims per lane.
__global__ void attention_combine_kernel(const float* __restrict__ o_part, const float* __restrict__ lse_part,
                                         __nv_bfloat16* __restrict__ o, int rows, int splits) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  pdl_wait();
  if (w >= rows) return;
  float m = -INFINITY;
  for (int s = 0; s < splits; ++s) m = fmaxf(m, lse_part[(size_t)s * rows + w]);
  float acc[4] = {0.f, 0.f, 0.f, 0.f}, tot = 0.f;
  if (m != -INFINITY) {
    for (int s = 0; s < splits; ++s) {
      const float l = lse_part[(size_t)s * rows + w];
      if (l == -INFINITY) continue;
      const float wgt = exp2f(l - m);
      tot += wgt;
      const float4 v = *reinterpret_cast<const float4*>(o_part + ((size_t)s * rows + w) * ATT_D + lane * 4);
      acc[0] += wgt * v.x;
      acc[1] += wgt * v.y;
      acc[2] += wgt * v.z;
      acc[3] += wgt * v.w;
    }
  }
  const float inv = tot > 0.f ? 1.f / tot : 0.f;
  uint2 out;
  out.x = pack_bf16x2(acc[0] * inv, acc[1] * inv);
  out.y = pack_bf16x2(acc[2] * inv, acc[3] * inv);
  *reinterpret_cast<uint2*>(o + (size_t)w * ATT_D + lane * 4) = out;
}

CUtensorMap make_tmap_bf16(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows);

template <int NWR, int KS>
static void launch_attn(dim3 grid, int smem, const CUtensorMap& tk, const CUtensorMap& tv, const AttnParams& p,
                        cudaStream_t stream) {
  static PerDeviceOnce smem_opt_in;
  smem_opt_in([smem] {
    C10_CUDA_CHECK(
        cudaFuncSetAttribute(paged_attention_kernel<NWR, KS>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  });
  launch_pdl(paged_attention_kernel<NWR, KS>, grid, dim3(32 * (NWR * KS + 1)), smem, stream, tk, tv, p);
}

void paged_attention_launch(const AttnLaunch& a, cudaStream_t stream) {
  TORCH_CHECK(a.head_dim == ATT_D, "paged attention supports head_dim 128");
  TORCH_CHECK(a.page % ATT_BK == 0, "page size must be a multiple of 64");
  const int64_t cache_rows = (int64_t)a.num_pages * a.hkv * a.page;
  CUtensorMap tk = make_tmap_bf16(a.k_cache, cache_rows, ATT_D, ATT_D, ATT_BK);
  CUtensorMap tv = make_tmap_bf16(a.v_cache, cache_rows, ATT_D, ATT_D, ATT_BK);
  AttnParams p{};
  p.q = a.q;
  p.o = a.o;
  p.o_part = a.o_part;
  p.lse_part = a.lse_part;
  p.block_tables = a.block_tables;
  p.bt_stride = a.bt_stride;
  p.prefix_lens = a.prefix_lens;
  p.suffix_mask = a.suffix_mask;
  p.cu_q = a.cu_q;
  p.cu_k = a.cu_k;
  p.Q = a.Q;
  p.hq = a.hq;
  p.hkv = a.hkv;
  p.group = a.hq / a.hkv;
  p.page = a.page;
  p.T = a.T;
  p.mode = a.mode;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.err = a.err;
  // rows per CTA: cover all (query, head) rows of a decode request when
  // possible (at most 8 compute warps = 128 rows); prefill uses 128-row blocks.
  int rows_needed = (a.mode == MODE_SUFFIX) ? a.Q * p.group : 128;
  // Row warps cover the (query, head) rows; small row sets split every 64-key
  // tile across KS warps as well so each SM keeps enough warps in flight.
  int nwr, ks;
  if (rows_needed <= 16) { nwr = 1; ks = 4; }
  else if (rows_needed <= 32) { nwr = 2; ks = 4; }
  else if (rows_needed <= 64) { nwr = 4; ks = 2; }
  else { nwr = 8; ks = 1; }
  p.rows_per_cta = nwr * 16;
  p.queries_per_cta = std::max(1, p.rows_per_cta / p.group);
  p.rows_per_cta = p.queries_per_cta * p.group;
  int qblocks = (a.mode == MODE_SUFFIX) ? (a.Q + p.queries_per_cta - 1) / p.queries_per_cta
                                        : (a.max_q + p.queries_per_cta - 1) / p.queries_per_cta;
  p.num_splits = std::max(1, a.num_splits);
  p.keys_per_split = a.keys_per_split;
  TORCH_CHECK(p.num_splits == 1 || (p.keys_per_split % ATT_BK == 0 && a.o_part && a.lse_part),
              "split attention needs 64-aligned splits and scratch");
  const int smem = 2 * ATT_STAGES * ATT_TILE_BYTES + 1024 + 128;
  dim3 grid(qblocks, a.B, a.hkv * p.num_splits);
  if (nwr == 1) launch_attn<1, 4>(grid, smem, tk, tv, p, stream);
  else if (nwr == 2) launch_attn<2, 4>(grid, smem, tk, tv, p, stream);
  else if (nwr == 4) launch_attn<4, 2>(grid, smem, tk, tv, p, stream);
  else launch_attn<8, 1>(grid, smem, tk, tv, p, stream);
  if (p.num_splits > 1) {
    const int rows = a.T * a.hq;
    launch_pdl(attention_combine_kernel, dim3((rows * 32 + 255) / 256), dim3(256), 0, stream, a.o_part,
               a.lse_part, a.o, rows, p.num_splits);
  }
}

}  // namespace uno
