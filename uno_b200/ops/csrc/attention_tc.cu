// Paged attention on the 5th-generation tensor cores (tcgen05 + TMEM), one
// persistent CTA per SM, for prefill, linear-block decode and tree verify.
//
// Visibility (one rule for every mode):
//   * MODE_SUFFIX (decode / tree): request b has prefix_lens[b] cached keys that
//     every query sees; query i also sees key prefix + j of its own forward iff
//     bit j of suffix_mask[b, i] is set (causal block or ancestor-or-self tree).
//   * MODE_CAUSAL (prefill): query i of a request with nq new and nk total keys
//     sees keys 0 .. nk - nq + i.
//
// Work decomposition.  A segment is (request b, 32-row block rb, kv head h):
// 32 rows = (query, GQA head) pairs sharing one K/V stream.  Its keys are cut
// into 128-key tiles.  All tiles of all segments form one list; CTA c takes the
// contiguous range [c*TT/G, (c+1)*TT/G) of it, so every SM streams the same
// number of K/V tiles whatever the request lengths (no host-side split plan,
// which a CUDA graph could not adapt).  A segment split across CTAs leaves one
// normalised partial (O, log2-sum-exp) per piece in scratch slot 2c or 2c+1;
// the last piece to finish (arrival counter per segment, reset after use)
// merges them into the output.
//
// Per tile, transposed so that the 128-key dimension is the MMA's M:
//   S^T[key, row] = K_tile[key, :] . Q[row, :]      (tcgen05, A = K, B = Q, K-major)
//   P^T = exp2(S^T * scale - m[row])                (4 softmax warps, 1 key per thread)
//   O^T[dim, row] += V_tile^T[dim, key] . P[row, key] (A = V MN-major, B = P K-major)
// Both accumulators live in TMEM.  The row max uses a lazy rescale: the running
// max moves only when a score exceeds it by more than 8 (log2 units), which a
// 128-thread bar.red.or detects in one barrier; the rare rescale multiplies the
// TMEM O columns in place.  Row sums stay per thread and are reduced once per
// piece with a 31-shuffle transpose-reduce.
//
// Warp roles (192 threads): warp 0 issues TMA (K/V tiles from the paged cache
// through the block table, 64-key boxes; Q rows through a 3-D map), warp 1
// allocates TMEM and issues tcgen05.mma from one lane, warps 2..5 run the
// softmax and the epilogue.  Every mbarrier wait is bounded; on expiry the
// kernel sets error bit 1, raises a CTA-wide abort flag and drains.
//
// Decode attention is bandwidth bound: the K/V ring holds three 64 KB tiles
// (K + V of 128 keys) so about 128 KB of HBM reads are in flight per SM.
//
// Reference behaviour: nano_vllm_uno/layers/attention.py (FlashAttention varlen
// prefill, paged block decode with a per-block causal mask, tree prefix + LSE
// merge); the math (softmax(QK^T * scale) V with these visibility rules) is the
// same, the decomposition is this file's own.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "uno_ops.h"

namespace uno {
namespace {

constexpr int TD = 128;                  // head dim
constexpr int TBK = 128;                 // keys per tile
constexpr int TR = 32;                   // rows (query, head) per segment
constexpr int TSTAGES = 3;
constexpr int REGION = TBK * 128;        // 128 keys x 64 dims (128 B rows): 16 KB
constexpr int KV_BYTES = 2 * REGION;     // one K or V tile (two 64-dim regions)
constexpr int STAGE_BYTES = 2 * KV_BYTES;
constexpr int QP_REGION = TR * 128;      // 32 rows x 64 dims (or 64 keys)
constexpr int QP_BYTES = 2 * QP_REGION;
constexpr int TMAX_B = 256;
constexpr int NTHREADS = 192;
constexpr int TMEM_COLS = 128;           // S[2] and O[2], TR columns each

constexpr int OFF_KV = 0;
constexpr int OFF_Q = OFF_KV + TSTAGES * STAGE_BYTES;
constexpr int OFF_P = OFF_Q + 2 * QP_BYTES;
constexpr int OFF_BAR = OFF_P + QP_BYTES;
constexpr int NUM_BARS = 2 * TSTAGES + 4 + 4 + 2 + 4;
constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;      // tmem base, abort, last flag
constexpr int OFF_RED = OFF_MISC + 16;                 // float [4][TR]
constexpr int OFF_FIN = OFF_RED + 4 * TR * 4;          // float [TR]
constexpr int OFF_MASK = OFF_FIN + TR * 4;             // int64 [TR]
constexpr int OFF_PREFIX = OFF_MASK + TR * 8;          // int [TMAX_B + 1]
constexpr int SMEM_USED = OFF_PREFIX + (TMAX_B + 1) * 4;
constexpr int SMEM_TOTAL = SMEM_USED + 1024;           // alignment slack
static_assert(SMEM_TOTAL <= 232448, "attention shared memory budget");

struct TcParams {
  const __nv_bfloat16* q;
  __nv_bfloat16* o;
  float* o_part;        // [2 * grid][TR][128] normalised partials
  float* lse_part;      // [2 * grid][TR] log2-sum-exp of each partial
  int* counters;        // [T * hkv] arrival counters (zero between launches)
  const int* block_tables;
  int bt_stride;
  const int* prefix_lens;
  const int64_t* suffix_mask;
  const int* cu_q;
  const int* cu_k;
  int B, Q, T, hq, hkv, group, page, mode, qpb;
  float scale_log2;
  int* err;
  unsigned long long* trace;  // optional timeline of CTA 0: [event][tile] globaltimer stamps
};

// Timeline probe (profiling aid, off unless a trace buffer is passed).
#define ATT_TRACE(ev, idx)                                                              \
  do {                                                                                  \
    if (p.trace != nullptr && blockIdx.x == 0 && (idx) < 64)                            \
      p.trace[(ev) * 64 + (idx)] = globaltimer_ns();                                    \
  } while (0)

enum : int { M_SUFFIX = 0, M_CAUSAL = 1 };

// ------------------------------------------------------------ request geometry
struct ReqGeo {
  int q_begin, nq, kv_len, prefix;
};

__device__ __forceinline__ ReqGeo req_geo(const TcParams& p, int b) {
  ReqGeo g;
  if (p.mode == M_SUFFIX) {
    g.prefix = p.prefix_lens[b];
    g.nq = p.Q;
    g.q_begin = b * p.Q;
    g.kv_len = g.prefix + p.Q;
  } else {
    g.q_begin = p.cu_q[b];
    g.nq = p.cu_q[b + 1] - g.q_begin;
    g.kv_len = p.cu_k[b + 1] - p.cu_k[b];
    g.prefix = g.kv_len - g.nq;
  }
  return g;
}

// keys a row block needs (causal: up to its last query's limit)
__device__ __forceinline__ int rb_keys(const TcParams& p, const ReqGeo& g, int rb) {
  if (p.mode == M_SUFFIX) return g.kv_len;
  const int last_q = min(g.nq, (rb + 1) * p.qpb);
  return min(g.kv_len, g.prefix + last_q);
}

__device__ __forceinline__ int num_rb(const TcParams& p, const ReqGeo& g) { return (g.nq + p.qpb - 1) / p.qpb; }

__device__ __forceinline__ int cdiv(int a, int b) { return (a + b - 1) / b; }

// A piece: tiles [t0, t1) of segment (b, rb, h), which has nt tiles.
struct Piece {
  int b, rb, h, t0, t1, nt;
  long long x0;  // global index of tile t0
};

// Walks the tile list of one CTA; every warp role runs an identical walker.
struct Walker {
  long long x, end;
  int b, rb, h, t, nt;
  ReqGeo g;
  int nrb;

  __device__ __forceinline__ void load_rb(const TcParams& p) { nt = cdiv(rb_keys(p, g, rb), TBK); }

  __device__ void init(const TcParams& p, const int* prefix, long long x_begin, long long x_end) {
    x = x_begin;
    end = x_end;
    if (x >= end) return;
    // request: last b with prefix[b] <= x
    int lo = 0, hi = p.B - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (prefix[mid] <= x) lo = mid;
      else hi = mid - 1;
    }
    b = lo;
    g = req_geo(p, b);
    nrb = num_rb(p, g);
    long long off = x - prefix[b];
    rb = 0;
    load_rb(p);
    while (off >= (long long)nt * p.hkv) {
      off -= (long long)nt * p.hkv;
      ++rb;
      load_rb(p);
    }
    h = (int)(off / nt);
    t = (int)(off % nt);
  }

  __device__ __forceinline__ bool done() const { return x >= end; }

  __device__ Piece next(const TcParams& p, const int* prefix) {
    Piece pc;
    pc.b = b;
    pc.rb = rb;
    pc.h = h;
    pc.t0 = t;
    pc.nt = nt;
    pc.x0 = x;
    const long long avail = end - x;
    pc.t1 = (int)min((long long)nt, (long long)t + avail);
    x += pc.t1 - t;
    // advance to the next segment
    t = 0;
    if (++h == p.hkv) {
      h = 0;
      if (++rb == nrb) {
        rb = 0;
        do {
          ++b;
        } while (b < p.B && prefix[b + 1] == prefix[b]);
        if (b < p.B) {
          g = req_geo(p, b);
          nrb = num_rb(p, g);
        }
      }
      if (b < p.B) load_rb(p);
    }
    return pc;
  }
};

__device__ __forceinline__ long long range_begin(long long c, long long TT, long long G) { return c * TT / G; }

// CTA that owns global tile x
__device__ __forceinline__ int tile_owner(long long x, long long TT, int G) {
  int c = (int)min((long long)G - 1, x * G / max(TT, 1LL));
  while (c + 1 < G && range_begin(c + 1, TT, G) <= x) ++c;
  while (c > 0 && range_begin(c, TT, G) > x) --c;
  return c;
}

// ------------------------------------------------------------------ helpers
// Bounded wait that also gives up when another role raised the abort flag.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err) {
  if (*abort_flag) return false;
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = globaltimer_ns();
  while (true) {
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - start > kWaitLimitNs) {
      set_error(err, 1);
      *abort_flag = 1;
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                            int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float* v) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const float* v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
               "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
               "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
               "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7]))
               : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ bool bar_red_or(int id, int nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.or.pred p, %2, %3, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void bar_named(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// After the call, lane l holds the sum (or max) over the warp of v[l].
template <bool MAX>
__device__ __forceinline__ float transpose_reduce32(float (&v)[TR], int lane) {
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) {
    const bool upper = (lane & s) != 0;
#pragma unroll
    for (int i = 0; i < s; ++i) {
      const float send = upper ? v[i] : v[i + s];
      const float keep = upper ? v[i + s] : v[i];
      const float got = __shfl_xor_sync(0xffffffff, send, s);
      v[i] = MAX ? fmaxf(keep, got) : keep + got;
    }
  }
  return v[0];
}

// MN-major (V^T) operand: 64-dim groups REGION bytes apart, 8-key groups 1024 B apart.
__device__ __forceinline__ uint64_t desc_v_mn(const void* smem) {
  uint64_t addr = smem_u32(smem);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3FFFull;
  d |= (uint64_t)(REGION >> 4) << 16;
  d |= (1024ull >> 4) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;
  return d;
}

// ------------------------------------------------------------------ kernel
__global__ void __launch_bounds__(NTHREADS, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                        const __grid_constant__ CUtensorMap tmQ, TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sKV = smem + OFF_KV;
  uint8_t* sQ = smem + OFF_Q;
  uint8_t* sP = smem + OFF_P;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* kv_full = bars;
  uint64_t* kv_empty = bars + TSTAGES;
  uint64_t* q_full = bars + 2 * TSTAGES;
  uint64_t* q_empty = q_full + 2;
  uint64_t* s_full = q_empty + 2;
  uint64_t* s_empty = s_full + 2;
  uint64_t* p_full = s_empty + 2;
  uint64_t* p_empty = p_full + 1;
  uint64_t* o_full = p_empty + 1;
  uint64_t* o_empty = o_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 4);
  volatile int* last_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 8);
  float* red = reinterpret_cast<float*>(smem + OFF_RED);
  float* fin = reinterpret_cast<float*>(smem + OFF_FIN);
  int64_t* rmask = reinterpret_cast<int64_t*>(smem + OFF_MASK);
  int* prefix = reinterpret_cast<int*>(smem + OFF_PREFIX);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // ---- tile counts per request and their prefix sums
  for (int b = threadIdx.x; b < p.B; b += NTHREADS) {
    const ReqGeo g = req_geo(p, b);
    int tiles = 0;
    const int nrb = num_rb(p, g);
    if (p.mode == M_SUFFIX) {
      tiles = nrb * cdiv(g.kv_len, TBK);
    } else {
      for (int rb = 0; rb < nrb; ++rb) tiles += cdiv(rb_keys(p, g, rb), TBK);
    }
    prefix[b + 1] = tiles * p.hkv;
  }
  if (threadIdx.x == 0) {
    prefix[0] = 0;
    *abort_flag = 0;
    for (int s = 0; s < TSTAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 4);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 4);
    }
    mbar_init(p_full, 4);
    mbar_init(p_empty, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int b = 0; b < p.B; ++b) prefix[b + 1] += prefix[b];
  }
  if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const long long TT = prefix[p.B];
  // at least one tile per CTA, so every CTA between two owners of a segment holds a piece of it
  const int G = (int)min((long long)gridDim.x, max(TT, 1LL));
  const bool active = (int)blockIdx.x < G;
  if (threadIdx.x == 0) ATT_TRACE(9, 0);
  const long long x_begin = active ? range_begin(blockIdx.x, TT, G) : 0;
  const long long x_end = active ? range_begin(blockIdx.x + 1, TT, G) : 0;

  if (warp == 0) {
    // ================================================================ TMA producer
    if (lane == 0 && x_begin < x_end) {
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmQ);
      Walker w;
      w.init(p, prefix, x_begin, x_end);
      int stage = 0;
      uint32_t phase = 0;
      int qn = 0;
      int pt = 0;
      uint32_t issued = 0, issued_phase = 0;  // bit s: stage s has a load in flight / its phase
      bool ok = true;
      while (ok && !w.done()) {
        const Piece pc = w.next(p, prefix);
        const ReqGeo g = req_geo(p, pc.b);
        // Q rows of this segment: queries i0.., heads h*group..
        const int qb = qn & 1;
        if (!wait_or_abort(&q_empty[qb], ((qn >> 1) & 1) ^ 1, abort_flag, p.err)) { ok = false; break; }
        mbar_arrive_expect_tx(&q_full[qb], QP_BYTES);
        const int z = g.q_begin + pc.rb * p.qpb;
        tma_load_3d(sQ + qb * QP_BYTES, &tmQ, &q_full[qb], 0, pc.h * p.group, z);
        tma_load_3d(sQ + qb * QP_BYTES + QP_REGION, &tmQ, &q_full[qb], 64, pc.h * p.group, z);
        ++qn;
        const int* bt = p.block_tables + (size_t)pc.b * p.bt_stride;
        for (int t = pc.t0; t < pc.t1; ++t) {
          if (!wait_or_abort(&kv_empty[stage], phase ^ 1, abort_flag, p.err)) { ok = false; break; }
          ATT_TRACE(0, pt);
          const int k0 = t * TBK;
          int rows[2];
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            int k = k0 + hh * 64;
            if (k >= g.kv_len) k = k0;  // keys past the end: reload a valid box (masked later)
            const int page_id = bt[k / p.page];
            rows[hh] = (page_id * p.hkv + pc.h) * p.page + (k % p.page);
          }
          uint8_t* sk = sKV + stage * STAGE_BYTES;
          uint8_t* sv = sk + KV_BYTES;
          mbar_arrive_expect_tx(&kv_full[stage], STAGE_BYTES);
#pragma unroll
          for (int dh = 0; dh < 2; ++dh)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              tma_load_2d(sk + dh * REGION + hh * (REGION / 2), &tmK, &kv_full[stage], dh * 64, rows[hh]);
              tma_load_2d(sv + dh * REGION + hh * (REGION / 2), &tmV, &kv_full[stage], dh * 64, rows[hh]);
            }
          ATT_TRACE(1, pt);
          ++pt;
          issued |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == TSTAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) {  // let copies in flight land before the CTA exits
        for (int s = 0; s < TSTAGES; ++s)
          if ((issued >> s) & 1) mbar_wait(&kv_full[s], (issued_phase >> s) & 1, nullptr);
      }
    }
  } else if (warp == 1) {
    // ================================================================ MMA issuer
    if (lane == 0 && x_begin < x_end) {
      constexpr uint32_t idesc_s = idesc_bf16(128, TR);
      constexpr uint32_t idesc_o = idesc_bf16(128, TR) | (1u << 15);  // A (V^T) MN-major
      Walker w;
      w.init(p, prefix, x_begin, x_end);
      int stage = 0;
      uint32_t phase = 0;
      int qn = 0, pn = 0, tn = 0;  // pieces, P buffers used, tiles
      bool ok = true;
      while (ok && !w.done()) {
        const Piece pc = w.next(p, prefix);
        const int qb = qn & 1, ob = qn & 1;
        if (!wait_or_abort(&q_full[qb], (qn >> 1) & 1, abort_flag, p.err)) { ok = false; break; }
        tc_fence_after();
        const uint64_t qdesc = smem_desc_sw128(sQ + qb * QP_BYTES);
        const uint32_t o_tm = tmem + 2 * TR + ob * TR;
        int prev_stage = -1;
        for (int t = pc.t0; t <= pc.t1 && ok; ++t) {
          if (t < pc.t1) {
            // S^T(t) = K_t . Q^T into S buffer tn % 2
            const int sb = tn & 1;
            if (!wait_or_abort(&kv_full[stage], phase, abort_flag, p.err)) { ok = false; break; }
            if (!wait_or_abort(&s_empty[sb], ((tn >> 1) & 1) ^ 1, abort_flag, p.err)) { ok = false; break; }
            ATT_TRACE(2, tn);
            tc_fence_after();
            const uint64_t kdesc = smem_desc_sw128(sKV + stage * STAGE_BYTES);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const uint64_t off_a = (uint64_t)((k >> 2) * (REGION >> 4) + (k & 3) * 2);
              const uint64_t off_b = (uint64_t)((k >> 2) * (QP_REGION >> 4) + (k & 3) * 2);
              tc_mma_bf16(tmem + sb * TR, kdesc + off_a, qdesc + off_b, idesc_s, k > 0);
            }
            tc_commit(&s_full[sb]);
            if (t + 1 == pc.t1) tc_commit(&q_empty[qb]);
            ++tn;
          }
          if (t > pc.t0) {
            // O^T += V_{t-1}^T . P^T(t-1)
            const int st = prev_stage;
            if (!wait_or_abort(p_full, pn & 1, abort_flag, p.err)) { ok = false; break; }
            ATT_TRACE(3, pn);
            if (t - 1 == pc.t0) {
              if (!wait_or_abort(&o_empty[ob], ((qn >> 1) & 1) ^ 1, abort_flag, p.err)) { ok = false; break; }
            }
            tc_fence_after();
            const uint64_t vdesc = desc_v_mn(sKV + st * STAGE_BYTES + KV_BYTES);
            const uint64_t pdesc = smem_desc_sw128(sP);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const uint64_t off_a = (uint64_t)(k * (2048 >> 4));  // 16 keys = 2 KB
              const uint64_t off_b = (uint64_t)((k >> 2) * (QP_REGION >> 4) + (k & 3) * 2);
              tc_mma_bf16(o_tm, vdesc + off_a, pdesc + off_b, idesc_o, (t - 1 > pc.t0) || k > 0);
            }
            tc_commit(&kv_empty[st]);
            tc_commit(p_empty);
            ATT_TRACE(4, pn);
            ++pn;
          }
          if (t < pc.t1) {
            prev_stage = stage;
            if (++stage == TSTAGES) { stage = 0; phase ^= 1; }
          }
        }
        if (!ok) break;
        tc_commit(&o_full[ob]);
        ++qn;
      }
      // drain: wait for every MMA this thread issued before TMEM is released
      tc_commit(p_empty);
      mbar_wait(p_empty, pn & 1, nullptr);
    }
  } else {
    // ================================================================ softmax + epilogue
    const int quarter = warp & 3;
    const int key = quarter * 32 + lane;        // this thread's key within a tile / dim of O
    const int sidx = (warp - 2) * 32 + lane;    // 0..127 within the softmax group
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    if (x_begin < x_end) {
      Walker w;
      w.init(p, prefix, x_begin, x_end);
      int qn = 0, tn = 0, pn = 0;
      while (!w.done()) {
        const Piece pc = w.next(p, prefix);
        const ReqGeo g = req_geo(p, pc.b);
        const int i0 = pc.rb * p.qpb;
        const int ob = qn & 1;
        // rows valid in this segment (query < nq)
        uint32_t valid = 0;
#pragma unroll
        for (int r = 0; r < TR; ++r)
          if (i0 + r / p.group < g.nq) valid |= 1u << r;
        if (p.mode == M_SUFFIX && sidx < TR) {
          const int i = i0 + sidx / p.group;
          rmask[sidx] = (i < g.nq) ? p.suffix_mask[(size_t)pc.b * p.Q + i] : 0;
        }
        bar_named(2, 128);
        float m_run[TR], l_run[TR];
#pragma unroll
        for (int r = 0; r < TR; ++r) {
          m_run[r] = -INFINITY;
          l_run[r] = 0.f;
        }
        for (int t = pc.t0; t < pc.t1; ++t) {
          const int sb = tn & 1;
          const int k0 = t * TBK;
          const int kg = k0 + key;
          wait_or_abort(&s_full[sb], (tn >> 1) & 1, abort_flag, p.err);
          if (sidx == 0) ATT_TRACE(5, tn);
          tc_fence_after();
          float s[TR];
          tmem_ld32(lane_base + sb * TR, s);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s_empty[sb]);
          ++tn;
          // ---- visibility + scale
          bool full_tile;
          if (p.mode == M_SUFFIX) full_tile = (k0 + TBK <= g.prefix);
          else full_tile = (k0 + TBK - 1 <= g.prefix + i0);
          if (full_tile) {
#pragma unroll
            for (int r = 0; r < TR; ++r) s[r] = ((valid >> r) & 1) ? s[r] * p.scale_log2 : -INFINITY;
          } else {
#pragma unroll
            for (int r = 0; r < TR; ++r) {
              bool vis = (valid >> r) & 1;
              if (p.mode == M_SUFFIX) {
                const int j = kg - g.prefix;
                vis = vis && kg < g.kv_len && (j < 0 || ((rmask[r] >> j) & 1));
              } else {
                vis = vis && kg <= g.prefix + i0 + r / p.group;
              }
              s[r] = vis ? s[r] * p.scale_log2 : -INFINITY;
            }
          }
          bool exceed = false;
#pragma unroll
          for (int r = 0; r < TR; ++r) exceed |= ((valid >> r) & 1) && (s[r] > m_run[r] + 8.f);
          exceed = bar_red_or(1, 128, exceed);
          // P buffer free (the previous P . V finished)
          if (sidx == 0) ATT_TRACE(6, pn);
          wait_or_abort(p_empty, (pn & 1) ^ 1, abort_flag, p.err);
          if (sidx == 0) ATT_TRACE(7, pn);
          ++pn;
          if (exceed) {
            float mx[TR];
#pragma unroll
            for (int r = 0; r < TR; ++r) mx[r] = s[r];
            const float wm = transpose_reduce32<true>(mx, lane);
            red[(warp - 2) * TR + lane] = wm;
            bar_named(2, 128);
            // mx[] now holds each row's correction factor
            bool any_corr = false;
#pragma unroll
            for (int r = 0; r < TR; ++r) {
              const float tm = fmaxf(fmaxf(red[r], red[TR + r]), fmaxf(red[2 * TR + r], red[3 * TR + r]));
              const float mn = (tm > m_run[r] + 8.f) ? tm : m_run[r];
              mx[r] = (m_run[r] == -INFINITY) ? 0.f : ex2(m_run[r] - mn);
              any_corr |= (mn != m_run[r]) && (m_run[r] != -INFINITY);
              m_run[r] = mn;
              l_run[r] *= mx[r];
            }
            if (t > pc.t0 && any_corr) {
              tc_fence_after();
              const uint32_t oaddr = lane_base + 2 * TR + ob * TR;
#pragma unroll
              for (int c = 0; c < TR; c += 8) {
                float ov[8];
                tmem_ld8(oaddr + c, ov);
#pragma unroll
                for (int r = 0; r < 8; ++r) ov[r] *= mx[c + r];
                tmem_st8(oaddr + c, ov);
              }
            }
          }
          // ---- P = exp2(S - m), row sums, P^T into shared memory (K-major, 128-byte swizzle)
          uint8_t* prow = sP + (key >> 6) * QP_REGION;
          const int kc = (key & 63) >> 3, kb = (key & 7) * 2;
#pragma unroll
          for (int r = 0; r < TR; ++r) {
            const float m = (m_run[r] == -INFINITY) ? 0.f : m_run[r];
            const float pv = ex2(s[r] - m);
            l_run[r] += pv;
            *reinterpret_cast<__nv_bfloat16*>(prow + r * 128 + ((kc ^ (r & 7)) << 4) + kb) = __float2bfloat16(pv);
          }
          fence_async_smem();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(p_full);
          if (sidx == 0) ATT_TRACE(8, pn - 1);
        }
        // ---- end of piece: O^T from TMEM, row sums, output or partial
        wait_or_abort(&o_full[ob], (qn >> 1) & 1, abort_flag, p.err);
        tc_fence_after();
        float ov[TR];
        tmem_ld32(lane_base + 2 * TR + ob * TR, ov);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&o_empty[ob]);
        ++qn;
        bar_named(2, 128);  // every thread is done reading red[] of the last rescale
        {
          const float ws = transpose_reduce32<false>(l_run, lane);
          red[(warp - 2) * TR + lane] = ws;
        }
        bar_named(2, 128);
        if (sidx < TR) fin[sidx] = red[sidx] + red[TR + sidx] + red[2 * TR + sidx] + red[3 * TR + sidx];
        bar_named(2, 128);
        const bool complete = (pc.t0 == 0 && pc.t1 == pc.nt);
        const bool aborted = *abort_flag != 0;
        if (complete) {
          if (!aborted) {
#pragma unroll
            for (int r = 0; r < TR; ++r) {
              if (!((valid >> r) & 1)) continue;
              const float l = fin[r];
              const float inv = l > 0.f ? 1.f / l : 0.f;
              const size_t row = (size_t)(g.q_begin + i0 + r / p.group) * p.hq + pc.h * p.group + r % p.group;
              p.o[row * TD + key] = __float2bfloat16(ov[r] * inv);
            }
          }
        } else {
          const int slot = 2 * blockIdx.x + (pc.x0 == x_begin ? 0 : 1);
          float* dst = p.o_part + (size_t)slot * TR * TD;
#pragma unroll
          for (int r = 0; r < TR; ++r) {
            const float l = fin[r];
            const float inv = l > 0.f ? 1.f / l : 0.f;
            dst[r * TD + key] = ov[r] * inv;
          }
          {
            float mr = 0.f;  // m_run[sidx] without a dynamic register index
#pragma unroll
            for (int r = 0; r < TR; ++r)
              if (r == sidx) mr = m_run[r];
            if (sidx < TR) {
              const float l = fin[sidx];
              p.lse_part[(size_t)slot * TR + sidx] = l > 0.f ? mr + __log2f(l) : -INFINITY;
            }
          }
          __threadfence();
          bar_named(2, 128);
          // segment's first global tile and its pieces' owners
          const long long seg_x0 = pc.x0 - pc.t0;
          const int c_first = tile_owner(seg_x0, TT, G);
          const int c_last = tile_owner(seg_x0 + pc.nt - 1, TT, G);
          const int n_pieces = c_last - c_first + 1;
          const size_t cidx = (size_t)(g.q_begin + i0) * p.hkv + pc.h;
          if (sidx == 0) {
            int last = 0;
            if (!aborted) last = (atomicAdd(p.counters + cidx, 1) == n_pieces - 1);
            *last_flag = last;
          }
          bar_named(2, 128);
          if (*last_flag) {
            __threadfence();
            for (int r = 0; r < TR; ++r) {
              if (!((valid >> r) & 1)) continue;
              float m = -INFINITY;
              for (int c = c_first; c <= c_last; ++c) {
                const int sl = 2 * c + (range_begin(c, TT, G) >= seg_x0 ? 0 : 1);
                m = fmaxf(m, __ldcg(p.lse_part + (size_t)sl * TR + r));
              }
              float acc = 0.f, tot = 0.f;
              if (m != -INFINITY) {
                for (int c = c_first; c <= c_last; ++c) {
                  const int sl = 2 * c + (range_begin(c, TT, G) >= seg_x0 ? 0 : 1);
                  const float lse = __ldcg(p.lse_part + (size_t)sl * TR + r);
                  if (lse == -INFINITY) continue;
                  const float wgt = ex2(lse - m);
                  tot += wgt;
                  acc += wgt * __ldcg(p.o_part + ((size_t)sl * TR + r) * TD + key);
                }
              }
              const size_t row = (size_t)(g.q_begin + i0 + r / p.group) * p.hq + pc.h * p.group + r % p.group;
              p.o[row * TD + key] = __float2bfloat16(tot > 0.f ? acc / tot : 0.f);
            }
            if (sidx == 0) p.counters[cidx] = 0;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace

CUtensorMap make_tmap_bf16(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows);
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();
int num_sms();

// Q viewed as [T][hq][128]: box = 64 dims x group heads x qpb queries.
static CUtensorMap make_q_map(const void* q, int T, int hq, int group, int qpb) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(q) % 16 == 0, "q must be 16-byte aligned");
  CUtensorMap m;
  cuuint64_t dims[3] = {(cuuint64_t)TD, (cuuint64_t)hq, (cuuint64_t)T};
  cuuint64_t strides[2] = {(cuuint64_t)TD * 2, (cuuint64_t)hq * TD * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)group, (cuuint32_t)qpb};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = tensor_map_encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(q), dims, strides, box,
                                    estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (q) failed: ", (int)r);
  return m;
}

int attention_tc_rows() { return TR; }

void attention_tc_launch(const AttnLaunch& a, int* counters, cudaStream_t stream, unsigned long long* trace) {
  TORCH_CHECK(a.head_dim == TD, "tcgen05 attention supports head_dim 128");
  TORCH_CHECK(a.page % 64 == 0, "page size must be a multiple of 64");
  const int group = a.hq / a.hkv;
  TORCH_CHECK(group >= 1 && group <= TR && TR % group == 0 && a.hq == group * a.hkv,
              "GQA group must divide ", TR);
  TORCH_CHECK(a.B <= TMAX_B, "at most ", TMAX_B, " requests per attention call");
  TORCH_CHECK(a.o_part && a.lse_part && counters, "attention scratch missing");
  const int64_t cache_rows = (int64_t)a.num_pages * a.hkv * a.page;
  CUtensorMap tk = make_tmap_bf16(a.k_cache, cache_rows, TD, TD, 64);
  CUtensorMap tv = make_tmap_bf16(a.v_cache, cache_rows, TD, TD, 64);
  const int qpb = TR / group;
  CUtensorMap tq = make_q_map(a.q, a.T, a.hq, group, qpb);
  TcParams p{};
  p.q = a.q;
  p.o = a.o;
  p.o_part = a.o_part;
  p.lse_part = a.lse_part;
  p.counters = counters;
  p.block_tables = a.block_tables;
  p.bt_stride = a.bt_stride;
  p.prefix_lens = a.prefix_lens;
  p.suffix_mask = a.suffix_mask;
  p.cu_q = a.cu_q;
  p.cu_k = a.cu_k;
  p.B = a.B;
  p.Q = a.Q;
  p.T = a.T;
  p.hq = a.hq;
  p.hkv = a.hkv;
  p.group = group;
  p.page = a.page;
  p.mode = a.mode;
  p.qpb = qpb;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.err = a.err;
  p.trace = trace;
  static PerDeviceOnce smem_opt_in;
  smem_opt_in([] {
    C10_CUDA_CHECK(
        cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_TOTAL));
  });
  attention_tc_kernel<<<num_sms(), NTHREADS, SMEM_TOTAL, stream>>>(tk, tv, tq, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace uno
