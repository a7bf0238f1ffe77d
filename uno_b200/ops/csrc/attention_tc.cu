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
//   P^T = exp2(S^T * scale - m[row])                (softmax warps, 1 key per thread)
//   O^T[dim, row] += V_tile^T[dim, key] . P[row, key] (A = V MN-major, B = P K-major)
// Both accumulators live in TMEM.  The row max uses a lazy rescale: the running
// max moves only when a score exceeds it by more than 8 (log2 units), which a
// 128-thread bar.red.or detects in one barrier; the rare rescale multiplies the
// TMEM O columns in place.  Row sums stay per thread and are reduced once per
// piece with warp shuffles.
//
// Warp roles (480 threads):
//   warp 0      TMA producer (one lane): Q rows of each piece through a 3-D map,
//               with the piece's geometry and suffix masks published next to
//               them; K and V tiles from the paged cache through the block table
//               (64-key boxes) on separate rings, polled without blocking so
//               that V loads keep flowing while a Q buffer is still in use;
//   warp 1      allocates TMEM and issues S = K.Q^T (one lane);
//   warps 2..9  softmax: two warps per TMEM lane quarter, 16 rows each;
//   warps 10..13 epilogue: O^T from TMEM, normalisation, output or partial
//               writes and the merge of split segments;
//   warp 14     issues O^T += V^T.P^T (one lane).
// Every mbarrier wait is bounded; on expiry the kernel sets error bit 1, raises
// a CTA-wide abort flag and drains its copies and MMAs before freeing TMEM.
//
// Shared memory: K ring 2 x 32 KB, V ring 3 x 32 KB, Q and P double buffers of
// 8 KB each, plus the epilogue staging of O^T (16 KB).
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
constexpr int KSTAGES = 2;               // K tiles in flight (freed when S = K.Q^T completes)
constexpr int VSTAGES = 3;               // V tiles in flight (freed when O += V^T.P completes)
constexpr int REGION = TBK * 128;        // 128 keys x 64 dims (128 B rows): 16 KB
constexpr int KV_BYTES = 2 * REGION;     // one K or V tile (two 64-dim regions)
constexpr int QP_REGION = TR * 128;      // 32 rows x 64 dims (Q) or 32 rows x 64 keys (P)
constexpr int QP_BYTES = 2 * QP_REGION;
constexpr int TMAX_B = 256;
constexpr int HR = TR / 2;               // rows per softmax warp (two warps share a TMEM lane quarter)
constexpr int NTHREADS = 480;            // producer, S issuer, 8 softmax, 4 epilogue warps, P.V issuer
constexpr int TMEM_COLS = 128;           // S[2] and O[2], TR columns each

constexpr int OFF_K = 0;
constexpr int OFF_V = OFF_K + KSTAGES * KV_BYTES;
constexpr int OFF_Q = OFF_V + VSTAGES * KV_BYTES;
constexpr int OFF_P = OFF_Q + 2 * QP_BYTES;
constexpr int OFF_BAR = OFF_P + 2 * QP_BYTES;
constexpr int NUM_BARS = 2 * KSTAGES + 2 * VSTAGES + 7 * 4 + 2;
constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;       // tmem base, abort, last flag
constexpr int OFF_RED = OFF_MISC + 16;                 // float [8 warps][HR] per-warp row maxima / sums
constexpr int OFF_MSM = OFF_RED + 8 * HR * 4;          // float [TR] running row maxima
constexpr int OFF_CSM = OFF_MSM + TR * 4;              // float [TR] last correction factors
constexpr int OFF_LFIN = OFF_CSM + TR * 4;             // float [2][TR] row sums per O buffer
constexpr int OFF_MFIN = OFF_LFIN + 2 * TR * 4;        // float [2][TR] row maxima per O buffer
constexpr int OFF_COL = OFF_MFIN + 2 * TR * 4;         // u32 [2 buffers][64] rows (bit r) that see suffix key j
constexpr int OFF_SMASK = OFF_COL + 2 * 64 * 4;        // int64 [2][TR] suffix masks of a piece's queries
constexpr int OFF_TROWS = OFF_SMASK + 2 * TR * 8;      // int2 [8] cache rows of queued tiles (K -> V)
constexpr int OFF_META = OFF_TROWS + 8 * 8;            // PieceMeta [2] (with the Q double buffer)
constexpr int OFF_CMB = OFF_META + 2 * 64;             // float [2][TR] merge maxima / inverse sums
constexpr int OFF_OST = OFF_CMB + 2 * TR * 4;          // float [TR][TD] epilogue staging of O^T (own column)
constexpr int OFF_PREFIX = OFF_OST + TR * TD * 4;      // int [TMAX_B + 1]
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
  int group_shift;  // log2(group): rows are (query << group_shift) | head-in-group
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

// Piece geometry that the producer publishes with the piece's Q tile.
struct PieceMeta {
  int b, rb, h, t0, t1, nt, q_begin, nq, kv_len, prefix;
  uint32_t valid[2];  // rows of each 16-row half whose query exists
};

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
__device__ __noinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err) {
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

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
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
  uint8_t* sK = smem + OFF_K;
  uint8_t* sV = smem + OFF_V;
  uint8_t* sQ = smem + OFF_Q;
  uint8_t* sP = smem + OFF_P;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* k_full = bars;
  uint64_t* k_empty = k_full + KSTAGES;
  uint64_t* v_full = k_empty + KSTAGES;
  uint64_t* v_empty = v_full + VSTAGES;
  uint64_t* q_full = v_empty + VSTAGES;
  uint64_t* q_empty = q_full + 2;
  uint64_t* s_full = q_empty + 2;
  uint64_t* s_empty = s_full + 2;
  uint64_t* p_full = s_empty + 2;
  uint64_t* p_empty = p_full + 2;
  uint64_t* o_full = p_empty + 2;
  uint64_t* o_empty = o_full + 2;
  uint64_t* l_full = o_empty + 2;
  uint64_t* drain_bar = l_full + 2;  // [0] S issuer, [1] P.V issuer: final commit before TMEM is freed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 4);
  volatile int* last_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 8);
  float* red = reinterpret_cast<float*>(smem + OFF_RED);
  float* lfin = reinterpret_cast<float*>(smem + OFF_LFIN);
  float* mfin = reinterpret_cast<float*>(smem + OFF_MFIN);
  uint32_t* colmask = reinterpret_cast<uint32_t*>(smem + OFF_COL);
  int64_t* smask_sm = reinterpret_cast<int64_t*>(smem + OFF_SMASK);
  int2* trows = reinterpret_cast<int2*>(smem + OFF_TROWS);
  float* cmb = reinterpret_cast<float*>(smem + OFF_CMB);
  float* msm = reinterpret_cast<float*>(smem + OFF_MSM);  // running row maxima (softmax)
  float* csm = reinterpret_cast<float*>(smem + OFF_CSM);  // their last correction factors
  PieceMeta* meta = reinterpret_cast<PieceMeta*>(smem + OFF_META);
  float* ostage = reinterpret_cast<float*>(smem + OFF_OST);
  int* prefix = reinterpret_cast<int*>(smem + OFF_PREFIX);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0 && p.trace != nullptr) p.trace[1024 + 4 * blockIdx.x] = globaltimer_ns();

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
    for (int s = 0; s < KSTAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < VSTAGES; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 3);  // S issuer (commit after the piece's last S), P.V issuer, softmax
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 8);
      mbar_init(&p_full[i], 8);
      mbar_init(&p_empty[i], 1);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 4);
      mbar_init(&l_full[i], 2);
      mbar_init(&drain_bar[i], 1);
    }
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
  if (threadIdx.x == 0 && p.trace != nullptr) p.trace[1024 + 4 * blockIdx.x + 1] = globaltimer_ns();
  const long long x_begin = active ? range_begin(blockIdx.x, TT, G) : 0;
  const long long x_end = active ? range_begin(blockIdx.x + 1, TT, G) : 0;

  if (warp == 0) {
    // ================================================================ TMA producer
    if (lane == 0 && x_begin < x_end) {
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmQ);
      // K loads run ahead of V loads: the K cursor walks the pieces (loading Q and the
      // piece metadata first) and queues each tile's cache rows; the V cursor follows.
      Walker w;
      w.init(p, prefix, x_begin, x_end);
      const long long n_tiles = x_end - x_begin;
      int kn = 0, vn = 0, qn = 0;
      int t_cur = 0, t_end = 0, cur_h = 0, cur_len = 0;  // K cursor inside the current piece
      Piece nx{};
      bool have_next = false;
      const int* bt = nullptr;
      uint32_t kin = 0, vin = 0;  // bit s: a load into stage s may still be in flight
      uint64_t idle_since = 0;
      bool ok = true;
      while (ok && vn < n_tiles) {
        bool progressed = false;  // set by any of the three sides below
        // ---- K side: next tile (and the piece's Q tile when a piece starts)
        if (kn < n_tiles && kn - vn < 8 && t_cur == t_end) {
          // start the next piece once its Q buffer is free (never block: V loads must keep flowing)
          if (!have_next) {
            nx = w.next(p, prefix);
            have_next = true;
          }
          const int qb = qn & 1;
          if (mbar_try_wait(&q_empty[qb], ((qn >> 1) & 1) ^ 1)) {
            const Piece pc = nx;
            have_next = false;
            const ReqGeo g = req_geo(p, pc.b);
            const int i0 = pc.rb * p.qpb;
            const int nrows = min(TR, (g.nq - i0) << p.group_shift);
            const uint32_t valid = nrows >= 32 ? ~0u : ((1u << nrows) - 1);
            if (p.mode == M_SUFFIX) {  // suffix masks of this piece's queries (0 past the request's last)
              const int64_t* src = p.suffix_mask + (size_t)pc.b * p.Q;
#pragma unroll 8
              for (int qi = 0; qi < p.qpb; ++qi) smask_sm[qb * TR + qi] = (i0 + qi < g.nq) ? src[i0 + qi] : 0;
            }
            meta[qb] = PieceMeta{pc.b, pc.rb, pc.h, pc.t0, pc.t1, pc.nt, g.q_begin, g.nq, g.kv_len, g.prefix,
                                 {valid & 0xFFFFu, valid >> 16}};
            mbar_arrive_expect_tx(&q_full[qb], QP_BYTES);  // releases the masks with the Q tile
            const int z = g.q_begin + pc.rb * p.qpb;
            tma_load_3d(sQ + qb * QP_BYTES, &tmQ, &q_full[qb], 0, pc.h * p.group, z);
            tma_load_3d(sQ + qb * QP_BYTES + QP_REGION, &tmQ, &q_full[qb], 64, pc.h * p.group, z);
            ++qn;
            t_cur = pc.t0;
            t_end = pc.t1;
            cur_h = pc.h;
            cur_len = g.kv_len;
            bt = p.block_tables + (size_t)pc.b * p.bt_stride;
            progressed = true;
          }
        }
        if (kn < n_tiles && kn - vn < 8 && t_cur < t_end) {
          const int ks = kn % KSTAGES;
          if (mbar_try_wait(&k_empty[ks], ((kn / KSTAGES) & 1) ^ 1)) {
            const int k0 = t_cur * TBK;
            int rows[2];
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              int k = k0 + hh * 64;
              if (k >= cur_len) k = k0;  // keys past the end: reload a valid box (masked later)
              rows[hh] = (bt[k / p.page] * p.hkv + cur_h) * p.page + (k % p.page);
            }
            ATT_TRACE(0, kn);
            mbar_arrive_expect_tx(&k_full[ks], KV_BYTES);
#pragma unroll
            for (int dh = 0; dh < 2; ++dh)
#pragma unroll
              for (int hh = 0; hh < 2; ++hh)
                tma_load_2d(sK + ks * KV_BYTES + dh * REGION + hh * (REGION / 2), &tmK, &k_full[ks], dh * 64,
                            rows[hh]);
            trows[kn & 7] = make_int2(rows[0], rows[1]);
            kin |= 1u << ks;
            ++kn;
            ++t_cur;
            progressed = true;
          }
        }
        // ---- V side
        if (vn < kn) {
          const int vs = vn % VSTAGES;
          if (mbar_try_wait(&v_empty[vs], ((vn / VSTAGES) & 1) ^ 1)) {
            const int2 rows = trows[vn & 7];
            ATT_TRACE(1, vn);
            mbar_arrive_expect_tx(&v_full[vs], KV_BYTES);
#pragma unroll
            for (int dh = 0; dh < 2; ++dh) {
              tma_load_2d(sV + vs * KV_BYTES + dh * REGION, &tmV, &v_full[vs], dh * 64, rows.x);
              tma_load_2d(sV + vs * KV_BYTES + dh * REGION + REGION / 2, &tmV, &v_full[vs], dh * 64, rows.y);
            }
            vin |= 1u << vs;
            ++vn;
            progressed = true;
          }
        }
        if (progressed) {
          idle_since = 0;
        } else {  // nothing ready: keep polling both rings, within the wait limit
          const uint64_t now = globaltimer_ns();
          if (idle_since == 0) idle_since = now;
          if (*abort_flag) { ok = false; break; }
          if (now - idle_since > kWaitLimitNs) {
            set_error(p.err, 1);
            *abort_flag = 1;
            ok = false;
            break;
          }
        }
      }
      if (!ok) {  // let copies in flight land before the CTA exits
        for (int i = 1; i <= 2 && i <= qn; ++i) {
          const int n = qn - i;
          mbar_wait(&q_full[n & 1], (n >> 1) & 1, nullptr);
        }
        for (int i = 1; i <= KSTAGES && i <= kn; ++i) {
          const int n = kn - i;
          if ((kin >> (n % KSTAGES)) & 1) mbar_wait(&k_full[n % KSTAGES], (n / KSTAGES) & 1, nullptr);
        }
        for (int i = 1; i <= VSTAGES && i <= vn; ++i) {
          const int n = vn - i;
          if ((vin >> (n % VSTAGES)) & 1) mbar_wait(&v_full[n % VSTAGES], (n / VSTAGES) & 1, nullptr);
        }
      }
    }
  } else if (warp == 1 || warp == 14) {
    // ================================================================ MMA issuers
    // warp 1 issues S^T = K.Q^T as soon as a K tile and an S buffer are free;
    // warp 14 issues O^T += V^T.P^T as soon as a V tile and a P tile are ready.
    // Each tracks its own tcgen05 operations, so neither waits for the other's.
    if (lane == 0 && x_begin < x_end) {
      constexpr uint32_t idesc_s = idesc_bf16(128, TR);
      constexpr uint32_t idesc_o = idesc_bf16(128, TR) | (1u << 15);  // A (V^T) MN-major
      const bool is_s = (warp == 1);
      const int n_tiles = (int)(x_end - x_begin);
      int qn = 0, tn = 0;  // pieces, tiles
      bool ok = true;
      while (ok && tn < n_tiles) {
        const int qb = qn & 1, ob = qn & 1;
        if (!wait_or_abort(&q_full[qb], (qn >> 1) & 1, abort_flag, p.err)) { ok = false; break; }
        const PieceMeta pc = meta[qb];
        if (is_s) {
          tc_fence_after();
          const uint64_t qdesc = smem_desc_sw128(sQ + qb * QP_BYTES);
          for (int t = pc.t0; t < pc.t1; ++t, ++tn) {
            const int sb = tn & 1, ks = tn % KSTAGES;
            if (!wait_or_abort(&k_full[ks], (tn / KSTAGES) & 1, abort_flag, p.err)) { ok = false; break; }
            if (!wait_or_abort(&s_empty[sb], ((tn >> 1) & 1) ^ 1, abort_flag, p.err)) { ok = false; break; }
            ATT_TRACE(2, tn);
            tc_fence_after();
            const uint64_t kdesc = smem_desc_sw128(sK + ks * KV_BYTES);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const uint64_t off_a = (uint64_t)((k >> 2) * (REGION >> 4) + (k & 3) * 2);
              const uint64_t off_b = (uint64_t)((k >> 2) * (QP_REGION >> 4) + (k & 3) * 2);
              tc_mma_bf16(tmem + sb * TR, kdesc + off_a, qdesc + off_b, idesc_s, k > 0);
            }
            tc_commit(&s_full[sb]);
            tc_commit(&k_empty[ks]);
            if (t + 1 == pc.t1) tc_commit(&q_empty[qb]);
          }
        } else {
          mbar_arrive(&q_empty[qb]);  // piece geometry read
          const uint32_t o_tm = tmem + 2 * TR + ob * TR;
          for (int t = pc.t0; t < pc.t1; ++t, ++tn) {
            const int vs = tn % VSTAGES, pb = tn & 1;
            if (!wait_or_abort(&v_full[vs], (tn / VSTAGES) & 1, abort_flag, p.err)) { ok = false; break; }
            if (!wait_or_abort(&p_full[pb], (tn >> 1) & 1, abort_flag, p.err)) { ok = false; break; }
            if (t == pc.t0) {
              if (!wait_or_abort(&o_empty[ob], ((qn >> 1) & 1) ^ 1, abort_flag, p.err)) { ok = false; break; }
            }
            ATT_TRACE(3, tn);
            tc_fence_after();
            const uint64_t vdesc = desc_v_mn(sV + vs * KV_BYTES);
            const uint64_t pdesc = smem_desc_sw128(sP + pb * QP_BYTES);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const uint64_t off_a = (uint64_t)(k * (2048 >> 4));  // 16 keys = 2 KB
              const uint64_t off_b = (uint64_t)((k >> 2) * (QP_REGION >> 4) + (k & 3) * 2);
              tc_mma_bf16(o_tm, vdesc + off_a, pdesc + off_b, idesc_o, (t > pc.t0) || k > 0);
            }
            tc_commit(&v_empty[vs]);
            tc_commit(&p_empty[pb]);
            ATT_TRACE(4, tn);
          }
          if (ok) tc_commit(&o_full[ob]);
        }
        ++qn;
      }
      // drain: wait for every MMA this thread issued before TMEM is released
      uint64_t* drain = &drain_bar[is_s ? 0 : 1];
      tc_commit(drain);
      mbar_wait(drain, 0, nullptr);
    }
  } else if (warp < 10) {
    // ================================================================ softmax
    // 8 warps: warp w reads TMEM lane quarter w % 4 (keys 32q..32q+31 of a tile)
    // and rows [HR*half, HR*half + HR) of S; the two halves are independent.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int key = quarter * 32 + lane;        // this thread's key within a tile
    const int hidx = ((warp - 2) & 3) * 32 + lane;  // 0..127 within this half
    const int r0 = half * HR;                   // first row of this half
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    const int bar_half = 1 + half;              // named barriers 1 and 2 (128 threads each)
    if (x_begin < x_end) {
      const int n_tiles = (int)(x_end - x_begin);
      int qn = 0, tn = 0, pn = 0;
      while (tn < n_tiles) {
        const int ob = qn & 1, qb = qn & 1;
        if (hidx == 0 && half == 0) ATT_TRACE(13, qn);
        // piece geometry and suffix masks arrive with the Q tile
        wait_or_abort(&q_full[qb], (qn >> 1) & 1, abort_flag, p.err);
        if (hidx == 0 && half == 0) ATT_TRACE(14, qn);
        const PieceMeta pc = meta[qb];
        struct { int prefix, kv_len; } g{pc.prefix, pc.kv_len};
        const int i0 = pc.rb * p.qpb;
        const uint32_t valid = half ? pc.valid[1] : pc.valid[0];
        // the suffix key (if any) that lands on this thread's TMEM lane: keys of a tile are 128 apart
        // per lane and a forward has at most 64, so one mask word per thread covers the whole piece
        const int j1 = ((key - g.prefix) % TBK + TBK) % TBK;
        uint32_t cm_mine = 0;  // rows of this half that see suffix key j1
        if (p.mode == M_SUFFIX && j1 < p.Q) {
          const uint64_t gbits = (1ull << p.group) - 1;
          for (int qi = r0 >> p.group_shift; qi <= (r0 + HR - 1) >> p.group_shift; ++qi)
            if ((smask_sm[qb * TR + qi] >> j1) & 1) cm_mine |= (uint32_t)((gbits << (qi << p.group_shift)) >> r0);
          cm_mine &= valid;
        }
        if (hidx < HR) msm[r0 + hidx] = -1e30f;
        bar_named(bar_half, 128);
        if (hidx == 0 && half == 0) mbar_arrive(&q_empty[qb]);  // the piece's masks are no longer read
        if (hidx == 0 && half == 0) ATT_TRACE(15, qn);
        float m_run[HR], l_run[HR];  // a row max of -1e30 stands for "no key yet" (exp2 of it is 0)
#pragma unroll
        for (int r = 0; r < HR; ++r) {
          m_run[r] = -1e30f;
          l_run[r] = 0.f;
        }
        for (int t = pc.t0; t < pc.t1; ++t) {
          const int sb = tn & 1, pb = pn & 1;
          const int kg = t * TBK + key;
          wait_or_abort(&s_full[sb], (tn >> 1) & 1, abort_flag, p.err);
          if (hidx == 0 && half == 0) ATT_TRACE(5, tn);
          tc_fence_after();
          float s[HR];
          tmem_ld16(lane_base + sb * TR + r0, s);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s_empty[sb]);
          ++tn;
          // ---- rows of this half that see this key
          uint32_t vm;
          if (p.mode == M_SUFFIX) {
            vm = kg < g.prefix ? valid : (kg < g.kv_len ? cm_mine : 0u);
          } else {
            const int d = kg - g.prefix - i0;  // rows of queries >= d see the key
            const int first = (d <= 0 ? 0 : d << p.group_shift) - r0;
            vm = first <= 0 ? valid : (first >= HR ? 0u : (valid & (~0u << first)));
          }
          bool exceed = false;
#pragma unroll
          for (int r = 0; r < HR; ++r) {
            s[r] = ((vm >> r) & 1) ? s[r] * p.scale_log2 : -INFINITY;
            exceed |= s[r] > m_run[r] + 8.f;
          }
          exceed = bar_red_or(bar_half, 128, exceed);
          // the P buffer of two tiles ago has been consumed
          if (hidx == 0 && half == 0) ATT_TRACE(6, pn);
          wait_or_abort(&p_empty[pb], ((pn >> 1) & 1) ^ 1, abort_flag, p.err);
          if (hidx == 0 && half == 0) ATT_TRACE(7, pn);
          if (exceed) {
            // row maxima: warp reduce (order-preserving int encoding), then every thread combines
            // the 4 warps of its half; a row's running maximum moves when it grew by > 8
#pragma unroll
            for (int r = 0; r < HR; ++r) {
              int v = __float_as_int(s[r]);
              v = v >= 0 ? v : v ^ 0x7fffffff;
              v = __reduce_max_sync(0xffffffff, v);
              if (lane == r) red[(warp - 2) * HR + r] = __int_as_float(v >= 0 ? v : v ^ 0x7fffffff);
            }
            bar_named(bar_half, 128);
            if (hidx < HR) {  // one thread per row of this half
              const float* rh = red + half * 4 * HR;
              const float tm = fmaxf(fmaxf(rh[hidx], rh[HR + hidx]), fmaxf(rh[2 * HR + hidx], rh[3 * HR + hidx]));
              const float mo = msm[r0 + hidx];
              const float mn = tm > mo + 8.f ? tm : mo;
              msm[r0 + hidx] = mn;
              csm[r0 + hidx] = ex2(mo - mn);  // 0 when the row had no key yet
            }
            bar_named(bar_half, 128);
            bool any_corr = false;
#pragma unroll
            for (int r = 0; r < HR; ++r) {
              const float c = csm[r0 + r];
              m_run[r] = msm[r0 + r];
              l_run[r] *= c;
              any_corr |= c != 1.f;
            }
            if (t > pc.t0 && any_corr) {
              // O holds the products of tiles < t: wait for the last one, then rescale in place
              const int prev = pn - 1;
              wait_or_abort(&p_empty[prev & 1], (prev >> 1) & 1, abort_flag, p.err);
              tc_fence_after();
              const uint32_t oaddr = lane_base + 2 * TR + ob * TR + r0;
#pragma unroll
              for (int c = 0; c < HR; c += 8) {
                float ov[8];
                tmem_ld8(oaddr + c, ov);
#pragma unroll
                for (int r = 0; r < 8; ++r) ov[r] *= csm[r0 + c + r];
                tmem_st8(oaddr + c, ov);
              }
            }
          }
          // ---- P = exp2(S - m), row sums, P^T into shared memory (K-major, 128-byte swizzle)
          uint8_t* prow = sP + pb * QP_BYTES + (key >> 6) * QP_REGION + r0 * 128;
          const int kc = (key & 63) >> 3, kb = (key & 7) * 2;
#pragma unroll
          for (int r = 0; r < HR; ++r) {
            const float pv = ex2(s[r] - m_run[r]);
            l_run[r] += pv;
            *reinterpret_cast<__nv_bfloat16*>(prow + r * 128 + ((kc ^ ((r0 + r) & 7)) << 4) + kb) =
                __float2bfloat16(pv);
          }
          fence_async_smem();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&p_full[pb]);
          if (hidx == 0 && half == 0) ATT_TRACE(8, pn);
          ++pn;
        }
        // ---- end of piece: row sums and maxima for the epilogue warps
#pragma unroll
        for (int r = 0; r < HR; ++r) {
          float v = l_run[r];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
          l_run[r] = v;
        }
        if (hidx == 0 && half == 0) ATT_TRACE(10, qn);
        // lfin/mfin[ob] and red[] are free once the epilogue released this O buffer's previous piece
        wait_or_abort(&o_empty[ob], ((qn >> 1) & 1) ^ 1, abort_flag, p.err);
        if (hidx == 0 && half == 0) ATT_TRACE(11, qn);
        bar_named(bar_half, 128);  // red[] of the last rescale has been read
        if (lane == 0) {
#pragma unroll
          for (int r = 0; r < HR; ++r) red[(warp - 2) * HR + r] = l_run[r];
        }
        bar_named(bar_half, 128);
        if (hidx < HR) {
          const int w0 = half * 4;
          lfin[ob * TR + r0 + hidx] = red[(w0 + 0) * HR + hidx] + red[(w0 + 1) * HR + hidx] +
                                      red[(w0 + 2) * HR + hidx] + red[(w0 + 3) * HR + hidx];
          mfin[ob * TR + r0 + hidx] = msm[r0 + hidx];
        }
        bar_named(bar_half, 128);
        if (hidx == 0) mbar_arrive(&l_full[ob]);  // one arrival per half
        if (hidx == 0 && half == 0) ATT_TRACE(12, qn);
        ++qn;
      }
    }
  } else if (warp < 14) {
    // ================================================================ epilogue
    const int quarter = warp & 3;
    const int dim = quarter * 32 + lane;        // this thread's output dimension
    const int eidx = (warp - 10) * 32 + lane;   // 0..127 within the epilogue group
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    if (x_begin < x_end) {
      Walker w;
      w.init(p, prefix, x_begin, x_end);
      int qn = 0;
      while (!w.done()) {
        const Piece pc = w.next(p, prefix);
        const ReqGeo g = req_geo(p, pc.b);
        const int i0 = pc.rb * p.qpb;
        const int ob = qn & 1;
        wait_or_abort(&o_full[ob], (qn >> 1) & 1, abort_flag, p.err);
        wait_or_abort(&l_full[ob], (qn >> 1) & 1, abort_flag, p.err);
        tc_fence_after();
        {
          // O^T column of this thread's dimension -> shared memory, so the loops below can stay rolled
          float ov[TR];
          tmem_ld32(lane_base + 2 * TR + ob * TR, ov);
#pragma unroll
          for (int r = 0; r < TR; ++r) ostage[r * TD + dim] = ov[r];
        }
        const float mrow_e = eidx < TR ? mfin[ob * TR + eidx] : 0.f;
        const float lrow_e = eidx < TR ? lfin[ob * TR + eidx] : 0.f;
        // normalise the staged column, then hand TMEM O[ob] and lfin/mfin[ob] back right away:
        // the output writes and any merge below only touch this thread's staging column
#pragma unroll 4
        for (int r = 0; r < TR; ++r) {
          const float l = lfin[ob * TR + r];
          ostage[r * TD + dim] *= (l > 0.f ? 1.f / l : 0.f);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&o_empty[ob]);
        ++qn;
        const bool complete = (pc.t0 == 0 && pc.t1 == pc.nt);
        const bool aborted = *abort_flag != 0;
        const size_t row0 = (size_t)(g.q_begin + i0) * p.hq + pc.h * p.group;  // row of r = 0
        const int slot = 2 * blockIdx.x + (pc.x0 == x_begin ? 0 : 1);
        float* part = p.o_part + (size_t)slot * TR * TD;
        const int nrows = min(TR, (g.nq - i0) << p.group_shift);  // rows whose query exists
#pragma unroll 4
        for (int r = 0; r < TR; ++r) {
          const float v = ostage[r * TD + dim];
          if (!complete) {
            part[r * TD + dim] = v;
          } else if (r < nrows && !aborted) {
            const size_t row = row0 + (size_t)(r >> p.group_shift) * p.hq + (r & (p.group - 1));
            p.o[row * TD + dim] = __float2bfloat16(v);
          }
        }
        if (!complete) {
        if (eidx < TR)
          p.lse_part[(size_t)slot * TR + eidx] = lrow_e > 0.f ? mrow_e + __log2f(lrow_e) : -INFINITY;
        __threadfence();
        bar_named(4, 128);
        const long long seg_x0 = pc.x0 - pc.t0;  // the segment's first global tile
        const int c_first = tile_owner(seg_x0, TT, G);
        const int c_last = tile_owner(seg_x0 + pc.nt - 1, TT, G);
        const int n_pieces = c_last - c_first + 1;
        const size_t cidx = (size_t)(g.q_begin + i0) * p.hkv + pc.h;
        if (eidx == 0) *last_flag = aborted ? 0 : (atomicAdd(p.counters + cidx, 1) == n_pieces - 1);
        bar_named(4, 128);
        if (*last_flag) {
          __threadfence();
          // merge the segment's pieces: per-row maxima and weight sums first (one row per thread),
          // then every thread accumulates its dimension of 8 rows at a time with independent loads
          if (eidx < TR) {
            float m = -INFINITY;
            for (int c = c_first; c <= c_last; ++c) {
              const int sl = 2 * c + (range_begin(c, TT, G) >= seg_x0 ? 0 : 1);
              m = fmaxf(m, __ldcg(p.lse_part + (size_t)sl * TR + eidx));
            }
            float tot = 0.f;
            if (m != -INFINITY) {
              for (int c = c_first; c <= c_last; ++c) {
                const int sl = 2 * c + (range_begin(c, TT, G) >= seg_x0 ? 0 : 1);
                const float lse = __ldcg(p.lse_part + (size_t)sl * TR + eidx);
                tot += lse == -INFINITY ? 0.f : ex2(lse - m);
              }
            }
            cmb[eidx] = m == -INFINITY ? 0.f : m;
            cmb[TR + eidx] = tot > 0.f ? 1.f / tot : 0.f;
          }
          bar_named(4, 128);
#pragma unroll 1
          for (int rb8 = 0; rb8 < nrows; rb8 += 8) {
            float acc[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] = 0.f;
            for (int c = c_first; c <= c_last; ++c) {
              const int sl = 2 * c + (range_begin(c, TT, G) >= seg_x0 ? 0 : 1);
              const float* lse = p.lse_part + (size_t)sl * TR + rb8;
              const float* op = p.o_part + ((size_t)sl * TR + rb8) * TD + dim;
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const float l = __ldcg(lse + j);
                const float wgt = l == -INFINITY ? 0.f : ex2(l - cmb[rb8 + j]);
                acc[j] += wgt * __ldcg(op + j * TD);
              }
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const int r = rb8 + j;
              if (r < nrows) {
                const size_t row = row0 + (size_t)(r >> p.group_shift) * p.hq + (r & (p.group - 1));
                p.o[row * TD + dim] = __float2bfloat16(acc[j] * cmb[TR + r]);
              }
            }
          }
          if (eidx == 0) p.counters[cidx] = 0;
        }
        bar_named(4, 128);  // last_flag is rewritten by the next partial piece
        }
      }
    }
  }
  __syncwarp();  // single-lane roles rejoin their warps before the CTA barrier
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    if (lane == 0 && p.trace != nullptr) p.trace[1024 + 4 * blockIdx.x + 2] = globaltimer_ns();
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
    if (lane == 0 && p.trace != nullptr) p.trace[1024 + 4 * blockIdx.x + 3] = globaltimer_ns();
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
  TORCH_CHECK(group >= 1 && group <= TR && (group & (group - 1)) == 0 && a.hq == group * a.hkv,
              "GQA group must be a power of two <= ", TR);
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
  p.group_shift = __builtin_ctz(group);
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
