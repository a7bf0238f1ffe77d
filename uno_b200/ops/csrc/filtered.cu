// Filtered (top-k / top-p) sampling and sparse Psi-Spec verification.
//
// Semantics (``nano_vllm_uno/layers/sampler.py:21-90``,
// ``nano_vllm_uno/engine/two_pass_decoding.py:56-97``):
// * top-k keeps the k most likely tokens and renormalises over them; top-p
//   then (or alone, relative to the full softmax) keeps a token while the
//   probability ranked strictly before it is <= top_p;
// * verification accepts the draft token s with probability min(1, p(s)/q(s))
//   on the filtered target p and draft q; on reject it resamples from
//   norm(max(p - q, 0)), or from p when that residual is empty.
//
// Representation.  Tokens are ranked by key(i) = ord(x_i) << 32 | (2^32-1-i),
// where ord is the order-preserving 16-bit image of the bf16 logit: key order
// is value descending, lowest id first among equal values -- a strict total
// order.  Every filtered distribution keeps a prefix of it, so three numbers
// describe one exactly:
//   m = max_i x_i / T,   K = key of the last kept token (i kept iff key(i) >= K),
//   S = sum over kept tokens of exp(x_i / T - m),   p_i = exp(x_i / T - m) / S.
// The sampler writes (K, m, S) per row next to the token; the verifier reads
// the draft's triple and the draft logits row, so no candidate list exists.
//
// Selection: one CTA of 1024 threads per row, the row re-read from L2.
//  1. stats: m, Z = sum exp(x/T - m), smallest finite x/T;
//  2. histogram: 2048 bins of d = m - x/T (bin index never decreases as the
//     key decreases), with token counts and, for the top-p criterion, masses
//     in 2^-40 fixed point held as three 14-bit limbs (native 32-bit shared
//     atomics, no carries within a row of < 2^18 tokens).  The sums are integer,
//     so they do not depend on thread timing and every tensor-parallel rank
//     that runs the same call selects the same set.  Top-p bins only
//     d <= ln(V / ((1 - top_p) Z)) + 1: the last kept token has at least
//     (1 - top_p) Z of mass at or after it, spread over at most V tokens of at
//     most exp(-d) each.  Top-p after top-k bins only the top-k tokens' range;
//  3. the boundary bin (where the count reaches k, or the last bin whose
//     preceding mass is <= P) is collected into shared memory, bitonic-sorted
//     by key and walked; a boundary bin of more than 4096 tokens is re-binned
//     over its exact key range (at most twice, 16-bit keys), and a single key
//     shared by many tokens is resolved by counting tied tokens in id order.
// The kept mass S is an exact integer sum, so every pass that forms it agrees.
// Randomness: Philox streams 4 (sample), 5 (accept test) and 6 (residual) of
// the (seed, offset, row, token id) keying used by every sampling kernel.
#include "common.cuh"
#include "sampling_common.cuh"
#include "uno_ops.h"

namespace uno {

namespace {

constexpr int FT = 1024;       // threads per row
constexpr int NB = 2048;       // histogram bins
constexpr int CAND = 4096;     // boundary-bin tokens sorted in shared memory
constexpr float FIX = 1099511627776.f;  // 2^40
typedef unsigned long long u64;

struct FiltSmem {
  u64 cand[CAND];
  uint32_t hcnt[NB];
  uint32_t hm[3][NB];  // mass limbs: bits 0-13, 14-27, 28-40 of the 2^-40 fixed-point weights
  u64 wsum[32];
  uint32_t wcnt[32];
  u64 ctot_w;
  uint32_t ctot_c;
  int bsel;
  uint32_t n_sel, c_above;
  u64 w_above;
  uint32_t kmin, kmax;
  uint32_t slot;
  int jstar;
  u64 sel_S;
  int tie_idx;
};

__device__ __forceinline__ uint32_t ord16(uint32_t h) { return (h & 0x8000u) ? (~h & 0xFFFFu) : (h | 0x8000u); }
__device__ __forceinline__ uint32_t unord16(uint32_t o) { return (o & 0x8000u) ? (o & 0x7FFFu) : (~o & 0xFFFFu); }
__device__ __forceinline__ float bits2f(uint32_t h) { return __uint_as_float(h << 16); }
__device__ __forceinline__ u64 make_key(uint32_t o, int i) {
  return ((u64)o << 32) | (u64)(0xFFFFFFFFu - (uint32_t)i);
}
// Scaled logit and its distance below the row max.  The _rn intrinsics are
// never contracted into FMAs, so every pass computes bit-identical values.
__device__ __forceinline__ float scaled(uint32_t h, float inv_temp) { return __fmul_rn(bits2f(h), inv_temp); }
// Histogram bin of a distance d in [0, dr]: floor(d * NB / dr), clamped.
__device__ __forceinline__ int bin_of(float d, float scale) { return min((int)__fmul_rn(d, scale), NB - 1); }
// floor(exp(-d) * 2^40): the token's mass in fixed point.
__device__ __forceinline__ u64 wfix(float d) { return __float2ull_rz(__fmul_rn(__expf(-d), FIX)); }
// Adds a token's mass to a bin as three 14-bit limbs (bits 0-13, 14-27, 28-40).
__device__ __forceinline__ void add_mass(FiltSmem& sm, int b, float d) {
  const u64 w = wfix(d);
  if (!w) return;
  atomicAdd(&sm.hm[0][b], (uint32_t)(w & 0x3FFFu));
  atomicAdd(&sm.hm[1][b], (uint32_t)((w >> 14) & 0x3FFFu));
  atomicAdd(&sm.hm[2][b], (uint32_t)(w >> 28));
}
// key(i) >= K with 32-bit operations: value above K's, or equal and id <= K's.
struct KeyCut {
  uint32_t o, idx;
  __device__ __forceinline__ explicit KeyCut(u64 K) : o((uint32_t)(K >> 32)), idx(0xFFFFFFFFu - (uint32_t)K) {}
  __device__ __forceinline__ bool keeps(uint32_t oi, int i) const { return oi > o || (oi == o && (uint32_t)i <= idx); }
};
__device__ __forceinline__ u64 bin_mass(const FiltSmem& sm, int b) {
  return (u64)sm.hm[0][b] + ((u64)sm.hm[1][b] << 14) + ((u64)sm.hm[2][b] << 28);
}

// Calls g(v, vector) for every 8-token vector v of a row (V % 8 == 0,
// 16-byte aligned rows).  A pass is bound by L2 round trips, so each thread
// issues four 16-byte loads before it processes them.
template <typename G>
__device__ __forceinline__ void row_vecs(const uint16_t* row, int V, G g) {
  const int nvec = V >> 3;
  const uint4* src = reinterpret_cast<const uint4*>(row);
  int k = threadIdx.x;
  for (; k + 3 * FT < nvec; k += 4 * FT) {
    uint4 w[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) w[u] = src[k + u * FT];
#pragma unroll
    for (int u = 0; u < 4; ++u) g(k + u * FT, w[u]);
  }
  for (; k < nvec; k += FT) g(k, src[k]);
}

// Calls f(i, bits) for every token of a row.
template <typename F>
__device__ __forceinline__ void row_each(const uint16_t* row, int V, F f) {
  row_vecs(row, V, [&](int v, const uint4& w) {
    const uint32_t p[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      f(v * 8 + 2 * j, p[j] & 0xFFFFu);
      f(v * 8 + 2 * j + 1, p[j] >> 16);
    }
  });
}

// Block-wide exclusive scan of (count, mass) pairs; also leaves the totals in
// sm.ctot_c / sm.ctot_w.
__device__ void scan2(uint32_t c, u64 w, uint32_t& ce, u64& we, FiltSmem& sm) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t ci = c;
  u64 wi = w;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t c2 = __shfl_up_sync(0xffffffffu, ci, o);
    const u64 w2 = __shfl_up_sync(0xffffffffu, wi, o);
    if (lane >= o) {
      ci += c2;
      wi += w2;
    }
  }
  if (lane == 31) {
    sm.wcnt[warp] = ci;
    sm.wsum[warp] = wi;
  }
  __syncthreads();
  if (warp == 0) {
    const uint32_t c0 = sm.wcnt[lane];
    const u64 w0 = sm.wsum[lane];
    uint32_t cs = c0;
    u64 ws = w0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t c2 = __shfl_up_sync(0xffffffffu, cs, o);
      const u64 w2 = __shfl_up_sync(0xffffffffu, ws, o);
      if (lane >= o) {
        cs += c2;
        ws += w2;
      }
    }
    if (lane == 31) {
      sm.ctot_c = cs;
      sm.ctot_w = ws;
    }
    sm.wcnt[lane] = cs - c0;
    sm.wsum[lane] = ws - w0;
  }
  __syncthreads();
  ce = sm.wcnt[warp] + ci - c;
  we = sm.wsum[warp] + wi - w;
  __syncthreads();  // wcnt / wsum are reused by the next scan
}

// After a histogram is built: find the boundary bin for "count reaches k"
// (k > 0) or "last non-empty bin whose preceding mass is <= P" (k == 0), with
// c_base / w_base the tokens and mass ranked before bin 0.  Leaves the bin in
// sm.bsel (-1 when the count never reaches k) and its tokens / preceding
// counts in sm.n_sel / sm.c_above / sm.w_above.
__device__ void find_boundary(int k, u64 P, uint32_t c_base, u64 w_base, FiltSmem& sm) {
  const int b0 = 2 * threadIdx.x, b1 = b0 + 1;
  const uint32_t c0 = sm.hcnt[b0], c1 = sm.hcnt[b1];
  const u64 w0 = k > 0 ? 0ull : bin_mass(sm, b0), w1 = k > 0 ? 0ull : bin_mass(sm, b1);
  if (threadIdx.x == 0) sm.bsel = -1;
  uint32_t ce;
  u64 we;
  scan2(c0 + c1, w0 + w1, ce, we, sm);  // its barriers order the bsel reset before the writes below
  ce += c_base;
  we += w_base;
  const uint32_t ce1 = ce + c0;
  const u64 we1 = we + w0;
  if (k > 0) {
    if (ce < (uint32_t)k && ce + c0 >= (uint32_t)k) sm.bsel = b0;
    else if (ce1 < (uint32_t)k && ce1 + c1 >= (uint32_t)k) sm.bsel = b1;
  } else {
    int best = -1;
    if (c0 > 0 && we <= P) best = b0;
    if (c1 > 0 && we1 <= P) best = b1;
    if (best >= 0) atomicMax(&sm.bsel, best);
  }
  __syncthreads();
  const int b = sm.bsel;
  if (b == b0) {
    sm.n_sel = c0;
    sm.c_above = ce;
    sm.w_above = we;
  } else if (b == b1) {
    sm.n_sel = c1;
    sm.c_above = ce1;
    sm.w_above = we1;
  }
  __syncthreads();
}

__device__ void clear_hist(FiltSmem& sm) {
  for (int b = threadIdx.x; b < NB; b += FT) {
    sm.hcnt[b] = 0;
    sm.hm[0][b] = 0;
    sm.hm[1][b] = 0;
    sm.hm[2][b] = 0;
  }
  __syncthreads();
}

struct Sel {
  u64 K;  // key of the last kept token
  u64 S;  // kept mass, 2^-40 units (0 when the count criterion chose the set: not formed)
};

// Sorts sm.cand[0, n) by key descending and picks the last kept token: the
// (k - c_above)-th one, or the last whose preceding mass is <= P.
__device__ Sel sort_and_walk(int n, int k, u64 P, uint32_t c_above, u64 w_above, float m, float inv_temp,
                             FiltSmem& sm) {
  int npad = 2;
  while (npad < n) npad <<= 1;
  for (int i = n + threadIdx.x; i < npad; i += FT) sm.cand[i] = 0ull;
  __syncthreads();
  for (int size = 2; size <= npad; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int t = threadIdx.x; t < (npad >> 1); t += FT) {
        const int i = 2 * stride * (t / stride) + (t % stride), j = i + stride;
        const u64 a = sm.cand[i], b = sm.cand[j];
        const bool desc = (i & size) == 0;
        if ((a < b) == desc) {
          sm.cand[i] = b;
          sm.cand[j] = a;
        }
      }
      __syncthreads();
    }
  }
  // prefix masses over the sorted tokens, four consecutive positions per thread
  const int j0 = 4 * threadIdx.x;
  u64 w[4];
  u64 local = 0;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int j = j0 + q;
    w[q] = 0;
    if (j < n) {
      const uint32_t h = unord16((uint32_t)(sm.cand[j] >> 32));
      w[q] = wfix(__fsub_rn(m, scaled(h, inv_temp)));
    }
    local += w[q];
  }
  if (threadIdx.x == 0) sm.jstar = -1;
  uint32_t unused;
  u64 excl;
  scan2(0u, local, unused, excl, sm);
  excl += w_above;
  const int target = k > 0 ? k - (int)c_above - 1 : -1;
  int mine = -1;
  u64 e = excl;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int j = j0 + q;
    if (j < n && (k > 0 ? j == target : e <= P)) mine = j;
    e += w[q];
  }
  if (mine >= 0) atomicMax(&sm.jstar, mine);
  __syncthreads();
  const int js = max(sm.jstar, 0);  // >= 0 whenever the histogram and the collection agree
  if (js >= j0 && js < j0 + 4) {
    u64 s = excl;
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (q <= js - j0) s += w[q];
    sm.sel_S = s;
  }
  __syncthreads();
  Sel out{sm.cand[js], sm.sel_S};
  __syncthreads();
  return out;
}

// Collects the tokens accepted by pred(i, bits, o) into sm.cand.
template <typename P>
__device__ void collect(const uint16_t* row, int V, P pred, FiltSmem& sm) {
  if (threadIdx.x == 0) sm.slot = 0;
  __syncthreads();
  row_each(row, V, [&](int i, uint32_t h) {
    const uint32_t o = ord16(h);
    if (pred(i, h, o)) {
      const uint32_t s = atomicAdd(&sm.slot, 1u);
      if (s < (uint32_t)CAND) sm.cand[s] = make_key(o, i);
    }
  });
  __syncthreads();
}

// n tokens share the key value o: keep r of them, lowest ids first.
__device__ Sel resolve_ties(const uint16_t* row, int V, uint32_t o, uint32_t n, int k, u64 P, uint32_t c_above,
                            u64 w_above, float m, float inv_temp, FiltSmem& sm) {
  const u64 wt = wfix(__fsub_rn(m, scaled(unord16(o), inv_temp)));
  uint32_t r;
  if (k > 0) {
    r = (uint32_t)k - c_above;
  } else if (wt == 0) {
    r = n;
  } else {
    const u64 avail = P >= w_above ? P - w_above : 0;
    const u64 q = avail / wt + 1;
    r = q < (u64)n ? (uint32_t)q : n;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) sm.tie_idx = -1;
  __syncthreads();
  uint32_t running = 0;
  for (int base = 0; base < V; base += FT) {
    const int i = base + threadIdx.x;
    const bool pred = i < V && ord16(row[i]) == o;
    const uint32_t bal = __ballot_sync(0xffffffffu, pred);
    if (lane == 0) sm.wcnt[warp] = __popc(bal);
    __syncthreads();
    uint32_t before = 0, total = 0;
    for (int w = 0; w < 32; ++w) {
      const uint32_t c = sm.wcnt[w];
      if (w < warp) before += c;
      total += c;
    }
    const uint32_t pos = running + before + __popc(bal & ((1u << lane) - 1u));
    if (pred && pos + 1 == r) sm.tie_idx = i;
    running += total;
    __syncthreads();
    if (running >= r) break;
  }
  const int idx = sm.tie_idx;
  __syncthreads();
  return Sel{make_key(o, idx < 0 ? 0 : idx), w_above + (u64)r * wt};
}

// The exact selection of one criterion over a row (see the file comment).
__device__ Sel select_tokens(const uint16_t* row, int V, float inv_temp, float m, float dr, int k, u64 P,
                             FiltSmem& sm) {
  clear_hist(sm);
  const float scale = dr > 0.f ? (float)NB / dr : 0.f;
  row_each(row, V, [&](int, uint32_t h) {
    const float d = __fsub_rn(m, scaled(h, inv_temp));
    if (d <= dr) {
      const int b = bin_of(d, scale);
      atomicAdd(&sm.hcnt[b], 1u);
      if (k == 0) add_mass(sm, b, d);
    }
  });
  __syncthreads();
  find_boundary(k, P, 0u, 0ull, sm);
  int b = sm.bsel;
  if (b < 0) return Sel{0ull, k > 0 ? 0ull : sm.ctot_w};  // fewer than k finite tokens: keep them all
  uint32_t n = sm.n_sel, c_above = sm.c_above;
  u64 w_above = sm.w_above;
  if (n <= (uint32_t)CAND) {
    const int bb = b;
    collect(row, V, [&](int, uint32_t h, uint32_t) {
      const float d = __fsub_rn(m, scaled(h, inv_temp));
      return d <= dr && bin_of(d, scale) == bb;
    }, sm);
    return sort_and_walk((int)n, k, P, c_above, w_above, m, inv_temp, sm);
  }
  // A crowded boundary bin: its exact key range, then re-bin over keys.
  if (threadIdx.x == 0) {
    sm.kmin = 0xFFFFu;
    sm.kmax = 0u;
  }
  __syncthreads();
  {
    uint32_t lo = 0xFFFFu, hi = 0u;
    const int bb = b;
    row_each(row, V, [&](int, uint32_t h) {
      const float d = __fsub_rn(m, scaled(h, inv_temp));
      if (d <= dr && bin_of(d, scale) == bb) {
        const uint32_t o = ord16(h);
        lo = min(lo, o);
        hi = max(hi, o);
      }
    });
    atomicMin(&sm.kmin, lo);
    atomicMax(&sm.kmax, hi);
  }
  __syncthreads();
  uint32_t klo = sm.kmin, khi = sm.kmax;
  for (int level = 0; level < 3; ++level) {
    if (klo == khi) break;
    const uint32_t span = khi - klo + 1;
    int shift = 0;
    while (((span - 1) >> shift) >= (uint32_t)NB) ++shift;
    clear_hist(sm);
    const uint32_t lo0 = klo, hi0 = khi;
    row_each(row, V, [&](int, uint32_t h) {
      const uint32_t o = ord16(h);
      if (o >= lo0 && o <= hi0) {
        const int sb = (int)((hi0 - o) >> shift);
        atomicAdd(&sm.hcnt[sb], 1u);
        if (k == 0) add_mass(sm, sb, __fsub_rn(m, scaled(h, inv_temp)));
      }
    });
    __syncthreads();
    find_boundary(k, P, c_above, w_above, sm);
    b = sm.bsel;
    if (b < 0) return Sel{0ull, k > 0 ? 0ull : sm.ctot_w + w_above};  // unreachable for a consistent histogram
    n = sm.n_sel;
    c_above = sm.c_above;
    w_above = sm.w_above;
    const uint32_t nhi = khi - ((uint32_t)b << shift);
    const uint32_t width = 1u << shift;
    const uint32_t nlo = (nhi - klo + 1 > width) ? nhi - width + 1 : klo;
    klo = nlo;
    khi = nhi;
    if (n <= (uint32_t)CAND) {
      const uint32_t lo = klo, hi = khi;
      collect(row, V, [&](int, uint32_t, uint32_t o) { return o >= lo && o <= hi; }, sm);
      return sort_and_walk((int)n, k, P, c_above, w_above, m, inv_temp, sm);
    }
  }
  return resolve_ties(row, V, khi, n, k, P, c_above, w_above, m, inv_temp, sm);
}

struct RowStats {
  float m, Z, lo;
};

// need_z: top-p alone needs Z; top-k only needs m and the smallest value.
__device__ RowStats row_stats(const uint16_t* row, int V, float inv_temp, bool need_z) {
  MaxSum ms{-INFINITY, 0.f};
  float lo = INFINITY;
  row_vecs(row, V, [&](int, const uint4& w) {
    const uint32_t p[4] = {w.x, w.y, w.z, w.w};
    float y[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      y[2 * j] = scaled(p[j] & 0xFFFFu, inv_temp);
      y[2 * j + 1] = scaled(p[j] >> 16, inv_temp);
    }
    float mx = y[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) mx = fmaxf(mx, y[j]);
    if (mx == -INFINITY) return;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (y[j] != -INFINITY) lo = fminf(lo, y[j]);
    if (need_z) {
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) s += __expf(y[j] - mx);
      ms = ms_merge(ms, MaxSum{mx, s});
    } else {
      ms.m = fmaxf(ms.m, mx);
    }
  });
  ms = block_maxsum(ms);
  const float mlo = -block_max(-lo);
  return RowStats{ms.m, ms.s, mlo};
}

// Block sum of 64-bit values in a fixed order (deterministic).
__device__ u64 block_sum_u64(u64 v, FiltSmem& sm) {
  uint32_t unused;
  u64 excl;
  scan2(0u, v, unused, excl, sm);
  return sm.ctot_w;
}

// Exact kept mass of the tokens with key >= K.
__device__ u64 kept_mass(const uint16_t* row, int V, float inv_temp, float m, u64 K, FiltSmem& sm) {
  u64 acc = 0;
  const KeyCut cut(K);
  row_each(row, V, [&](int i, uint32_t h) {
    if (cut.keeps(ord16(h), i)) acc += wfix(__fsub_rn(m, scaled(h, inv_temp)));
  });
  const u64 tot = block_sum_u64(acc, sm);
  return tot;
}

__device__ __forceinline__ float key_dist(u64 K, float m, float inv_temp) {
  return __fsub_rn(m, scaled(unord16((uint32_t)(K >> 32)), inv_temp));
}

// Top-k then top-p (either may be off: k == 0, top_p >= 1).  S of the result
// is 0 when only the count criterion ran.
__device__ Sel filtered_select(const uint16_t* row, int V, float inv_temp, int k, float top_p, const RowStats& st,
                               FiltSmem& sm) {
  const float dfull = st.m - st.lo;
  if (k > 0) {
    Sel s = select_tokens(row, V, inv_temp, st.m, dfull, k, 0ull, sm);
    s.S = 0;  // the count criterion forms no mass above its boundary bin
    if (top_p < 1.f) {
      const u64 Sk = kept_mass(row, V, inv_temp, st.m, s.K, sm);
      const u64 P = (u64)((double)top_p * (double)Sk);
      // the nucleus lies inside the top-k set, whose last token is at distance key_dist(K)
      s = select_tokens(row, V, inv_temp, st.m, fminf(dfull, key_dist(s.K, st.m, inv_temp)), 0, P, sm);
    }
    return s;
  }
  const u64 P = (u64)((double)top_p * (double)st.Z * (double)FIX);
  const float bound = __logf((float)V / ((1.f - top_p) * fmaxf(st.Z, 1.f))) + 1.f;
  return select_tokens(row, V, inv_temp, st.m, fminf(dfull, bound), 0, P, sm);
}

__device__ __forceinline__ float sel_mass(const Sel& s) { return (float)((double)s.S / (double)FIX); }

}  // namespace

__global__ void __launch_bounds__(FT, 1)
    filtered_sample_kernel(const uint16_t* __restrict__ x, RowMap rm, int V, float inv_temp, int k, float top_p,
                           uint32_t seed, uint32_t offset, int64_t* __restrict__ tokens, int64_t* __restrict__ params) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  FiltSmem& sm = *reinterpret_cast<FiltSmem*>(smem_raw);
  const int r = blockIdx.x;
  const uint16_t* row = x + rm.off(r);
  const RowStats st = row_stats(row, V, inv_temp, k == 0);
  const Sel s = filtered_select(row, V, inv_temp, k, top_p, st, sm);
  const KeyCut cut(s.K);
  ArgBest best{-INFINITY, 0x7fffffff};
  u64 acc = 0;
  row_each(row, V, [&](int i, uint32_t h) {
    if (cut.keeps(ord16(h), i)) {
      const float y = scaled(h, inv_temp);
      acc += wfix(__fsub_rn(st.m, y));
      best = better(best, ArgBest{y + gumbel1(seed, offset, r, 4u, i), i});
    }
  });
  best = block_best(best);
  const u64 S_fix = block_sum_u64(acc, sm);
  if (threadIdx.x == 0) {
    tokens[r] = best.i;
    params[2 * r] = (int64_t)s.K;
    const float S = sel_mass(Sel{s.K, S_fix});
    params[2 * r + 1] = (int64_t)(((u64)__float_as_uint(S) << 32) | (u64)__float_as_uint(st.m));
  }
}

__global__ void __launch_bounds__(FT, 1)
    filtered_verify_kernel(const uint16_t* __restrict__ clean, RowMap cm_, const uint16_t* __restrict__ draft,
                           RowMap dm_, const int64_t* __restrict__ dparams, const int64_t* __restrict__ spec, int V,
                           float inv_temp, int k, float top_p, uint32_t seed, uint32_t offset,
                           int32_t* __restrict__ accepted, int64_t* __restrict__ corr) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  FiltSmem& sm = *reinterpret_cast<FiltSmem*>(smem_raw);
  const int r = blockIdx.x;
  const uint16_t* c = clean + cm_.off(r);
  const uint16_t* d = draft + dm_.off(r);
  const RowStats st = row_stats(c, V, inv_temp, k == 0);
  Sel sc = filtered_select(c, V, inv_temp, k, top_p, st, sm);
  if (sc.S == 0) sc.S = kept_mass(c, V, inv_temp, st.m, sc.K, sm);
  const u64 Kc = sc.K, Kd = (u64)dparams[2 * r];
  const u64 packed = (u64)dparams[2 * r + 1];
  const float md = __uint_as_float((uint32_t)packed), Sd = __uint_as_float((uint32_t)(packed >> 32));
  const float mc = st.m, Sc = sel_mass(sc);
  const float ic = 1.f / Sc, id = 1.f / Sd;
  const int64_t s = spec[r];
  const bool s_ok = s >= 0 && s < V;  // an out-of-range draft token has probability 0 and is rejected
  const uint32_t hs = s_ok ? c[s] : 0u, hd = s_ok ? d[s] : 0u;
  const KeyCut cc(Kc), cd(Kd);
  const float ps = s_ok && cc.keeps(ord16(hs), (int)s) ? __expf(scaled(hs, inv_temp) - mc) * ic : 0.f;
  const float qs = s_ok && cd.keeps(ord16(hd), (int)s) ? __expf(scaled(hd, inv_temp) - md) * id : 0.f;
  const float ratio = qs > 0.f ? ps / qs : 0.f;
  const Philox4 ur = philox4x32_10(0u, (uint32_t)r, 5u, 0u, seed, offset);
  if (u01(ur.x) < fminf(ratio, 1.f)) {
    if (threadIdx.x == 0) {
      accepted[r] = 1;
      corr[r] = 0;
    }
    return;
  }
  // residual max(p - q, 0): both rows in one pass, exps only for kept tokens
  const int nvec = V >> 3;
  ArgBest best{-INFINITY, 0x7fffffff};
  for (int kk = threadIdx.x; kk < nvec; kk += FT) {
    const uint4 wc = *reinterpret_cast<const uint4*>(c + (int64_t)kk * 8);
    const uint4 wd = *reinterpret_cast<const uint4*>(d + (int64_t)kk * 8);
    const uint32_t pc[4] = {wc.x, wc.y, wc.z, wc.w}, pd[4] = {wd.x, wd.y, wd.z, wd.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = kk * 8 + j;
      const uint32_t h1 = (j & 1) ? pc[j >> 1] >> 16 : pc[j >> 1] & 0xFFFFu;
      if (!cc.keeps(ord16(h1), i)) continue;
      const uint32_t h2 = (j & 1) ? pd[j >> 1] >> 16 : pd[j >> 1] & 0xFFFFu;
      const float p = __expf(scaled(h1, inv_temp) - mc) * ic;
      const float q = cd.keeps(ord16(h2), i) ? __expf(scaled(h2, inv_temp) - md) * id : 0.f;
      const float res = p - q;
      if (res > 0.f) best = better(best, ArgBest{__logf(res) + gumbel1(seed, offset, r, 6u, i), i});
    }
  }
  best = block_best(best);
  if (best.i == 0x7fffffff) {  // p == q on the support: sample p itself
    best = ArgBest{-INFINITY, 0x7fffffff};
    row_each(c, V, [&](int i, uint32_t h) {
      if (cc.keeps(ord16(h), i))
        best = better(best, ArgBest{scaled(h, inv_temp) + gumbel1(seed, offset, r, 6u, i), i});
    });
    best = block_best(best);
  }
  if (threadIdx.x == 0) {
    accepted[r] = 0;
    corr[r] = best.i == 0x7fffffff ? s : best.i;
  }
}

namespace {
void filtered_smem_attr() {
  static int done_mask = 0;
  int dev = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 31 && (done_mask >> dev) & 1) return;
  C10_CUDA_CHECK(cudaFuncSetAttribute(filtered_sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)sizeof(FiltSmem)));
  C10_CUDA_CHECK(cudaFuncSetAttribute(filtered_verify_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)sizeof(FiltSmem)));
  if (dev < 31) done_mask |= 1 << dev;
}
}  // namespace

void filtered_sample_launch(const at::Tensor& x, double inv_temp, int64_t k, double top_p, int64_t seed,
                            int64_t offset, at::Tensor& tokens, at::Tensor& params) {
  check_dev(x, "logits");
  check_dev(tokens, "tokens");
  check_dev(params, "params");
  int rows, V;
  RowMap m = row_map(x, rows, V);  // bf16, unit stride, strides % 8, 16-byte aligned
  TORCH_CHECK(V % 8 == 0 && V < (1 << 18), "filtered_sample: the vocabulary must be a multiple of 8 below 2^18 "
              "(the 14-bit mass limbs of a bin sum without carries up to 2^18 tokens)");
  TORCH_CHECK(k >= 0 && k < V, "top_k must be in [0, V)");
  TORCH_CHECK(top_p > 0.0 && top_p <= 1.0, "top_p must be in (0, 1]");
  TORCH_CHECK(k > 0 || top_p < 1.0, "filtered_sample needs top_k or top_p");
  TORCH_CHECK(tokens.scalar_type() == at::kLong && tokens.is_contiguous() && tokens.numel() == rows,
              "tokens: int64 [rows]");
  TORCH_CHECK(params.scalar_type() == at::kLong && params.is_contiguous() && params.numel() == 2 * (int64_t)rows,
              "params: int64 [rows, 2]");
  if (rows == 0) return;
  filtered_smem_attr();
  filtered_sample_kernel<<<rows, FT, sizeof(FiltSmem), cur_stream()>>>(
      reinterpret_cast<const uint16_t*>(x.data_ptr()), m, V, (float)inv_temp, (int)k, (float)top_p,
      (uint32_t)seed, (uint32_t)offset, tokens.data_ptr<int64_t>(), params.data_ptr<int64_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void filtered_verify_launch(const at::Tensor& clean, const at::Tensor& draft, const at::Tensor& dparams,
                            const at::Tensor& spec, double inv_temp, int64_t k, double top_p, int64_t seed,
                            int64_t offset, at::Tensor& accepted, at::Tensor& corr) {
  check_dev(clean, "clean");
  check_dev(draft, "draft");
  check_dev(dparams, "draft params");
  check_dev(spec, "spec");
  check_dev(accepted, "accepted");
  check_dev(corr, "corr");
  int rows, V, rows2, V2;
  RowMap cm = row_map(clean, rows, V);
  RowMap dm = row_map(draft, rows2, V2);
  TORCH_CHECK(rows == rows2 && V == V2 && spec.numel() == rows, "filtered_verify shapes");
  TORCH_CHECK(V % 8 == 0 && V < (1 << 18), "filtered_verify: the vocabulary must be a multiple of 8 below 2^18");
  TORCH_CHECK(k >= 0 && k < V && top_p > 0.0 && top_p <= 1.0 && (k > 0 || top_p < 1.0),
              "filtered_verify needs top_k in (0, V) or top_p in (0, 1)");
  TORCH_CHECK(dparams.scalar_type() == at::kLong && dparams.is_contiguous() && dparams.numel() == 2 * (int64_t)rows,
              "draft params: int64 [rows, 2]");
  TORCH_CHECK(spec.scalar_type() == at::kLong && spec.is_contiguous(), "spec: contiguous int64");
  TORCH_CHECK(accepted.scalar_type() == at::kInt && corr.scalar_type() == at::kLong && accepted.is_contiguous() &&
                  corr.is_contiguous() && accepted.numel() == rows && corr.numel() == rows,
              "accepted int32 / corr int64 [rows]");
  if (rows == 0) return;
  filtered_smem_attr();
  filtered_verify_kernel<<<rows, FT, sizeof(FiltSmem), cur_stream()>>>(
      reinterpret_cast<const uint16_t*>(clean.data_ptr()), cm, reinterpret_cast<const uint16_t*>(draft.data_ptr()),
      dm, dparams.data_ptr<int64_t>(), spec.data_ptr<int64_t>(), V, (float)inv_temp, (int)k, (float)top_p,
      (uint32_t)seed, (uint32_t)offset, accepted.data_ptr<int32_t>(), corr.data_ptr<int64_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace uno
