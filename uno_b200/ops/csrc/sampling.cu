// Sampling, Psi-Spec verification and draft-tree kernels.
//
// Randomness: element v of row r in call (seed, offset) uses Philox-4x32-10
// with key (seed, offset) and counter (v / 4, r, stream id, 0); the four 32-bit
// outputs serve four consecutive vocabulary entries.  The values depend only on
// (seed, offset, row, v), so every TP rank that makes the same call draws the
// same numbers and a partial vocabulary shard can be sampled consistently.
//
// * argmax_kernel           greedy decoding (lowest index wins ties)
// * gumbel_sample_kernel    categorical sample of softmax(x / T) as
//                           argmax(x / T - log(E)), E ~ Exp(1)
// * fused_verify_kernel     speculative acceptance test + residual resample
//                           from raw target/draft logits (two passes over V);
//                           semantics of ``engine/fused_verify_kernel.py:8-98``
// * topk_lse_kernel         per-row top-K token ids with log-softmax values
//                           (draft-tree candidates, ``engine/tree_builder.py:8-127``)
// * build_tree_kernel       best-first fixed-budget tree, one warp per request
//                           (``engine/tree_builder.py:130-330``)
// * walk_tree_kernel        target-sample walk of the tree (``engine/tree_walk.py:8-146``)
#include "common.cuh"
#include "sampling_common.cuh"
#include "uno_ops.h"

namespace uno {

// ------------------------------------------------------------------ argmax
__global__ void __launch_bounds__(SAMPLE_THREADS) argmax_kernel(const __nv_bfloat16* __restrict__ x, RowMap rm, int V,
                                                               int64_t* __restrict__ out) {
  const __nv_bfloat16* row = x + rm.off(blockIdx.x);
  ArgBest best{-INFINITY, 0x7fffffff};
  const int nvec = V / 8;
  for (int c = threadIdx.x; c < nvec; c += blockDim.x) {
    float v[8];
    load8(row + c * 8, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) best = better(best, ArgBest{v[i], c * 8 + i});
  }
  for (int i = nvec * 8 + threadIdx.x; i < V; i += blockDim.x) best = better(best, ArgBest{__bfloat162float(row[i]), i});
  best = block_best(best);
  if (threadIdx.x == 0) out[blockIdx.x] = best.i;
}

// ---------------------------------------------------------- gumbel sample
__global__ void __launch_bounds__(SAMPLE_THREADS)
    gumbel_sample_kernel(const __nv_bfloat16* __restrict__ x, RowMap rm, int V, float inv_temp, uint32_t seed,
                         uint32_t offset, int64_t* __restrict__ out) {
  const __nv_bfloat16* row = x + rm.off(blockIdx.x);
  ArgBest best{-INFINITY, 0x7fffffff};
  const int nvec = V / 8;
  for (int c = threadIdx.x; c < nvec; c += blockDim.x) {
    float v[8], g[8];
    load8(row + c * 8, v);
    gumbel8(seed, offset, blockIdx.x, 1u, c * 8, g);
#pragma unroll
    for (int i = 0; i < 8; ++i) best = better(best, ArgBest{v[i] * inv_temp + g[i], c * 8 + i});
  }
  for (int i = nvec * 8 + threadIdx.x; i < V; i += blockDim.x)
    best = better(best, ArgBest{__bfloat162float(row[i]) * inv_temp + gumbel1(seed, offset, blockIdx.x, 1u, i), i});
  best = block_best(best);
  if (threadIdx.x == 0) out[blockIdx.x] = best.i;
}

// ------------------------------------------------------------ fused verify
__global__ void __launch_bounds__(SAMPLE_THREADS)
    fused_verify_kernel(const __nv_bfloat16* __restrict__ clean, RowMap cm_, const __nv_bfloat16* __restrict__ draft,
                        RowMap dm_, const int64_t* __restrict__ spec, int V, float inv_temp, uint32_t seed,
                        uint32_t offset, int32_t* __restrict__ accepted, int64_t* __restrict__ corr) {
  const int r = blockIdx.x;
  const __nv_bfloat16* c = clean + cm_.off(r);
  const __nv_bfloat16* d = draft + dm_.off(r);
  const int nvec = V / 8;
  // pass 1: softmax statistics of both rows (one read of each)
  float cm, cs, dm, ds;
  row_stats2(c, d, V, inv_temp, cm, cs, dm, ds);
  const int64_t s = spec[r];
  const float ps = __expf(__bfloat162float(c[s]) * inv_temp - cm) / cs;
  const float qs = __expf(__bfloat162float(d[s]) * inv_temp - dm) / ds;
  const float ratio = qs > 0.f ? ps / qs : 0.f;
  Philox4 ur = philox4x32_10(0u, (uint32_t)r, 2u, 0u, seed, offset);
  const float u = u01(ur.x);
  const bool acc = (ratio >= 1.f) || (u < ratio);
  if (acc) {
    if (threadIdx.x == 0) {
      accepted[r] = 1;
      corr[r] = 0;
    }
    return;
  }
  // pass 2: Gumbel-max over log(max(p - q, 0))
  const float cinv = 1.f / cs, dinv = 1.f / ds;
  ArgBest best{-INFINITY, 0x7fffffff};
  for (int k = threadIdx.x; k < nvec; k += blockDim.x) {
    float a[8], b[8], g[8];
    load8(c + k * 8, a);
    load8(d + k * 8, b);
    gumbel8(seed, offset, r, 3u, k * 8, g);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float res = __expf(a[i] * inv_temp - cm) * cinv - __expf(b[i] * inv_temp - dm) * dinv;
      if (res > 0.f) best = better(best, ArgBest{__logf(res) + g[i], k * 8 + i});
    }
  }
  for (int i = nvec * 8 + threadIdx.x; i < V; i += blockDim.x) {
    const float res = __expf(__bfloat162float(c[i]) * inv_temp - cm) * cinv -
                      __expf(__bfloat162float(d[i]) * inv_temp - dm) * dinv;
    if (res > 0.f) best = better(best, ArgBest{__logf(res) + gumbel1(seed, offset, r, 3u, i), i});
  }
  best = block_best(best);
  if (threadIdx.x == 0) {
    accepted[r] = 0;
    corr[r] = best.i == 0x7fffffff ? s : best.i;
  }
}

// ----------------------------------------------------------- top-K + LSE
// One CTA per draft row.  Each thread keeps a sorted local top-K of its strided
// slice; the CTA then extracts the global top-K by K rounds of block argmax.
constexpr int TOPK_MAX = 32;
constexpr int TOPK_THREADS = 256;

__global__ void __launch_bounds__(TOPK_THREADS)
    topk_lse_kernel(const __nv_bfloat16* __restrict__ x, int64_t ld, int V, int K, float inv_temp,
                    int64_t* __restrict__ top_ids, float* __restrict__ top_lp) {
  __shared__ float cand_v[TOPK_THREADS * 8];
  __shared__ int cand_i[TOPK_THREADS * 8];
  const __nv_bfloat16* row = x + (size_t)blockIdx.x * ld;
  // local top-min(K,8) per thread, kept sorted descending
  const int L = K < 8 ? K : 8;
  float lv[8];
  int li[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    lv[i] = -INFINITY;
    li[i] = 0x7fffffff;
  }
  float m = -INFINITY;
  for (int v = threadIdx.x; v < V; v += blockDim.x) {
    const float val = __bfloat162float(row[v]) * inv_temp;
    m = fmaxf(m, val);
    if (val > lv[L - 1] || (val == lv[L - 1] && v < li[L - 1])) {
      int pos = L - 1;
      while (pos > 0 && (val > lv[pos - 1] || (val == lv[pos - 1] && v < li[pos - 1]))) {
        lv[pos] = lv[pos - 1];
        li[pos] = li[pos - 1];
        --pos;
      }
      lv[pos] = val;
      li[pos] = v;
    }
  }
  m = block_max(m);
  float s = 0.f;
  for (int v = threadIdx.x; v < V; v += blockDim.x) s += __expf(__bfloat162float(row[v]) * inv_temp - m);
  s = block_sum(s);
  const float lse = m + __logf(s);
  // A thread contributes at most L candidates; if K > L a thread could own
  // more than L of the global top-K, so rescan in that case (K > 8 is rare).
  if (K > L) {
    // fallback: K rounds of exclusion argmax over the whole row
    float last_v = INFINITY;
    int last_i = -1;
    for (int k = 0; k < K; ++k) {
      ArgBest best{-INFINITY, 0x7fffffff};
      for (int v = threadIdx.x; v < V; v += blockDim.x) {
        const float val = __bfloat162float(row[v]) * inv_temp;
        const bool after = (val < last_v) || (val == last_v && v > last_i);
        if (after) best = better(best, ArgBest{val, v});
      }
      best = block_best(best);
      if (threadIdx.x == 0) {
        top_ids[(size_t)blockIdx.x * K + k] = best.i;
        top_lp[(size_t)blockIdx.x * K + k] = best.v - lse;
      }
      last_v = best.v;
      last_i = best.i;
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    cand_v[threadIdx.x * 8 + i] = lv[i];
    cand_i[threadIdx.x * 8 + i] = li[i];
  }
  __syncthreads();
  for (int k = 0; k < K; ++k) {
    ArgBest best{-INFINITY, 0x7fffffff};
    int slot = -1;
    for (int j = threadIdx.x; j < TOPK_THREADS * 8; j += blockDim.x) {
      ArgBest c{cand_v[j], cand_i[j]};
      ArgBest nb = better(best, c);
      if (nb.i != best.i || nb.v != best.v) {
        best = nb;
        slot = j;
      }
    }
    ArgBest win = block_best(best);
    if (best.i == win.i && best.v == win.v && slot >= 0 && win.i != 0x7fffffff) {
      cand_v[slot] = -INFINITY;
      cand_i[slot] = 0x7fffffff;
    }
    if (threadIdx.x == 0) {
      top_ids[(size_t)blockIdx.x * K + k] = win.i;
      top_lp[(size_t)blockIdx.x * K + k] = win.v - lse;
    }
    __syncthreads();
  }
}

// --------------------------------------------------------------- tree build
// One warp per request.  Node n's next candidate is its lowest-rank unused
// child among the depth-d top-K list (children are added in rank order), so the
// global best candidate is the best head over all nodes.  Priority: larger
// cumulative log-prob, then smaller depth, rank, token id, parent index.
__global__ void build_tree_kernel(const int64_t* __restrict__ roots, const int64_t* __restrict__ cand_ids,
                                  const float* __restrict__ cand_lp, int D, int K, int Qn,
                                  int64_t* __restrict__ tok, int64_t* __restrict__ par, int64_t* __restrict__ dep,
                                  float* __restrict__ mass, int* __restrict__ count_out) {
  const int b = blockIdx.x, lane = threadIdx.x;
  __shared__ int s_ptr[64];
  __shared__ int s_dep[64];
  __shared__ float s_mass[64];
  const int64_t* ids = cand_ids + (size_t)b * D * K;
  const float* lps = cand_lp + (size_t)b * D * K;
  int64_t* T = tok + (size_t)b * Qn;
  int64_t* P = par + (size_t)b * Qn;
  int64_t* Dp = dep + (size_t)b * Qn;
  float* Ms = mass + (size_t)b * Qn;
  if (lane == 0) {
    T[0] = roots[b];
    P[0] = -1;
    Dp[0] = 0;
    Ms[0] = 0.f;
  }
  for (int i = lane; i < 64; i += 32) {
    s_ptr[i] = 0;
    s_dep[i] = 0;
    s_mass[i] = 0.f;
  }
  __syncwarp();
  int n = 1;
  for (; n < Qn; ++n) {
    // each lane examines nodes lane and lane + 32
    float bv = -INFINITY;
    int bd = 0x7fffffff, br = 0x7fffffff, bnode = -1;
    int64_t btok = 0x7fffffffffffffffll;
    for (int node = lane; node < n; node += 32) {
      const int d = s_dep[node], r = s_ptr[node];
      if (d >= D || r >= K) continue;
      const float v = s_mass[node] + lps[d * K + r];
      const int64_t t = ids[d * K + r];
      bool take = false;
      if (bnode < 0 || v > bv) take = true;
      else if (v == bv) {
        if (d + 1 < bd) take = true;
        else if (d + 1 == bd) {
          if (r < br) take = true;
          else if (r == br) {
            if (t < btok) take = true;
            else if (t == btok && node < bnode) take = true;
          }
        }
      }
      if (take) {
        bv = v;
        bd = d + 1;
        br = r;
        btok = t;
        bnode = node;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffff, bv, o);
      const int od = __shfl_xor_sync(0xffffffff, bd, o);
      const int orr = __shfl_xor_sync(0xffffffff, br, o);
      const long long ot = __shfl_xor_sync(0xffffffff, (long long)btok, o);
      const int on = __shfl_xor_sync(0xffffffff, bnode, o);
      bool take = false;
      if (on >= 0) {
        if (bnode < 0 || ov > bv) take = true;
        else if (ov == bv) {
          if (od < bd) take = true;
          else if (od == bd) {
            if (orr < br) take = true;
            else if (orr == br) {
              if (ot < btok) take = true;
              else if (ot == btok && on < bnode) take = true;
            }
          }
        }
      }
      if (take) {
        bv = ov;
        bd = od;
        br = orr;
        btok = ot;
        bnode = on;
      }
    }
    if (bnode < 0) break;  // candidate set exhausted
    if (lane == 0) {
      T[n] = btok;
      P[n] = bnode;
      Dp[n] = bd;
      Ms[n] = bv;
      s_ptr[bnode] += 1;
      s_dep[n] = bd;
      s_mass[n] = bv;
      s_ptr[n] = 0;
    }
    __syncwarp();
  }
  if (lane == 0) count_out[b] = n;
  for (int i = n + lane; i < Qn; i += 32) {  // unused slots: unreachable padding
    T[i] = 0;
    P[i] = -2;  // never equals a walk position, never an ancestor
    Dp[i] = 1;
    Ms[i] = -INFINITY;
  }
}

// --------------------------------------------------------------- tree walk
__global__ void walk_tree_kernel(const int64_t* __restrict__ tok, const int64_t* __restrict__ par,
                                 const int64_t* __restrict__ tgt, int Qn, int max_depth, int64_t pad,
                                 int64_t* __restrict__ committed, int64_t* __restrict__ accepted,
                                 int64_t* __restrict__ lengths) {
  const int b = blockIdx.x, lane = threadIdx.x;
  const int n_cached = max_depth + 1;
  const int64_t* T = tok + (size_t)b * Qn;
  const int64_t* P = par + (size_t)b * Qn;
  const int64_t* G = tgt + (size_t)b * Qn;
  int64_t* C = committed + (size_t)b * (n_cached + 1);
  int64_t* A = accepted + (size_t)b * n_cached;
  for (int i = lane; i <= n_cached; i += 32) C[i] = pad;
  for (int i = lane; i < n_cached; i += 32) A[i] = -1;
  __syncwarp();
  int cur = 0;
  int64_t len = 1;
  if (lane == 0) {
    C[0] = T[0];
    A[0] = 0;
  }
  for (int step = 1; step <= n_cached; ++step) {
    const int64_t s = G[cur];
    if (lane == 0) C[step] = s;
    len = step + 1;
    if (step > max_depth) break;
    int child = 0x7fffffff;
    for (int j = lane; j < Qn; j += 32)
      if (P[j] == cur && T[j] == s && j < child) child = j;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) child = min(child, __shfl_xor_sync(0xffffffff, child, o));
    if (child == 0x7fffffff) break;
    if (lane == 0) A[step] = child;
    cur = child;
  }
  if (lane == 0) lengths[b] = len;
}

// ----------------------------------------------------------- cycle payload
// One thread per request: committed tokens of a linear Psi-Spec cycle, then
// their count, in one [B, L+2] int64 row.  Proposals 1..L-1 are accepted left
// to right until the first rejection, which is replaced by its residual
// resample; with every proposal accepted the lookahead sample is the (L+1)-th
// token.  Acceptance comes from the verify kernel (accepted != 0) or, for
// greedy decoding, from proposal == target.  Unless ignore_eos, the row ends
// at its first stop token (kept).  Semantics of the eager assembly it replaces
// (``engine/two_pass_decoding.py`` payload + stop truncation of the reference).
__global__ void cycle_payload_kernel(const int64_t* __restrict__ proposal, const int32_t* __restrict__ accepted,
                                     const int64_t* __restrict__ target, const int64_t* __restrict__ corr,
                                     const int64_t* __restrict__ lookahead, const int64_t* __restrict__ stops,
                                     int n_stops, int B, int L, int64_t* __restrict__ payload) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int64_t* prop = proposal + (size_t)b * L;
  int64_t* out = payload + (size_t)b * (L + 2);
  int len = L + 1;
  for (int i = 0; i < L; ++i) out[i] = prop[i];
  out[L] = lookahead[b];
  for (int i = 0; i + 1 < L; ++i) {
    const bool ok = target != nullptr ? prop[i + 1] == target[(size_t)b * (L - 1) + i]
                                      : accepted[(size_t)b * (L - 1) + i] != 0;
    if (!ok) {
      out[i + 1] = target != nullptr ? target[(size_t)b * (L - 1) + i] : corr[(size_t)b * (L - 1) + i];
      len = i + 2;
      break;
    }
  }
  for (int j = 0; j < len && n_stops > 0; ++j) {
    bool hit = false;
    for (int k = 0; k < n_stops; ++k) hit |= out[j] == stops[k];
    if (hit) {
      len = j + 1;
      break;
    }
  }
  out[L + 1] = len;
}

// One warp per request: ancestor-or-self bitmasks of a draft tree (parents
// before children, root parent -1) and node positions prefix + depth, written
// straight into the forward's metadata buffers.
__global__ void tree_meta_kernel(const int64_t* __restrict__ parents, const int64_t* __restrict__ depths,
                                 const int* __restrict__ prefix, int B, int Q, int64_t* __restrict__ masks,
                                 int64_t* __restrict__ positions) {
  const int b = blockIdx.x;
  if (b >= B || threadIdx.x != 0) return;
  const int64_t* par = parents + (size_t)b * Q;
  int64_t* m = masks + (size_t)b * Q;
  for (int i = 0; i < Q; ++i) {
    const int64_t pa = par[i];
    uint64_t v = 1ull << i;
    if (pa >= 0 && pa < i) v |= (uint64_t)m[pa];
    m[i] = (int64_t)v;
    positions[(size_t)b * Q + i] = (int64_t)prefix[b] + depths[(size_t)b * Q + i];
  }
}

// ------------------------------------------------------------------- host
void cycle_payload_launch(const at::Tensor& proposal, c10::optional<at::Tensor> accepted,
                          c10::optional<at::Tensor> target, c10::optional<at::Tensor> corr, const at::Tensor& lookahead,
                          const at::Tensor& stops, at::Tensor& payload) {
  check_dev(proposal, "proposal");
  check_dev(lookahead, "lookahead");
  check_dev(payload, "payload");
  const int B = proposal.size(0), L = proposal.size(1);
  TORCH_CHECK(proposal.scalar_type() == at::kLong && proposal.is_contiguous(), "proposal: contiguous int64 [B, L]");
  TORCH_CHECK(payload.scalar_type() == at::kLong && payload.is_contiguous() && payload.numel() == (int64_t)B * (L + 2),
              "payload: contiguous int64 [B, L+2]");
  TORCH_CHECK(lookahead.scalar_type() == at::kLong && lookahead.numel() == B, "lookahead: int64 [B]");
  TORCH_CHECK(stops.scalar_type() == at::kLong && (stops.numel() == 0 || stops.is_cuda()), "stops: int64");
  const int64_t* tgt = nullptr;
  const int32_t* acc = nullptr;
  const int64_t* cor = nullptr;
  if (L > 1) {
    if (target.has_value()) {
      check_dev(*target, "target");
      TORCH_CHECK(target->scalar_type() == at::kLong && target->is_contiguous() && target->numel() == (int64_t)B * (L - 1),
                  "target: int64 [B, L-1]");
      tgt = target->data_ptr<int64_t>();
    } else {
      TORCH_CHECK(accepted.has_value() && corr.has_value(), "payload needs accepted + corr or a greedy target");
      check_dev(*accepted, "accepted");
      check_dev(*corr, "corr");
      TORCH_CHECK(accepted->scalar_type() == at::kInt && accepted->is_contiguous() &&
                      accepted->numel() == (int64_t)B * (L - 1), "accepted: int32 [B, L-1]");
      TORCH_CHECK(corr->scalar_type() == at::kLong && corr->is_contiguous() && corr->numel() == (int64_t)B * (L - 1),
                  "corr: int64 [B, L-1]");
      acc = accepted->data_ptr<int32_t>();
      cor = corr->data_ptr<int64_t>();
    }
  }
  if (B == 0) return;
  cycle_payload_kernel<<<(B + 127) / 128, 128, 0, cur_stream()>>>(
      proposal.data_ptr<int64_t>(), acc, tgt, cor, lookahead.data_ptr<int64_t>(),
      stops.numel() ? stops.data_ptr<int64_t>() : nullptr, (int)stops.numel(), B, L, payload.data_ptr<int64_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void tree_meta_launch(const at::Tensor& parents, const at::Tensor& depths, const at::Tensor& prefix, at::Tensor& masks,
                      at::Tensor& positions) {
  check_dev(parents, "parents");
  check_dev(depths, "depths");
  check_dev(prefix, "prefix_lens");
  check_dev(masks, "masks");
  check_dev(positions, "positions");
  const int B = parents.size(0), Q = parents.size(1);
  TORCH_CHECK(Q <= 64, "tree masks support at most 64 nodes");
  TORCH_CHECK(parents.scalar_type() == at::kLong && depths.scalar_type() == at::kLong && parents.is_contiguous() &&
                  depths.is_contiguous() && depths.numel() == (int64_t)B * Q, "parents / depths: int64 [B, Q]");
  TORCH_CHECK(prefix.scalar_type() == at::kInt && prefix.numel() >= B, "prefix_lens: int32 [B]");
  TORCH_CHECK(masks.scalar_type() == at::kLong && positions.scalar_type() == at::kLong &&
                  masks.numel() >= (int64_t)B * Q && positions.numel() >= (int64_t)B * Q,
              "masks / positions: int64 [B * Q]");
  if (B == 0) return;
  tree_meta_kernel<<<B, 32, 0, cur_stream()>>>(parents.data_ptr<int64_t>(), depths.data_ptr<int64_t>(),
                                               prefix.data_ptr<int>(), B, Q, masks.data_ptr<int64_t>(),
                                               positions.data_ptr<int64_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void argmax_launch(const at::Tensor& x, at::Tensor& out) {
  check_dev(x, "logits");
  check_dev(out, "out");
  int rows, V;
  RowMap m = row_map(x, rows, V);
  TORCH_CHECK(out.numel() == rows, "argmax output size");
  if (rows == 0) return;
  argmax_kernel<<<rows, SAMPLE_THREADS, 0, cur_stream()>>>(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), m, V,
                                                           out.data_ptr<int64_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gumbel_sample_launch(const at::Tensor& x, at::Tensor& out, double inv_temp, int64_t seed, int64_t offset) {
  check_dev(x, "logits");
  check_dev(out, "out");
  int rows, V;
  RowMap m = row_map(x, rows, V);
  TORCH_CHECK(out.numel() == rows, "sample output size");
  if (rows == 0) return;
  gumbel_sample_kernel<<<rows, SAMPLE_THREADS, 0, cur_stream()>>>(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
                                                                  m, V, (float)inv_temp, (uint32_t)seed,
                                                                  (uint32_t)offset, out.data_ptr<int64_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void fused_verify_launch(const at::Tensor& clean, const at::Tensor& draft, const at::Tensor& spec, double inv_temp,
                         int64_t seed, int64_t offset, at::Tensor& accepted, at::Tensor& corr) {
  check_dev(clean, "clean");
  check_dev(draft, "draft");
  check_dev(spec, "spec");
  check_dev(accepted, "accepted");
  check_dev(corr, "corr");
  int rows, V, rows2, V2;
  RowMap cm = row_map(clean, rows, V);
  RowMap dm = row_map(draft, rows2, V2);
  TORCH_CHECK(rows == rows2 && V == V2 && spec.numel() == rows, "verify shapes");
  if (rows == 0) return;
  fused_verify_kernel<<<rows, SAMPLE_THREADS, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(clean.data_ptr()), cm,
      reinterpret_cast<const __nv_bfloat16*>(draft.data_ptr()), dm, spec.data_ptr<int64_t>(), V, (float)inv_temp,
      (uint32_t)seed, (uint32_t)offset, accepted.data_ptr<int32_t>(), corr.data_ptr<int64_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void topk_lse_launch(const at::Tensor& x, int K, double inv_temp, at::Tensor& ids, at::Tensor& lp) {
  check_dev(x, "logits");
  check_dev(ids, "ids");
  check_dev(lp, "lp");
  const int rows = x.size(0), V = x.size(1);
  TORCH_CHECK(K >= 1 && K <= TOPK_MAX, "candidate top-k must be in [1, 32]");
  if (rows == 0) return;
  topk_lse_kernel<<<rows, TOPK_THREADS, 0, cur_stream()>>>(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
                                                           x.stride(0), V, K, (float)inv_temp,
                                                           ids.data_ptr<int64_t>(), lp.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void build_tree_launch(const at::Tensor& roots, const at::Tensor& ids, const at::Tensor& lp, int Qn, at::Tensor& tok,
                       at::Tensor& par, at::Tensor& dep, at::Tensor& mass, at::Tensor& count) {
  check_dev(roots, "roots");
  check_dev(ids, "ids");
  check_dev(lp, "lp");
  check_dev(tok, "tok");
  check_dev(par, "par");
  check_dev(dep, "dep");
  check_dev(mass, "mass");
  check_dev(count, "count");
  const int B = ids.size(0), D = ids.size(1), K = ids.size(2);
  TORCH_CHECK(Qn <= 64, "tree verification supports at most 64 nodes");
  if (B == 0) return;
  build_tree_kernel<<<B, 32, 0, cur_stream()>>>(roots.data_ptr<int64_t>(), ids.data_ptr<int64_t>(),
                                                lp.data_ptr<float>(), D, K, Qn, tok.data_ptr<int64_t>(),
                                                par.data_ptr<int64_t>(), dep.data_ptr<int64_t>(),
                                                mass.data_ptr<float>(), count.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void walk_tree_launch(const at::Tensor& tok, const at::Tensor& par, const at::Tensor& tgt, int max_depth, int64_t pad,
                      at::Tensor& committed, at::Tensor& accepted, at::Tensor& lengths) {
  check_dev(tok, "tok");
  check_dev(par, "par");
  check_dev(tgt, "tgt");
  check_dev(committed, "committed");
  check_dev(accepted, "accepted");
  check_dev(lengths, "lengths");
  const int B = tok.size(0), Qn = tok.size(1);
  if (B == 0) return;
  walk_tree_kernel<<<B, 32, 0, cur_stream()>>>(tok.data_ptr<int64_t>(), par.data_ptr<int64_t>(),
                                               tgt.data_ptr<int64_t>(), Qn, max_depth, pad,
                                               committed.data_ptr<int64_t>(), accepted.data_ptr<int64_t>(),
                                               lengths.data_ptr<int64_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace uno
