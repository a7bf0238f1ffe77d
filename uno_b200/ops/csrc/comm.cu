// Tensor-parallel communication over NVLink peer memory (no NCCL on the hot path).
//
// Symmetric workspace: every TP rank cudaMallocs the same layout and opens its
// peers' allocations through CUDA IPC handles, so a kernel can store into any
// rank's memory directly.  Layout of each rank's workspace (bytes):
//   [0, 4096)                 control words: epoch counter, CTA arrival
//                             counter, arrive flags [8], done flags [8]
//   [4096, +recv_bytes)       receive slots: recv[src][R][H] bf16 partial rows
//                             that rank `src` computed for the rows this rank owns
//   [.., +gather_bytes)       gathered activations [T][H] bf16 (every rank's
//                             normalised rows, written by their owners)
//
// Row ownership: with T rows and tp ranks, rank r owns rows [r*R, (r+1)*R),
// R = ceil(T / tp).  The residual stream stays sharded by rows.
//
// A row-parallel projection (o_proj, down_proj) and the vocab-parallel
// embedding write their partial rows straight into the owner's receive slot
// from their epilogue (P2P stores), which overlaps the transfer with the GEMM
// tile by tile.  reduce_norm_gather_kernel then, per launch:
//   1. CTA 0 publishes "my partials are written" to every peer (system-scope
//      release), and every CTA waits for all peers' flags (bounded spin);
//   2. each owned row: sum of the tp partial slots (+ residual shard) ->
//      residual shard; RMSNorm -> bf16 row stored into every rank's gathered
//      buffer (P2P broadcast);
//   3. the last CTA to finish publishes "done" and waits for every peer's done
//      flag, so the next (column-parallel) GEMM can read the gathered buffer
//      locally and the receive slots may be rewritten.
// Flags carry a per-rank device epoch (2e+1 arrive, 2e+2 done) advanced by the
// kernel itself, so the kernel can be captured in a CUDA graph and replayed.
// Every wait is bounded; on timeout the kernel sets the error word (code 3)
// and returns instead of hanging.
#include "common.cuh"
#include "uno_ops.h"

namespace uno {

constexpr int MAX_TP = 8;
constexpr uint64_t kPeerWaitNs = 5000000000ull;  // 5 s

struct CommCtl {
  unsigned long long epoch;
  unsigned int cta_count;
  unsigned int pad;
  unsigned long long arrive[MAX_TP];
  unsigned long long done[MAX_TP];
};

static_assert(offsetof(CommCtl, epoch) == COMM_EPOCH_OFF && offsetof(CommCtl, done) == COMM_DONE_OFF,
              "control block layout shared with the GEMM");

struct RsParams {
  uint8_t* peers[MAX_TP];       // base of every rank's workspace (own included)
  int tp, rank;
  int T, R, H;                  // rows, rows per rank, hidden
  int recv_off, gather_off;     // byte offsets inside the workspace
  __nv_bfloat16* residual;      // [R, H] this rank's residual shard (in/out)
  int add_residual;             // 0: first layer (residual := sum)
  const __nv_bfloat16* weight;  // RMSNorm weight [H]
  int groups;
  float eps;
  int wait_all;                 // 1: return only after every rank's rows have arrived
  int* err;
};

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ bool wait_flags(const unsigned long long* flags, int tp, unsigned long long target, int* err) {
  uint64_t start = 0;
  for (int j = 0; j < tp; ++j) {
    while (ld_acquire_sys(flags + j) < target) {
      if (start == 0) start = globaltimer_ns();
      if (globaltimer_ns() - start > kPeerWaitNs) {
        set_error(err, 3);
        return false;
      }
    }
  }
  return true;
}

// One CTA per owned row chunk; each thread owns 8 columns of a row.
__global__ void __launch_bounds__(512) reduce_norm_gather_kernel(RsParams p) {
  CommCtl* ctl = reinterpret_cast<CommCtl*>(p.peers[p.rank]);
  __shared__ unsigned long long s_epoch;
  __shared__ int s_ok;
  __shared__ float red[64];
  pdl_wait();  // this rank's GEMM (its partial rows, its fence) has completed
  if (threadIdx.x == 0) {
    const unsigned long long e = *((volatile unsigned long long*)&ctl->epoch);
    s_epoch = e;
    if (blockIdx.x == 0) {
      __threadfence_system();
      for (int j = 0; j < p.tp; ++j) {
        CommCtl* peer = reinterpret_cast<CommCtl*>(p.peers[j]);
        st_release_sys(&peer->arrive[p.rank], 2 * e + 1);
      }
    }
    s_ok = wait_flags(ctl->arrive, p.tp, 2 * e + 1, p.err);
  }
  __syncthreads();
  const unsigned long long epoch = s_epoch;
  const int H = p.H;
  const int nvec = H / 8;
  const int lo = p.rank * p.R;
  const int rows = max(0, min(p.R, p.T - lo));
  if (s_ok) {
    const __nv_bfloat16* recv = reinterpret_cast<const __nv_bfloat16*>(p.peers[p.rank] + p.recv_off);
    for (int lr = blockIdx.x; lr < rows; lr += gridDim.x) {
      float v[8];
      bool active = threadIdx.x < nvec;
      if (active) {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.f;
        for (int src = 0; src < p.tp; ++src) {
          const uint4 w = reinterpret_cast<const uint4*>(recv + ((size_t)src * p.R + lr) * H)[threadIdx.x];
          const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(h2[i]);
            v[2 * i] += f.x;
            v[2 * i + 1] += f.y;
          }
        }
        // the partial sum is rounded like a bf16 all-reduce result
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = bf16r(v[i]);
        uint4* res = reinterpret_cast<uint4*>(p.residual + (size_t)lr * H);
        if (p.add_residual) {
          const uint4 rr = res[threadIdx.x];
          const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&rr);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(r2[i]);
            v[2 * i] += f.x;
            v[2 * i + 1] += f.y;
          }
        }
        uint4 out;
        out.x = pack_bf16x2(v[0], v[1]);
        out.y = pack_bf16x2(v[2], v[3]);
        out.z = pack_bf16x2(v[4], v[5]);
        out.w = pack_bf16x2(v[6], v[7]);
        res[threadIdx.x] = out;
        if (p.groups > 1 || !p.add_residual) {
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = bf16r(v[i]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.f;
      }
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
      float inv;
      if (p.groups == 1) {
        ss = warp_sum(ss);
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        if (warp == 0) {
          float t = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
          t = warp_sum(t);
          if (lane == 0) red[32] = t;
        }
        __syncthreads();
        inv = rsqrtf(red[32] / H + p.eps);
        __syncthreads();
      } else {
        // threads of a group are contiguous (group size / 8 threads); reduce with shuffles
        const int per = (H / p.groups) / 8;
        float t = ss;
        for (int o = 1; o < per && o < 32; o <<= 1) t += __shfl_xor_sync(0xffffffff, t, o);
        if (per > 32) {  // groups wider than a warp: combine warp sums
          const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
          if (lane == 0) red[warp] = t;
          __syncthreads();
          const int wpg = per / 32, g0 = (warp / wpg) * wpg;
          t = 0.f;
          for (int k = 0; k < wpg; ++k) t += red[g0 + k];
          __syncthreads();
        }
        inv = rsqrtf(t / (H / p.groups) + p.eps);
      }
      if (active) {
        const uint4 wr = reinterpret_cast<const uint4*>(p.weight)[threadIdx.x];
        const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&wr);
        float o[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __bfloat1622float2(w2[i]);
          o[2 * i] = bf16r(bf16r(v[2 * i] * inv) * f.x);
          o[2 * i + 1] = bf16r(bf16r(v[2 * i + 1] * inv) * f.y);
        }
        uint4 out;
        out.x = pack_bf16x2(o[0], o[1]);
        out.y = pack_bf16x2(o[2], o[3]);
        out.z = pack_bf16x2(o[4], o[5]);
        out.w = pack_bf16x2(o[6], o[7]);
        const size_t goff = (size_t)p.gather_off + ((size_t)(lo + lr) * H) * 2;
        for (int j = 0; j < p.tp; ++j) reinterpret_cast<uint4*>(p.peers[j] + goff)[threadIdx.x] = out;
      }
    }
  }
  // ---- completion: the last CTA publishes "done" and waits for every peer
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned int prev = atomicAdd(&ctl->cta_count, 1u);
    if (prev == gridDim.x - 1) {
      ctl->cta_count = 0;
      for (int j = 0; j < p.tp; ++j) {
        CommCtl* peer = reinterpret_cast<CommCtl*>(p.peers[j]);
        st_release_sys(&peer->done[p.rank], 2 * epoch + 2);
      }
      // Normally no wait here: the GEMM that reads the gathered rows waits for
      // exactly their owners' done flags (wait_row_owners), tile by tile.  The
      // last norm of a forward waits for all of them, since its rows leave the
      // fused path (row selection, host reads, the next forward's scatter).
      if (p.wait_all) {
        wait_flags(ctl->done, p.tp, 2 * epoch + 2, p.err);
        asm volatile("fence.proxy.async.global;" ::: "memory");
      }
      ctl->epoch = epoch + 1;
      __threadfence();
    }
  }
}

// Vocab-parallel embedding with the reduce-scatter send fused in: the partial
// row (zero when the id is outside this rank's vocab shard) goes straight into
// the owner's receive slot.
__global__ void embedding_scatter_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                                         int64_t start, int64_t rows, int H, RsParams p) {
  const int t = blockIdx.x;
  pdl_wait();
  const int64_t id = ids[t] - start;
  const bool ok = id >= 0 && id < rows;
  const int owner = t / p.R, lr = t % p.R;
  const uint4* src = reinterpret_cast<const uint4*>(table + (ok ? id : 0) * (int64_t)H);
  uint4* dst = reinterpret_cast<uint4*>(p.peers[owner] + p.recv_off + (((size_t)p.rank * p.R + lr) * H) * 2);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = ok ? src[i] : make_uint4(0, 0, 0, 0);
  __threadfence_system();
}

// ------------------------------------------------------------------ host
static RsParams make_params(const std::vector<int64_t>& peers, int64_t rank, int64_t T, int64_t H, int64_t recv_off,
                            int64_t gather_off) {
  RsParams p{};
  const int tp = (int)peers.size();
  TORCH_CHECK(tp >= 1 && tp <= MAX_TP, "tp must be in [1, 8]");
  TORCH_CHECK(H % 8 == 0 && H / 8 <= 512, "hidden size must be a multiple of 8 and <= 4096");
  for (int j = 0; j < tp; ++j) p.peers[j] = reinterpret_cast<uint8_t*>(peers[j]);
  p.tp = tp;
  p.rank = (int)rank;
  p.T = (int)T;
  p.R = (int)((T + tp - 1) / tp);
  p.H = (int)H;
  p.recv_off = (int)recv_off;
  p.gather_off = (int)gather_off;
  p.err = device_error_flag();
  return p;
}

void reduce_norm_gather_launch(const std::vector<int64_t>& peers, int64_t rank, int64_t T, int64_t H,
                               int64_t recv_off, int64_t gather_off, at::Tensor& residual, bool add_residual,
                               const at::Tensor& weight, int64_t groups, double eps, bool wait_all) {
  check_dev(residual, "residual shard");
  check_dev(weight, "norm weight");
  RsParams p = make_params(peers, rank, T, H, recv_off, gather_off);
  TORCH_CHECK(residual.is_contiguous() && residual.numel() >= (int64_t)p.R * H, "residual shard too small");
  TORCH_CHECK(groups >= 1 && H % groups == 0 && ((H / groups) % 8) == 0, "bad RMSNorm group count");
  const int per = (int)(H / groups) / 8;
  TORCH_CHECK(groups == 1 || per <= 32 || per % 32 == 0, "unsupported RMSNorm group width");
  p.residual = reinterpret_cast<__nv_bfloat16*>(residual.data_ptr());
  p.add_residual = add_residual ? 1 : 0;
  p.weight = reinterpret_cast<const __nv_bfloat16*>(weight.data_ptr());
  p.groups = (int)groups;
  p.eps = (float)eps;
  p.wait_all = wait_all ? 1 : 0;
  const int rows = std::max(1, p.R);
  const int grid = std::min(rows, 4 * num_sms());
  const int threads = std::max(64, ((int)(H / 8) + 31) / 32 * 32);
  launch_pdl(reduce_norm_gather_kernel, dim3(grid), dim3(threads), 0, cur_stream(), p);
}

void embedding_scatter_launch(const std::vector<int64_t>& peers, int64_t rank, const at::Tensor& ids,
                              const at::Tensor& table, int64_t start, int64_t recv_off, int64_t gather_off) {
  check_dev(ids, "ids");
  check_dev(table, "embedding table");
  const int64_t T = ids.numel(), H = table.size(1);
  RsParams p = make_params(peers, rank, T, H, recv_off, gather_off);
  if (T == 0) return;
  embedding_scatter_kernel<<<T, 256, 0, cur_stream()>>>(ids.data_ptr<int64_t>(),
                                                       reinterpret_cast<const __nv_bfloat16*>(table.data_ptr()), start,
                                                       table.size(0), (int)H, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// IPC plumbing -----------------------------------------------------------
std::vector<int64_t> symm_alloc(int64_t nbytes) {
  void* ptr = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&ptr, nbytes));
  C10_CUDA_CHECK(cudaMemset(ptr, 0, nbytes));
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, ptr));
  std::vector<int64_t> out;
  out.push_back(reinterpret_cast<int64_t>(ptr));
  const unsigned char* b = reinterpret_cast<const unsigned char*>(&h);
  for (size_t i = 0; i < sizeof(h); ++i) out.push_back(b[i]);
  return out;
}

int64_t symm_open(const std::vector<int64_t>& handle_bytes) {
  cudaIpcMemHandle_t h;
  TORCH_CHECK(handle_bytes.size() == sizeof(h), "bad IPC handle size");
  unsigned char* b = reinterpret_cast<unsigned char*>(&h);
  for (size_t i = 0; i < sizeof(h); ++i) b[i] = (unsigned char)handle_bytes[i];
  void* ptr = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(ptr);
}

void symm_close(int64_t ptr, bool owned) {
  if (ptr == 0) return;
  if (owned)
    cudaFree(reinterpret_cast<void*>(ptr));
  else
    cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr));
}

}  // namespace uno
