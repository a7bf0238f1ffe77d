// LoRA optimizer step fused with its collectives over NVLink peer memory.
//
// ZeRO-2 style data parallelism (the reference runs DeepSpeed stage 2 over the
// LoRA parameters: ``training/configs/deepspeed_zero2.json:18-27``, AdamW
// ``training/train.py:285-290``, clip 1.0): every rank holds all fp32 LoRA
// parameters and a full local gradient, but only the Adam moments of its own
// 1/world shard.  One kernel does what is otherwise reduce-scatter -> global
// grad-norm all-reduce -> clip -> AdamW on the shard -> all-gather:
//
//   ready    CTA 0 of each rank tells every peer that this rank's gradient for
//            the step is complete (the backward ran before this kernel on the
//            same stream); every CTA waits for all ranks before reading;
//   phase 1  each rank sums its shard of every rank's gradient (P2P loads from
//            the peers' gradient buffers), scales by 1/world, keeps the result
//            in local scratch and accumulates its squared norm;
//   sync     the last CTA of each rank stores the shard's squared norm into
//            every peer's control block and releases a flag; every CTA waits
//            for all ranks' flags and forms the global norm;
//   phase 2  clip coefficient min(1, max_norm / (norm + 1e-6)), decoupled-decay
//            AdamW with bias correction on the shard, and the updated fp32
//            values are stored into every rank's parameter buffer (P2P);
//   done     the last CTA releases a done flag to every peer and waits until
//            all ranks have delivered their shards, so the parameters are
//            complete on this rank when the kernel ends.
//
// Buffers: ``params`` and ``grads`` are flat fp32 arrays at the same offsets in
// every rank's symmetric workspace; ``ctl`` is an OptCtl at the same offset.
// The grid is at most one CTA per SM so every CTA is resident while others
// wait; all waits are bounded (error code 5).
#include "common.cuh"
#include "uno_ops.h"

namespace uno {

constexpr int OPT_MAX_RANKS = 8;

struct OptCtl {
  unsigned long long epoch;       // steps completed on this rank
  unsigned int count1, count2;    // CTA arrival counters of the two grid syncs
  double sumsq;                   // this rank's shard sum of squares (accumulated by CTAs)
  double norm_part[OPT_MAX_RANKS];          // written by each rank
  unsigned long long norm_flag[OPT_MAX_RANKS];
  unsigned long long done_flag[OPT_MAX_RANKS];
  unsigned long long ready_flag[OPT_MAX_RANKS];  // rank j's gradient of step `value` is complete
};

struct AdamWArgs {
  uint8_t* ws[OPT_MAX_RANKS];  // every rank's workspace base (own included)
  int world, rank;
  int64_t params_off, grads_off, ctl_off;  // byte offsets inside every workspace
  int64_t n;                               // parameters (multiple of world)
  float* m;                                // this rank's moments [n / world]
  float* v;
  float* scratch;                          // reduced gradient of this rank's shard [n / world]
  float lr, beta1, beta2, eps, weight_decay, max_norm;
  float bc1, bc2;                          // 1 - beta^t
  float* norm_out;                         // global gradient norm before clipping
  int* err;
};

__device__ __forceinline__ void st_rel_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ bool opt_wait(const unsigned long long* f, unsigned long long target, int* err) {
  const uint64_t t0 = globaltimer_ns();
  while (ld_acquire_sys_u64(f) < target) {
    if (*reinterpret_cast<volatile int*>(err) != 0) return false;
    if (globaltimer_ns() - t0 > 5000000000ull) {
      set_error(err, 5);
      return false;
    }
  }
  return true;
}

__global__ void __launch_bounds__(512) fused_adamw_kernel(AdamWArgs a) {
  OptCtl* ctl = reinterpret_cast<OptCtl*>(a.ws[a.rank] + a.ctl_off);
  const unsigned long long epoch = *reinterpret_cast<volatile unsigned long long*>(&ctl->epoch);
  const unsigned long long target = epoch + 1;
  const int64_t shard = a.n / a.world;
  const int64_t s0 = shard * a.rank;
  const float inv_world = 1.f / (float)a.world;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  __shared__ double red[32];
  __shared__ float s_coef;

  // ---- ready: no rank reads a peer's gradient before the peer's backward has finished
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0) {
      __threadfence_system();
      for (int j = 0; j < a.world; ++j) {
        OptCtl* peer = reinterpret_cast<OptCtl*>(a.ws[j] + a.ctl_off);
        st_rel_u64(&peer->ready_flag[a.rank], target);
      }
    }
    for (int j = 0; j < a.world; ++j) opt_wait(&ctl->ready_flag[j], target, a.err);
  }
  __syncthreads();

  // ---- phase 1: reduce-scatter of the gradient + shard sum of squares
  double ss = 0.0;
  for (int64_t i = tid; i < shard; i += stride) {
    float g = 0.f;
    for (int j = 0; j < a.world; ++j) {
      const float* gj = reinterpret_cast<const float*>(a.ws[j] + a.grads_off);
      g += __ldcv(gj + s0 + i);  // volatile: peers' memory, never cached here
    }
    g *= inv_world;
    a.scratch[i] = g;
    ss += (double)g * g;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffff, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    atomicAdd(&ctl->sumsq, t);
    __threadfence();
    const unsigned int prev = atomicAdd(&ctl->count1, 1u);
    if (prev == gridDim.x - 1) {
      const double mine = *reinterpret_cast<volatile double*>(&ctl->sumsq);
      ctl->sumsq = 0.0;
      ctl->count1 = 0;
      for (int j = 0; j < a.world; ++j) {
        OptCtl* peer = reinterpret_cast<OptCtl*>(a.ws[j] + a.ctl_off);
        *reinterpret_cast<volatile double*>(&peer->norm_part[a.rank]) = mine;
        st_rel_u64(&peer->norm_flag[a.rank], target);
      }
    }
    // ---- every CTA: wait for all ranks' shard norms
    double total = 0.0;
    for (int j = 0; j < a.world; ++j) {
      opt_wait(&ctl->norm_flag[j], target, a.err);
      total += *reinterpret_cast<volatile double*>(&ctl->norm_part[j]);
    }
    const float norm = (float)sqrt(total);
    s_coef = a.max_norm > 0.f ? fminf(1.f, a.max_norm / (norm + 1e-6f)) : 1.f;
    if (blockIdx.x == 0) *a.norm_out = norm;
  }
  __syncthreads();
  const float coef = s_coef;

  // ---- phase 2: clipped AdamW on the shard, updated values to every rank
  for (int64_t i = tid; i < shard; i += stride) {
    const float g = a.scratch[i] * coef;
    float* pown = reinterpret_cast<float*>(a.ws[a.rank] + a.params_off) + s0 + i;
    float p = *pown;
    const float m = a.beta1 * a.m[i] + (1.f - a.beta1) * g;
    const float v = a.beta2 * a.v[i] + (1.f - a.beta2) * g * g;
    a.m[i] = m;
    a.v[i] = v;
    p -= a.lr * a.weight_decay * p;
    p -= a.lr * (m / a.bc1) / (sqrtf(v / a.bc2) + a.eps);
    for (int j = 0; j < a.world; ++j) reinterpret_cast<float*>(a.ws[j] + a.params_off)[s0 + i] = p;
  }

  // ---- done: publish, then wait for every rank's shard
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned int prev = atomicAdd(&ctl->count2, 1u);
    if (prev == gridDim.x - 1) {
      ctl->count2 = 0;
      for (int j = 0; j < a.world; ++j) {
        OptCtl* peer = reinterpret_cast<OptCtl*>(a.ws[j] + a.ctl_off);
        st_rel_u64(&peer->done_flag[a.rank], target);
      }
      for (int j = 0; j < a.world; ++j) opt_wait(&ctl->done_flag[j], target, a.err);
      *reinterpret_cast<volatile unsigned long long*>(&ctl->epoch) = target;
      __threadfence_system();
    }
  }
}

int64_t opt_ctl_bytes() { return (int64_t)((sizeof(OptCtl) + 255) / 256 * 256); }

void fused_adamw_launch(const std::vector<int64_t>& ws, int64_t rank, int64_t params_off, int64_t grads_off,
                        int64_t ctl_off, int64_t n, at::Tensor& m, at::Tensor& v, at::Tensor& scratch,
                        at::Tensor& norm_out, double lr, double beta1, double beta2, double eps, double weight_decay,
                        double max_norm, int64_t step) {
  const int world = (int)ws.size();
  TORCH_CHECK(world >= 1 && world <= OPT_MAX_RANKS, "fused AdamW supports 1..8 ranks");
  TORCH_CHECK(rank >= 0 && rank < world, "bad rank");
  TORCH_CHECK(n % world == 0, "parameter count must be a multiple of the world size");
  TORCH_CHECK(step >= 1, "AdamW step counts from 1");
  const int64_t shard = n / world;
  at::Tensor* shards[3] = {&m, &v, &scratch};
  for (at::Tensor* t : shards) {
    check_dev(*t, "optimizer state");
    TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() >= shard, "fp32 shard buffer");
  }
  TORCH_CHECK(params_off % 16 == 0 && grads_off % 16 == 0 && ctl_off % 16 == 0, "workspace offsets");
  check_dev(norm_out, "norm output");
  TORCH_CHECK(norm_out.scalar_type() == at::kFloat && norm_out.numel() >= 1, "norm output must be fp32");
  AdamWArgs a{};
  for (int j = 0; j < world; ++j) a.ws[j] = reinterpret_cast<uint8_t*>(ws[j]);
  a.world = world;
  a.rank = (int)rank;
  a.params_off = params_off;
  a.grads_off = grads_off;
  a.ctl_off = ctl_off;
  a.n = n;
  a.m = m.data_ptr<float>();
  a.v = v.data_ptr<float>();
  a.scratch = scratch.data_ptr<float>();
  a.lr = (float)lr;
  a.beta1 = (float)beta1;
  a.beta2 = (float)beta2;
  a.eps = (float)eps;
  a.weight_decay = (float)weight_decay;
  a.max_norm = (float)max_norm;
  a.bc1 = (float)(1.0 - std::pow(beta1, (double)step));
  a.bc2 = (float)(1.0 - std::pow(beta2, (double)step));
  a.norm_out = norm_out.data_ptr<float>();
  a.err = device_error_flag();
  const int grid = std::max(1, std::min<int>(num_sms(), (int)((shard + 511) / 512)));
  fused_adamw_kernel<<<grid, 512, 0, cur_stream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace uno
