// Host-side declarations shared by the uno_b200 CUDA translation units.
#pragma once

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAException.h>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <utility>

namespace uno {

// Parameters of the tcgen05 GEMM (gemm_tcgen05.cu) and its fused epilogues.
struct GemmParams {
  int M, N, K;
  int num_m, num_n;
  __nv_bfloat16* C;
  int ldc;
  const __nv_bfloat16* R;  // residual input (ADD)
  int ldr;
  int K2;                  // K extension length (0 = none)
  float lora_scale;
  const float* row_mask;
  // QK-norm / RoPE / KV store
  __nv_bfloat16* q_out;
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  const int64_t* slots;
  const int64_t* positions;
  const float* cos_sin;
  const __nv_bfloat16* q_norm_w;
  const __nv_bfloat16* k_norm_w;
  float eps;
  int num_q_heads, num_kv_heads, page_size;
  int* err;
  // split-K: number of K splits, fp32 partial workspace, per-tile arrival counters
  int splits;
  float* ws;
  int* counters;
  // reduce-scatter send (row-parallel TP): row r goes to rank r / rs_R, slot
  // rs_rank, at byte offset rs_recv_off of that rank's symmetric workspace
  uint8_t* rs_peers[8];
  int rs_enable, rs_rank, rs_R, rs_recv_off;
  // all-gathered A operand (fused TP collectives): before loading the A rows
  // of a tile, wait until their owner ranks (row / ag_R) have published
  // "done" for the current epoch in this rank's workspace control block
  const uint8_t* ag_base;
  int ag_R;
  // weight-gradient GEMM (EPI_WGRAD): C32[M, N] += A^T B in fp32
  float* C32;
  int ldc32;
};
void gemm_dispatch(int epi, int bn, const void* a, int64_t lda, const void* b, int64_t ldb, const void* a2,
                   int64_t lda2, const void* b2, int64_t ldb2, GemmParams& p, cudaStream_t stream, int max_ctas);
int pick_bn(int M, int N, int forced);
int pick_splits(int M, int N, int K, int bn, int forced);
void pick_tile(int M, int N, int K, int epi, int forced_bn, int forced_splits, int* bn, int* splits);
void gemm_wgrad_dispatch(const void* a, int64_t lda, const void* b, int64_t ldb, GemmParams& p, int bn,
                         cudaStream_t stream);
int num_sms();

// Output tiles a split-K launch of tile width bn can index: 128-row tiles, or
// 256-row CTA pairs counted as two 128-row tiles (M = 384 uses four).  The
// split-K scratch holds tiles * splits * 128 * bn partials and one counter per
// tile, so every scratch-size check uses this count.
inline int64_t splitk_tiles(int M, int N, int bn) {
  const int64_t m_tiles = std::max<int64_t>((M + 127) / 128, (int64_t)((M + 255) / 256) * 2);
  return m_tiles * ((N + bn - 1) / bn);
}

// Runs a set-up step once per CUDA device.  Function attributes such as the
// dynamic shared-memory opt-in belong to (function, device): a process that
// launches on several devices must set them on each one.
// Launch with programmatic stream serialisation (PDL): the kernel may be scheduled while the
// previous kernel of the stream drains; it must call pdl_wait() before reading what that kernel
// wrote.  UNO_PDL=0 launches normally (for A/B timing).
bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

class PerDeviceOnce {
 public:
  template <class F>
  void operator()(F&& f) {
    int dev = 0;
    C10_CUDA_CHECK(cudaGetDevice(&dev));
    TORCH_CHECK(dev >= 0 && dev < 64, "device index ", dev, " out of range");
    const uint64_t bit = uint64_t(1) << dev;
    if (done_.load(std::memory_order_acquire) & bit) return;
    f();
    done_.fetch_or(bit, std::memory_order_acq_rel);
  }

 private:
  std::atomic<uint64_t> done_{0};
};

// Per-device scratch shared by the GEMM split-K path (fp32 partials and
// self-resetting tile counters) and the device error word.
struct DeviceScratch {
  int* err;
  int* counters;
  float* ws;
  size_t ws_floats;
  int max_counters;
};
DeviceScratch& device_scratch();

struct AttnLaunch {
  const __nv_bfloat16* q;
  __nv_bfloat16* o;
  float* o_part;
  float* lse_part;
  const __nv_bfloat16* k_cache;
  const __nv_bfloat16* v_cache;
  int num_pages;
  const int* block_tables;
  int bt_stride;
  const int* prefix_lens;
  const int64_t* suffix_mask;
  const int* cu_q;
  const int* cu_k;
  int B, Q, T, max_q;
  int hq, hkv, head_dim, page;
  int num_splits, keys_per_split;
  float scale;
  int mode;
  int* err;
};
void paged_attention_launch(const AttnLaunch& a, cudaStream_t stream);
// tcgen05 paged attention (attention_tc.cu): one persistent CTA per SM; o_part
// holds 2 * SMs * rows * 128 floats, lse_part 2 * SMs * rows, counters T * hkv
// ints that are zero between launches (the kernel resets the ones it uses).
void attention_tc_launch(const AttnLaunch& a, int* counters, cudaStream_t stream,
                         unsigned long long* trace = nullptr);
int attention_tc_rows();
int num_sms();

// Control block at the start of every rank's symmetric workspace (comm.cu):
// u64 epoch, u32 CTA counter, u32 pad, u64 arrive[8], u64 done[8].
constexpr int COMM_EPOCH_OFF = 0;
constexpr int COMM_DONE_OFF = 80;

// Device error word (allocated once per device by the bindings).
inline int* device_error_flag() { return device_scratch().err; }

// Every pointer handed to a kernel must live on the current CUDA device: a
// host or foreign-device tensor is rejected on the host instead of faulting.
inline void check_dev(const at::Tensor& t, const char* what) {
  TORCH_CHECK(t.is_cuda(), what, " must be a CUDA tensor");
  int dev;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  TORCH_CHECK(t.get_device() == dev, what, " is on cuda:", t.get_device(), " but the current device is cuda:", dev);
}

inline cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

#define UNO_CHECK_CUDA(t) TORCH_CHECK((t).is_cuda(), #t " must be a CUDA tensor")
#define UNO_CHECK_BF16(t) TORCH_CHECK((t).scalar_type() == at::kBFloat16, #t " must be bfloat16")
#define UNO_CHECK_CONTIG(t) TORCH_CHECK((t).is_contiguous(), #t " must be contiguous")

}  // namespace uno
