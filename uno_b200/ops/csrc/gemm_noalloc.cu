// Split-K GEMM entry point that allocates no memory (plain C ABI, declared in
// uno_noalloc.h).
//
// This entry point has no counterpart in the reference implementation.
//
//   out[M, N] (bf16) = A[M, K] . B[N, K]^T   (bf16 operands, fp32 accumulation)
//
// It runs the same tcgen05 kernels as the regular GEMM entry point
// (uno_b200._C.gemm, STORE epilogue, split-K inside the kernel).  The only
// difference is where the split-K scratch lives.  The regular entry point
// takes its fp32 partial-sum workspace and per-tile arrival counters from a
// device buffer that it cudaMalloc's the first time a device is used.  This
// one keeps them in fixed-size arrays that are part of the loaded module
// (file-scope __device__ arrays below), so a call never allocates device or
// host memory and never goes through the PyTorch caching allocator.
//
// Who needs that: callers that are not allowed to allocate at call time, e.g.
// code that runs inside a custom device allocator or its out-of-memory path
// (an allocation there could recurse or fail), or a serving process that
// sizes every device buffer at start-up and treats later growth as a bug.
// A C or C++ host can call it through uno_noalloc.h; the library links
// libtorch, which must be loadable, but no PyTorch allocator is involved.
// All buffers (A, B, out) belong to the caller.
//
// Limits: a split-K launch needs tiles * splits * 128 * tile_width fp32
// partials and one counter per output tile (uno::splitk_tiles).  The fixed
// scratch holds kNoAllocWsFloats floats (4 MiB) and kNoAllocCounters
// counters.  With splits == 0 (automatic) a problem whose split does not fit
// runs without a K split, as the regular entry point does; an explicit split
// count that does not fit is rejected with UNO_NOALLOC_TOO_LARGE before
// anything is launched (uno_noalloc_last_error() says why).  splits == 1
// needs no scratch.
//
// Set-up: uno_gemm_noalloc_setup() waits for the device to be idle, looks up
// the device addresses of the arrays for the current device
// (cudaGetSymbolAddress) and clears the counters and the error word, which
// must start at zero; the kernel returns each counter to zero after use.  The
// first call on a device runs the set-up itself; run it explicitly, with the
// device current, before capturing a stream that will contain a call, since
// the set-up synchronises with the device.
//
// Errors on the device: the kernels' bounded waits write this module's own
// error word, read with uno_noalloc_error_flag(); a non-zero value means the
// output is incomplete and the counters must be cleared by running the
// set-up again.
//
// Concurrency: all calls on a device share one scratch area, which keeps the
// last call's contents.  Calls that can overlap in time (different streams,
// or host threads without ordering between their launches) race on it and
// give wrong results; issue them on a single stream.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <exception>

#include "uno_noalloc.h"
#include "uno_ops.h"

namespace {

constexpr size_t kNoAllocWsFloats = size_t(1) << 20;  // 4 MiB of fp32 partials
constexpr int kNoAllocCounters = 1024;                // output tiles per call
constexpr int kMaxDevices = 64;

__device__ __align__(256) float g_noalloc_ws[kNoAllocWsFloats];
__device__ __align__(256) int g_noalloc_counters[kNoAllocCounters];
__device__ __align__(256) int g_noalloc_err[1];

struct DevicePtrs {
  float* ws;
  int* counters;
  int* err;
  bool ready;
};
DevicePtrs g_devices[kMaxDevices];
thread_local char g_message[512];

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(g_message, sizeof(g_message), fmt, ap);
  va_end(ap);
  return code;
}

}  // namespace

extern "C" {

__attribute__((visibility("default"))) const char* uno_noalloc_last_error() { return g_message; }

__attribute__((visibility("default"))) int uno_gemm_noalloc_setup() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(UNO_NOALLOC_CUDA_ERROR, "cudaGetDevice failed: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(UNO_NOALLOC_BAD_ARGS, "device index %d out of range", dev);
  // never clear counters under a call that is still running on this device
  e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return fail(UNO_NOALLOC_CUDA_ERROR, "waiting for the device failed: %s", cudaGetErrorString(e));
  DevicePtrs d{};
  e = cudaGetSymbolAddress(reinterpret_cast<void**>(&d.ws), g_noalloc_ws);
  if (e != cudaSuccess) return fail(UNO_NOALLOC_CUDA_ERROR, "cudaGetSymbolAddress(workspace) failed: %s", cudaGetErrorString(e));
  e = cudaGetSymbolAddress(reinterpret_cast<void**>(&d.counters), g_noalloc_counters);
  if (e != cudaSuccess) return fail(UNO_NOALLOC_CUDA_ERROR, "cudaGetSymbolAddress(counters) failed: %s", cudaGetErrorString(e));
  e = cudaGetSymbolAddress(reinterpret_cast<void**>(&d.err), g_noalloc_err);
  if (e != cudaSuccess) return fail(UNO_NOALLOC_CUDA_ERROR, "cudaGetSymbolAddress(error word) failed: %s", cudaGetErrorString(e));
  // the arrival counters and the error word must start at zero
  e = cudaMemset(d.counters, 0, sizeof(int) * kNoAllocCounters);
  if (e == cudaSuccess) e = cudaMemset(d.err, 0, sizeof(int));
  if (e != cudaSuccess) return fail(UNO_NOALLOC_CUDA_ERROR, "clearing the counters failed: %s", cudaGetErrorString(e));
  d.ready = true;
  g_devices[dev] = d;
  g_message[0] = '\0';
  return UNO_NOALLOC_OK;
}

// Returns 0 on success, else an UNO_NOALLOC_* code with a message in
// uno_noalloc_last_error().  Leading dimensions are in elements; every
// pointer must be 16-byte aligned and every leading dimension a multiple of 8.
// splits == 0 picks the split count the regular entry point would use, and no
// split when that does not fit the fixed scratch.
__attribute__((visibility("default"))) int uno_gemm_splitk_noalloc(const void* a, long long lda, const void* b,
                                                                    long long ldb, void* out, long long ldo, int M,
                                                                    int N, int K, int splits, void* stream) {
  if (!a || !b || !out) return fail(UNO_NOALLOC_BAD_ARGS, "null operand pointer");
  if (M <= 0 || N <= 0 || K <= 0 || splits < 0)
    return fail(UNO_NOALLOC_BAD_ARGS, "bad sizes M=%d N=%d K=%d splits=%d", M, N, K, splits);
  if (lda < K || ldb < K || ldo < N || lda % 8 || ldb % 8 || ldo % 8)
    return fail(UNO_NOALLOC_BAD_ARGS, "leading dimensions must cover the rows and be multiples of 8");
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(out)) % 16)
    return fail(UNO_NOALLOC_BAD_ARGS, "operands must be 16-byte aligned");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(UNO_NOALLOC_CUDA_ERROR, "cudaGetDevice failed: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(UNO_NOALLOC_BAD_ARGS, "device index %d out of range", dev);
  if (!g_devices[dev].ready) {
    const int rc = uno_gemm_noalloc_setup();
    if (rc != UNO_NOALLOC_OK) return rc;
  }
  const DevicePtrs& d = g_devices[dev];
  try {
    uno::GemmParams p{};
    p.M = M;
    p.N = N;
    p.K = K;
    p.C = reinterpret_cast<__nv_bfloat16*>(out);
    p.ldc = ldo;
    p.err = d.err;
    int bn = 0;
    uno::pick_tile(M, N, K, 0 /* STORE */, 0, splits, &bn, &p.splits);
    if (p.splits > 1) {
      const long long tiles = uno::splitk_tiles(M, N, bn);
      const long long need = tiles * p.splits * 128LL * bn;
      const bool fits = tiles <= kNoAllocCounters && need <= (long long)kNoAllocWsFloats;
      if (!fits && splits == 0) {
        p.splits = 1;  // automatic split count: run unsplit, as the regular entry point does
      } else if (!fits) {
        return fail(UNO_NOALLOC_TOO_LARGE,
                    "split-K scratch too small: %lld tiles x %d splits x 128 x %d needs %lld floats and %lld "
                    "counters; the fixed scratch holds %zu floats and %d counters (use fewer splits or a "
                    "smaller problem)",
                    tiles, p.splits, bn, need, tiles, kNoAllocWsFloats, kNoAllocCounters);
      }
    }
    if (p.splits > 1) {
      p.ws = d.ws;
      p.counters = d.counters;
    }
    uno::gemm_dispatch(0 /* STORE */, bn, a, lda, b, ldb, nullptr, 0, nullptr, 0, p,
                       reinterpret_cast<cudaStream_t>(stream), 0);
  } catch (const std::exception& ex) {
    return fail(UNO_NOALLOC_CUDA_ERROR, "%s", ex.what());
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(UNO_NOALLOC_CUDA_ERROR, "launch failed: %s", cudaGetErrorString(e));
  g_message[0] = '\0';
  return UNO_NOALLOC_OK;
}

__attribute__((visibility("default"))) int uno_noalloc_error_flag(int reset) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices || !g_devices[dev].ready) return 0;  // nothing ran here
  int word = 0;  // host stack memory: a plain synchronous copy allocates nothing
  e = cudaMemcpy(&word, g_devices[dev].err, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) {
    fail(UNO_NOALLOC_CUDA_ERROR, "reading the error word failed: %s", cudaGetErrorString(e));
    return -1;
  }
  if (reset) {
    const int zero = 0;
    e = cudaMemcpy(g_devices[dev].err, &zero, sizeof(int), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
      fail(UNO_NOALLOC_CUDA_ERROR, "clearing the error word failed: %s", cudaGetErrorString(e));
      return -1;
    }
  }
  return word;
}

}  // extern "C"
