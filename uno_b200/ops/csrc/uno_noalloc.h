/* C interface of the fixed-scratch split-K GEMM (gemm_noalloc.cu).
 *
 * This interface has no counterpart in the reference implementation.
 *
 * Plain C: no PyTorch or C++ headers, so a C or C++ host can include it and
 * link the extension library (uno_b200/_C*.so) directly.  The library itself
 * links libtorch, which must be loadable; no PyTorch allocator is used by
 * these calls.
 *
 *   out[M, N] (bf16) = A[M, K] . B[N, K]^T   (bf16 operands, fp32 accumulation)
 *
 * Every call returns UNO_NOALLOC_OK or one of the error codes below; the text
 * of the last failure on the calling host thread is returned by
 * uno_noalloc_last_error().
 */
#ifndef UNO_NOALLOC_H_
#define UNO_NOALLOC_H_

#ifdef __cplusplus
extern "C" {
#endif

enum {
  UNO_NOALLOC_OK = 0,
  UNO_NOALLOC_BAD_ARGS = 1,   /* null pointer, bad size, misaligned operand or leading dimension */
  UNO_NOALLOC_TOO_LARGE = 2,  /* the requested K split count needs more than the fixed scratch */
  UNO_NOALLOC_CUDA_ERROR = 3, /* a CUDA runtime call failed (message says which) */
};

/* Looks up the fixed scratch of the current device and clears its counters
 * and error word.  It first waits for all work on the device to finish, so it
 * never clears counters under a running call; do not call it while a stream
 * of this device is being captured.  The first GEMM call on a device runs it
 * implicitly. */
int uno_gemm_noalloc_setup(void);

/* Launches the GEMM on `stream` (a cudaStream_t; NULL is the legacy default
 * stream).  Leading dimensions are in elements; pointers must be 16-byte
 * aligned and leading dimensions multiples of 8.  splits == 0 picks the split
 * count automatically and falls back to no split when the fixed scratch is
 * too small; an explicit splits > 1 that does not fit is rejected with
 * UNO_NOALLOC_TOO_LARGE before anything is launched. */
int uno_gemm_splitk_noalloc(const void* a, long long lda, const void* b, long long ldb, void* out, long long ldo,
                            int M, int N, int K, int splits, void* stream);

/* Reads the device-side error word of these calls on the current device
 * (waits for the device first: a synchronous 4-byte copy into host stack
 * memory, no allocation).  Non-zero means a kernel gave up on a bounded wait
 * and returned early: its output is incomplete and the split-K counters may
 * be left non-zero, so run uno_gemm_noalloc_setup() before the next call.
 * reset != 0 clears the word after reading it. */
int uno_noalloc_error_flag(int reset);

/* Text of the last failure on this host thread ("" after a success). */
const char* uno_noalloc_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* UNO_NOALLOC_H_ */
