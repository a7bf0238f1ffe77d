// Shared device helpers for the uno_b200 sm_100a kernels.
//
// * bounded mbarrier waits: every spin has a wall-clock limit (%globaltimer);
//   on expiry the kernel records an error code in a device flag and returns
//   instead of hanging the GPU;
// * TMA (cp.async.bulk.tensor) and tcgen05 (MMA / TMEM) inline-PTX wrappers;
// * Philox-4x32-10 counter RNG (Salmon, Moraes, Dror, Shaw: "Parallel random
//   numbers: as easy as 1, 2, 3", SC'11) for sampling;
// * small warp/block reductions.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace uno {

// ------------------------------------------------------------------ errors
// Device error word shared by all kernels of the extension (host reads it with
// uno_error_flag()).  Codes: 1 = barrier wait timed out, 2 = bad argument seen
// on device, 3 = peer wait timed out.
__device__ __forceinline__ void set_error(int* flag, int code) {
  if (flag) atomicOr(flag, 1 << code);
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s per wait

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for phase `parity` of `bar` to complete.  Returns false (and flags the
// error word) when the wall-clock limit expires.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t start = globaltimer_ns();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - start > kWaitLimitNs) {
      set_error(err, 1);
      return false;
    }
  }
}

// System-scope acquire load (flags written by peer GPUs over NVLink).
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Wait until every rank owning a row of [r0, r1) has published flag value
// >= target in done[]; then make the peers' generic-proxy stores visible to
// this thread's TMA (async-proxy) loads.  Bounded: sets error code 3.
__device__ __forceinline__ bool wait_row_owners(const unsigned long long* done, int r0, int r1, int rows_per_rank,
                                                unsigned long long target, int* err) {
  uint64_t start = 0;
  for (int j = r0 / rows_per_rank; j <= (r1 - 1) / rows_per_rank; ++j) {
    while (ld_acquire_sys_u64(done + j) < target) {
      if (start == 0) start = globaltimer_ns();
      if (globaltimer_ns() - start > 5000000000ull) {
        set_error(err, 3);
        return false;
      }
    }
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
  return true;
}

// --------------------------------------------- programmatic dependent launch
// Kernels launched with launch_pdl() may start while the previous kernel of the
// stream is still running.  pdl_wait() blocks until that kernel has completed
// and its writes are visible (a no-op without the launch attribute);
// pdl_trigger() lets the next kernel begin launching once every CTA of this
// grid has triggered or exited.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x,
                                            int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ------------------------------------------------------------------ tcgen05
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Allocate `ncols` TMEM columns (power of two >= 32); the base address is
// written to shared memory.  Must be executed by one full warp.
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D(tmem) (+)= A(smem desc) * B(smem desc)^T, kind::f16 (bf16 inputs, fp32 accumulate).
__device__ __forceinline__ void tc_mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Load 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor for a K-major bf16 tile written by TMA with
// 128-byte swizzle: rows of 64 elements (128 B), 8-row atoms 1024 B apart.
__device__ __forceinline__ uint64_t smem_desc_sw128(const void* smem) {
  uint64_t addr = smem_u32(smem);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3FFFull;      // start address
  d |= 1ull << 16;                   // leading byte offset (unused for swizzled K-major)
  d |= (1024ull >> 4) << 32;         // stride byte offset: 8 rows * 128 B
  d |= 1ull << 46;                   // descriptor version (sm_100)
  d |= 2ull << 61;                   // layout: 128-byte swizzle
  return d;
}

// MN-major operand tile staged as BK-row boxes of 64 contiguous MN elements
// (128 B rows, 128-byte swizzle): 8-row K groups are 1024 B apart (stride byte
// offset) and consecutive 64-element MN groups are one 64 x 128 B box apart
// (leading byte offset, 8 KB).  One 16-deep MMA step advances 16 rows = 2 KB.
__device__ __forceinline__ uint64_t smem_desc_mn_sw128(const void* smem) {
  uint64_t addr = smem_u32(smem);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3FFFull;      // start address
  d |= (8192ull >> 4) << 16;         // leading byte offset: next 64-element MN group
  d |= (1024ull >> 4) << 32;         // stride byte offset: next 8 K rows
  d |= 1ull << 46;                   // descriptor version (sm_100)
  d |= 2ull << 61;                   // layout: 128-byte swizzle
  return d;
}

// Instruction descriptor: kind::f16, A/B bf16, D fp32, both K-major.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4)                    // D format fp32
         | (1u << 7)                  // A bf16
         | (1u << 10)                 // B bf16
         | ((uint32_t)(N >> 3) << 17) // N / 8
         | ((uint32_t)(M >> 4) << 24);// M / 16
}

// ------------------------------------------------------- CTA pairs (clusters)
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t num_clusters_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}

// shared::cluster address of the same shared variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrive on an mbarrier given by its shared::cluster address (possibly in the peer CTA).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// 2-D TMA load into this CTA's shared memory whose completion is counted on an
// mbarrier of the CTA pair's leader (cta_group::2 form; no multicast).
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t leader_bar, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(leader_bar), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D(tmem, 256 rows across the pair) (+)= A(smem, 128 rows per CTA) * B(smem, N/2 rows per CTA)^T
__device__ __forceinline__ void tc_mma_bf16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the mbarrier at `cluster_addr` (this CTA's or the peer's) once the
// pair MMAs issued so far complete.
__device__ __forceinline__ void tc_commit_pair(uint32_t cluster_addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_addr)
               : "memory");
}

// ------------------------------------------------------------------ numeric
__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16(x)); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffff, v, o));
  return v;
}

// -------------------------------------------------------------------- Philox
// Philox-4x32 with 10 rounds; multipliers and Weyl constants are the values
// published in the SC'11 paper.
struct Philox4 {
  uint32_t x, y, z, w;
};

__host__ __device__ __forceinline__ Philox4 philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3,
                                                         uint32_t k0, uint32_t k1) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
  const uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    uint64_t p0 = (uint64_t)M0 * c0;
    uint64_t p1 = (uint64_t)M1 * c2;
    uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    uint32_t n0 = hi1 ^ c1 ^ k0;
    uint32_t n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
    k0 += W0;
    k1 += W1;
  }
  return {c0, c1, c2, c3};
}

// Uniform in (0, 1): 24 random bits, offset by half an ulp so 0 never occurs.
__host__ __device__ __forceinline__ float u01(uint32_t bits) {
  return ((bits >> 8) + 0.5f) * (1.0f / 16777216.0f);
}

}  // namespace uno
