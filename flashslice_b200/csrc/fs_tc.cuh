// flashslice_b200 -- sm_100a tensor-core primitives: mbarriers, TMA tile
// loads, TMEM allocation, tcgen05.mma (kind::f16, bf16 operands, fp32
// accumulators), tcgen05.commit / ld, and the shared-memory and instruction
// descriptors of the canonical no-swizzle operand layouts.
//
// Every wait is bounded: after kWaitNs it records an error code in the
// kernel's status word and returns false, so that a lost arrival ends the
// kernel instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace fs {
namespace tc {

// A bounded wait gives up after this long (ns of %globaltimer); a poll of
// mbarrier.try_wait suspends the thread for microseconds, so the count of
// polls says little about the time waited.
constexpr uint64_t kWaitNs = 2000000000ull;

enum : int { kErrNone = 0, kErrTimeout = 1 };

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

// make initialised barriers visible to the async proxy (TMA, tensor core)
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
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

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Non-blocking probe: has the phase with the given parity completed?
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete; false (and *status
// set) if it does not within limit_ns (kWaitNs in the kernels). A try_wait
// may itself suspend the thread for longer than a short limit, so limits
// below the default are kept by polling with the non-blocking test_wait.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status,
                                          uint64_t limit_ns = kWaitNs) {
  if (limit_ns >= kWaitNs) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 0; i < (1u << 30); ++i) {
      if (mbar_try_wait(bar, parity)) return true;
      if (globaltimer_ns() - t0 > limit_ns) break;
    }
  } else {
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 0; i < (1u << 30); ++i) {
      if (mbar_test_wait(bar, parity)) return true;
      if (globaltimer_ns() - t0 > limit_ns) break;
    }
  }
  if (status) atomicExch(status, kErrTimeout);
  return false;
}

// ------------------------------------------------------------------ TMA
// 4-D tile load (coordinates innermost first) into shared memory, completing
// `bytes` of transaction count on `bar`.
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, int c3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
      "l"((uint64_t)map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

// Contiguous global -> shared copy of `bytes` (a multiple of 16; both
// addresses 16-byte aligned), completing that many bytes of transaction
// count on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"((uint64_t)src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// generic-proxy shared-memory writes -> visible to the async proxy (MMA, TMA)
__device__ __forceinline__ void fence_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------------------ TMEM
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, bf16 operands, fp32 accumulators. Issued
// by one thread.
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, bool accumulate) {
  const uint32_t acc = accumulate ? 1u : 0u, z = 0u;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(acc), "r"(z), "r"(z), "r"(z), "r"(z)
      : "memory");
}

// arrive on `bar` once every MMA this thread issued so far has completed
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::
                   "r"(smem_u32(bar))
               : "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane (warp w reads lanes
// 32w .. 32w+31; taddr carries the lane in its upper 16 bits)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// ------------------------------------------------------------------ descriptors
// Shared-memory matrix descriptor, no swizzle ("interleaved" core matrices of
// 8 rows x 16 bytes, 128 contiguous bytes each). For a K-major operand, LBO
// is the byte distance between the two K-adjacent core matrices of one MMA
// (K = 16 bf16) and SBO the distance between 8-row groups along M (or N).
// For an MN-major operand, LBO is the distance between groups of 8 K-rows
// and SBO between 16-byte groups along M (or N).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  // base offset 0, absolute LBO mode 0, layout type 0 = no swizzle
  return d;
}

// Instruction descriptor: bf16 x bf16 -> fp32, M x N, A and B majors
// (0 = K-major, 1 = MN-major).
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, int a_mn_major, int b_mn_major) {
  return (1u << 4)                            // D format fp32
         | (1u << 7)                          // A format bf16
         | (1u << 10)                         // B format bf16
         | ((uint32_t)a_mn_major << 15)       // A major
         | ((uint32_t)b_mn_major << 16)       // B major
         | ((uint32_t)(N >> 3) << 17)         // N / 8
         | ((uint32_t)(M >> 4) << 24);        // M / 16
}

// Byte offset of element (row, k) in a K-major no-swizzle bf16 operand of
// K extent kext (a multiple of 8): core matrices along K contiguous (LBO =
// 128 B), 8-row groups SBO = kext * 16 bytes apart.
__host__ __device__ constexpr uint32_t kmajor_off(int row, int k, int kext) {
  return (uint32_t)((row >> 3) * (kext * 16) + (k >> 3) * 128 + (row & 7) * 16 + (k & 7) * 2);
}

// Byte offset of element (mn, k) in an MN-major no-swizzle bf16 operand of
// MN extent mnext (a multiple of 8): 8-element MN groups SBO = 128 B apart
// inside a group of 8 K-rows, K-row groups LBO = mnext * 16 bytes apart.
__host__ __device__ constexpr uint32_t mnmajor_off(int mn, int k, int mnext) {
  return (uint32_t)((k >> 3) * (mnext * 16) + (mn >> 3) * 128 + (k & 7) * 16 + (mn & 7) * 2);
}

// ------------------------------------------------------------------ splits
// x = hi + mid + lo exactly, each a bf16 (8 significant bits each, 24 in all).
__device__ __forceinline__ void split3(float x, __nv_bfloat16& h, __nv_bfloat16& m,
                                       __nv_bfloat16& l) {
  h = __float2bfloat16_rn(x);
  const float r1 = x - __bfloat162float(h);
  m = __float2bfloat16_rn(r1);
  const float r2 = r1 - __bfloat162float(m);
  l = __float2bfloat16_rn(r2);
}

// x = hi + mid + r, |r| <= 2^-17 |x|: two bf16 parts carry 16 significant bits
__device__ __forceinline__ void split2(float x, __nv_bfloat16& h, __nv_bfloat16& m) {
  h = __float2bfloat16_rn(x);
  m = __float2bfloat16_rn(x - __bfloat162float(h));
}

}  // namespace tc
}  // namespace fs
