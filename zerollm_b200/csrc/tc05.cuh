// tcgen05 (5th-generation tensor core) helpers shared by the GEMM kernels of libzllm_cuda.so: TMEM
// allocation, the MMA and its commit, TMEM loads and stores, shared-memory matrix descriptors for the
// K-major 128-byte-swizzled layout, and the bounded mbarrier waits of the warp-specialized pipelines.
// Every wait gives up after WAIT_DEADLINE_NS (common.cuh): it sets the status word and an abort flag
// that ends every loop of the kernel.
#pragma once
#include "common.cuh"

namespace zllm {

// ---------------------------------------------------------------------------- tcgen05 wrappers
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// arrive on `bar` once this thread's earlier cp.async copies have landed (no pending-count increment:
// the barrier's expected count includes these arrivals)
__device__ __forceinline__ void cp_async_arrive(uint64_t *bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// D[tmem] (+)= A[smem] . B[smem]^T, both K-major f16, f32 accumulation
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(acc)
      : "memory");
}
// arrive on `bar` once every tcgen05 operation this thread issued before has completed
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// 32 lanes x 32 consecutive f32 columns: thread i gets lane (base lane + i), columns col..col+31
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu)      // start address
         | ((uint64_t)1 << 16)                   // leading byte offset (unused for swizzled K-major)
         | ((uint64_t)(1024 >> 4) << 32)         // stride byte offset: 8 rows x 128 B
         | ((uint64_t)1 << 46)                   // descriptor version
         | ((uint64_t)2 << 61);                  // 128-byte swizzle
}
// Instruction descriptor of kind::f16: f16 A and B, f32 D, both K-major, M x N (N a multiple of 16,
// in bits 17..22 as N / 8; M in bits 24..28 as M / 16).
__host__ __device__ __forceinline__ constexpr uint32_t idesc_f16(int m, int n) {
  return (1u << 4) | ((uint32_t)(m >> 4) << 24) | ((uint32_t)(n >> 3) << 17);
}

// byte offset of element (row, k) of a [rows][64] f16 tile in the 128-byte-swizzled layout
__host__ __device__ __forceinline__ uint32_t sw128_off(int row, int k) {
  return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((((k >> 3) ^ (row & 7)) & 7) << 4) + (k & 7) * 2);
}

// ---------------------------------------------------------------------------- bounded waits
// try_wait without a suspend-time hint: the thread polls instead of sleeping between tries, which
// keeps the reaction to a completed phase short in these tightly coupled pipelines
__device__ __forceinline__ bool try_wait_spin(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// test_wait: never suspends -- the cheap check when the phase has most likely completed already
__device__ __forceinline__ bool test_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
struct Ctl {
  volatile int *abort;
  unsigned *status;
};
// one thread; false after a give-up (sets the status bit and the abort flag) or when aborted.
// Sleep: tries that may suspend the thread until the phase completes (mbar_try_wait's hint), for
// roles off the critical path, whose polling would take issue slots from the others.
template <bool Sleep = false>
__device__ __forceinline__ bool wait1(uint64_t *bar, uint32_t parity, const Ctl &c, uint32_t bit) {
  if (test_wait(bar, parity)) return true;           // the common case: no abort check needed
  if (*c.abort) return false;
  for (int i = 0; i < (Sleep ? 1 : 64); i++)
    if (Sleep ? mbar_try_wait(bar, parity) : try_wait_spin(bar, parity)) return true;
  const uint64_t deadline = globaltimer_ns() + WAIT_DEADLINE_NS;
  uint32_t n = 0;
  while (!(Sleep ? mbar_try_wait(bar, parity) : try_wait_spin(bar, parity))) {
    if (*c.abort) return false;
    if ((++n & (Sleep ? 0u : 63u)) == 0 && globaltimer_ns() > deadline) {
      atomicOr(c.status, bit);
      *c.abort = 1;
      return false;
    }
  }
  return true;
}
// a warp: lane 0 waits, the verdict is broadcast
template <bool Sleep = false>
__device__ __forceinline__ bool waitw(uint64_t *bar, uint32_t parity, const Ctl &c, uint32_t bit, int lane) {
  bool ok = true;
  if (lane == 0) ok = wait1<Sleep>(bar, parity, c, bit);
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  return ok;
}

// 32 lanes x 32 consecutive f32 columns from registers: thread i writes lane (base lane + i)
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
      ::"r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])),
        "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
        "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])),
        "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])),
        "r"(__float_as_uint(v[23])), "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
        "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])),
        "r"(__float_as_uint(v[31]))
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

}  // namespace zllm
