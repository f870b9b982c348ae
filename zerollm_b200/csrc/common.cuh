// Shared device helpers for the sm_100a kernels of libzllm_cuda.so: bounded mbarrier waits,
// 1D bulk (TMA) copies, programmatic-dependent-launch controls, status reporting.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace zllm {

// ---------------------------------------------------------------------------- status word
// Kernels never trap.  A wait that runs past its deadline sets a bit in the context's device
// status word, drains its own copies in flight and returns; the host reads the word after the
// stream synchronises and turns it into ZLLM_E_TIMEOUT.
enum : uint32_t {
  ST_FULL_TIMEOUT = 1u << 0,   // consumer waited too long for a bulk copy
  ST_EMPTY_TIMEOUT = 1u << 1,  // producer waited too long for a free stage
  ST_DRAIN_TIMEOUT = 1u << 2,  // copies still in flight at exit did not land in time
  ST_BAD_ARGS = 1u << 3,       // launch geometry rejected inside the kernel
  ST_PEER_TIMEOUT = 1u << 4,   // a peer GPU's all-reduce slice did not arrive in time
};

// 2 s: far above any legitimate wait (microseconds), far below a box-level hang.
constexpr uint64_t WAIT_DEADLINE_NS = 2000000000ull;

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0;
}
// Wait for the phase with the given parity to complete, at most until `deadline`.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, uint64_t deadline) {
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() > deadline) return false;
  }
  return true;
}
// The same with the 2 s limit counted from the first unsuccessful try: the clock (a slow read) is
// only consulted when the phase is not already complete.
__device__ __forceinline__ bool mbar_wait_lazy(uint64_t *bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t deadline = globaltimer_ns() + WAIT_DEADLINE_NS;
  return mbar_wait_bounded(bar, parity, deadline);
}

// ---------------------------------------------------------------------------- thread-block clusters
// every thread of every CTA of the cluster arrives, then waits (release / acquire: shared-memory
// writes before the barrier are visible to the cluster's reads after it)
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// a float at the same shared-memory offset as `local` in the cluster's CTA of rank `rank`
__device__ __forceinline__ float ld_dsmem_f32(const float *local, uint32_t rank) {
  uint32_t ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_u32(local)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(ra) : "memory");
  return v;
}

// ---------------------------------------------------------------------------- 1D bulk copy
// global -> shared, completion counted on `bar` (bytes and both addresses 16-byte aligned).
__device__ __forceinline__ void bulk_g2s(void *dst_smem, const void *src_gmem, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------- cp.async (16 bytes)
// global -> shared through L2 only; per-thread groups: commit closes the thread's group of copies
// issued since the last commit, wait<N> returns once at most N of the thread's groups are pending
// (hardware-tracked: no spin loop of ours).  Both addresses 16-byte aligned.
__device__ __forceinline__ void cp_async16(uint32_t dst_smem, const void *src_gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst_smem), "l"(src_gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// ---------------------------------------------------------------------------- PDL
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------- named barriers
__device__ __forceinline__ void named_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
// Barrier over `nthreads` threads that also returns the OR of `pred` across them (uniform result).
__device__ __forceinline__ bool named_sync_or(uint32_t id, uint32_t nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

// ---------------------------------------------------------------------------- shared / global loads
// shared-memory loads by 32-bit shared-window address (volatile: never hoisted above an mbarrier wait)
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds16(uint32_t a) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ float lds_f(uint32_t a) { return __uint_as_float(lds32(a)); }
__device__ __forceinline__ float2 lds_f2(uint32_t a) {
  const uint2 v = lds64(a);
  return make_float2(__uint_as_float(v.x), __uint_as_float(v.y));
}
// ---------------------------------------------------------------------------- packed f32 pairs
// Blackwell's f32x2 arithmetic: element x in the low word, y in the high word; each element rounds
// exactly as the scalar instruction would.
typedef unsigned long long f2v;
__device__ __forceinline__ f2v f2pack(float x, float y) {
  f2v r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(x), "f"(y));
  return r;
}
__device__ __forceinline__ f2v f2bits(uint32_t x, uint32_t y) {
  f2v r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(x), "r"(y));
  return r;
}
__device__ __forceinline__ void f2unpack(f2v v, float &x, float &y) { asm("mov.b64 {%0, %1}, %2;" : "=f"(x), "=f"(y) : "l"(v)); }
__device__ __forceinline__ f2v f2fma(f2v a, f2v b, f2v c) {
  f2v d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ f2v f2mul(f2v a, f2v b) {
  f2v d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f2v f2add(f2v a, f2v b) {
  f2v d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f2v f2sub(f2v a, f2v b) {
  f2v d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ uint4 ldg128(const void *p) { return __ldg(reinterpret_cast<const uint4 *>(p)); }
// The same load issued where it stands in the program: a prefetch the compiler may not sink to the
// first use of its result (volatile asm keeps its place among the other volatile statements).
__device__ __forceinline__ uint4 ldg128_now(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
// int32 -> double without the conversion pipe: (2^52 + 2^31 + v) - (2^52 + 2^31) is exact in double.
// i2d_biased takes v + 2^31 (mod 2^32), which an integer multiply-add produces for free.
__device__ __forceinline__ double i2d_biased(uint32_t v_plus_2p31) {
  return __dsub_rn(__hiloint2double(0x43300000, (int)v_plus_2p31), 4503601774854144.0);
}
__device__ __forceinline__ double i2d_exact(int v) { return i2d_biased((uint32_t)v + 0x80000000u); }

// ---------------------------------------------------------------------------- numbers
__device__ __forceinline__ float h2f(uint32_t bits16) { return __half2float(__ushort_as_half((unsigned short)bits16)); }
__device__ __forceinline__ float bf2f(uint32_t bits16) { return __uint_as_float(bits16 << 16); }

__device__ __forceinline__ double warp_sum_f64(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum_f32(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace zllm
