// Decode GEMV for float weights (F16, BF16, F32) against the f32 activation: the output head of
// the decode step (151936 x 4096 F16 for Qwen3-8B, the largest matrix of the pass).
//
// Replaces the reference's float matvec, src/compute/ref-kernels.js:278-299 (y[r] = sum f32(w)*x,
// x not quantized), which the worker pool runs in plain JS even with the SIMD kernels
// (src/compute/worker.js:263-268).
//
// Memory-bound streaming: a warp owns whole rows; each lane reads 16 weight bytes per step with
// coalesced 128-bit loads (a row of 4096 F16 values is 16 loads per lane, all issued before the
// first is used), widens them to f32 and accumulates x * w with fused multiply-adds; the
// activation of up to 8 tokens sits in shared memory.  A row's lane sums are reduced by a
// butterfly in a fixed order, so results do not depend on the launch shape or on how many tokens
// share the pass.  The reference accumulates in double; f32 accumulation differs by ~1e-7
// relative.
#include "common.cuh"
#include "internal.h"

namespace zllm {

namespace {

constexpr int kWarpsF = 16;
constexpr int kThreadsF = kWarpsF * 32;
constexpr int kMaxTokF = 8;
constexpr int kUnroll = 8;          // 16-byte loads per lane in flight per row

template <int T> struct FloatFmt;
template <> struct FloatFmt<T_F16> {
  static constexpr int PER = 8;     // values per 16 bytes
  __device__ static void widen(const uint4 &q, float (&v)[8]) {
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; i++) { v[2 * i] = h2f(w[i] & 0xffffu); v[2 * i + 1] = h2f(w[i] >> 16); }
  }
};
template <> struct FloatFmt<T_BF16> {
  static constexpr int PER = 8;
  __device__ static void widen(const uint4 &q, float (&v)[8]) {
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; i++) { v[2 * i] = __uint_as_float(w[i] << 16); v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u); }
  }
};
template <> struct FloatFmt<T_F32> {
  static constexpr int PER = 4;
  __device__ static void widen(const uint4 &q, float (&v)[4]) {
    v[0] = __uint_as_float(q.x); v[1] = __uint_as_float(q.y); v[2] = __uint_as_float(q.z); v[3] = __uint_as_float(q.w);
  }
};

struct FloatArgs {
  const uint8_t *w;
  int64_t row_stride;   // bytes
  int64_t rows, cols;
  const float *x;       // [ntok][cols]
  int ntok;
  float *y;
  const float *y_add;
  int64_t y_stride;
};

template <int T, int NTOK>
__global__ void __launch_bounds__(kThreadsF, 1) float_gemv_kernel(const FloatArgs p) {
  using F = FloatFmt<T>;
  constexpr int PER = F::PER;
  extern __shared__ __align__(16) float sx[];                 // [NTOK][cols]
  pdl_launch_dependents();
  pdl_wait();                                                 // the activation comes from the previous kernel
  const int64_t n4 = p.cols / 4;
  for (int64_t i = threadIdx.x; i < NTOK * n4; i += kThreadsF) {
    const int tok = (int)(i / n4);
    const float4 v = tok < p.ntok ? __ldg(reinterpret_cast<const float4 *>(p.x + (int64_t)tok * p.cols) + (i - tok * n4))
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
    reinterpret_cast<float4 *>(sx)[i] = v;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t nw = (int64_t)gridDim.x * kWarpsF;
  const int nstep = (int)(p.cols / PER / 32);                 // 16-byte steps per lane per row
  const int tail = (int)(p.cols / PER - (int64_t)nstep * 32); // leftover 16-byte units (cols not a multiple of 32*PER)
  for (int64_t r = (int64_t)blockIdx.x * kWarpsF + warp; r < p.rows; r += nw) {
    const uint4 *wr = reinterpret_cast<const uint4 *>(p.w + r * p.row_stride);
    float acc[NTOK];
#pragma unroll
    for (int k = 0; k < NTOK; k++) acc[k] = 0.f;
    for (int s0 = 0; s0 < nstep; s0 += kUnroll) {
      uint4 q[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; u++) q[u] = s0 + u < nstep ? __ldg(wr + (int64_t)(s0 + u) * 32 + lane) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int u = 0; u < kUnroll; u++) {
        if (s0 + u >= nstep) break;
        float v[PER];
        F::widen(q[u], v);
        const int c0 = ((s0 + u) * 32 + lane) * PER;
#pragma unroll
        for (int k = 0; k < NTOK; k++) {
          const float4 *xp = reinterpret_cast<const float4 *>(sx + (int64_t)k * p.cols + c0);
#pragma unroll
          for (int i = 0; i < PER / 4; i++) {
            const float4 xv = xp[i];
            acc[k] = __fmaf_rn(v[4 * i], xv.x, acc[k]);
            acc[k] = __fmaf_rn(v[4 * i + 1], xv.y, acc[k]);
            acc[k] = __fmaf_rn(v[4 * i + 2], xv.z, acc[k]);
            acc[k] = __fmaf_rn(v[4 * i + 3], xv.w, acc[k]);
          }
        }
      }
    }
    if (lane < tail) {
      float v[PER];
      F::widen(__ldg(wr + (int64_t)nstep * 32 + lane), v);
      const int c0 = (nstep * 32 + lane) * PER;
#pragma unroll
      for (int k = 0; k < NTOK; k++)
#pragma unroll
        for (int i = 0; i < PER; i++) acc[k] = __fmaf_rn(v[i], sx[(int64_t)k * p.cols + c0 + i], acc[k]);
    }
#pragma unroll
    for (int k = 0; k < NTOK; k++) acc[k] = warp_sum_f32(acc[k]);
    if (lane < NTOK && lane < p.ntok) {
      float out = 0.f;
#pragma unroll
      for (int k = 0; k < NTOK; k++) if (k == lane) out = acc[k];
      const int64_t o = (int64_t)lane * p.y_stride + r;
      if (p.y_add) out = __fadd_rn(p.y_add[o], out);
      p.y[o] = out;
    }
  }
}

template <int T, int NTOK>
cudaError_t launch_float_t(const FloatArgs &a, int grid, size_t smem, cudaStream_t s, bool pdl) {
  auto kern = float_gemv_kernel<T, NTOK>;
  static bool granted[64] = {false};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!granted[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    granted[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreadsF);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <int T>
cudaError_t launch_float_n(const FloatArgs &a, int nt, int grid, size_t smem, cudaStream_t s, bool pdl) {
  switch (nt) {
    case 1: return launch_float_t<T, 1>(a, grid, smem, s, pdl);
    case 2: return launch_float_t<T, 2>(a, grid, smem, s, pdl);
    case 3: case 4: return launch_float_t<T, 4>(a, grid, smem, s, pdl);
    default: return launch_float_t<T, 8>(a, grid, smem, s, pdl);
  }
}

}  // namespace

bool float_type(int t) { return t == T_F16 || t == T_BF16 || t == T_F32; }

cudaError_t launch_gemv_float(const DevMatrix &m, const ActView &act, int ntok, float *y, int64_t y_stride,
                              const float *y_add, int num_sms, cudaStream_t s, bool pdl, const char **why) {
  if (!act.x) { *why = "float weights need the f32 activation"; return cudaErrorInvalidValue; }
  if (m.cols % (m.type == T_F32 ? 4 : 8)) { *why = "float rows must be a multiple of 16 bytes"; return cudaErrorInvalidValue; }
  // tokens per pass: the activations of one pass share the shared memory
  int per = kMaxTokF;
  while (per > 1 && (size_t)per * m.cols * 4 > 200 * 1024) per /= 2;
  if ((size_t)m.cols * 4 > 200 * 1024) { *why = "float rows too long for the staged activation"; return cudaErrorInvalidValue; }
  for (int t0 = 0; t0 < ntok; t0 += per) {
    const int nt = ntok - t0 < per ? ntok - t0 : per;
    const int ntp = nt <= 2 ? nt : (nt <= 4 ? 4 : 8);
    FloatArgs a{};
    a.w = m.data; a.row_stride = m.row_stride; a.rows = m.rows; a.cols = m.cols;
    a.x = act.x + (int64_t)t0 * m.cols; a.ntok = nt;
    a.y = y + (int64_t)t0 * y_stride; a.y_add = y_add ? y_add + (int64_t)t0 * y_stride : nullptr; a.y_stride = y_stride;
    const size_t smem = (size_t)ntp * m.cols * 4;
    int64_t grid = (m.rows + kWarpsF - 1) / kWarpsF;
    if (grid > num_sms) grid = num_sms;
    cudaError_t e;
    switch (m.type) {
      case T_F16: e = launch_float_n<T_F16>(a, ntp, (int)grid, smem, s, pdl); break;
      case T_BF16: e = launch_float_n<T_BF16>(a, ntp, (int)grid, smem, s, pdl); break;
      default: e = launch_float_n<T_F32>(a, ntp, (int)grid, smem, s, pdl); break;
    }
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace zllm
