// Activation quantization: f32 -> int8 per 32-value block with an f32 scale and the block's
// integer sum.  Replaces quantizeAct (src/compute/ref-kernels.js:44-62) as called by the worker's
// `prep` (src/compute/worker.js:238-249).
//
// Bit-exact with the reference: amax is exact in f32, the scale amax/127, its reciprocal and
// x * (1/scale) are computed in IEEE double with correctly rounded division and
// multiplication, and the rounding is half away from zero like the JS
// `v < 0 ? -Math.round(-v) : Math.round(v)`.  Non-finite inputs follow the JS typed-array
// stores: a NaN quantized value stores 0 in the Int8Array and a NaN block sum stores 0 in the
// Int32Array.
#include "common.cuh"
#include "internal.h"

namespace zllm {

// One warp per 32-value block, lane i owns value i.
__global__ void quantize_act_kernel(const float *__restrict__ x, int64_t nblocks, int8_t *__restrict__ xq,
                                    float *__restrict__ xd, int32_t *__restrict__ xs) {
  // let the consumer GEMV launch now and start streaming its weights; it waits for this grid to
  // finish before it reads xq / xd / xs
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t b = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < nblocks; b += warps) {
    const float v = x[b * 32 + lane];
    float a = fabsf(v);
    if (!(a == a)) a = 0.f;                     // a NaN never raises amax (`Math.abs(NaN) > amax` is false)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    const double scale = __ddiv_rn((double)a, 127.0);
    const double inv = scale != 0.0 ? __ddiv_rn(1.0, scale) : 0.0;
    const double t = __dmul_rn((double)v, inv);
    const double r = round(t);                  // half away from zero
    const bool nan = !(r == r);
    xq[b * 32 + lane] = nan ? (int8_t)0 : (int8_t)(int)r;
    int s = nan ? 0 : (int)r;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const bool any_nan = __any_sync(0xffffffffu, nan);
    if (lane == 0) {
      xd[b] = __double2float_rn(scale);
      xs[b] = any_nan ? 0 : s;
    }
  }
}

cudaError_t launch_quantize(const float *x, int64_t k, int ntok, int8_t *xq, float *xd, int32_t *xs, unsigned *status,
                            cudaStream_t s, bool pdl) {
  (void)status;
  const int64_t nblocks = k / 32 * ntok;
  if (nblocks <= 0) return cudaSuccess;
  const int threads = 256;
  int64_t grid = (nblocks + (threads / 32) - 1) / (threads / 32);
  if (grid > 4096) grid = 4096;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(threads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, quantize_act_kernel, x, nblocks, xq, xd, xs);
}

}  // namespace zllm
