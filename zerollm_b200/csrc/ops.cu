// Per-token glue of the decode step, each fused with the activation quantization its consumer
// needs: token embedding (dequantized row), RMSNorm + quantize, SwiGLU + quantize, greedy argmax.
//
// Arithmetic follows the reference: rmsnorm src/compute/ref-kernels.js:305-310 (double sum of
// squares, s = 1/sqrt(ss/n + eps), f32(x * s * w)); silu :322 and the SwiGLU product
// src/compute/worker.js:426 (double, stored f32); dequantRow :80-120 with quant.js:121-202;
// quantizeAct :44-62 (see quant.cu); argmax src/model/generate.js:4-10 (first maximum wins).
// The double sums of squares are reduced as a fixed tree rather than left to right, so a result can
// differ from the reference's in the last bit of the double -- and only then, rarely, in the f32.
#include "common.cuh"
#include "internal.h"
#include "kq_layout.h"

namespace zllm {

// ---------------------------------------------------------------------------- block quantization
// One warp quantizes one 32-value block held one value per lane (same arithmetic as quant.cu).
__device__ __forceinline__ void quantize_block_warp(float v, int lane, int8_t *q, float *d, int32_t *s) {
  float a = fabsf(v);
  if (!(a == a)) a = 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
  const double scale = __ddiv_rn((double)a, 127.0);
  const double inv = scale != 0.0 ? __ddiv_rn(1.0, scale) : 0.0;
  const double r = round(__dmul_rn((double)v, inv));
  const bool nan = !(r == r);
  q[lane] = nan ? (int8_t)0 : (int8_t)(int)r;
  int sum = nan ? 0 : (int)r;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const bool any_nan = __any_sync(0xffffffffu, nan);
  if (lane == 0) {
    *d = __double2float_rn(scale);
    *s = any_nan ? 0 : sum;
  }
}

// ---------------------------------------------------------------------------- RMSNorm + quantize
// grid (ntok, nsplit): every CTA of a token computes the token's sum of squares (the same reduction
// in the same order, so the same bits) and then normalizes / quantizes its own share of the 32-value
// blocks.  xb (optional) receives the normalized f32 vector; xq/xd/xs (optional) its quantization.
// n must be a multiple of 32 when quantizing.
__global__ void rmsnorm_quant_kernel(const float *__restrict__ x, const float *__restrict__ w, int n, double eps,
                                     float *xb, int8_t *xq, float *xd, int32_t *xs) {
  __shared__ double red[32];
  pdl_launch_dependents();
  pdl_wait();
  const int t = blockIdx.x;
  const float *xt = x + (int64_t)t * n;
  double ss = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) ss = __dadd_rn(ss, __dmul_rn((double)xt[i], (double)xt[i]));
  ss = warp_sum_f64(ss);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  double tot = lane < nw ? red[lane] : 0.0;
  tot = warp_sum_f64(tot);                      // every warp reduces the same values in the same order
  const double s = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(tot, (double)n), eps)));
  const int nblk = n / 32, per = (nblk + gridDim.y - 1) / gridDim.y;
  const int b0 = blockIdx.y * per, b1 = min(nblk, b0 + per);
  if (xq) {
    for (int b = b0 + warp; b < b1; b += nw) {
      const int i = b * 32 + lane;
      const float v = __double2float_rn(__dmul_rn(__dmul_rn((double)xt[i], s), (double)w[i]));
      if (xb) xb[(int64_t)t * n + i] = v;
      quantize_block_warp(v, lane, xq + (int64_t)t * n + b * 32, xd + (int64_t)t * (n / 32) + b, xs + (int64_t)t * (n / 32) + b);
    }
  } else {
    const int i0 = blockIdx.y == 0 ? 0 : b0 * 32, i1 = blockIdx.y == gridDim.y - 1 ? n : b1 * 32;
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x)
      xb[(int64_t)t * n + i] = __double2float_rn(__dmul_rn(__dmul_rn((double)xt[i], s), (double)w[i]));
  }
}

// ---------------------------------------------------------------------------- SwiGLU + quantize
// hb = f32(silu(gate) * up) with silu(z) = z / (1 + exp(-z)) in double; then quantized per 32.
__global__ void swiglu_quant_kernel(const float *__restrict__ gate, const float *__restrict__ up, int n, int ntok,
                                    int64_t stride, float *hb, int8_t *xq, float *xd, int32_t *xs) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t nblk = (int64_t)ntok * (n / 32);
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t gb = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); gb < nblk; gb += warps) {
    const int t = (int)(gb / (n / 32)), b = (int)(gb % (n / 32));
    const int64_t i = (int64_t)t * stride + b * 32 + lane;
    const double z = gate[i];
    const double sl = __ddiv_rn(z, __dadd_rn(1.0, exp(-z)));
    const float v = __double2float_rn(__dmul_rn(sl, (double)up[i]));
    if (hb) hb[(int64_t)t * n + b * 32 + lane] = v;
    if (xq) quantize_block_warp(v, lane, xq + (int64_t)t * n + b * 32, xd + (int64_t)t * (n / 32) + b, xs + (int64_t)t * (n / 32) + b);
  }
}

// ---------------------------------------------------------------------------- embedding
// value i of row r of a device-layout matrix (the repacked layouts of gemv.cu), as f32
__device__ float dequant_at(const DevMatrix &m, int64_t r, int64_t i) {
  const uint8_t *row = m.data + r * m.row_stride;
  switch (m.type) {
    case T_F32: return reinterpret_cast<const float *>(row)[i];
    case T_F16: return h2f(reinterpret_cast<const uint16_t *>(row)[i]);
    case T_BF16: return bf2f(reinterpret_cast<const uint16_t *>(row)[i]);
    case T_Q8_0: {
      const int64_t nb = m.cols / 32, b = i / 32;
      const double d = h2f(*reinterpret_cast<const uint16_t *>(row + 32 * nb + 2 * b));
      return __double2float_rn(__dmul_rn(d, (double)(int8_t)row[b * 32 + i % 32]));
    }
    case T_Q4_0: case T_Q5_0: {
      const int64_t nb = m.cols / 32, b = i / 32;
      const int j = (int)(i % 32);
      const uint8_t byte = row[b * 16 + (j & 15)];
      int q = j < 16 ? (byte & 15) : (byte >> 4);
      const bool five = m.type == T_Q5_0;
      if (five) q |= (int)((*reinterpret_cast<const uint32_t *>(row + 16 * nb + 4 * b) >> j) & 1u) << 4;
      const double d = h2f(*reinterpret_cast<const uint16_t *>(row + (five ? 20 : 16) * nb + 2 * b));
      return __double2float_rn(__dmul_rn(d, (double)(q - (five ? 16 : 8))));
    }
    case T_Q4_K: case T_Q5_K: {
      const bool five = m.type == T_Q5_K;
      const int bs = five ? 176 : 144;
      const int64_t nb = m.cols / 256, sb = i / 256;
      const int e = (int)(i % 256), s = e / 32, l = e % 32, c = s >> 1;
      // raw GGUF byte positions, mapped to the device layout (kq_layout.h)
      auto at = [&](int64_t raw) { return m.data[kq_dev_pos(m.type, r, sb * bs + raw, nb)]; };
      const uint8_t byte = at((five ? 48 : 16) + c * 32 + l);
      int v = (s & 1) ? byte >> 4 : byte & 15;
      if (five) v |= ((at(16 + l) >> s) & 1) << 4;
      // the repacked scale field of chunk c: sc(2c) | sc(2c+1) << 6 | mn(2c) << 12 | mn(2c+1) << 18
      const uint32_t F = (uint32_t)at(4 + 3 * c) | ((uint32_t)at(5 + 3 * c) << 8) | ((uint32_t)at(6 + 3 * c) << 16);
      const int sc = (s & 1) ? (F >> 6) & 63 : F & 63, mn = (s & 1) ? (F >> 18) & 63 : (F >> 12) & 63;
      const double d = h2f(at(0) | (at(1) << 8)), dmin = h2f(at(2) | (at(3) << 8));
      // quant.js:150: d * sc * v - dmin * mn
      return __double2float_rn(__dsub_rn(__dmul_rn(__dmul_rn(d, (double)sc), (double)v), __dmul_rn(dmin, (double)mn)));
    }
    case T_Q6_K: {
      const int64_t nb = m.cols / 256, sb = i / 256, rb = sb * 210;
      const int e = (int)(i % 256), half = e / 128, k = (e % 128) / 32, l = e % 32;
      auto at = [&](int64_t raw) { return m.data[kq_dev_pos(T_Q6_K, r, rb + raw, nb)]; };
      const uint8_t ql = at(half * 64 + (k & 1) * 32 + l);
      const uint8_t qh = at(128 + half * 32 + l);
      const int q = (int)(((k < 2 ? ql & 15 : ql >> 4)) | (((qh >> (2 * k)) & 3) << 4)) - 32;
      const int scale = (int8_t)at(192 + half * 8 + (l >> 4) + 2 * k);
      const double d = h2f(at(208) | (at(209) << 8));
      // quant.js:194-197: d * scale * q
      return __double2float_rn(__dmul_rn(__dmul_rn(d, (double)scale), (double)q));
    }
  }
  return 0.f;
}

// CTA (t, c): columns [c * kEmbedCols, (c + 1) * kEmbedCols) of token t's row
constexpr int kEmbedCols = 1024;
__global__ void embed_kernel(const DevMatrix m, const int32_t *tokens, int ntok, float *x) {
  pdl_launch_dependents();
  pdl_wait();
  const int t = blockIdx.x;
  if (t >= ntok) return;
  const int64_t r = tokens[t];
  const int64_t i1 = min(m.cols, (int64_t)(blockIdx.y + 1) * kEmbedCols);
  for (int64_t i = (int64_t)blockIdx.y * kEmbedCols + threadIdx.x; i < i1; i += blockDim.x)
    x[(int64_t)t * m.cols + i] = dequant_at(m, r, i);
}

// ---------------------------------------------------------------------------- argmax
// The first maximum of each token's logits (src/model/generate.js:4-10), in two stages: CTA (c, t)
// reduces chunk c of token t's row, then one warp per token combines the chunks with the same rule,
// which picks the largest value and, among equal ones, the smallest index -- so the answer does not
// depend on the chunking.
__device__ __forceinline__ void argmax_merge(float &best, int &idx, float ob, int oi) {
  if (ob > best || (ob == best && oi >= 0 && (idx < 0 || oi < idx)) || (idx < 0 && oi >= 0)) { best = ob; idx = oi; }
}
__device__ __forceinline__ void argmax_warp(float &best, int &idx) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    argmax_merge(best, idx, ob, oi);
  }
}
__global__ void argmax_part_kernel(const float *logits, int64_t n, int64_t stride, int64_t chunk, float *pv, int *pi) {
  __shared__ float bv[32];
  __shared__ int bi[32];
  pdl_launch_dependents();
  pdl_wait();
  const int c = blockIdx.x, t = blockIdx.y;
  const float *l = logits + (int64_t)t * stride;
  const int64_t i1 = min(n, (int64_t)(c + 1) * chunk);
  float best = -INFINITY;
  int idx = -1;
  for (int64_t i = (int64_t)c * chunk + threadIdx.x; i < i1; i += blockDim.x) {
    const float v = l[i];
    if (v > best || idx < 0) { best = v; idx = (int)i; }
  }
  argmax_warp(best, idx);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { bv[warp] = best; bi[warp] = idx; }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? bv[lane] : -INFINITY;
    idx = lane < nw ? bi[lane] : -1;
    argmax_warp(best, idx);
    if (lane == 0) { pv[(int64_t)t * gridDim.x + c] = best; pi[(int64_t)t * gridDim.x + c] = idx; }
  }
}
__global__ void argmax_final_kernel(const float *pv, const int *pi, int nchunk, int32_t *out) {
  pdl_launch_dependents();
  pdl_wait();
  const int t = blockIdx.x, lane = threadIdx.x;
  float best = -INFINITY;
  int idx = -1;
  for (int c = lane; c < nchunk; c += 32) argmax_merge(best, idx, pv[(int64_t)t * nchunk + c], pi[(int64_t)t * nchunk + c]);
  argmax_warp(best, idx);
  if (lane == 0) out[t] = idx;
}

// ---------------------------------------------------------------------------- launchers
static cudaLaunchConfig_t cfg_of(dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl, cudaLaunchAttribute *attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cfg;
}

cudaError_t launch_rmsnorm_quant(const float *x, const float *w, int n, int ntok, double eps, float *xb, int8_t *xq, float *xd,
                                 int32_t *xs, cudaStream_t s, bool pdl) {
  cudaLaunchAttribute attr[1];
  // split each token's blocks over CTAs, one block per warp (each CTA re-reads the token to get the
  // same sum of squares): the quantization's double divisions are the long chain, not the reads
  const int nblk = n / 32 > 0 ? n / 32 : 1;
  const int split = nblk / 8 > 0 ? nblk / 8 : 1;
  cudaLaunchConfig_t cfg = cfg_of(dim3(ntok, split), dim3(256), 0, s, pdl, attr);
  return cudaLaunchKernelEx(&cfg, rmsnorm_quant_kernel, x, w, n, eps, xb, xq, xd, xs);
}

cudaError_t launch_swiglu_quant(const float *gate, const float *up, int n, int ntok, int64_t stride, float *hb, int8_t *xq,
                                float *xd, int32_t *xs, cudaStream_t s, bool pdl) {
  const int64_t blocks = (int64_t)ntok * (n / 32);
  int64_t grid = (blocks + 7) / 8;
  if (grid > 2048) grid = 2048;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = cfg_of(dim3((unsigned)grid), dim3(256), 0, s, pdl, attr);
  return cudaLaunchKernelEx(&cfg, swiglu_quant_kernel, gate, up, n, ntok, stride, hb, xq, xd, xs);
}

cudaError_t launch_embed(const DevMatrix &m, const int32_t *tokens, int ntok, float *x, cudaStream_t s, bool pdl) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = cfg_of(dim3(ntok, (unsigned)((m.cols + kEmbedCols - 1) / kEmbedCols)), dim3(256), 0, s, pdl, attr);
  return cudaLaunchKernelEx(&cfg, embed_kernel, m, tokens, ntok, x);
}

// Greedy feedback between decode passes on the device: each sequence's next input is the argmax of
// its logits (src/model/generate.js:4-10 picks the first maximum), at the next position; the token
// is also recorded as output `step` (a device counter advanced here).
__global__ void advance_kernel(const int32_t *arg, int n, int32_t *tok, int32_t *pos, int32_t *npos, int32_t *out,
                               int32_t *step) {
  pdl_launch_dependents();
  pdl_wait();
  const int i = threadIdx.x;
  const int st = *step;
  if (i < n) {
    const int32_t a = arg[i];
    tok[i] = a;
    pos[i] += 1;
    npos[i] += 1;
    out[(int64_t)st * n + i] = a;
  }
  __syncthreads();
  if (i == 0) *step = st + 1;
}

cudaError_t launch_advance(const int32_t *arg, int n, int32_t *tok, int32_t *pos, int32_t *npos, int32_t *out,
                           int32_t *step, cudaStream_t s, bool pdl) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = cfg_of(dim3(1), dim3(64), 0, s, pdl, attr);
  return cudaLaunchKernelEx(&cfg, advance_kernel, arg, n, tok, pos, npos, out, step);
}

cudaError_t launch_argmax(const float *logits, int64_t n, int64_t stride, int ntok, int32_t *out, float *pv, int *pi,
                          cudaStream_t s, bool pdl) {
  const int64_t chunk = (n + kArgmaxChunks - 1) / kArgmaxChunks;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = cfg_of(dim3(kArgmaxChunks, ntok), dim3(256), 0, s, pdl, attr);
  cudaError_t e = cudaLaunchKernelEx(&cfg, argmax_part_kernel, logits, n, stride, chunk, pv, pi);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg2 = cfg_of(dim3(ntok), dim3(32), 0, s, false, attr);
  return cudaLaunchKernelEx(&cfg2, argmax_final_kernel, (const float *)pv, (const int *)pi, kArgmaxChunks, out);
}

}  // namespace zllm
