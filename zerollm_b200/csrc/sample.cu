// Device-side candidate selection for sampling: the k largest logits of each row, so that only k
// (id, value) pairs leave the GPU instead of the whole vocabulary row.
//
// Follows src/sampling/sampler.js: the penalties of :98-112 are applied first (repetition penalty
// divides a positive logit and multiplies a negative one, then count * frequency + presence is
// subtracted, all in double, the result stored back as f32), then topKSelect (:20-42) keeps the k
// largest values sorted descending.  Its size-k heap keeps, among equal values at the boundary,
// the ones seen first, and sorts equal values by index: together that is the order "larger value
// first, then smaller index", which is the only order used here, so the set and its order do not
// depend on how the row is split.  NaN logits are never candidates.  The softmax, min-p, top-p
// and the seeded draw over the k candidates stay with the caller (host doubles).
//
// Two stages: CTA (c, t) loads chunk c of row t into shared memory, applies the penalties that
// fall in the chunk, and each thread sorts its own few elements; k block-wide rounds then take the
// best of the threads' list heads (the winner's owner moves on), giving the chunk's k best in
// order.  One warp per row merges the kTopkChunks sorted lists the same way, by shuffles alone.
#include "capi_internal.h"
#include "common.cuh"
#include "internal.h"

namespace zllm {

// a strictly before b: larger value first, then smaller index; an invalid entry (index < 0) last
__device__ __forceinline__ bool cand_before(float av, int ai, float bv, int bi) {
  if (ai < 0) return false;
  if (bi < 0) return true;
  return av > bv || (av == bv && ai < bi);
}

// sampler.js:103-108 in double with explicit rounding (no contraction into fused multiply-adds)
__device__ __forceinline__ float penalize(float l, int cnt, double rp, double freq, double pres) {
  double v = (double)l;
  if (rp != 1.0) v = l > 0.f ? __ddiv_rn(v, rp) : __dmul_rn(v, rp);
  v = __dsub_rn(v, __dadd_rn(__dmul_rn((double)cnt, freq), pres));
  return __double2float_rn(v);
}

// the best (value, index) over the block; every thread returns it
__device__ __forceinline__ void block_best(float &bv, int &bi, float *wv, int *wi) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (cand_before(ov, oi, bv, bi)) { bv = ov; bi = oi; }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { wv[warp] = bv; wi[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    bv = lane < nw ? wv[lane] : -INFINITY;
    bi = lane < nw ? wi[lane] : -1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (cand_before(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    __syncwarp();
    if (lane == 0) { wv[32] = bv; wi[32] = bi; }
  }
  __syncthreads();
  bv = wv[32];
  bi = wi[32];
  __syncthreads();                                       // wv / wi are rewritten by the next round
}

__global__ void topk_part_kernel(const float *logits, int64_t n, int64_t stride, int64_t chunk, int k,
                                 const int32_t *pen_tok, const int32_t *pen_cnt, int n_pen, double rp, double freq,
                                 double pres, float *pv, int *pi) {
  extern __shared__ float sv[];                          // [chunk] values, then [chunk] indices
  int *si = (int *)(sv + chunk);
  __shared__ float wv[33];
  __shared__ int wi[33];
  const int c = blockIdx.x, t = blockIdx.y, tid = threadIdx.x, nt = blockDim.x;
  const float *l = logits + (int64_t)t * stride;
  const int64_t i0 = (int64_t)c * chunk, i1 = min(n, i0 + chunk);
  const int len = i1 > i0 ? (int)(i1 - i0) : 0;
  for (int j = tid; j < len; j += nt) sv[j] = l[i0 + j];
  __syncthreads();
  for (int j = tid; j < n_pen; j += nt) {
    const int tok = pen_tok[j];
    if (tok >= i0 && tok < i1) sv[tok - i0] = penalize(l[tok], pen_cnt[j], rp, freq, pres);
  }
  __syncthreads();
  // each thread sorts its own elements (positions tid, tid + nt, ...) in the order above, NaN last
  const int cnt = tid < len ? (len - tid + nt - 1) / nt : 0;
  for (int q = 0; q < cnt; q++) {
    const int j = tid + q * nt;
    const float v = sv[j];
    const int iv = v != v ? -1 : (int)(i0 + j);
    int p = q;
    while (p > 0 && cand_before(v, iv, sv[tid + (p - 1) * nt], si[tid + (p - 1) * nt])) {
      sv[tid + p * nt] = sv[tid + (p - 1) * nt];
      si[tid + p * nt] = si[tid + (p - 1) * nt];
      p--;
    }
    sv[tid + p * nt] = v;
    si[tid + p * nt] = iv;
  }
  float *ov = pv + ((int64_t)t * gridDim.x + c) * k;
  int *oi = pi + ((int64_t)t * gridDim.x + c) * k;
  // each round the block takes the best of the threads' list heads; the owner (indices are
  // unique) moves to its next element
  int p = 0;
  for (int r = 0; r < k; r++) {
    float hv = -INFINITY;
    int hi = -1;
    if (p < cnt) { hv = sv[tid + p * nt]; hi = si[tid + p * nt]; }
    float bv = hv;
    int bi = hi;
    block_best(bv, bi, wv, wi);
    if (tid == 0) { ov[r] = bv; oi[r] = bi; }
    if (bi >= 0 && bi == hi) p++;
  }
}

// One warp per row merges the nchunk (<= 64) sorted lists of k: lane L owns lists L and L + 32.
__global__ void topk_final_kernel(const float *pv, const int *pi, int nchunk, int k, float *out_v, int32_t *out_i) {
  const int t = blockIdx.x, lane = threadIdx.x;
  const float *cv = pv + (int64_t)t * nchunk * k;
  const int *ci = pi + (int64_t)t * nchunk * k;
  const int la = lane, lb = lane + 32;
  int pa = 0, pb = 0;
  for (int r = 0; r < k; r++) {
    float va = -INFINITY, vb = -INFINITY;
    int ia = -1, ib = -1;
    if (la < nchunk && pa < k) { va = cv[la * k + pa]; ia = ci[la * k + pa]; }
    if (lb < nchunk && pb < k) { vb = cv[lb * k + pb]; ib = ci[lb * k + pb]; }
    const bool from_b = cand_before(vb, ib, va, ia);
    float bv = from_b ? vb : va;
    int bi = from_b ? ib : ia;
    const int mine = bi;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (cand_before(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) { out_v[(int64_t)t * k + r] = bv; out_i[(int64_t)t * k + r] = bi; }
    if (bi >= 0 && bi == mine) { if (from_b) pb++; else pa++; }
  }
}

cudaError_t launch_topk(const float *logits, int64_t n, int64_t stride, int ntok, int k, const int32_t *pen_tok,
                        const int32_t *pen_cnt, int n_pen, double rp, double freq, double pres, float *pv, int *pi,
                        float *out_v, int32_t *out_i, cudaStream_t s) {
  if (ntok <= 0 || k <= 0 || k > kTopkMax || n <= 0) return cudaErrorInvalidValue;
  const int64_t chunk = (n + kTopkChunks - 1) / kTopkChunks;
  if (chunk * (int64_t)(sizeof(float) + sizeof(int)) > kTopkSmem) return cudaErrorInvalidValue;
  topk_part_kernel<<<dim3(kTopkChunks, ntok), 256, chunk * (sizeof(float) + sizeof(int)), s>>>(
      logits, n, stride, chunk, k, pen_tok, pen_cnt, n_pen, rp, freq, pres, pv, pi);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  topk_final_kernel<<<ntok, 32, 0, s>>>(pv, pi, kTopkChunks, k, out_v, out_i);
  return cudaGetLastError();
}

}  // namespace zllm

using namespace zllm;

// Kernel-level entry on host buffers: the same selection over `rows` rows of n logits each.
extern "C" int zllm_topk(zllm_ctx *c, const float *logits_host, int rows, int64_t n, int k, const int32_t *pen_tok,
                         const int32_t *pen_cnt, int n_pen, double repeat_penalty, double frequency, double presence,
                         int32_t *ids_host, float *vals_host) {
  if (!c) return ZLLM_E_ARG;
  if (!logits_host || !ids_host || !vals_host || rows < 1 || n < 1 || k < 1 || k > kTopkMax || k > n || n_pen < 0 ||
      n_pen > kTopkMaxPen || (n_pen && (!pen_tok || !pen_cnt)) ||
      (n + kTopkChunks - 1) / kTopkChunks * (int64_t)(sizeof(float) + sizeof(int)) > kTopkSmem) {
    zllm_set_error(c, "zllm_topk: bad argument");
    return ZLLM_E_ARG;
  }
  for (int j = 0; j < n_pen; j++)
    if (pen_tok[j] < 0 || pen_tok[j] >= n) { zllm_set_error(c, "token id %d out of range", pen_tok[j]); return ZLLM_E_TOKEN; }
  cudaSetDevice(c->device);
  void *l_, *pen_, *pv_, *pi_, *ov_, *oi_;
  int rc;
  if ((rc = zllm_scratch(c, 0, sizeof(float) * n * rows, &l_))) return rc;
  if ((rc = zllm_scratch(c, 1, sizeof(int32_t) * 2 * (n_pen + 1), &pen_))) return rc;
  if ((rc = zllm_scratch(c, 2, sizeof(float) * rows * kTopkChunks * k, &pv_))) return rc;
  if ((rc = zllm_scratch(c, 3, sizeof(int32_t) * rows * kTopkChunks * k, &pi_))) return rc;
  if ((rc = zllm_scratch(c, 4, sizeof(float) * rows * k, &ov_))) return rc;
  if ((rc = zllm_scratch(c, 5, sizeof(int32_t) * rows * k, &oi_))) return rc;
  int32_t *pen = (int32_t *)pen_;
  cudaError_t e = cudaMemcpyAsync(l_, logits_host, sizeof(float) * n * rows, cudaMemcpyHostToDevice, c->stream);
  if (e == cudaSuccess && n_pen) e = cudaMemcpyAsync(pen, pen_tok, sizeof(int32_t) * n_pen, cudaMemcpyHostToDevice, c->stream);
  if (e == cudaSuccess && n_pen)
    e = cudaMemcpyAsync(pen + n_pen, pen_cnt, sizeof(int32_t) * n_pen, cudaMemcpyHostToDevice, c->stream);
  if (e == cudaSuccess)
    e = launch_topk((const float *)l_, n, n, rows, k, pen, pen + n_pen, n_pen, repeat_penalty, frequency, presence,
                    (float *)pv_, (int *)pi_, (float *)ov_, (int32_t *)oi_, c->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(ids_host, oi_, sizeof(int32_t) * rows * k, cudaMemcpyDeviceToHost, c->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(vals_host, ov_, sizeof(float) * rows * k, cudaMemcpyDeviceToHost, c->stream);
  if (e != cudaSuccess) return zllm_cuda_fail(c, e, "zllm_topk");
  return zllm_sync(c);
}
