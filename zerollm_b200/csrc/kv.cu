// KV cache and GQA decode attention for the attention layers of the hot path.
//
//  * qkv_post_kernel -- per token: optional q/k/v biases, per-head q-norm and k-norm (RMSNorm), RoPE
//    on q and k, and the append of k and v to the cache at the token's position, cast f32 -> f16
//    (round to nearest even, NaN as the reference encodes it) or stored as f32.
//    Replaces src/compute/worker.js:296-309 (k-norm :301, RoPE :302, f32ToF16 :305 / f32 copy
//    :307-308) and the q side :313-315; RefModel: src/model/forward.js:113-121.
//  * attn_decode_kernel -- softmax(q K^T / sqrt(hd)) V for the query heads of one KV head over
//    positions [0, npos), split over the context (flash decoding): each CTA streams a range of K/V
//    rows through shared memory with 1D bulk copies, keeps an online softmax, and the last CTA of a
//    (sequence, KV head) merges the partial results.  Replaces the per-head attention of
//    src/compute/worker.js:310-337 (JS loop :320-333, WASM attn_scores / attn_av
//    src/compute/wasm/attn-kernels.js:26-194) and src/model/forward.js:123-140.
//  * kv_convert_kernel -- kvSet / kvGet: f32 [n][kvDim] staging <-> the per-head cache layout
//    (src/compute/worker.js:457-472, src/compute/pool.js:225-238).
//
// Cache layout (per sequence): [layer][k|v][kv_head][ctx][head_dim], element f16 or f32.
#include "common.cuh"
#include "internal.h"

namespace zllm {

// f32 -> f16 bits, round to nearest even; NaN -> sign | 0x7e00 like src/util/f16.js:15.
__device__ __forceinline__ uint16_t f32_to_f16_bits(float x) {
  if (x != x) return (uint16_t)(((__float_as_uint(x) >> 16) & 0x8000u) | 0x7e00u);
  return __half_as_ushort(__float2half_rn(x));
}

// ============================================================================ q/k/v post-processing + append
// One warp per head: heads [0, n_head) are query heads, [n_head, n_head + n_kv) key heads (whose
// value head is appended alongside).  Token t of the batch is at position pos[t] of sequence seq[t].
__global__ void qkv_post_kernel(const QkvPostArgs a) {
  extern __shared__ float sh[];                     // one head_dim row per warp
  pdl_launch_dependents();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int heads = a.n_head + a.n_kv;
  const int gw = blockIdx.x * (blockDim.x >> 5) + warp;
  if (gw >= heads * a.ntok) return;
  const int t = gw / heads, h = gw % heads;
  const bool isq = h < a.n_head;
  const int hd = a.head_dim;
  float *row = sh + warp * hd;
  const float *src = isq ? a.q + (int64_t)t * a.q_stride + h * hd : a.k + (int64_t)t * a.kv_stride + (h - a.n_head) * hd;
  const float *bias = isq ? (a.bq ? a.bq + h * hd : nullptr) : (a.bk ? a.bk + (h - a.n_head) * hd : nullptr);
  const float *norm = isq ? a.q_norm : a.k_norm;
  // bias (worker.js:290-292: f32 += f32)
  for (int i = lane; i < hd; i += 32) {
    float v = src[i];
    if (bias) v = __fadd_rn(v, bias[i]);
    row[i] = v;
  }
  __syncwarp();
  if (norm) {
    // rmsnorm (ref-kernels.js:305-310): ss summed in double in element order (as the JS loop), then
    // s = 1 / sqrt(ss / n + eps) and out = f32(x * s * w)
    double ss = 0.0;
    if (lane == 0)
      for (int i = 0; i < hd; i++) ss = __dadd_rn(ss, __dmul_rn((double)row[i], (double)row[i]));
    ss = __shfl_sync(0xffffffffu, ss, 0);
    const double s = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, (double)hd), a.eps)));
    for (int i = lane; i < hd; i += 32) row[i] = __double2float_rn(__dmul_rn(__dmul_rn((double)row[i], s), (double)norm[i]));
  }
  __syncwarp();
  // RoPE (ref-kernels.js:349-363): v[i0] = a*c - b*s, v[i1] = a*s + b*c in double, stored as f32
  const int pos = a.pos[t];
  const int half = a.n_rot / 2;
  const float *ct = a.rope_cos + (int64_t)pos * half, *st = a.rope_sin + (int64_t)pos * half;
  for (int i = lane; i < half; i += 32) {
    const int i0 = a.neox ? i : 2 * i, i1 = a.neox ? i + half : 2 * i + 1;
    const double x0 = row[i0], x1 = row[i1], c = ct[i], s = st[i];
    const float r0 = __double2float_rn(__dsub_rn(__dmul_rn(x0, c), __dmul_rn(x1, s)));
    const float r1 = __double2float_rn(__dadd_rn(__dmul_rn(x0, s), __dmul_rn(x1, c)));
    row[i0] = r0;
    row[i1] = r1;
  }
  __syncwarp();
  if (isq) {
    float *dst = a.q_out + (int64_t)t * a.q_out_stride + h * hd;
    for (int i = lane; i < hd; i += 32) dst[i] = row[i];
    return;
  }
  // append k and v at `pos` of this sequence's cache (worker.js:303-308)
  const int kh = h - a.n_head;
  const int64_t base = (int64_t)a.seq[t] * a.seq_stride + (int64_t)kh * a.head_stride + (int64_t)pos * hd;
  const float *vsrc = a.v + (int64_t)t * a.kv_stride + kh * hd;
  const float *bv = a.bv ? a.bv + kh * hd : nullptr;
  if (a.kv_f16) {
    uint16_t *kc = reinterpret_cast<uint16_t *>(a.kcache) + base, *vc = reinterpret_cast<uint16_t *>(a.vcache) + base;
    for (int i = lane; i < hd; i += 32) {
      kc[i] = f32_to_f16_bits(row[i]);
      float v = vsrc[i];
      if (bv) v = __fadd_rn(v, bv[i]);
      vc[i] = f32_to_f16_bits(v);
    }
  } else {
    float *kc = reinterpret_cast<float *>(a.kcache) + base, *vc = reinterpret_cast<float *>(a.vcache) + base;
    for (int i = lane; i < hd; i += 32) {
      kc[i] = row[i];
      float v = vsrc[i];
      if (bv) v = __fadd_rn(v, bv[i]);
      vc[i] = v;
    }
  }
}

cudaError_t launch_qkv_post(const QkvPostArgs &a, cudaStream_t s, bool pdl) {
  const int heads = (a.n_head + a.n_kv) * a.ntok;
  if (heads <= 0) return cudaSuccess;
  const int wpb = 8;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((heads + wpb - 1) / wpb);
  cfg.blockDim = dim3(32 * wpb);
  cfg.dynamicSmemBytes = (size_t)wpb * a.head_dim * sizeof(float);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, qkv_post_kernel, a);
}

// ============================================================================ decode attention
// CTA = 8 warps, one (sequence, KV head, context split).  Tiles of TP positions of K and V are bulk
// copied into a ring of shared-memory stages.  Per tile: (1) scores -- LP lanes share one position,
// each dotting HD/LP dims for all G query heads of the group, reduced across the LP lanes; (2) an
// online-softmax update of the running max / sum per head; (3) P.V -- each lane owns HD/32 dims of
// every head of the group and accumulates over the warp's positions.  At the end the 8 warps'
// accumulators are added, and the CTA either writes the final output (one split) or a partial
// (max, sum, acc) that the last CTA of the (sequence, KV head) merges in split order.
constexpr int kAttnWarps = 8;
constexpr int kAttnTP = 64;                          // positions per tile

template <typename T, int HD, int G>
struct AttnCfg {
  static constexpr int LP = G >= 8 ? 16 : (G >= 4 ? 8 : 4);   // lanes per position in the score phase
  static constexpr int DPL = HD / LP;                        // dims per lane in the score phase
  static constexpr int PPW = kAttnTP / kAttnWarps;           // positions per warp per tile
  static constexpr int DPV = HD / 32;                        // dims per lane in the P.V phase
  static constexpr int ROW = HD * (int)sizeof(T);            // bytes per cached position
  static constexpr int TILE = kAttnTP * ROW;                 // bytes of one K (or V) tile
  static constexpr int NS = sizeof(T) == 2 ? 3 : 2;          // stages (shared memory budget)
};

__device__ __forceinline__ void load_row(const uint8_t *p, float *out, int n, bool f16) {
  if (f16 && n % 8) {
    for (int i = 0; i < n; i += 4) {
      const uint2 v = *reinterpret_cast<const uint2 *>(p + 2 * i);
      out[i] = h2f(v.x & 0xffffu); out[i + 1] = h2f(v.x >> 16); out[i + 2] = h2f(v.y & 0xffffu); out[i + 3] = h2f(v.y >> 16);
    }
  } else if (f16) {
    for (int i = 0; i < n; i += 8) {
      const uint4 v = *reinterpret_cast<const uint4 *>(p + 2 * i);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; j++) {
        out[i + 2 * j] = h2f(w[j] & 0xffffu);
        out[i + 2 * j + 1] = h2f(w[j] >> 16);
      }
    }
  } else {
    for (int i = 0; i < n; i += 4) {
      const float4 v = *reinterpret_cast<const float4 *>(p + 4 * i);
      out[i] = v.x; out[i + 1] = v.y; out[i + 2] = v.z; out[i + 3] = v.w;
    }
  }
}

template <typename T, int HD, int G>
__global__ void __launch_bounds__(kAttnWarps * 32, 1) attn_decode_kernel(const AttnArgs a) {
  using C = AttnCfg<T, HD, G>;
  constexpr bool F16 = sizeof(T) == 2;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t *stage = smem;                                                     // [stages][K tile | V tile]
  float *sc = reinterpret_cast<float *>(smem + C::NS * 2 * C::TILE);   // scores / probs [G][TP]
  float *stat = sc + G * kAttnTP;                                            // m_new[G], alpha[G], l[G], m[G]
  float *red = stat + 4 * G;                                                 // [warps][G][HD] accumulators
  uint64_t *full = reinterpret_cast<uint64_t *>(red + kAttnWarps * G * HD);
  uint64_t *empty = full + C::NS;
  int *last_flag = reinterpret_cast<int *>(empty + C::NS);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
  if (threadIdx.x == 0) {
    for (int i = 0; i < C::NS; i++) { mbar_init(&full[i], 1); mbar_init(&empty[i], kAttnWarps); }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();
  pdl_wait();                                         // q and the newest K/V row come from the previous kernel

  // split s covers positions [s * kAttnSplit, (s + 1) * kAttnSplit): the partition depends on the
  // sequence's own length only, so a query gets the same bits alone or in any batch
  const int npos = a.npos[b];
  const int active = npos > 0 ? (npos + kAttnSplit - 1) / kAttnSplit : 1;
  if (split >= active) return;                        // nothing of this sequence here (no partial, no count)
  const int t0 = min(npos, split * kAttnSplit), t1 = min(npos, t0 + kAttnSplit);
  const int ntiles = (t1 - t0 + kAttnTP - 1) / kAttnTP;
  const int64_t cs = a.seq ? a.seq[b] : b;            // cache sequence of this query
  const uint8_t *kbase = reinterpret_cast<const uint8_t *>(a.kcache) +
                         (cs * a.seq_stride + (int64_t)kh * a.head_stride + (int64_t)t0 * HD) * sizeof(T);
  const uint8_t *vbase = reinterpret_cast<const uint8_t *>(a.vcache) +
                         (cs * a.seq_stride + (int64_t)kh * a.head_stride + (int64_t)t0 * HD) * sizeof(T);

  // q of the group's heads: lane holds dims [dc*DPL, +DPL) for the score phase
  const int p_in = lane / C::LP, dc = lane % C::LP;
  float q[G][C::DPL];
#pragma unroll
  for (int g = 0; g < G; g++) {
    const float *qs = a.q + ((int64_t)b * a.n_head + kh * G + g) * HD + dc * C::DPL;
#pragma unroll
    for (int i = 0; i < C::DPL; i++) q[g][i] = qs[i];
  }
  float acc[G][C::DPV];
#pragma unroll
  for (int g = 0; g < G; g++)
#pragma unroll
    for (int i = 0; i < C::DPV; i++) acc[g][i] = 0.f;
  if (threadIdx.x < G) { stat[3 * G + threadIdx.x] = -INFINITY; stat[2 * G + threadIdx.x] = 0.f; }

  int issued = 0;
  auto issue = [&](int i) {                            // thread 0 only
    const int s = i % C::NS;
    const int rows = min(kAttnTP, t1 - t0 - i * kAttnTP);
    const uint32_t bytes = (uint32_t)(rows * C::ROW);
    mbar_arrive_expect_tx(&full[s], 2 * bytes);
    bulk_g2s(stage + (size_t)s * 2 * C::TILE, kbase + (int64_t)i * C::TILE, bytes, &full[s]);
    bulk_g2s(stage + (size_t)s * 2 * C::TILE + C::TILE, vbase + (int64_t)i * C::TILE, bytes, &full[s]);
  };
  if (threadIdx.x == 0)
    for (; issued < ntiles && issued < C::NS; issued++) issue(issued);
  issued = min(ntiles, C::NS);
  __syncthreads();

  const uint64_t deadline = globaltimer_ns() + WAIT_DEADLINE_NS;
  bool aborted = false;
  for (int i = 0; i < ntiles; i++) {
    const int s = i % C::NS;
    const bool ok = mbar_wait_bounded(&full[s], (i / C::NS) & 1, deadline);
    if (!__syncthreads_and(ok)) { aborted = true; break; }   // uniform across the CTA
    const uint8_t *kt = stage + (size_t)s * 2 * C::TILE, *vt = kt + C::TILE;
    const int rows = min(kAttnTP, t1 - t0 - i * kAttnTP);
    // (1) scores
#pragma unroll
    for (int pass = 0; pass < C::PPW * C::LP / 32; pass++) {
      const int tp = warp * C::PPW + pass * (32 / C::LP) + p_in;
      float kv[C::DPL];
      load_row(kt + (size_t)min(tp, rows - 1) * C::ROW + dc * C::DPL * sizeof(T), kv, C::DPL, F16);
      float d[G];
#pragma unroll
      for (int g = 0; g < G; g++) {
        float s0 = 0.f;
#pragma unroll
        for (int j = 0; j < C::DPL; j++) s0 = __fmaf_rn(q[g][j], kv[j], s0);
        d[g] = s0;
      }
#pragma unroll
      for (int o = C::LP / 2; o > 0; o >>= 1)
#pragma unroll
        for (int g = 0; g < G; g++) d[g] = __fadd_rn(d[g], __shfl_xor_sync(0xffffffffu, d[g], o));
      if (dc == 0)
#pragma unroll
        for (int g = 0; g < G; g++) sc[g * kAttnTP + tp] = tp < rows ? d[g] * a.scale : -INFINITY;
    }
    __syncthreads();
    // (2) online softmax: warp g < G owns head g
    if (warp < G) {
      const float v0 = sc[warp * kAttnTP + lane], v1 = sc[warp * kAttnTP + lane + 32];
      float mx = fmaxf(v0, v1);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float m_old = stat[3 * G + warp];
      const float m_new = fmaxf(m_old, mx);
      const float p0 = expf(v0 - m_new), p1 = expf(v1 - m_new);
      sc[warp * kAttnTP + lane] = p0;
      sc[warp * kAttnTP + lane + 32] = p1;
      float ps = p0 + p1;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
      if (lane == 0) {
        const float alpha = m_old == -INFINITY ? 0.f : expf(m_old - m_new);
        stat[G + warp] = alpha;
        stat[2 * G + warp] = stat[2 * G + warp] * alpha + ps;
        stat[3 * G + warp] = m_new;
      }
    }
    __syncthreads();
    // (3) P.V over this warp's positions
#pragma unroll
    for (int g = 0; g < G; g++) {
      const float al = stat[G + g];
#pragma unroll
      for (int i2 = 0; i2 < C::DPV; i2++) acc[g][i2] *= al;
    }
    for (int j = 0; j < C::PPW; j++) {
      const int tp = warp * C::PPW + j;
      if (tp >= rows) break;
      float vv[C::DPV];
      const uint8_t *vr = vt + (size_t)tp * C::ROW + lane * C::DPV * sizeof(T);
      if (F16) {
        if (C::DPV == 4) {
          const uint2 w = *reinterpret_cast<const uint2 *>(vr);
          vv[0] = h2f(w.x & 0xffffu); vv[1] = h2f(w.x >> 16); vv[2] = h2f(w.y & 0xffffu); vv[3] = h2f(w.y >> 16);
        } else {
          const uint32_t w = *reinterpret_cast<const uint32_t *>(vr);
          vv[0] = h2f(w & 0xffffu); vv[C::DPV - 1] = h2f(w >> 16);
        }
      } else {
#pragma unroll
        for (int i2 = 0; i2 < C::DPV; i2++) vv[i2] = reinterpret_cast<const float *>(vr)[i2];
      }
#pragma unroll
      for (int g = 0; g < G; g++) {
        const float pg = sc[g * kAttnTP + tp];
#pragma unroll
        for (int i2 = 0; i2 < C::DPV; i2++) acc[g][i2] = __fmaf_rn(pg, vv[i2], acc[g][i2]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (threadIdx.x == 0 && issued < ntiles) {
      if (mbar_wait_bounded(&empty[s], (i / C::NS) & 1, deadline)) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        issue(issued);
      } else {
        atomicOr(a.status, ST_EMPTY_TIMEOUT);
      }
    }
    issued = min(issued + (issued < ntiles ? 1 : 0), ntiles);
    __syncthreads();                                  // scores are rewritten by the next tile
  }
  if (aborted) {
    if (threadIdx.x == 0) atomicOr(a.status, ST_FULL_TIMEOUT);
  }
  if (threadIdx.x == 0) {
    // copies still in flight (only after an abort) must land before the CTA exits
    const uint64_t dd = globaltimer_ns() + WAIT_DEADLINE_NS;
    for (int s = 0; s < C::NS && s < issued; s++) {
      const int last = s + ((issued - 1 - s) / C::NS) * C::NS;
      if (!mbar_wait_bounded(&full[s], (last / C::NS) & 1, dd)) atomicOr(a.status, ST_DRAIN_TIMEOUT);
    }
  }
  // add the warps' accumulators
#pragma unroll
  for (int g = 0; g < G; g++)
#pragma unroll
    for (int i2 = 0; i2 < C::DPV; i2++) red[((size_t)warp * G + g) * HD + lane * C::DPV + i2] = acc[g][i2];
  __syncthreads();
  for (int e = threadIdx.x; e < G * HD; e += blockDim.x) {
    float sum = 0.f;
    for (int w = 0; w < kAttnWarps; w++) sum += red[(size_t)w * G * HD + e];
    red[e] = sum;                                       // warp 0's slot now holds the CTA total
  }
  __syncthreads();
  const int64_t grp = (int64_t)b * a.n_kv + kh;
  if (active == 1) {
    for (int e = threadIdx.x; e < G * HD; e += blockDim.x) {
      const int g = e / HD;
      const float l = stat[2 * G + g];
      a.out[((int64_t)b * a.n_head + kh * G) * HD + e] = l > 0.f ? red[e] / l : 0.f;
    }
    return;
  }
  // partial: [grp][split] -> m[G], l[G], acc[G][HD]
  float *part = a.partial + (grp * a.nsplit + split) * (size_t)(G * (HD + 2));
  for (int e = threadIdx.x; e < G * HD; e += blockDim.x) part[2 * G + e] = red[e];
  if (threadIdx.x < G) { part[threadIdx.x] = stat[3 * G + threadIdx.x]; part[G + threadIdx.x] = stat[2 * G + threadIdx.x]; }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int done = atomicAdd(a.counters + grp, 1);
    *last_flag = done == active - 1;
  }
  __syncthreads();
  if (!*last_flag) return;
  __threadfence();
  // merge the active splits in split order (deterministic)
  for (int e = threadIdx.x; e < G * HD; e += blockDim.x) {
    const int g = e / HD;
    float M = -INFINITY;
#pragma unroll 8
    for (int j = 0; j < active; j++) M = fmaxf(M, __ldcg(a.partial + (grp * a.nsplit + j) * (size_t)(G * (HD + 2)) + g));
    float L = 0.f, O = 0.f;
#pragma unroll 8
    for (int j = 0; j < active; j++) {
      const float *pj = a.partial + (grp * a.nsplit + j) * (size_t)(G * (HD + 2));
      const float mj = __ldcg(pj + g);
      if (mj == -INFINITY) continue;
      const float f = expf(mj - M);
      L = __fmaf_rn(__ldcg(pj + G + g), f, L);
      O = __fmaf_rn(__ldcg(pj + 2 * G + e), f, O);
    }
    a.out[((int64_t)b * a.n_head + kh * G) * HD + e] = L > 0.f ? O / L : 0.f;
  }
  if (threadIdx.x == 0) a.counters[grp] = 0;            // ready for the next launch
}

size_t attn_smem_bytes(int head_dim, int group, bool f16) {
  const size_t tile = (size_t)kAttnTP * head_dim * (f16 ? 2 : 4);
  const int ns = f16 ? 3 : 2;
  return ns * 2 * tile + sizeof(float) * (group * kAttnTP + 4 * group + (size_t)kAttnWarps * group * head_dim) +
         2 * ns * 8 + 16;
}

template <typename T, int HD, int G>
static cudaError_t launch_attn_t(const AttnArgs &a, cudaStream_t s, bool pdl) {
  auto kern = attn_decode_kernel<T, HD, G>;
  const size_t smem = attn_smem_bytes(HD, G, sizeof(T) == 2);
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
  cfg.gridDim = dim3(a.nsplit, a.n_kv, a.nseq);
  cfg.blockDim = dim3(kAttnWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <typename T, int HD>
static cudaError_t launch_attn_hd(const AttnArgs &a, int group, cudaStream_t s, bool pdl) {
  switch (group) {
    case 1: return launch_attn_t<T, HD, 1>(a, s, pdl);
    case 2: return launch_attn_t<T, HD, 2>(a, s, pdl);
    case 4: return launch_attn_t<T, HD, 4>(a, s, pdl);
    case 8: return launch_attn_t<T, HD, 8>(a, s, pdl);
  }
  return cudaErrorInvalidValue;
}

bool attn_supported(int head_dim, int group) {
  return (head_dim == 64 || head_dim == 128) && (group == 1 || group == 2 || group == 4 || group == 8);
}

cudaError_t launch_attn(const AttnArgs &a, bool f16, cudaStream_t s, bool pdl) {
  const int group = a.n_head / a.n_kv;
  if (!attn_supported(a.head_dim, group)) return cudaErrorInvalidValue;
  if (f16) return a.head_dim == 128 ? launch_attn_hd<uint16_t, 128>(a, group, s, pdl) : launch_attn_hd<uint16_t, 64>(a, group, s, pdl);
  return a.head_dim == 128 ? launch_attn_hd<float, 128>(a, group, s, pdl) : launch_attn_hd<float, 64>(a, group, s, pdl);
}

// ============================================================================ kvSet / kvGet
// dir 0: staging f32 [n][kvDim] -> cache (f16 cast or f32 copy); dir 1: cache -> staging.
__global__ void kv_convert_kernel(float *stage, void *cache, int n, int n_kv, int hd, int64_t head_stride, int kv_f16,
                                  int dir) {
  const int64_t total = (int64_t)n * n_kv * hd;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int i = (int)(e % hd);
    const int64_t th = e / hd;
    const int kh = (int)(th % n_kv);
    const int64_t t = th / n_kv;
    const int64_t c = (int64_t)kh * head_stride + t * hd + i;
    if (kv_f16) {
      uint16_t *cc = reinterpret_cast<uint16_t *>(cache);
      if (dir == 0) cc[c] = f32_to_f16_bits(stage[e]);
      else stage[e] = h2f(cc[c]);
    } else {
      float *cc = reinterpret_cast<float *>(cache);
      if (dir == 0) cc[c] = stage[e];
      else stage[e] = cc[c];
    }
  }
}

cudaError_t launch_kv_convert(float *stage, void *cache, int n, int n_kv, int hd, int64_t head_stride, bool f16, int dir,
                              cudaStream_t s) {
  const int64_t total = (int64_t)n * n_kv * hd;
  if (total <= 0) return cudaSuccess;
  int64_t grid = (total + 255) / 256;
  if (grid > 8192) grid = 8192;
  kv_convert_kernel<<<(unsigned)grid, 256, 0, s>>>(stage, cache, n, n_kv, hd, head_stride, f16 ? 1 : 0, dir);
  return cudaGetLastError();
}

}  // namespace zllm
