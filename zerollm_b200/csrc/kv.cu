// KV cache and GQA decode attention for the attention layers of the hot path.
//
//  * qkv_post_kernel -- per token: optional q/k/v biases, per-head q-norm and k-norm (RMSNorm), RoPE
//    on q and k, and the append of k and v to the cache at the token's position, cast f32 -> f16
//    (round to nearest even, NaN as the reference encodes it) or stored as f32.
//    Replaces src/compute/worker.js:296-309 (k-norm :301, RoPE :302, f32ToF16 :305 / f32 copy
//    :307-308) and the q side :313-315; RefModel: src/model/forward.js:113-121.
//  * attn_mma_kernel (f16 caches) / attn_decode_kernel (f32 caches) -- softmax(q K^T / sqrt(hd)) V
//    for the query heads of one KV head over positions [0, npos), split over the context (flash
//    decoding): each warp of a CTA streams its own run of K/V rows (through a shared-memory stage and
//    the tensor cores, or straight into registers), keeps an online softmax, and the last CTA of a
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
// Head h of token t, by one warp with a head_dim row of shared memory: heads [0, n_head) are query
// heads (the roped query is left in `row`, and copied to q_out unless it is NULL), [n_head, n_head
// + n_kv) key heads (k is normalized, roped and appended with its value head).  Token t of the
// batch is at position pos[t] of sequence seq[t].
__device__ void post_head(const QkvPostArgs &a, int t, int h, float *row, float *q_out, int lane) {
  const bool isq = h < a.n_head;
  const int hd = a.head_dim;
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
    // rmsnorm (ref-kernels.js:305-310): ss summed in double, then s = 1 / sqrt(ss / n + eps) and
    // out = f32(x * s * w).  The sum is a fixed tree (each lane its elements in order, then a
    // butterfly over the lanes) rather than the JS loop's left-to-right order: the double can differ
    // in its last bits, and the f32 outputs then only when that crosses an f32 rounding boundary
    // (as rmsnorm_quant_kernel's tree)
    double ss = 0.0;
    for (int i = lane; i < hd; i += 32) ss = __dadd_rn(ss, __dmul_rn((double)row[i], (double)row[i]));
    ss = warp_sum_f64(ss);
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
    if (q_out)
      for (int i = lane; i < hd; i += 32) q_out[i] = row[i];
    return;
  }
  // append k and v at `pos` of this sequence's cache (worker.js:303-308)
  const int kh = h - a.n_head;
  const int64_t base = a.pages.table ? kv_page_row(a.pages, a.seq[t], a.n_kv, kh, pos, hd, a.status)
                                     : (int64_t)a.seq[t] * a.seq_stride + (int64_t)kh * a.head_stride + (int64_t)pos * hd;
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

// One warp per head of every token.
__global__ void qkv_post_kernel(const QkvPostArgs a) {
  extern __shared__ float sh[];                     // one head_dim row per warp
  pdl_launch_dependents();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int heads = a.n_head + a.n_kv;
  const int gw = blockIdx.x * (blockDim.x >> 5) + warp;
  if (gw >= heads * a.ntok) return;
  const int t = gw / heads, h = gw % heads;
  post_head(a, t, h, sh + warp * a.head_dim, h < a.n_head ? a.q_out + (int64_t)t * a.q_out_stride + h * a.head_dim : nullptr,
            lane);
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
// CTA = W warps (attn_warps(n_kv): 8, or 16 with at most 2 KV heads), one (sequence, KV head,
// context split); the splits of a sequence of n positions are attn_nsplit(n, W) runs of
// W x attn_warp_len(n, W) positions, and each warp streams its own
// attn_warp_len(n, W) positions with no CTA barrier until the end.  Lane l holds dims
// [l*DPL, (l+1)*DPL) of the G query heads and of their output accumulators.  Positions go in
// batches of NB: K and V rows are read straight from HBM (coalesced, the next batch in flight
// while the current one is used); a batch's NI = NB x G partial dot products are added across the
// lanes by a butterfly reduce-scatter (lane l ends with index l / R, R = 32 / NI lanes holding each
// score); an online softmax per head follows (the reference's softmax, ref-kernels.js:313-320,
// computed with a running maximum); the batch's probabilities go through shared memory to every
// lane for P.V.  At the end the 8 warps' (max, sum, acc) are merged in warp order, and a CTA
// either writes the output (one split) or a partial that the last CTA of the (sequence, KV head)
// merges in split order.  Every order is fixed by the sequence's length alone.

template <typename T, int HD>
struct KvRow {
  static constexpr int DPL = HD / 32;                  // dims per lane
  static constexpr int WORDS = DPL * (int)sizeof(T) / 4;  // 32-bit words per lane per row
  uint32_t w[WORDS > 0 ? WORDS : 1];
  // `fresh`: a row this launch wrote (the fused append) -- read through L2, not the read-only path
  __device__ __forceinline__ void load(const T *row, int lane, bool fresh = false) {
    const uint8_t *p = reinterpret_cast<const uint8_t *>(row) + lane * DPL * sizeof(T);
    if (fresh) {
      if constexpr (WORDS == 4) { const uint4 v = __ldcg(reinterpret_cast<const uint4 *>(p)); w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w; }
      else if constexpr (WORDS == 2) { const uint2 v = __ldcg(reinterpret_cast<const uint2 *>(p)); w[0] = v.x; w[1] = v.y; }
      else { w[0] = __ldcg(reinterpret_cast<const uint32_t *>(p)); }
      return;
    }
    if constexpr (WORDS == 4) { const uint4 v = __ldg(reinterpret_cast<const uint4 *>(p)); w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w; }
    else if constexpr (WORDS == 2) { const uint2 v = __ldg(reinterpret_cast<const uint2 *>(p)); w[0] = v.x; w[1] = v.y; }
    else { w[0] = __ldg(reinterpret_cast<const uint32_t *>(p)); }
  }
  __device__ __forceinline__ float get(int i) const {
    if constexpr (sizeof(T) == 2) return h2f((w[i >> 1] >> (16 * (i & 1))) & 0xffffu);
    else return __uint_as_float(w[i]);
  }
  // dims 2 ip and 2 ip + 1 as a packed pair (the same values get() gives)
  __device__ __forceinline__ f2v get2(int ip) const {
    if constexpr (sizeof(T) == 2) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[ip]));
      return f2pack(f.x, f.y);
    } else {
      return f2bits(w[2 * ip], w[2 * ip + 1]);
    }
  }
};

// The end of a decode-attention CTA, after its warps stored their running max / sum (sm, sl) and
// accumulators (sacc(w): warp w's [G][HD] f32) and the CTA synchronised: the W warps merged in warp
// order, then the output (one split) or this split's partial, which the last CTA of the (sequence,
// KV head) merges in split order.
template <int G, int HD, int W, typename Sacc>
__device__ __forceinline__ void attn_finish(const AttnArgs &a, const float (*sm)[G], const float (*sl)[G], Sacc sacc,
                                            int active, int split, int b, int kh, int &last_flag) {
  const int64_t grp = (int64_t)b * a.n_kv + kh;
  float *part = a.partial + (grp * a.nsplit + split) * (size_t)(G * (HD + 2));
  for (int e = threadIdx.x; e < G * HD; e += blockDim.x) {
    const int g = e / HD, d = e % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < W; w++) M = fmaxf(M, sm[w][g]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < W; w++) {
      if (sm[w][g] == -INFINITY) continue;
      const float f = expf(sm[w][g] - M);
      L = __fmaf_rn(sl[w][g], f, L);
      O = __fmaf_rn(sacc(w)[g * HD + d], f, O);
    }
    if (active == 1) {
      a.out[((int64_t)b * a.n_head + kh * G) * HD + e] = L > 0.f ? O / L : 0.f;
    } else {
      part[2 * G + e] = O;
      if (d == 0) { part[g] = M; part[G + g] = L; }
    }
  }
  if (active == 1) return;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int done = atomicAdd(a.counters + grp, 1);
    last_flag = done == active - 1;
  }
  __syncthreads();
  if (!last_flag) return;
  __threadfence();
  // merge the active splits in split order (deterministic).  Up to kMergeFast splits: warp g
  // (< G <= W) reads every split's maximum and sum of head g at once (lane l: splits l, l + 32),
  // finds the maximum M, the factors exp(m_j - M) (0 for a split without a finite maximum, which
  // then adds nothing) and L = sum of l_j f_j (a fixed butterfly); then each thread adds its
  // elements' accumulators over the splits in split order, up to 32 loads in flight.  (Rounds of
  // dependent L2 reads are what this costs: a load-compare-load chain per split measured ~15 us at
  // 37 splits.)  More splits (contexts beyond ~64k positions) take the same arithmetic one split at
  // a time.
  constexpr int kMergeFast = 64;
  constexpr size_t PS = (size_t)G * (HD + 2);
  const float *pbase = a.partial + grp * a.nsplit * PS;
  __shared__ float sf[G][kMergeFast];
  __shared__ float sL[G];
  if (active <= kMergeFast) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp < G) {
      const int g = warp;
      const bool ha = lane < active, hb = lane + 32 < active;
      const float ma = ha ? __ldcg(pbase + lane * PS + g) : -INFINITY, la = ha ? __ldcg(pbase + lane * PS + G + g) : 0.f;
      const float mb = hb ? __ldcg(pbase + (lane + 32) * PS + g) : -INFINITY;
      const float lb = hb ? __ldcg(pbase + (lane + 32) * PS + G + g) : 0.f;
      float M = fmaxf(ma, mb);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
      const float fa = ma == -INFINITY ? 0.f : expf(ma - M), fb = mb == -INFINITY ? 0.f : expf(mb - M);
      if (ha) sf[g][lane] = fa;
      if (hb) sf[g][lane + 32] = fb;
      float L = (fa != 0.f ? la * fa : 0.f) + (fb != 0.f ? lb * fb : 0.f);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
      if (lane == 0) sL[g] = L;
    }
    __syncthreads();
    constexpr int NT = W * 32, EPT = (G * HD + NT - 1) / NT, RND = EPT >= 4 ? 8 : 32 / EPT;
    float O[EPT];
#pragma unroll
    for (int k = 0; k < EPT; k++) O[k] = 0.f;
    for (int j0 = 0; j0 < active; j0 += RND) {
      float o[EPT][RND];
#pragma unroll
      for (int k = 0; k < EPT; k++) {
        const int e = threadIdx.x + k * NT;
#pragma unroll
        for (int jj = 0; jj < RND; jj++)
          o[k][jj] = e < G * HD && j0 + jj < active ? __ldcg(pbase + (j0 + jj) * PS + 2 * G + e) : 0.f;
      }
#pragma unroll
      for (int k = 0; k < EPT; k++) {
        const int e = threadIdx.x + k * NT, g = (e < G * HD ? e : 0) / HD;
#pragma unroll
        for (int jj = 0; jj < RND; jj++) {
          const float f = j0 + jj < active ? sf[g][j0 + jj] : 0.f;
          if (f != 0.f) O[k] = __fmaf_rn(o[k][jj], f, O[k]);
        }
      }
    }
#pragma unroll
    for (int k = 0; k < EPT; k++) {
      const int e = threadIdx.x + k * NT;
      if (e < G * HD) {
        const float L = sL[e / HD];
        a.out[((int64_t)b * a.n_head + kh * G) * HD + e] = L > 0.f ? O[k] / L : 0.f;
      }
    }
  } else {
    for (int e = threadIdx.x; e < G * HD; e += blockDim.x) {
      const int g = e / HD;
      float M = -INFINITY;
      for (int j = 0; j < active; j++) M = fmaxf(M, __ldcg(pbase + j * PS + g));
      float L = 0.f, O = 0.f;
      for (int j = 0; j < active; j++) {
        const float *pj = pbase + j * PS;
        const float mj = __ldcg(pj + g);
        if (mj == -INFINITY) continue;
        const float f = expf(mj - M);
        L = __fmaf_rn(__ldcg(pj + G + g), f, L);
        O = __fmaf_rn(__ldcg(pj + 2 * G + e), f, O);
      }
      a.out[((int64_t)b * a.n_head + kh * G) * HD + e] = L > 0.f ? O / L : 0.f;
    }
  }
  if (threadIdx.x == 0) a.counters[grp] = 0;            // ready for the next launch
}

template <typename T, int HD, int G, bool PAGED, int W>
__global__ void __launch_bounds__(W * 32, 16 / W) attn_decode_kernel(const AttnArgs a) {
  constexpr int kAttnWarps = W;
  constexpr int DPL = HD / 32;
  // batch: 32 / G positions, fewer where K and V of two batches would not fit in registers
  constexpr int NBMAX = 16 / KvRow<T, HD>::WORDS;
  constexpr int NB = 32 / G < NBMAX ? 32 / G : NBMAX;
  constexpr int NI = NB * G, R = 32 / NI;
  __shared__ float sp[kAttnWarps][NB][G];               // a batch's probabilities
  __shared__ float sa[kAttnWarps][G];                   // a batch's rescale factors
  __shared__ float sm[kAttnWarps][G], sl[kAttnWarps][G];
  extern __shared__ __align__(16) float attn_dyn[];
  float(*sacc)[G][HD] = reinterpret_cast<float(*)[G][HD]>(attn_dyn);   // [W][G][HD], dynamic
  __shared__ float sq[G][HD];                           // fused: this KV head's roped queries
  __shared__ int last_flag;

  // Under programmatic dependent launch this runs while the q/k/v projection finishes: in a fused
  // decode pass the cache rows of earlier positions and the lengths are not that kernel's output, so
  // the first K/V batch streams in before griddepcontrol.wait; q and the newest row are read after.
  pdl_launch_dependents();
  if (!a.fused) pdl_wait();                           // unfused: every input may be the previous kernel's
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
  // the partition depends on the sequence's own length only, so a query gets the same bits alone
  // or in any batch
  const int npos = a.npos[b];
  const int ppw = attn_warp_len(npos, W), slen = ppw * kAttnWarps;
  const int active = npos > 0 ? (npos + slen - 1) / slen : 1;
  if (split >= active) return;                        // nothing of this sequence here (no partial, no count)
  const int t0 = min(npos, split * slen), t1 = min(npos, t0 + slen);
  const int w0 = min(t1, t0 + warp * ppw), w1 = min(t1, w0 + ppw);
  const int64_t cs = a.seq ? a.seq[b] : b;            // cache sequence of this query
  const T *kpool = reinterpret_cast<const T *>(a.kcache), *vpool = reinterpret_cast<const T *>(a.vcache);
  const int64_t cbase = PAGED ? 0 : cs * a.seq_stride + (int64_t)kh * a.head_stride;
  // element offset of position p's K (and V) row: contiguous, or through query b's page-table row
  auto row = [&](int p) -> int64_t {
    if constexpr (PAGED) return kv_page_row(a.pages, b, a.n_kv, kh, p, HD, a.status);
    else return cbase + (int64_t)p * HD;
  };
  // fused decode: this launch appends the query's own position npos - 1 (the last split's CTA does)
  const int newp = a.fused ? npos - 1 : -1;

  KvRow<T, HD> kr[NB], vr[NB];
  auto load_batch = [&](int p0, KvRow<T, HD> (&k)[NB], KvRow<T, HD> (&v)[NB]) {
#pragma unroll
    for (int j = 0; j < NB; j++) {
      const int p = min(p0 + j, w1 - 1);               // past the end: repeat the last row (masked below)
      const int64_t o = row(p);
      k[j].load(kpool + o, lane, p == newp);
      v[j].load(vpool + o, lane, p == newp);
    }
  };
  // fused: the first batch streams in during the wait and the prologue unless it holds the row this
  // kernel appends; unfused, the previous kernel may have appended any of the rows (zllm_qkv_append
  // just before), so every load waits
  const bool early = a.fused && !(w0 <= newp && newp < w0 + NB);
  if (w0 < w1 && early) load_batch(w0, kr, vr);
  if (a.fused) pdl_wait();                            // q / k / v come from the previous kernel
  if (a.fused) {
    // q/k/v post-processing of this query (qkv_post_kernel's arithmetic): warps take the KV head's
    // G query heads, and in the last split also the key / value head, which is appended before any
    // warp reads the row
    const int nh = G + (split == active - 1 ? 1 : 0);
    for (int hh = warp; hh < nh; hh += kAttnWarps)
      post_head(a.post, b, hh < G ? kh * G + hh : a.n_head + kh, hh < G ? &sq[hh][0] : &sacc[warp][0][0], nullptr, lane);
    __syncthreads();
  }
  if (w0 < w1 && !early) load_batch(w0, kr, vr);

  // packed pairs (f32x2): the query as pairs of heads (GP of them; a lone head stays scalar), the
  // accumulators as pairs of dims -- every element still takes the scalar code's roundings in the
  // scalar code's order
  constexpr int GP = G / 2, DP = DPL / 2;
  float q[G][DPL];
  f2v qh[GP > 0 ? GP : 1][DPL], acc[G][DP];
#pragma unroll
  for (int g = 0; g < G; g++) {
    const float *qs = a.fused ? &sq[g][lane * DPL] : a.q + ((int64_t)b * a.n_head + kh * G + g) * HD + lane * DPL;
#pragma unroll
    for (int i = 0; i < DPL; i++) q[g][i] = qs[i];
#pragma unroll
    for (int ip = 0; ip < DP; ip++) acc[g][ip] = 0ull;
  }
#pragma unroll
  for (int gp = 0; gp < GP; gp++)
#pragma unroll
    for (int i = 0; i < DPL; i++) qh[gp][i] = f2pack(q[2 * gp][i], q[2 * gp + 1][i]);
  // running max / sum of head (lane % G), kept identically by every lane of that head
  float m_run = -INFINITY, l_run = 0.f;
  const int my_i = lane / R, my_h = my_i % G, my_p = my_i / G;
  for (int p0 = w0; p0 < w1; p0 += NB) {
    KvRow<T, HD> kc[NB], vc[NB];
#pragma unroll
    for (int j = 0; j < NB; j++) { kc[j] = kr[j]; vc[j] = vr[j]; }
    if (p0 + NB < w1) load_batch(p0 + NB, kr, vr);    // the next batch streams while this one is used
    // partial scores, index j * G + g
    float v32[NI];
#pragma unroll
    for (int j = 0; j < NB; j++) {
      float kf[DPL];
#pragma unroll
      for (int ip = 0; ip < DP; ip++) f2unpack(kc[j].get2(ip), kf[2 * ip], kf[2 * ip + 1]);
      if constexpr (GP > 0) {
#pragma unroll
        for (int gp = 0; gp < GP; gp++) {
          f2v d = 0ull;
#pragma unroll
          for (int i = 0; i < DPL; i++) d = f2fma(qh[gp][i], f2pack(kf[i], kf[i]), d);
          f2unpack(d, v32[j * G + 2 * gp], v32[j * G + 2 * gp + 1]);
        }
      } else {
        float d = 0.f;
#pragma unroll
        for (int i = 0; i < DPL; i++) d = __fmaf_rn(q[0][i], kf[i], d);
        v32[j * G] = d;
      }
    }
    // butterfly reduce-scatter: lane l ends with the full sum of index l / R (the R lanes of an
    // index add the same two values at each step, so they hold the same bits)
#pragma unroll
    for (int o = 16, n = NI; o > 0; o >>= 1, n >>= 1) {
      if (n > 1) {
        const bool up = lane & o;
#pragma unroll
        for (int i = 0; i < n / 2; i++) {
          const float send = up ? v32[i] : v32[i + n / 2];
          const float keep = up ? v32[i + n / 2] : v32[i];
          v32[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, o));
        }
      } else {
        v32[0] = __fadd_rn(v32[0], __shfl_xor_sync(0xffffffffu, v32[0], o));
      }
    }
    const bool valid = p0 + my_p < w1;
    const float sc = valid ? v32[0] * a.scale : -INFINITY;
    // online softmax per head over the batch (the positions of one head differ in the lane bits
    // >= log2(R * G); the R copies of a score are not added twice)
    float mx = sc;
#pragma unroll
    for (int o = R * G; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float m_new = fmaxf(m_run, mx);
    const float pr = valid ? expf(sc - m_new) : 0.f;
    float ps = pr;
#pragma unroll
    for (int o = R * G; o < 32; o <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
    const float alpha = m_run == -INFINITY ? 0.f : expf(m_run - m_new);
    l_run = __fmaf_rn(l_run, alpha, ps);
    m_run = m_new;
    if (lane % R == 0) {
      sp[warp][my_p][my_h] = pr;
      if (my_i < G) sa[warp][my_i] = alpha;
    }
    __syncwarp();
#pragma unroll
    for (int g = 0; g < G; g++) {
      const float al = sa[warp][g];
      const f2v al2 = f2pack(al, al);
#pragma unroll
      for (int ip = 0; ip < DP; ip++) acc[g][ip] = f2mul(acc[g][ip], al2);
    }
#pragma unroll
    for (int j = 0; j < NB; j++) {
      f2v pj[G];
#pragma unroll
      for (int g = 0; g < G; g++) {
        const float pg = sp[warp][j][g];
        pj[g] = f2pack(pg, pg);
      }
#pragma unroll
      for (int ip = 0; ip < DP; ip++) {
        const f2v vv = vc[j].get2(ip);
#pragma unroll
        for (int g = 0; g < G; g++) acc[g][ip] = f2fma(pj[g], vv, acc[g][ip]);
      }
    }
    __syncwarp();                                      // sp / sa are rewritten by the next batch
  }
  // merge the 8 warps in warp order (lane g * R holds head g's running max and sum)
#pragma unroll
  for (int g = 0; g < G; g++) {
    const float lg = __shfl_sync(0xffffffffu, l_run, g * R);
    const float mg = __shfl_sync(0xffffffffu, m_run, g * R);
    if (lane == 0) { sl[warp][g] = lg; sm[warp][g] = mg; }
  }
#pragma unroll
  for (int g = 0; g < G; g++)
#pragma unroll
    for (int ip = 0; ip < DP; ip++) f2unpack(acc[g][ip], sacc[warp][g][lane * DPL + 2 * ip], sacc[warp][g][lane * DPL + 2 * ip + 1]);
  __syncthreads();
  attn_finish<G, HD, W>(a, sm, sl, [&](int w) { return &sacc[w][0][0]; }, active, split, b, kh, last_flag);
}

// ============================================================================ decode attention on the tensor cores (f16 KV)
// The same grid, context partition, fused prologue and merges as attn_decode_kernel, for f16
// caches.  A warp streams its positions in chunks of 16 K and V rows through its own shared-memory
// stage (16-byte cp.async, each row's 16-byte pieces XOR-swizzled by row so ldmatrix is free of bank
// conflicts; the next chunk's K rows load during this chunk's softmax and P.V, its V rows during the
// next chunk's Q.K) and does both products with mma.sync m16n8k16 (f16 operands, f32 accumulators):
//   S^T (16 positions x 8 heads) = K (16 x HD) . Q^T       Q as an f16 pair hi + lo: two MMAs per step
//   O^T (HD x 8 heads)          += V^T (HD x 16) . P^T      P = exp(S - max) as an f16 pair hi + lo
// K and V are f16 already, every f16 x f16 product is exact in f32, and the pairs carry q and p to
// ~22 bits, so the result stays within ~1e-6 of the CUDA-core kernel's f32 arithmetic (the f16-KV
// contract is 2e-3).  The online softmax per head is the same running-max form (per chunk of 16
// positions).  P goes from the score layout (positions x heads) to the operand layout (heads x
// positions) in registers with movmatrix.  Heads beyond G are zero queries and never stored.
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
               "{%0, %1, %2, %3};"
               : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
               : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t movm_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
// (x0, x1) as f16 hi and lo pairs: hi = f16(x), lo = f16(x - hi), element 0 in the low half
__device__ __forceinline__ void f16_pair(float x0, float x1, uint32_t &hi, uint32_t &lo) {
  const __half2 h = __floats2half2_rn(x0, x1);
  const __half2 l = __floats2half2_rn(x0 - __low2float(h), x1 - __high2float(h));
  hi = *reinterpret_cast<const uint32_t *>(&h);
  lo = *reinterpret_cast<const uint32_t *>(&l);
}

constexpr int kAttnChunk = 16;
template <int HD> constexpr int attn_stage_bytes() { return 2 * kAttnChunk * HD * 2; }   // K then V rows

template <int HD, int G, bool PAGED, int W>
__global__ void __launch_bounds__(W * 32, 16 / W) attn_mma_kernel(const AttnArgs a) {
  constexpr int ROWB = HD * 2, CH = ROWB / 16, KS = HD / 16, STAGE = attn_stage_bytes<HD>();
  constexpr int PIECES = kAttnChunk * CH / 32;          // 16-byte pieces per lane per tensor
  static_assert(G <= 8 && G * HD * 4 <= STAGE, "a warp's accumulators fit its stage");
  extern __shared__ __align__(128) uint8_t attn_stage[];  // [W][STAGE]; after the loop warp w's [G][HD] f32
  __shared__ float sm[W][G], sl[W][G];
  __shared__ float sq[G][HD];                           // fused: this KV head's roped queries
  __shared__ float srow[HD];                            // fused: the appended key row's staging
  __shared__ int last_flag;

  pdl_launch_dependents();
  if (!a.fused) pdl_wait();                           // unfused: every input may be the previous kernel's
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int split = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
  const int npos = a.npos[b];
  const int ppw = attn_warp_len(npos, W), slen = ppw * W;
  const int active = npos > 0 ? (npos + slen - 1) / slen : 1;
  if (split >= active) return;                        // nothing of this sequence here (no partial, no count)
  const int t0 = min(npos, split * slen), t1 = min(npos, t0 + slen);
  const int w0 = min(t1, t0 + warp * ppw), w1 = min(t1, w0 + ppw);
  const int64_t cs = a.seq ? a.seq[b] : b;
  const uint16_t *kpool = reinterpret_cast<const uint16_t *>(a.kcache), *vpool = reinterpret_cast<const uint16_t *>(a.vcache);
  const int64_t cbase = PAGED ? 0 : cs * a.seq_stride + (int64_t)kh * a.head_stride;
  auto row = [&](int p) -> int64_t {
    if constexpr (PAGED) return kv_page_row(a.pages, b, a.n_kv, kh, p, HD, a.status);
    else return cbase + (int64_t)p * HD;
  };
  const int newp = a.fused ? npos - 1 : -1;
  uint8_t *stage = attn_stage + (size_t)warp * STAGE;
  const uint32_t kst = smem_u32(stage), vst = kst + kAttnChunk * ROWB;
  // one commit group: the 16 K (or V) rows from position p0 (past w1: the last row again, masked)
  auto issue = [&](const uint16_t *pool, uint32_t dst0, int p0) {
#pragma unroll
    for (int k = 0; k < PIECES; k++) {
      const int q = lane + 32 * k, r = q / CH, c = q % CH;
      const int64_t o = row(min(p0 + r, w1 - 1));
      cp_async16(dst0 + r * ROWB + ((c ^ (r & 7)) << 4), pool + o + c * 8);
    }
    cp_async_commit();
  };
  // Q^T as B operands: step j, lane (g, t): head g, dims 16 j + 2 t (+1) and 16 j + 2 t + 8 (+9).
  // Unfused, the query is read before the first copies are issued: loads issued behind a warp's
  // burst of cp.async wait for it to drain (measured ~4 us at 32k positions x 1 sequence).
  uint32_t qh[KS][2], ql[KS][2];
  auto load_q = [&]() {
    const float *qs = a.fused ? &sq[g < G ? g : 0][0] : a.q + ((int64_t)b * a.n_head + kh * G + (g < G ? g : 0)) * HD;
#pragma unroll
    for (int j = 0; j < KS; j++)
#pragma unroll
      for (int e = 0; e < 2; e++) {
        const int d = 16 * j + 2 * t + 8 * e;
        const float x0 = g < G ? qs[d] : 0.f, x1 = g < G ? qs[d + 1] : 0.f;
        f16_pair(x0, x1, qh[j][e], ql[j][e]);
      }
  };
  const bool early = a.fused && !(w0 <= newp && newp < w0 + kAttnChunk);
  if (!a.fused) load_q();
  if (w0 < w1 && (early || !a.fused)) { issue(kpool, kst, w0); issue(vpool, vst, w0); }
  if (a.fused) {
    pdl_wait();                                       // q / k / v come from the previous kernel
    const int nh = G + (split == active - 1 ? 1 : 0);
    for (int hh = warp; hh < nh; hh += W)
      post_head(a.post, b, hh < G ? kh * G + hh : a.n_head + kh, hh < G ? &sq[hh][0] : srow, nullptr, lane);
    __threadfence();                                  // the appended row reaches L2 before any cp.async reads it
    __syncthreads();
    if (w0 < w1 && !early) { issue(kpool, kst, w0); issue(vpool, vst, w0); }
    load_q();
  }
  // running max / sum of heads 2t and 2t + 1, and O^T: m-tile i, lane (g, t) holds dims 16 i + g
  // (c0: head 2t, c1: 2t + 1) and 16 i + g + 8 (c2, c3)
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  float acc[KS][4];
#pragma unroll
  for (int i = 0; i < KS; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  const int lq = lane >> 3, lr = lane & 7;            // ldmatrix: this lane's matrix and row in it
  for (int p0 = w0; p0 < w1; p0 += kAttnChunk) {
    const bool more = p0 + kAttnChunk < w1;
    cp_async_wait<1>();                               // this chunk's K rows (its V rows may still load)
    __syncwarp();
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < KS; j++) {
      uint32_t ka[4];
      const int r = (lq & 1) * 8 + lr, c = 2 * j + (lq >> 1);
      ldsm_x4(kst + r * ROWB + ((c ^ (r & 7)) << 4), ka);
      mma_16816(sc, ka, qh[j][0], qh[j][1]);
      mma_16816(sc, ka, ql[j][0], ql[j][1]);
    }
    __syncwarp();                                     // every lane's K reads are done
    if (more) issue(kpool, kst, p0 + kAttnChunk); else cp_async_commit();
    // online softmax over the chunk: rows g (position p0 + g) and g + 8
    const bool v0 = p0 + g < w1, v1 = p0 + g + 8 < w1;
    const float x0 = v0 ? sc[0] * a.scale : -INFINITY, x1 = v0 ? sc[1] * a.scale : -INFINITY;
    const float x2 = v1 ? sc[2] * a.scale : -INFINITY, x3 = v1 ? sc[3] * a.scale : -INFINITY;
    float mx0 = fmaxf(x0, x2), mx1 = fmaxf(x1, x3);
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
    }
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float al0 = m0 == -INFINITY ? 0.f : expf(m0 - mn0), al1 = m1 == -INFINITY ? 0.f : expf(m1 - mn1);
    const float p_0 = v0 ? expf(x0 - mn0) : 0.f, p_1 = v0 ? expf(x1 - mn1) : 0.f;
    const float p_2 = v1 ? expf(x2 - mn0) : 0.f, p_3 = v1 ? expf(x3 - mn1) : 0.f;
    float ps0 = p_0 + p_2, ps1 = p_1 + p_3;
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      ps0 += __shfl_xor_sync(0xffffffffu, ps0, o);
      ps1 += __shfl_xor_sync(0xffffffffu, ps1, o);
    }
    l0 = __fmaf_rn(l0, al0, ps0);
    l1 = __fmaf_rn(l1, al1, ps1);
    m0 = mn0;
    m1 = mn1;
#pragma unroll
    for (int i = 0; i < KS; i++) {
      acc[i][0] *= al0; acc[i][1] *= al1; acc[i][2] *= al0; acc[i][3] *= al1;
    }
    // P^T operands: rows g / g + 8 of the score layout, transposed
    uint32_t h01, l01, h23, l23;
    f16_pair(p_0, p_1, h01, l01);
    f16_pair(p_2, p_3, h23, l23);
    const uint32_t bh0 = movm_t(h01), bh1 = movm_t(h23), bl0 = movm_t(l01), bl1 = movm_t(l23);
    cp_async_wait<1>();                               // this chunk's V rows
    __syncwarp();
#pragma unroll
    for (int i = 0; i < KS; i++) {
      uint32_t va[4];
      const int r = (lq >> 1) * 8 + lr, c = 2 * i + (lq & 1);
      ldsm_x4_t(vst + r * ROWB + ((c ^ (r & 7)) << 4), va);
      mma_16816(acc[i], va, bh0, bh1);
      mma_16816(acc[i], va, bl0, bl1);
    }
    __syncwarp();                                     // every lane's V reads are done
    if (more) issue(vpool, vst, p0 + kAttnChunk); else cp_async_commit();
  }
  cp_async_wait<0>();
  __syncwarp();
  // this warp's state into its own stage (no other warp reads a stage) and the CTA's max / sum table
  float *sw = reinterpret_cast<float *>(stage);
#pragma unroll
  for (int i = 0; i < KS; i++) {
    if (2 * t < G) { sw[(2 * t) * HD + 16 * i + g] = acc[i][0]; sw[(2 * t) * HD + 16 * i + g + 8] = acc[i][2]; }
    if (2 * t + 1 < G) { sw[(2 * t + 1) * HD + 16 * i + g] = acc[i][1]; sw[(2 * t + 1) * HD + 16 * i + g + 8] = acc[i][3]; }
  }
  if (g == 0) {
    if (2 * t < G) { sm[warp][2 * t] = m0; sl[warp][2 * t] = l0; }
    if (2 * t + 1 < G) { sm[warp][2 * t + 1] = m1; sl[warp][2 * t + 1] = l1; }
  }
  __syncthreads();
  attn_finish<G, HD, W>(a, sm, sl, [&](int w) { return reinterpret_cast<const float *>(attn_stage + (size_t)w * STAGE); },
                        active, split, b, kh, last_flag);
}

// ============================================================================ KV block copy
// nblk blocks of `rows` rows of row_bytes (a multiple of 16) each, between arbitrary row / block
// strides: the prefix-slot save and restore (every layer's K and V of a sequence in one launch) and
// zllm_kv_copy.  16-byte loads and stores, grid-stride; a byte copy, so bit-exact by construction.
__global__ void kv_block_copy_kernel(uint8_t *__restrict__ dst, int64_t dst_row, int64_t dst_blk,
                                     const uint8_t *__restrict__ src, int64_t src_row, int64_t src_blk, int64_t row_bytes,
                                     int rows, int nblk) {
  const int64_t per_row = row_bytes / 16, per_blk = per_row * rows, total = per_blk * nblk;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / per_blk, rem = i % per_blk, r = rem / per_row, c = rem % per_row;
    const uint4 v = __ldg(reinterpret_cast<const uint4 *>(src + b * src_blk + r * src_row) + c);
    reinterpret_cast<uint4 *>(dst + b * dst_blk + r * dst_row)[c] = v;
  }
}

cudaError_t launch_kv_block_copy(void *dst, int64_t dst_row, int64_t dst_blk, const void *src, int64_t src_row,
                                 int64_t src_blk, int64_t row_bytes, int rows, int nblk, int num_sms, cudaStream_t s) {
  const int64_t chunks = row_bytes / 16 * rows * nblk;
  if (chunks <= 0) return cudaSuccess;
  int64_t grid = (chunks + 255) / 256;
  if (grid > (int64_t)num_sms * 8) grid = (int64_t)num_sms * 8;
  kv_block_copy_kernel<<<(unsigned)grid, 256, 0, s>>>((uint8_t *)dst, dst_row, dst_blk, (const uint8_t *)src, src_row,
                                                       src_blk, row_bytes, rows, nblk);
  return cudaGetLastError();
}

template <typename T, int HD, int G, int W>
static cudaError_t launch_attn_w(const AttnArgs &a, cudaStream_t s, bool pdl) {
  constexpr bool MMA = sizeof(T) == 2;                // f16 caches: the tensor-core kernel
  void (*kern)(AttnArgs);
  if constexpr (MMA) kern = a.pages.table ? attn_mma_kernel<HD, G, true, W> : attn_mma_kernel<HD, G, false, W>;
  else kern = a.pages.table ? attn_decode_kernel<T, HD, G, true, W> : attn_decode_kernel<T, HD, G, false, W>;
  const size_t smem = MMA ? (size_t)W * attn_stage_bytes<HD>() : (size_t)W * G * HD * sizeof(float);
  // above 48 KB of dynamic shared memory a kernel must be granted it (once per kernel and device)
  static bool granted[2][64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  bool &gr = granted[a.pages.table ? 1 : 0][dev];
  if (!gr) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    gr = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.nsplit, a.n_kv, a.nseq);
  cfg.blockDim = dim3(W * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <typename T, int HD, int G>
static cudaError_t launch_attn_t(const AttnArgs &a, cudaStream_t s, bool pdl) {
  return attn_warps(a.n_kv) == 16 ? launch_attn_w<T, HD, G, 16>(a, s, pdl) : launch_attn_w<T, HD, G, 8>(a, s, pdl);
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
