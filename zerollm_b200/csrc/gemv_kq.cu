// Decode GEMV for the k-quant formats (Q4_K, Q5_K, Q6_K) with the integer dot products on the
// tensor cores.
//
// Replaces the reference's k-quant matvec kernels: src/compute/ref-kernels.js:196-277 (oracle)
// and the WASM matvec_q4_k / matvec_q5_k / matvec_q6_k and mm_* exports
// (src/compute/wasm/kquant-kernels.js:337-504), dispatched by ggml type as in
// src/compute/worker.js:184-197 / :251-270.
//
// What a launch computes, for 1..8 tokens:  y[t][r] = (y_add) + sum over blocks of
//   Q4_K / Q5_K:  xd * (d*sc*lo - dmin*mn*xs)       per 32-value sub-block (ref-kernels.js:235-236)
//   Q6_K:         xd * d * scale * gsum             per 16-value group     (ref-kernels.js:271)
// where lo / gsum are exact integer dot products of the weight quants with the int8 activation.
//
// The weights are stored as units of (16-row tile, super-block) (kq_layout.h); a CTA owns a
// contiguous range of tiles, i.e. one contiguous range of HBM.  The integer dots are warp-level
// MMAs (mma.sync m16n8k32 / m16n8k16, uint8 or int8 x int8 -> int32, exact) on a unit:
//   * one token (kq_stream_kernel): the B operand is block-diagonal -- column j carries the
//     activation of sub-block (group) j and is zero elsewhere -- so the 8 MMAs of a unit leave the
//     16 rows x 8 sub-blocks of integer dots in one accumulator, one value per lane and row pair.
//     Every warp streams its share of the CTA's units straight from HBM into registers (coalesced
//     16-byte loads, a few units in flight), with no shared-memory staging of the weights;
//   * 2..8 tokens (kq_tok_kernel): B column j carries token j, one MMA per sub-block (group); runs
//     of units are staged in shared memory by 1D bulk copies (one per stage, completion on an
//     mbarrier) and shared by the 8 warps.
// Each integer dot becomes its block term in IEEE double with the reference's operations and
// rounding (no fused multiply-add where the JS rounds twice), so every block term is bit-identical
// to the oracle's.  Only the order of the final double additions differs from the reference, and
// it is fixed: each super-block's terms are added as a pairwise tree (Q4_K / Q5_K:
// ((T0 + T1) + (T2 + T3)) + ((T4 + T5) + (T6 + T7)); Q6_K: the same over groups 0..7 plus the same
// over 8..15) and the super-block sums are added in super-block order.  That order depends on
// nothing but the row, so a token gets the same bits alone, in a batch, or in any launch shape.
// A one-token launch may take the f32 activation (optionally RMSNorm-ed first) and quantize it
// itself, bit-exact with quantize_act_kernel, so a lone matvec is one kernel.
#include "common.cuh"
#include "internal.h"
#include "kq_layout.h"

namespace zllm {

namespace {

constexpr int kTile = kKqTile;               // rows per unit (the MMA's M)
constexpr int kMaxTok = 8;                   // tokens per launch of the token kernel (the MMA's N)

// unit regions (kq_layout.h)
template <int FMT> constexpr int unit_bytes() { return FMT == T_Q4_K ? 2304 : FMT == T_Q5_K ? 2816 : 3360; }
template <int FMT> constexpr int hdr_off() { return FMT == T_Q4_K ? 2048 : 2560; }   // Q4_K / Q5_K header region
constexpr int kE5 = 2048;                                  // Q5_K high bits
constexpr int kQ6H = 2048, kQ6S = 3072, kQ6D = 3328;        // Q6_K qh, scales, d

// ---------------------------------------------------------------------------- tensor-core dots
// C += A . B with A 16 x K uint8 (weights), B K x 8 int8 (activations), exact int32 accumulation.
__device__ __forceinline__ void mma_k32(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_k16(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm("mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5}, {%6}, {%0, %1, %2, %3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(b0));
}

// C += A . B, both int8 (the signed Q6_K quants q - 32 against the activation)
__device__ __forceinline__ void mma_k16s(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm("mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5}, {%6}, {%0, %1, %2, %3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(b0));
}

// f16 bits -> double (exact)
__device__ __forceinline__ double h2d(uint32_t bits16) {
  double d;
  asm("cvt.f64.f16 %0, %1;" : "=d"(d) : "h"((unsigned short)bits16));
  return d;
}

// Bounded wait on an mbarrier phase by lane 0 alone (the other lanes would only queue on the same
// word); the result is broadcast and __syncwarp orders the stage's data for the whole warp.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t *bar, uint32_t parity, int lane) {
  bool ok = true;
  if (lane == 0) ok = mbar_wait_lazy(bar, parity);
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  return ok;
}

__device__ __forceinline__ double dshfl_xor(double v, int m) { return __shfl_xor_sync(0xffffffffu, v, m); }
// Sum over the 4 lanes t of a lane quad: ((v0 + v1) + (v2 + v3)) in every lane of the quad.
__device__ __forceinline__ double quad_tree(double v) {
  v = __dadd_rn(v, dshfl_xor(v, 1));
  return __dadd_rn(v, dshfl_xor(v, 2));
}

// ---------------------------------------------------------------------------- block terms
// Q4_K / Q5_K sub-block term xd * (d*sc*lo - dmin*mn*xs).  sc*lo and mn*xs are exact int32, so
// d*(sc*lo) and dmin*(mn*xs) are the JS products (d*sc)*lo and (dmin*mn)*xs exactly; the fused
// multiply-add rounds once where the JS subtraction rounds; the product by xd rounds like the JS.
__device__ __forceinline__ double k45_term(double d, double dmin, int sc, int mn, int lo, int xs, double xd) {
  const double p = i2d_biased((uint32_t)(sc * lo) + 0x80000000u);
  const double m = __dmul_rn(dmin, i2d_biased((uint32_t)(mn * xs) + 0x80000000u));
  return __dmul_rn(xd, __fma_rn(d, p, -m));
}
// Q6_K group term xd * d * scale * gsum: xd*d (35 bits) and (xd*d)*scale are exact in double, so the
// JS left-to-right product equals (xd*d) * (scale*gsum) rounded once.
__device__ __forceinline__ double q6_term(double xdd, int scale, int gsum) {
  return __dmul_rn(xdd, i2d_exact(scale * gsum));
}
// the 24-bit scale/min field of chunk c from header words 1..3 of a Q4_K / Q5_K block
__device__ __forceinline__ uint32_t k45_field(const uint4 &h, int c) {
  const uint32_t lo = c < 2 ? h.y : (c == 2 ? h.z : h.w);
  const uint32_t hi = c == 0 ? h.y : (c == 1 ? h.z : (c == 2 ? h.w : 0u));
  return __funnelshift_r(lo, hi, (24 * c) & 31);
}
// Q6_K quants of one (row, half, 16-value run) for group k = 0..3 from ql words (p0, p1) and the qh word
__device__ __forceinline__ uint32_t q6_unpack(uint32_t w0, uint32_t w1, uint32_t h, int k) {
  switch (k) {
    case 0: return (w0 & 0x0f0f0f0fu) | ((h << 4) & 0x30303030u);
    case 1: return (w1 & 0x0f0f0f0fu) | ((h << 2) & 0x30303030u);
    case 2: return ((w0 >> 4) & 0x0f0f0f0fu) | (h & 0x30303030u);
    default: return ((w1 >> 4) & 0x0f0f0f0fu) | ((h >> 2) & 0x30303030u);
  }
}

// ---------------------------------------------------------------------------- activation views
// One-token activation staged in shared memory: xq [K] int8, xd [K/32] f64 (the f32 scales,
// widened once), xs [K/32] i32, and for Q6_K xs16 [K/16] i32 (sums of the stored int8 per
// 16-value group).  sel[s] = 1 when the lane's MMA column is s, else 0: the block-diagonal B
// operand is x * sel[s], a multiply on the FMA pipe instead of a select on the integer pipe.
struct SAct {
  uint32_t xq, xd, xs, xs16;    // shared-window addresses
  uint32_t sel[8];
};
// 2..8 tokens, read from global memory
struct GAct {
  const int8_t *xq;     // [ntok][k]
  const float *xd;      // [ntok][k/32]
  const int32_t *xs;    // [ntok][k/32]
  int64_t k;
  int ntok;
};

struct KqArgs {
  const uint8_t *w;     // first unit of the launch's first tile
  int64_t rows;         // rows of the launch (the last tile may be partial)
  int nb;               // super-blocks per row
  int nchunk;           // token kernel: chunks of super-blocks per tile
  int nst;              // token kernel: stages in the ring
  int ntok;             // tokens in this launch (1..8)
  const int8_t *xq;     // quantized activation [ntok][k] (one token: may be NULL with x set)
  const float *xd;
  const int32_t *xs;
  const float *x;       // f32 activation, quantized in the kernel when xq is NULL
  const float *norm_w;  // with x: RMSNorm x with these weights before quantizing (NULL: none)
  double norm_eps;
  int swiglu;           // rows are (gate, up) pairs: y gets silu(gate) * up, one value per pair
  int64_t k;
  float *y;
  const float *y_add;
  int64_t y_stride;
  unsigned *status;
  int x_off, part_off, bar_off;   // shared-memory regions
};

// tiles [T0, T1) of a CTA: an even split of the launch's tiles
__device__ __forceinline__ void cta_tiles(int64_t rows, int &T0, int &T1) {
  const int64_t nt = (rows + kTile - 1) / kTile;
  T0 = (int)((int64_t)blockIdx.x * nt / gridDim.x);
  T1 = (int)((int64_t)(blockIdx.x + 1) * nt / gridDim.x);
}

// y for output row r (launch-relative) from its f64 total; with swiglu the (gate, up) pair
// r, r + 1 is written once, by r (src/compute/worker.js:426, ref-kernels.js:322: silu in double,
// the product rounded to f32)
__device__ __forceinline__ void store_row(const KqArgs &p, int tok, int64_t r, float out, float up) {
  if (p.swiglu) {
    const double z = out;
    const double sl = __ddiv_rn(z, __dadd_rn(1.0, exp(-z)));
    p.y[(int64_t)tok * p.y_stride + r / 2] = __double2float_rn(__dmul_rn(sl, (double)up));
  } else {
    const int64_t o = (int64_t)tok * p.y_stride + r;
    if (p.y_add) out = __fadd_rn(p.y_add[o], out);
    p.y[o] = out;
  }
}

// RMSNorm scale 1 / sqrt(mean(x^2) + eps) of one token, with exactly the reduction of
// rmsnorm_quant_kernel (ops.cu): 256 partial sums, sum i = t (mod 256) for thread t, then a
// butterfly within each of 8 warps and one over the 8 warp sums -- so both give the same bits.
template <int NT>
__device__ double rms_scale(const float *x, int64_t n, double eps, int warp, int lane) {
  static_assert(NT >= 256, "rms_scale needs 256 threads");
  __shared__ double red[8];
  double ss = 0.0;
  if (threadIdx.x < 256)
    for (int64_t i = threadIdx.x; i < n; i += 256) ss = __dadd_rn(ss, __dmul_rn((double)x[i], (double)x[i]));
  if (warp < 8) {
    ss = warp_sum_f64(ss);
    if (lane == 0) red[warp] = ss;
  }
  __syncthreads();
  double tot = lane < 8 ? red[lane] : 0.0;
  tot = warp_sum_f64(tot);
  return __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(tot, (double)n), eps)));
}

// Quantize one token's f32 activation into shared memory; bit-exact with quantize_act_kernel
// (quantizeAct, src/compute/ref-kernels.js:44-62).  Lane pairs own a 32-value block, 16 values each.
// With norm_w the values are first f32(x * s * w) with s the RMSNorm scale (ref-kernels.js:305-310),
// as rmsnorm_quant_kernel writes them.
template <int NT>
__device__ void quantize_to_smem(const float *x, int64_t k, const float *norm_w, double eps, uint8_t *sxq, double *sxd,
                                 int32_t *sxs, int32_t *sxs16, int warp, int lane) {
  const double rs = norm_w ? rms_scale<NT>(x, k, eps, warp, lane) : 0.0;
  const int nhb = (int)(k / 16);
  for (int base = warp * 32; base < nhb; base += NT) {
    const int hb = base + lane;
    const bool act = hb < nhb;
    float v[16];
    if (act) {
      const float4 *p = reinterpret_cast<const float4 *>(x + (int64_t)hb * 16);
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const float4 f = __ldg(p + i);
        v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
      }
      if (norm_w) {
        const float4 *wp = reinterpret_cast<const float4 *>(norm_w + (int64_t)hb * 16);
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const float4 f = __ldg(wp + i);
          const float wv[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
          for (int j = 0; j < 4; j++) v[4 * i + j] = __double2float_rn(__dmul_rn(__dmul_rn((double)v[4 * i + j], rs), (double)wv[j]));
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 16; i++) v[i] = 0.f;
    }
    float a = 0.f;
#pragma unroll
    for (int i = 0; i < 16; i++) {
      const float m = fabsf(v[i]);
      if (m > a) a = m;                         // NaN never raises amax (as `Math.abs(NaN) > amax`)
    }
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
    const double scale = __ddiv_rn((double)a, 127.0);
    const double inv = scale != 0.0 ? __ddiv_rn(1.0, scale) : 0.0;
    uint32_t words[4] = {0, 0, 0, 0};
    int sum = 0;
    bool nan = false;
#pragma unroll
    for (int i = 0; i < 16; i++) {
      const double r = round(__dmul_rn((double)v[i], inv));   // half away from zero
      const bool bad = !(r == r);
      const int q = bad ? 0 : (int)r;
      nan |= bad;
      sum += q;
      words[i >> 2] |= (uint32_t)(q & 0xff) << (8 * (i & 3));
    }
    const int osum = __shfl_xor_sync(0xffffffffu, sum, 1);
    const bool onan = __shfl_xor_sync(0xffffffffu, (int)nan, 1) != 0;
    if (act) {
      reinterpret_cast<uint4 *>(sxq)[hb] = make_uint4(words[0], words[1], words[2], words[3]);
      if (sxs16) sxs16[hb] = sum;
      if ((lane & 1) == 0) {
        sxd[hb >> 1] = (double)__double2float_rn(scale);
        sxs[hb >> 1] = (nan || onan) ? 0 : sum + osum;
      }
    }
  }
}

// ---------------------------------------------------------------------------- 2..8 tokens
// One unit in shared memory at `u` (kq_layout.h): lane (g, t) computes rows g and g + 8 for tokens
// 2t and 2t + 1.  S[e] (e = 2 * row half + token parity) = the super-block sum in the canonical
// tree order.
template <bool FIVE>
__device__ __forceinline__ void sb_k45_tok(uint32_t u, int lane, int g, int t, const GAct &x, int sb, double (&S)[4]) {
  constexpr int HO = FIVE ? 2560 : 2048;
  const uint4 hdr[2] = {lds128(u + HO + 16 * g), lds128(u + HO + 16 * (g + 8))};
  const bool live = g < x.ntok;
  const uint32_t *xw = reinterpret_cast<const uint32_t *>(x.xq + (live ? g : 0) * x.k + (int64_t)sb * 256);
  const int t0 = 2 * t < x.ntok ? 2 * t : 0, t1 = 2 * t + 1 < x.ntok ? 2 * t + 1 : 0;   // padding tokens read token 0
  const float *xd0 = x.xd + t0 * (x.k / 32) + sb * 8, *xd1 = x.xd + t1 * (x.k / 32) + sb * 8;
  const int32_t *xs0 = x.xs + t0 * (x.k / 32) + sb * 8, *xs1 = x.xs + t1 * (x.k / 32) + sb * 8;
  double dd[2], dm[2];
#pragma unroll
  for (int ri = 0; ri < 2; ri++) { dd[ri] = h2d(hdr[ri].x & 0xffffu); dm[ri] = h2d(hdr[ri].x >> 16); }
  uint2 eg = make_uint2(0, 0), eh = make_uint2(0, 0);
  if (FIVE) { eg = lds64(u + kE5 + 8 * lane); eh = lds64(u + kE5 + 256 + 8 * lane); }
  double q01[4];
#pragma unroll
  for (int cp = 0; cp < 2; cp++) {
    const uint4 wq = lds128(u + (cp * 32 + lane) * 16), vq = lds128(u + ((2 + cp) * 32 + lane) * 16);
#pragma unroll
    for (int ci = 0; ci < 2; ci++) {
      const int c = 2 * cp + ci;
      const uint32_t wx = ci ? wq.z : wq.x, wy = ci ? wq.w : wq.y, vx = ci ? vq.z : vq.x, vy = ci ? vq.w : vq.y;
      uint32_t lg0 = wx & 0x0f0f0f0fu, lg1 = wy & 0x0f0f0f0fu, lh0 = vx & 0x0f0f0f0fu, lh1 = vy & 0x0f0f0f0fu;
      uint32_t ug0, ug1, uh0, uh1;
      if (FIVE) {
        lg0 |= ((eg.x >> (2 * c)) & 0x01010101u) << 4; lg1 |= ((eg.y >> (2 * c)) & 0x01010101u) << 4;
        lh0 |= ((eh.x >> (2 * c)) & 0x01010101u) << 4; lh1 |= ((eh.y >> (2 * c)) & 0x01010101u) << 4;
        ug0 = ((wx >> 4) & 0x0f0f0f0fu) | (((eg.x >> (2 * c + 1)) & 0x01010101u) << 4);
        ug1 = ((wy >> 4) & 0x0f0f0f0fu) | (((eg.y >> (2 * c + 1)) & 0x01010101u) << 4);
        uh0 = ((vx >> 4) & 0x0f0f0f0fu) | (((eh.x >> (2 * c + 1)) & 0x01010101u) << 4);
        uh1 = ((vy >> 4) & 0x0f0f0f0fu) | (((eh.y >> (2 * c + 1)) & 0x01010101u) << 4);
      } else {
        ug0 = wx & 0xf0f0f0f0u; ug1 = wy & 0xf0f0f0f0u; uh0 = vx & 0xf0f0f0f0u; uh1 = vy & 0xf0f0f0f0u;
      }
      // token g's activation of sub-blocks 2c (lo) and 2c+1 (hi)
      const uint32_t xla = live ? __ldg(xw + 16 * c + t) : 0u, xlb = live ? __ldg(xw + 16 * c + 4 + t) : 0u;
      const uint32_t xua = live ? __ldg(xw + 16 * c + 8 + t) : 0u, xub = live ? __ldg(xw + 16 * c + 12 + t) : 0u;
      int L[4] = {0, 0, 0, 0}, U[4] = {0, 0, 0, 0};
      mma_k32(L, lg0, lh0, lg1, lh1, xla, xlb);
      mma_k32(U, ug0, uh0, ug1, uh1, xua, xub);
      const float2 d0 = __ldg(reinterpret_cast<const float2 *>(xd0 + 2 * c)), d1 = __ldg(reinterpret_cast<const float2 *>(xd1 + 2 * c));
      const int2 s0 = __ldg(reinterpret_cast<const int2 *>(xs0 + 2 * c)), s1 = __ldg(reinterpret_cast<const int2 *>(xs1 + 2 * c));
      const uint32_t F[2] = {k45_field(hdr[0], c), k45_field(hdr[1], c)};
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int ri = e >> 1, ti = e & 1;
        const int hi = FIVE ? U[e] : U[e] >> 4;
        const double xdl = (double)(ti ? d1.x : d0.x), xdu = (double)(ti ? d1.y : d0.y);
        const int xsl = ti ? s1.x : s0.x, xsu = ti ? s1.y : s0.y;
        const double P = __dadd_rn(k45_term(dd[ri], dm[ri], F[ri] & 63, (F[ri] >> 12) & 63, L[e], xsl, xdl),
                                   k45_term(dd[ri], dm[ri], (F[ri] >> 6) & 63, (F[ri] >> 18) & 63, hi, xsu, xdu));
        // pairwise tree over the four pairs: ((P0 + P1) + (P2 + P3))
        if (c == 0 || c == 2) q01[e] = P;
        else if (c == 1) S[e] = __dadd_rn(q01[e], P);
        else S[e] = __dadd_rn(S[e], __dadd_rn(q01[e], P));
      }
    }
  }
}

// Q6_K, 2..8 tokens: Sh[e][h] = tree8 of half h, ((P0 + P1) + (P2 + P3)) with P_k the pair of
// groups 8h + 2k, 8h + 2k + 1 (the pair lane k holds in the one-token path).
__device__ __forceinline__ void sb_q6_tok(uint32_t u, int lane, int g, int t, const GAct &x, int sb,
                                          double (&Sh)[4][2]) {
  const double d[2] = {h2d(lds16(u + kQ6D + 2 * g)), h2d(lds16(u + kQ6D + 2 * (g + 8)))};
  const uint4 scw[2] = {lds128(u + kQ6S + 16 * g), lds128(u + kQ6S + 16 * (g + 8))};   // the rows' 16 scales
  const uint4 qhw[2] = {lds128(u + kQ6H + 16 * lane), lds128(u + kQ6H + 512 + 16 * lane)};
  const bool live = g < x.ntok;
  const uint32_t *xw = reinterpret_cast<const uint32_t *>(x.xq + (live ? g : 0) * x.k + (int64_t)sb * 256);
  const int t0 = 2 * t < x.ntok ? 2 * t : 0, t1 = 2 * t + 1 < x.ntok ? 2 * t + 1 : 0;
  const float *xd0 = x.xd + t0 * (x.k / 32) + sb * 8, *xd1 = x.xd + t1 * (x.k / 32) + sb * 8;
#pragma unroll
  for (int h = 0; h < 2; h++) {
    // this lane's quants of half h: ql words [u][p], qh words [u] (values 4t..4t+3 of each group)
    const uint4 lg = lds128(u + (h * 32 + lane) * 16), lh = lds128(u + ((2 + h) * 32 + lane) * 16);
    const uint32_t gw[4] = {lg.x, lg.y, lg.z, lg.w}, hw[4] = {lh.x, lh.y, lh.z, lh.w};
    const uint32_t gq[2] = {h ? qhw[0].z : qhw[0].x, h ? qhw[0].w : qhw[0].y};
    const uint32_t hq[2] = {h ? qhw[1].z : qhw[1].x, h ? qhw[1].w : qhw[1].y};
    double q[4][2];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      // scales of groups 8h + 2k + uu (reordered table: byte 4k + 2h + uu) and their 32-block's xd
      const uint32_t swd[2] = {k == 0 ? scw[0].x : k == 1 ? scw[0].y : k == 2 ? scw[0].z : scw[0].w,
                               k == 0 ? scw[1].x : k == 1 ? scw[1].y : k == 2 ? scw[1].z : scw[1].w};
      const uint32_t sw[2] = {(swd[0] >> (16 * h)) & 0xffffu, (swd[1] >> (16 * h)) & 0xffffu};
      const double xdv[2] = {(double)__ldg(xd0 + 4 * h + k), (double)__ldg(xd1 + 4 * h + k)};
      double P[4];
#pragma unroll
      for (int uu = 0; uu < 2; uu++) {
        // signed quants q - 32 (bytes in [0, 63]: + 96 never carries, then flip the top bit)
        const uint32_t a0 = (q6_unpack(gw[uu * 2], gw[uu * 2 + 1], gq[uu], k) + 0x60606060u) ^ 0x80808080u;
        const uint32_t a1 = (q6_unpack(hw[uu * 2], hw[uu * 2 + 1], hq[uu], k) + 0x60606060u) ^ 0x80808080u;
        const uint32_t xa = live ? __ldg(xw + 4 * (8 * h + 2 * k + uu) + t) : 0u;
        int Cm[4] = {0, 0, 0, 0};
        mma_k16s(Cm, a0, a1, xa);
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const int ri = e >> 1, ti = e & 1;
          const int scale = (int)(int8_t)((sw[ri] >> (8 * uu)) & 0xffu);
          const double T = q6_term(__dmul_rn(xdv[ti], d[ri]), scale, Cm[e]);
          P[e] = uu == 0 ? T : __dadd_rn(P[e], T);
        }
      }
#pragma unroll
      for (int e = 0; e < 4; e++) {
        if (k == 0 || k == 2) q[e][k >> 1] = P[e];
        else q[e][k >> 1] = __dadd_rn(q[e][k >> 1], P[e]);
      }
    }
#pragma unroll
    for (int e = 0; e < 4; e++) Sh[e][h] = __dadd_rn(q[e][0], q[e][1]);
  }
}

// super-blocks per staged chunk (Q6_K: more bytes and twice the MMAs per super-block)
template <int FMT> constexpr int chunk_sb() { return FMT == T_Q6_K ? 8 : 16; }
constexpr int chunk_sb_of(int type) { return type == T_Q6_K ? 8 : 16; }
constexpr int kTokWarps = 8;
constexpr int kMaxStages = 8;
constexpr int64_t kTokBudget = 200 * 1024;   // one CTA per SM (the grid is at most one per SM)

// 2..8 tokens.  A CTA owns tiles [T0, T1) and walks them in chunks of up to kChunk super-blocks:
// stage s of the ring holds one chunk (one bulk copy of its contiguous units, issued by lane 0 of
// warp 0, completion on full[s]).  Warp w takes super-blocks w and w + 8 of every chunk; each
// lane writes its super-block sums to a per-chunk slot array, one CTA barrier (which also carries
// the bounded waits' give-up flag to every warp) publishes them, and one thread per (row, token)
// adds them in super-block order while warp 0 refills the freed stage.
template <int FMT>
__global__ void __launch_bounds__(kTokWarps * 32, 1) kq_tok_kernel(const KqArgs p) {
  constexpr int US = unit_bytes<FMT>();
  constexpr int NTP = kMaxTok, NT = kTokWarps * 32;
  constexpr int kChunk = chunk_sb<FMT>();
  constexpr int kSlots = 16;                    // per-chunk slots of super-block sums (Q6_K: 8 x 2 halves)
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int nst = p.nst;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + p.bar_off);
  uint8_t *stages = smem;
  double *part = reinterpret_cast<double *>(smem + p.part_off);    // [2][slot][row][NTP]
  int T0, T1;
  cta_tiles(p.rows, T0, T1);
  const int nunit = (T1 - T0) * p.nchunk;       // this CTA's (tile, chunk) units of work
  const int stage_bytes = kChunk * US;

  auto issue = [&](int u) {                     // lane 0 of warp 0
    const int s = u % nst, tile = u / p.nchunk, c = u % p.nchunk;
    const int sb0 = c * kChunk, nsb = min(kChunk, p.nb - sb0);
    const uint32_t bytes = (uint32_t)(nsb * US);
    mbar_arrive_expect_tx(&full[s], bytes);
    bulk_g2s(stages + (size_t)s * stage_bytes, p.w + ((int64_t)(T0 + tile) * p.nb + sb0) * US, bytes, &full[s]);
  };

  int issued = 0;                               // units issued so far (tracked by lane 0 of warp 0)
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < nst; s++) mbar_init(&full[s], 1);
    fence_mbar_init();
    for (; issued < nunit && issued < nst; issued++) issue(issued);
  }
  pdl_launch_dependents();
  __syncthreads();                              // barriers initialised before anyone waits on them
  pdl_wait();                                   // the activation comes from the previous kernel

  GAct ga{};
  ga.xq = p.xq; ga.xd = p.xd; ga.xs = p.xs; ga.k = p.k; ga.ntok = p.ntok;
  const uint32_t sbase = smem_u32(stages);
  const bool adder = threadIdx.x < kTile * NTP;
  double tot = 0.0;
  bool aborted = false;
  for (int u = 0; u < nunit; u++) {
    const int s = u % nst, tile = u / p.nchunk, c = u % p.nchunk;
    // after one give-up the warp waits no more: it only passes the barriers until all stop together
    const bool ok = !aborted && mbar_wait_warp(&full[s], (uint32_t)(u / nst) & 1u, lane);
    const int sb0 = c * kChunk, nsb = min(kChunk, p.nb - sb0);
    double *pu = part + (size_t)(u & 1) * kSlots * kTile * NTP;
    if (ok) {
      const uint32_t st = sbase + (uint32_t)(s * stage_bytes);
#pragma unroll
      for (int jj = 0; jj < kChunk / kTokWarps; jj++) {
        const int j = warp + kTokWarps * jj;
        if (j >= nsb) break;
        const uint32_t un = st + (uint32_t)(j * US);
        if constexpr (FMT == T_Q6_K) {
          double Sh[4][2];
          sb_q6_tok(un, lane, g, t, ga, sb0 + j, Sh);
#pragma unroll
          for (int e = 0; e < 4; e++)
#pragma unroll
            for (int h = 0; h < 2; h++)
              pu[((j + 8 * h) * kTile + g + 8 * (e >> 1)) * NTP + 2 * t + (e & 1)] = Sh[e][h];
        } else {
          double S[4];
          sb_k45_tok<FMT == T_Q5_K>(un, lane, g, t, ga, sb0 + j, S);
#pragma unroll
          for (int e = 0; e < 4; e++) pu[(j * kTile + g + 8 * (e >> 1)) * NTP + 2 * t + (e & 1)] = S[e];
        }
      }
    }
    // every warp is done with stage s and has published its sums
    if (named_sync_or(1, NT, aborted || !ok)) { aborted = true; break; }
    if (u + nst < nunit && warp == 0 && lane == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(u + nst);
      issued = u + nst + 1;
    }
    if (adder) {
      // the chunk's super-block sums in super-block order (Q6_K: half 0 + half 1 first)
      constexpr int NJ = FMT == T_Q6_K ? 8 : 16;
      double v[NJ];
#pragma unroll
      for (int j = 0; j < NJ; j++)
        if (j < nsb)
          v[j] = FMT == T_Q6_K ? __dadd_rn(pu[j * kTile * NTP + threadIdx.x], pu[(j + 8) * kTile * NTP + threadIdx.x])
                               : pu[j * kTile * NTP + threadIdx.x];
#pragma unroll
      for (int j = 0; j < NJ; j++)
        if (j < nsb) tot = __dadd_rn(tot, v[j]);
      if (c == p.nchunk - 1) {
        const int row = threadIdx.x / NTP, tk = threadIdx.x % NTP;
        const int64_t r = (int64_t)(T0 + tile) * kTile + row;
        const float out = __double2float_rn(tot);
        // rows r (gate) and r + 1 (up) are the adders threadIdx.x and threadIdx.x + NTP, in one warp
        const float up = __shfl_xor_sync(0xffffffffu, out, NTP);
        if (tk < p.ntok && r < p.rows && (!p.swiglu || (row & 1) == 0)) store_row(p, tk, r, out, up);
        tot = 0.0;
      }
    }
  }
  if (aborted) {
    if (lane == 0) atomicOr(p.status, ST_FULL_TIMEOUT);
    if (warp == 0 && lane == 0) {
      // copies still in flight must land before the CTA's shared memory is released
      const uint64_t drain_deadline = globaltimer_ns() + WAIT_DEADLINE_NS;
      for (int v = issued - nst > 0 ? issued - nst : 0; v < issued; v++)
        if (!mbar_wait_bounded(&full[v % nst], (uint32_t)(v / nst) & 1u, drain_deadline))
          atomicOr(p.status, ST_DRAIN_TIMEOUT);
    }
  }
}

// ---------------------------------------------------------------------------- one token, register streaming
// A unit as lane (g, t) needs it: its pieces of rows g and g + 8, loaded straight from HBM; every
// load but the headers and d reads 512 (Q5_K high bits: 256; Q6_K scales: 128) contiguous bytes
// across the warp.
template <int FMT> struct PairRegs;
template <> struct PairRegs<T_Q4_K> { uint4 q[2][2]; uint4 h[2]; };             // quants [row][half], header [row]
template <> struct PairRegs<T_Q5_K> { uint4 q[2][2]; uint4 h[2]; uint2 e[2]; }; // + high bits [row]
template <> struct PairRegs<T_Q6_K> { uint4 l[2][2]; uint4 qh[2]; uint32_t sc[2]; uint32_t d[2]; };

template <int FMT>
__device__ __forceinline__ void load_unit(PairRegs<FMT> &R, const uint8_t *u, int lane, int g) {
#pragma unroll
  for (int r = 0; r < 2; r++) {
    if constexpr (FMT == T_Q6_K) {
      R.l[r][0] = ldg128(u + ((2 * r) * 32 + lane) * 16);
      R.l[r][1] = ldg128(u + ((2 * r + 1) * 32 + lane) * 16);
      R.qh[r] = ldg128(u + kQ6H + (r * 32 + lane) * 16);
      R.sc[r] = __ldg(reinterpret_cast<const uint32_t *>(u + kQ6S + (r * 32 + lane) * 4));
      R.d[r] = __ldg(reinterpret_cast<const unsigned short *>(u + kQ6D + 2 * (8 * r + g)));
    } else {
      R.q[r][0] = ldg128(u + ((2 * r) * 32 + lane) * 16);
      R.q[r][1] = ldg128(u + ((2 * r + 1) * 32 + lane) * 16);
      R.h[r] = ldg128(u + hdr_off<FMT>() + 16 * (8 * r + g));
      if constexpr (FMT == T_Q5_K) R.e[r] = __ldg(reinterpret_cast<const uint2 *>(u + kE5 + (r * 32 + lane) * 8));
    }
  }
}

// The super-block sums of rows g (p0) and g + 8 (p1) of one unit from registers, in the canonical
// order: the quad tree over lanes t of (T(2t) + T(2t+1)) (Q6_K: half 0's tree plus half 1's tree,
// each over the pairs of groups 8h + 2t, 8h + 2t + 1).
template <int FMT>
__device__ __forceinline__ void pair_sums(const PairRegs<FMT> &R, int g, int t, const SAct &x, int sb, double &p0,
                                          double &p1) {
  if constexpr (FMT == T_Q6_K) {
    double ph[2][2];
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const uint32_t lgw[4] = {R.l[0][h].x, R.l[0][h].y, R.l[0][h].z, R.l[0][h].w};
      const uint32_t lhw[4] = {R.l[1][h].x, R.l[1][h].y, R.l[1][h].z, R.l[1][h].w};
      const uint32_t qgw[2] = {h ? R.qh[0].z : R.qh[0].x, h ? R.qh[0].w : R.qh[0].y};
      const uint32_t qhw[2] = {h ? R.qh[1].z : R.qh[1].x, h ? R.qh[1].w : R.qh[1].y};
      const uint32_t xa = lds32(x.xq + sb * 256 + 16 * (8 * h + g) + 4 * t);
      int C[4] = {0, 0, 0, 0};
#pragma unroll
      for (int u = 0; u < 2; u++) {
#pragma unroll
        for (int k = 0; k < 4; k++) {
          const uint32_t a0 = q6_unpack(lgw[u * 2], lgw[u * 2 + 1], qgw[u], k);
          const uint32_t a1 = q6_unpack(lhw[u * 2], lhw[u * 2 + 1], qhw[u], k);
          mma_k16(C, a0, a1, xa * x.sel[2 * k + u]);
        }
      }
      const uint2 s2 = lds64(x.xs16 + 4 * (sb * 16 + 8 * h + 2 * t));
      const uint2 xdw = lds64(x.xd + 8 * (sb * 8 + 4 * h + t));
      const double xdv = __hiloint2double((int)xdw.y, (int)xdw.x);
#pragma unroll
      for (int r = 0; r < 2; r++) {
        const uint32_t scw = (R.sc[r] >> (16 * h)) & 0xffffu;
        const double xdd = __dmul_rn(xdv, h2d(R.d[r]));
        const double pr = __dadd_rn(q6_term(xdd, (int)(int8_t)(scw & 0xff), C[2 * r] - 32 * (int)s2.x),
                                    q6_term(xdd, (int)(int8_t)(scw >> 8), C[2 * r + 1] - 32 * (int)s2.y));
        ph[h][r] = quad_tree(pr);
      }
    }
    p0 = __dadd_rn(ph[0][0], ph[1][0]);
    p1 = __dadd_rn(ph[0][1], ph[1][1]);
  } else {
    constexpr bool FIVE = FMT == T_Q5_K;
    uint2 eg = make_uint2(0, 0), eh = make_uint2(0, 0);
    if constexpr (FIVE) { eg = R.e[0]; eh = R.e[1]; }
    const uint32_t xa = lds32(x.xq + sb * 256 + 32 * g + 4 * t), xb = lds32(x.xq + sb * 256 + 32 * g + 16 + 4 * t);
    int C0[4] = {0, 0, 0, 0}, C1[4] = {0, 0, 0, 0};
#pragma unroll
    for (int cp = 0; cp < 2; cp++) {
      const uint4 wq = R.q[0][cp], vq = R.q[1][cp];
      const uint32_t wg[4] = {wq.x, wq.y, wq.z, wq.w}, wh[4] = {vq.x, vq.y, vq.z, vq.w};
#pragma unroll
      for (int ci = 0; ci < 2; ci++) {
        const int c = 2 * cp + ci;
        uint32_t lg0 = wg[2 * ci] & 0x0f0f0f0fu, lg1 = wg[2 * ci + 1] & 0x0f0f0f0fu;
        uint32_t lh0 = wh[2 * ci] & 0x0f0f0f0fu, lh1 = wh[2 * ci + 1] & 0x0f0f0f0fu;
        uint32_t ug0, ug1, uh0, uh1;
        if constexpr (FIVE) {
          lg0 |= ((eg.x >> (2 * c)) & 0x01010101u) << 4; lg1 |= ((eg.y >> (2 * c)) & 0x01010101u) << 4;
          lh0 |= ((eh.x >> (2 * c)) & 0x01010101u) << 4; lh1 |= ((eh.y >> (2 * c)) & 0x01010101u) << 4;
          ug0 = ((wg[2 * ci] >> 4) & 0x0f0f0f0fu) | (((eg.x >> (2 * c + 1)) & 0x01010101u) << 4);
          ug1 = ((wg[2 * ci + 1] >> 4) & 0x0f0f0f0fu) | (((eg.y >> (2 * c + 1)) & 0x01010101u) << 4);
          uh0 = ((wh[2 * ci] >> 4) & 0x0f0f0f0fu) | (((eh.x >> (2 * c + 1)) & 0x01010101u) << 4);
          uh1 = ((wh[2 * ci + 1] >> 4) & 0x0f0f0f0fu) | (((eh.y >> (2 * c + 1)) & 0x01010101u) << 4);
        } else {
          ug0 = wg[2 * ci] - lg0; ug1 = wg[2 * ci + 1] - lg1;
          uh0 = wh[2 * ci] - lh0; uh1 = wh[2 * ci + 1] - lh1;
        }
        int(&C)[4] = (c & 1) ? C1 : C0;
        mma_k32(C, lg0, lh0, lg1, lh1, xa * x.sel[2 * c], xb * x.sel[2 * c]);
        mma_k32(C, ug0, uh0, ug1, uh1, xa * x.sel[2 * c + 1], xb * x.sel[2 * c + 1]);
      }
    }
    int v0 = C0[0] + C1[0], v1 = C0[1] + C1[1], v2 = C0[2] + C1[2], v3 = C0[3] + C1[3];
    if (!FIVE) { v1 >>= 4; v3 >>= 4; }
    const uint4 xdw = lds128(x.xd + 8 * (sb * 8 + 2 * t));
    const double xd0 = __hiloint2double((int)xdw.y, (int)xdw.x), xd1 = __hiloint2double((int)xdw.w, (int)xdw.z);
    const uint2 xs = lds64(x.xs + 4 * (sb * 8 + 2 * t));
#pragma unroll
    for (int r = 0; r < 2; r++) {
      const uint4 hd = R.h[r];
      const uint32_t F = k45_field(hd, t);
      const double d = h2d(hd.x & 0xffffu), dmin = h2d(hd.x >> 16);
      const double pr = __dadd_rn(k45_term(d, dmin, F & 63, (F >> 12) & 63, r ? v2 : v0, (int)xs.x, xd0),
                                  k45_term(d, dmin, (F >> 6) & 63, (F >> 18) & 63, r ? v3 : v1, (int)xs.y, xd1));
      if (r) p1 = quad_tree(pr); else p0 = quad_tree(pr);
    }
  }
}

// Stage one token's activation in shared memory (quantized here from f32, or copied when the
// caller quantized it) and return its view.
template <int FMT, int NT>
__device__ __forceinline__ SAct stage_token(const KqArgs &p, uint8_t *base, int warp, int lane, int g) {
  uint8_t *sxq = base;
  double *sxd = reinterpret_cast<double *>(sxq + p.k);
  int32_t *sxs = reinterpret_cast<int32_t *>(sxd + p.k / 32);
  int32_t *sxs16 = FMT == T_Q6_K ? sxs + p.k / 32 : nullptr;
  if (p.xq == nullptr) {
    quantize_to_smem<NT>(p.x, p.k, p.norm_w, p.norm_eps, sxq, sxd, sxs, sxs16, warp, lane);
  } else {
    const uint4 *q4 = reinterpret_cast<const uint4 *>(p.xq);
    for (int i = threadIdx.x; i < p.k / 16; i += NT) {
      const uint4 v = __ldg(q4 + i);
      reinterpret_cast<uint4 *>(sxq)[i] = v;
      if (sxs16) sxs16[i] = __dp4a((int)v.x, 0x01010101, __dp4a((int)v.y, 0x01010101,
                                   __dp4a((int)v.z, 0x01010101, __dp4a((int)v.w, 0x01010101, 0))));
    }
    for (int i = threadIdx.x; i < p.k / 32; i += NT) { sxd[i] = (double)__ldg(p.xd + i); sxs[i] = __ldg(p.xs + i); }
  }
  SAct sa{};
  sa.xq = smem_u32(sxq); sa.xd = smem_u32(sxd); sa.xs = smem_u32(sxs); sa.xs16 = sxs16 ? smem_u32(sxs16) : 0u;
#pragma unroll
  for (int i = 0; i < 8; i++) sa.sel[i] = g == i ? 1u : 0u;
  return sa;
}

// One token.  A CTA owns tiles [T0, T1); their units, (tile, super-block) in order, are one
// contiguous range, cut into 16 equal runs, one per warp.  A warp keeps D units of loads in flight
// in registers -- the first ones issued before griddepcontrol.wait -- and writes each unit's two
// super-block sums to shared memory.  After one CTA barrier a thread per row adds its super-block
// sums in super-block order and applies the epilogue.  No waits on other warps or copies: nothing
// to bound.
constexpr int kStreamWarps = 16;
constexpr int kStreamDepth = 2;

template <int FMT>
__global__ void __launch_bounds__(kStreamWarps * 32, 1) kq_stream_kernel(const KqArgs p) {
  constexpr int NT = kStreamWarps * 32, D = kStreamDepth, US = unit_bytes<FMT>();
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  int T0, T1;
  cta_tiles(p.rows, T0, T1);
  const int nb = p.nb;
  const int npair = (T1 - T0) * nb;
  const int i0 = (int)((int64_t)warp * npair / kStreamWarps), i1 = (int)((int64_t)(warp + 1) * npair / kStreamWarps);
  const int64_t row0 = (int64_t)T0 * kTile;
  const int nrows = (int)(min((int64_t)T1 * kTile, p.rows) - row0);
  double *sums = reinterpret_cast<double *>(smem + p.part_off);    // [pair][16 rows]
  const uint8_t *base = p.w + (int64_t)T0 * nb * US;

  PairRegs<FMT> R[D];
#pragma unroll
  for (int d = 0; d < D; d++)
    if (i0 + d < i1) load_unit<FMT>(R[d], base + (int64_t)(i0 + d) * US, lane, g);   // not the previous kernel's output
  pdl_launch_dependents();
  pdl_wait();                                   // the activation is
  const SAct sa = stage_token<FMT, NT>(p, smem + p.x_off, warp, lane, g);
  __syncthreads();

  int sb = nb > 0 ? i0 % nb : 0;                // super-block of unit i
  for (int i = i0; i < i1; i += D) {
#pragma unroll
    for (int d = 0; d < D; d++) {
      const int ii = i + d;
      if (ii < i1) {
        double S0, S1;
        pair_sums<FMT>(R[d], g, t, sa, sb, S0, S1);
        if (ii + D < i1) load_unit<FMT>(R[d], base + (int64_t)(ii + D) * US, lane, g);
        if (t == 0) { sums[ii * kTile + g] = S0; sums[ii * kTile + g + 8] = S1; }
        if (++sb == nb) sb = 0;
      }
    }
  }
  __syncthreads();

  // one thread per row (per (gate, up) pair with swiglu): the super-block sums in order
  const int step = p.swiglu ? 2 : 1;
  for (int row = step * threadIdx.x; row < nrows; row += step * NT) {
    float o[2] = {0.f, 0.f};
    for (int e = 0; e < step; e++) {
      const int rr = row + e;
      const double *sr = sums + (int64_t)(rr / kTile) * nb * kTile + rr % kTile;
      double tot = 0.0;
      for (int s = 0; s < nb; s++) tot = __dadd_rn(tot, sr[s * kTile]);
      o[e] = __double2float_rn(tot);
    }
    store_row(p, 0, row0 + row, o[0], o[1]);
  }
}

// ---------------------------------------------------------------------------- host side
int kq_x_bytes(const DevMatrix &m) {
  return (int)((m.cols + 12 * (m.cols / 32) + (m.type == T_Q6_K ? 4 * (m.cols / 16) : 0) + 127) / 128 * 128);
}

// one shared-memory grant per kernel (the template parameter) and device
template <void (*kern)(KqArgs)>
cudaError_t launch_ex(int64_t max_smem, const KqArgs &a, int grid, int block, int smem, cudaStream_t s, bool pdl) {
  static bool granted[64] = {false};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!granted[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)max_smem);
    if (e != cudaSuccess) return e;
    granted[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

// The one-token launches over a matrix: each takes whole tiles, at most as many per CTA as leave
// the CTA's super-block sums room in shared memory next to the staged activation.
constexpr int64_t kStreamBudget = 200 * 1024;

cudaError_t launch_stream(const DevMatrix &m, const ActView &act, float *y, const float *y_add, const GemvFuse &fz,
                          unsigned *status, int num_sms, cudaStream_t s, bool pdl, const char **why) {
  const int64_t nb = m.cols / 256;
  const int64_t x_bytes = kq_x_bytes(m);
  const int64_t cap = (kStreamBudget - x_bytes) / (nb * kTile * 8);       // tiles per CTA
  if (cap < 1) { *why = "k-quant rows too long for the one-token GEMV"; return cudaErrorInvalidValue; }
  const int64_t tiles_all = (m.rows + kTile - 1) / kTile, per_launch = cap * num_sms;
  const int us = kq_unit_bytes(m.type);
  for (int64_t tb = 0; tb < tiles_all; tb += per_launch) {
    const int64_t nt = tiles_all - tb < per_launch ? tiles_all - tb : per_launch;
    const int64_t rb = tb * kTile;
    const int grid = (int)(nt < num_sms ? nt : num_sms);
    const int64_t tiles_cta = (nt + grid - 1) / grid;
    KqArgs a{};
    a.w = m.data + tb * nb * us;
    a.rows = m.rows - rb < nt * kTile ? m.rows - rb : nt * kTile;
    a.nb = (int)nb; a.ntok = 1; a.k = m.cols;
    a.xq = act.xq; a.xd = act.xd; a.xs = act.xs; a.x = act.x;
    a.y = y + (fz.swiglu ? rb / 2 : rb);
    a.y_add = y_add ? y_add + rb : nullptr;
    a.norm_w = fz.norm_w; a.norm_eps = fz.eps; a.swiglu = fz.swiglu ? 1 : 0;
    a.status = status;
    a.x_off = 0; a.part_off = (int)x_bytes;
    const int smem = (int)(x_bytes + tiles_cta * nb * kTile * 8);
    const int block = kStreamWarps * 32;
    cudaError_t e;
    switch (m.type) {
      case T_Q4_K: e = launch_ex<kq_stream_kernel<T_Q4_K>>(kStreamBudget, a, grid, block, smem, s, pdl); break;
      case T_Q5_K: e = launch_ex<kq_stream_kernel<T_Q5_K>>(kStreamBudget, a, grid, block, smem, s, pdl); break;
      default: e = launch_ex<kq_stream_kernel<T_Q6_K>>(kStreamBudget, a, grid, block, smem, s, pdl); break;
    }
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// 2..8 tokens per launch, tokens in groups of 8.
cudaError_t launch_tok(const DevMatrix &m, const ActView &act, int ntok, float *y, int64_t y_stride, const float *y_add,
                       const GemvFuse &fz, unsigned *status, int num_sms, cudaStream_t s, bool pdl, const char **why) {
  if (!act.xq) { *why = "the in-kernel activation quantization takes one token"; return cudaErrorInvalidValue; }
  const int64_t nb = m.cols / 256;
  const int kChunk = chunk_sb_of(m.type), us = kq_unit_bytes(m.type);
  const int nchunk = (int)((nb + kChunk - 1) / kChunk);
  const int64_t tiles_all = (m.rows + kTile - 1) / kTile;
  const int grid = (int)(tiles_all < num_sms ? tiles_all : num_sms);
  const int64_t units = (tiles_all + grid - 1) / grid * nchunk;           // per CTA, at most
  const int64_t stage = (int64_t)kChunk * us;
  const int64_t part_bytes = 2LL * 16 * kTile * kMaxTok * 8;
  int64_t nst = (kTokBudget - part_bytes - 8 * kMaxStages) / stage;
  if (nst > kMaxStages) nst = kMaxStages;
  if (nst > units) nst = units;
  if (nst < 1) { *why = "k-quant rows too long for the shared-memory stages"; return cudaErrorInvalidValue; }
  const int part_off = (int)(nst * stage), bar_off = (int)(part_off + part_bytes);
  const int smem = bar_off + 8 * (int)nst;
  for (int t0 = 0; t0 < ntok; t0 += kMaxTok) {
    const int nt = ntok - t0 < kMaxTok ? ntok - t0 : kMaxTok;
    KqArgs a{};
    a.w = m.data; a.rows = m.rows; a.nb = (int)nb; a.nchunk = nchunk; a.nst = (int)nst;
    a.ntok = nt; a.k = m.cols;
    a.xq = act.xq + (int64_t)t0 * m.cols;
    a.xd = act.xd + (int64_t)t0 * (m.cols / 32);
    a.xs = act.xs + (int64_t)t0 * (m.cols / 32);
    a.y = y + (int64_t)t0 * y_stride;
    a.y_add = y_add ? y_add + (int64_t)t0 * y_stride : nullptr;
    a.y_stride = y_stride;
    a.swiglu = fz.swiglu ? 1 : 0;
    a.status = status;
    a.part_off = part_off; a.bar_off = bar_off;
    const int block = kTokWarps * 32;
    cudaError_t e;
    switch (m.type) {
      case T_Q4_K: e = launch_ex<kq_tok_kernel<T_Q4_K>>(kTokBudget + 1024, a, grid, block, smem, s, pdl); break;
      case T_Q5_K: e = launch_ex<kq_tok_kernel<T_Q5_K>>(kTokBudget + 1024, a, grid, block, smem, s, pdl); break;
      default: e = launch_ex<kq_tok_kernel<T_Q6_K>>(kTokBudget + 1024, a, grid, block, smem, s, pdl); break;
    }
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace

bool kq_type(int t) { return t == T_Q4_K || t == T_Q5_K || t == T_Q6_K; }

cudaError_t launch_gemv_kq(const DevMatrix &m, const ActView &act, int ntok, float *y, int64_t y_stride,
                           const float *y_add, unsigned *status, int num_sms, cudaStream_t s, bool pdl, const char **why) {
  return launch_gemv_kq_ex(m, act, ntok, y, y_stride, y_add, GemvFuse{}, status, num_sms, s, pdl, why);
}

cudaError_t launch_gemv_kq_ex(const DevMatrix &m, const ActView &act, int ntok, float *y, int64_t y_stride,
                              const float *y_add, const GemvFuse &fz, unsigned *status, int num_sms, cudaStream_t s,
                              bool pdl, const char **why) {
  if (m.cols % 256 || m.cols < 256) { *why = "k-quant rows must be a whole number of 256-value super-blocks"; return cudaErrorInvalidValue; }
  if (fz.norm_w && (act.xq || !act.x || ntok != 1)) { *why = "the fused RMSNorm takes one f32 token"; return cudaErrorInvalidValue; }
  if (fz.swiglu && (m.rows % 2 || y_add)) { *why = "the SwiGLU epilogue takes (gate, up) row pairs and no residual"; return cudaErrorInvalidValue; }
  if (act.xq == nullptr && (ntok != 1 || act.x == nullptr)) {
    *why = "the in-kernel activation quantization takes one token";
    return cudaErrorInvalidValue;
  }
  if (ntok == 1) return launch_stream(m, act, y, y_add, fz, status, num_sms, s, pdl, why);
  return launch_tok(m, act, ntok, y, y_stride, y_add, fz, status, num_sms, s, pdl, why);
}

}  // namespace zllm
