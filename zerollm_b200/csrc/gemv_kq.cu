// Decode GEMV for the k-quant formats (Q4_K, Q5_K, Q6_K) with the integer dot products on the
// tensor cores.
//
// Replaces the reference's k-quant matvec kernels: src/compute/ref-kernels.js:196-277 (oracle)
// and the WASM matvec_q4_k / matvec_q5_k / matvec_q6_k and mm_* exports
// (src/compute/wasm/kquant-kernels.js:337-504), dispatched by ggml type as in
// src/compute/worker.js:184-197 / :251-270.
//
// What a launch computes, for each token t and row r:  y[t][r] = (y_add) + sum over blocks of
//   Q4_K / Q5_K:  xd * (d*sc*lo - dmin*mn*xs)       per 32-value sub-block (ref-kernels.js:235-236)
//   Q6_K:         xd * d * scale * gsum             per 16-value group     (ref-kernels.js:271)
// where lo / gsum are exact integer dot products of the weight quants with the int8 activation.
//
// The weights are stored as units of (16-row tile, super-block) (kq_layout.h); a CTA owns a
// contiguous range of tiles.  The integer dots are warp-level MMAs (mma.sync m16n8k32 / m16n8k16,
// uint8 or int8 x int8 -> int32, exact) on a unit, whose A operand is the unit itself:
//   * one token (kq_ring_kernel): the B operand is block-diagonal -- column j carries the
//     activation of sub-block (group) j and is zero elsewhere -- so the 8 MMAs of a unit leave the
//     16 rows x 8 sub-blocks of integer dots in one accumulator.  Every warp stages its share of
//     the CTA's units through a shared-memory ring with 16-byte cp.async (coalesced 512-byte warp
//     copies, several units in flight);
//   * 2..16 tokens per launch (kq_batch_kernel): B column j carries token j, one MMA per sub-block
//     (group) and group of 8 tokens.  The CTA's units are walked super-block by super-block, so a
//     warp loads a super-block's activation fragments once and reuses them for every tile; the
//     block terms of a token pair are computed with packed f32x2 arithmetic, element for element
//     the same rounding as the one-token kernel's scalar formula.
// Block terms are f32 with a fixed formula shared by both kernels (k45_pair / q6_pair below); an
// integer dot leaves the MMA already biased by 1.5 * 2^23 (the accumulator starts there), so one
// subtraction turns it into the exact float.  The order of the additions is fixed as well: each
// super-block's terms are added as a pairwise tree (Q4_K / Q5_K: ((P0 + P1) + (P2 + P3)) over the
// sub-block pairs; Q6_K: the same over the group pairs of each 128-value half, then half 0 + half
// 1), and the super-block sums are added in super-block order.  That order depends on nothing but
// the row, so a token gets the same bits alone, in a batch, or in any launch shape.  Against the
// oracle's double arithmetic the outputs differ by f32 rounding only (max|d| / max|y| ~ 1e-6).
// A one-token launch may take the f32 activation (optionally RMSNorm-ed first) and quantize it
// itself, bit-exact with quantize_act_kernel, so a lone matvec is one kernel.
#include "common.cuh"
#include "internal.h"
#include "kq_layout.h"

namespace zllm {

namespace {

constexpr int kTile = kKqTile;               // rows per unit (the MMA's M)
constexpr int kBatchTok = 16;                // tokens per launch of the batch kernel (two MMA N groups)

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

// ---------------------------------------------------------------------------- exact int -> f32
// An int32 accumulator that started at kBias holds kBias + v; for |v| < 2^22 its bits are the float
// 1.5 * 2^23 + v exactly (a float with unit spacing), so one subtraction yields v.  Every integer dot
// here is below 2^22 in magnitude (Q5_K: 32 * 31 * 127 = 125,984).
constexpr int kBias = 0x4B400000;
constexpr float kBiasF = 12582912.0f;
__device__ __forceinline__ float biased_f(int acc) { return __fsub_rn(__int_as_float(acc), kBiasF); }
// small ints (|v| < 2^22) to float on the integer + FMA pipes instead of the conversion pipe
__device__ __forceinline__ float small_f(int v) { return biased_f(v + kBias); }

__device__ __forceinline__ float fshfl_xor(float v, int m) { return __shfl_xor_sync(0xffffffffu, v, m); }
// Sum over the 4 lanes t of a lane quad: ((v0 + v1) + (v2 + v3)) in every lane of the quad.
__device__ __forceinline__ float quad_tree(float v) {
  v = __fadd_rn(v, fshfl_xor(v, 1));
  return __fadd_rn(v, fshfl_xor(v, 2));
}

// ---------------------------------------------------------------------------- block terms
// Scales of one Q4_K / Q5_K row for a sub-block pair (2c, 2c + 1): d*sc and dmin*mn, exact in f32
// (an f16 times a 6-bit integer).
struct K45Sc { float ds0, ds1, dm0, dm1; };
__device__ __forceinline__ K45Sc k45_sc(float d, float dmin, uint32_t F) {
  K45Sc s;
  s.ds0 = __fmul_rn(d, small_f((int)(F & 63)));
  s.ds1 = __fmul_rn(d, small_f((int)((F >> 6) & 63)));
  s.dm0 = __fmul_rn(dmin, small_f((int)((F >> 12) & 63)));
  s.dm1 = __fmul_rn(dmin, small_f((int)((F >> 18) & 63)));
  return s;
}
// The pair term T(2c) + T(2c + 1) of one (row, token): with xdm = (xd0, xd1, xd0*xs0, xd1*xs1) of the
// token's two 32-blocks, xd * (d*sc*lo - dmin*mn*xs) summed over the pair as
//   fma(xd1*ds1, lo1, fma(xd0*ds0, lo0, -(fma(dm1, xm1, dm0*xm0)))).
__device__ __forceinline__ float k45_pair(const K45Sc &s, float lo0, float lo1, const float4 &xdm) {
  const float m = __fmaf_rn(s.dm1, xdm.w, __fmul_rn(s.dm0, xdm.z));
  return __fmaf_rn(__fmul_rn(xdm.y, s.ds1), lo1, __fmaf_rn(__fmul_rn(xdm.x, s.ds0), lo0, -m));
}
// The Q6_K pair term of groups (G, G + 1), which share the 32-block b: (xd_b * d) * (sc_G * g_G +
// sc_G+1 * g_G+1); the integer combination is exact in f32 (|.| < 2^24).
__device__ __forceinline__ float q6_pair(float xd, float d, float sc0, float g0, float sc1, float g1) {
  return __fmul_rn(__fmul_rn(xd, d), __fmaf_rn(sc1, g1, __fmul_rn(sc0, g0)));
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
// int8 scale byte i of a word as float
__device__ __forceinline__ float sbyte_f(uint32_t w, int i) { return small_f((int)(int8_t)((w >> (8 * i)) & 0xffu)); }

// ---------------------------------------------------------------------------- launch arguments
struct KqArgs {
  const uint8_t *w;     // first unit of the launch's first tile
  int64_t rows;         // rows of the launch (the last tile may be partial)
  int nb;               // super-blocks per row
  int ntok;             // tokens in this launch
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
  int x_off, part_off, ring_off;  // shared-memory regions
};

// tiles [T0, T1) of a CTA: an even split of the launch's tiles
__device__ __forceinline__ void cta_tiles(int64_t rows, int &T0, int &T1) {
  const int64_t nt = (rows + kTile - 1) / kTile;
  T0 = (int)((int64_t)blockIdx.x * nt / gridDim.x);
  T1 = (int)((int64_t)(blockIdx.x + 1) * nt / gridDim.x);
}

// y for output row r (launch-relative) from its f32 total; with swiglu the (gate, up) pair
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

// ---------------------------------------------------------------------------- one-token activation
// One token's activation staged in shared memory:
//   xq   [K] int8;
//   Q4_K / Q5_K: xdm [K/64] float4 = (xd of 32-blocks 2p, 2p + 1, then xd * xs of the same);
//   Q6_K:        xd6 [K/256][4] float2 = (xd of 32-blocks t, 4 + t of the super-block) and
//                moff [K/256][4] float4 = kBiasF + 32 * (sum of the int8 of groups 2t, 2t + 1,
//                8 + 2t, 9 + 2t): the unsigned-quant dot minus moff is the signed group dot.
// sel[s] = 1 when the lane's MMA column is s, else 0: the block-diagonal B operand is x * sel[s].
struct SAct {
  uint32_t xq, sc0, sc1;    // shared-window addresses: xq, xdm / xd6, moff
  uint32_t sel[8];
};

template <int FMT>
__device__ __forceinline__ void put_block_scales(float *ssc0, int b, float xd, int xs) {
  if constexpr (FMT == T_Q6_K) {
    ssc0[((b >> 3) * 4 + (b & 3)) * 2 + ((b >> 2) & 1)] = xd;
  } else {
    ssc0[(b >> 1) * 4 + (b & 1)] = xd;
    ssc0[(b >> 1) * 4 + 2 + (b & 1)] = __fmul_rn(xd, __int2float_rn(xs));
  }
}
// moff of 16-value group G (global index) from the sum of its int8
__device__ __forceinline__ void put_group_off(float *ssc1, int G, int s16) {
  const int gg = G & 15;
  ssc1[((G >> 4) * 4 + ((gg >> 1) & 3)) * 4 + 2 * (gg >> 3) + (gg & 1)] = __fadd_rn(kBiasF, __int2float_rn(32 * s16));
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

// ---------------------------------------------------------------------------- exact quantizeAct, f32 fast path
// quantizeAct (src/compute/ref-kernels.js:44-62) computes, per 32-value block with maximum |x| amax,
//   scale = amax / 127, d = f32(scale), inv = 1 / scale, q = round-half-away(x * inv)   (doubles).
// The same integers come out of f32 arithmetic almost always:
//   * d: for every float amax, f32(amax / 127 in double) equals the f32 quotient amax / 127.f --
//     127's binary expansion repeats with period 7, so the double quotient can never sit on an
//     f32 rounding midpoint (checked exhaustively over all positive floats);
//   * q: r = x * f32(127 / amax) is within |r| * 2^-23 <= 1.6e-5 of the double product, so it rounds
//     the same way unless its fraction is within 2^-12 of one half; those values (about 5 in 10^4
//     of random inputs) and every value of a block whose amax is below 2^-96 (where 127 / amax
//     leaves f32's range) take the double formula itself.
// amax == 0 and amax == inf both give inv == 0 in the reference (1 / inf), hence invf = 0.
struct QuantBlock { float d, invf; bool dbl; };
__device__ __forceinline__ QuantBlock quant_block(float amax) {
  QuantBlock b;
  b.d = __fdiv_rn(amax, 127.f);
  b.dbl = amax > 0.f && amax < 0x1p-96f;
  b.invf = (amax == 0.f || isinf(amax) || b.dbl) ? 0.f : __fdiv_rn(127.f, amax);
  return b;
}
// q of one value from the f32 estimate; `slow` is set (and q is meaningless) when the value must take
// the double formula (quant_value_dbl): a fraction within 2^-12 of one half, a NaN, or a block whose
// amax is below 2^-96.  The rounding adds 1.5 * 2^23, which leaves r rounded to the nearest integer
// (ties to even) in the low mantissa bits; away from the ties that is round-half-away, and the ties
// are among the slow values.
__device__ __forceinline__ int quant_value_fast(float x, const QuantBlock &b, bool &slow) {
  const float r = __fmul_rn(x, b.invf);
  const float t = __fadd_rn(r, kBiasF);
  const float e = __fsub_rn(r, __fsub_rn(t, kBiasF));   // r minus its rounded value, exactly
  slow = b.dbl || !(fabsf(e) < 0.5f - 0x1p-12f);          // NaN lands here too
  return __float_as_int(t) - kBias;
}
// the reference's double formula itself (bad: the value is NaN or NaN after scaling -- q is 0 and the
// block sum becomes 0)
__device__ __noinline__ int quant_value_dbl(float x, float amax, bool &bad) {
  const double scale = __ddiv_rn((double)amax, 127.0);
  const double inv = scale != 0.0 ? __ddiv_rn(1.0, scale) : 0.0;
  const double rd = round(__dmul_rn((double)x, inv));       // half away from zero
  bad = !(rd == rd);
  return bad ? 0 : (int)rd;
}

// Quantize one token's f32 activation into shared memory; bit-exact with quantize_act_kernel
// (quantizeAct, src/compute/ref-kernels.js:44-62).  32 / V lanes own a 32-value block, V values each
// (V = 8 when the token fits one round of the CTA's threads -- K <= 4096 -- else 16: fewer rounds of
// the double-precision scale chain).  With norm_w the values are first f32(x * s * w) with s the
// RMSNorm scale (ref-kernels.js:305-310), as rmsnorm_quant_kernel writes them.
template <int FMT, int NT, int V>
__device__ void quantize_rounds(const float *x, int64_t k, const float *norm_w, double rs, uint8_t *sxq, float *ssc0,
                                float *ssc1, int warp, int lane) {
  constexpr int LPB = 32 / V;                   // lanes per 32-value block
  const int nqb = (int)(k / V);
  for (int base = warp * 32; base < nqb; base += NT) {
    const int qb = base + lane;
    const bool act = qb < nqb;
    float v[V];
    if (act) {
      const float4 *p = reinterpret_cast<const float4 *>(x + (int64_t)qb * V);
#pragma unroll
      for (int i = 0; i < V / 4; i++) {
        const float4 f = __ldg(p + i);
        v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
      }
      if (norm_w) {
        const float4 *wp = reinterpret_cast<const float4 *>(norm_w + (int64_t)qb * V);
#pragma unroll
        for (int i = 0; i < V / 4; i++) {
          const float4 f = __ldg(wp + i);
          const float wv[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
          for (int j = 0; j < 4; j++) v[4 * i + j] = __double2float_rn(__dmul_rn(__dmul_rn((double)v[4 * i + j], rs), (double)wv[j]));
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < V; i++) v[i] = 0.f;
    }
    float a = 0.f;
#pragma unroll
    for (int i = 0; i < V; i++) a = fmaxf(a, fabsf(v[i]));   // NaN never raises amax (as `Math.abs(NaN) > amax`)
#pragma unroll
    for (int o = 1; o < LPB; o <<= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    const QuantBlock qb_ = quant_block(a);
    int qv[V];
    uint32_t slow = 0u;
#pragma unroll
    for (int i = 0; i < V; i++) {
      bool sl;
      qv[i] = quant_value_fast(v[i], qb_, sl);
      slow |= (uint32_t)sl << i;
    }
    bool nan = false;
    while (slow) {                              // rare: the values the f32 estimate cannot settle
      const int i = __ffs(slow) - 1;
      slow &= slow - 1u;
      bool bad;
      float xi = v[0];
#pragma unroll
      for (int j = 1; j < V; j++) xi = j == i ? v[j] : xi;
      const int q = quant_value_dbl(xi, a, bad);
      nan |= bad;
#pragma unroll
      for (int j = 0; j < V; j++) qv[j] = j == i ? q : qv[j];
    }
    uint32_t words[V / 4];
    int sum = 0;
#pragma unroll
    for (int i = 0; i < V / 4; i++) {           // the low bytes of four q, then their sum
      words[i] = __byte_perm(__byte_perm(qv[4 * i], qv[4 * i + 1], 0x0040), __byte_perm(qv[4 * i + 2], qv[4 * i + 3], 0x0040),
                             0x5410);
      sum = __dp4a((int)words[i], 0x01010101, sum);
    }
    const int s16 = V == 16 ? sum : sum + __shfl_xor_sync(0xffffffffu, sum, 1);   // the 16-value group
    int s32 = s16;
#pragma unroll
    for (int o = 16 / V; o < LPB; o <<= 1) s32 += __shfl_xor_sync(0xffffffffu, s32, o);
    const bool nan32 = ((__ballot_sync(0xffffffffu, nan) >> (lane & ~(LPB - 1))) & ((1u << LPB) - 1u)) != 0;
    if (act) {
      if constexpr (V == 16) reinterpret_cast<uint4 *>(sxq)[qb] = make_uint4(words[0], words[1], words[2], words[3]);
      else reinterpret_cast<uint2 *>(sxq)[qb] = make_uint2(words[0], words[1]);
      if constexpr (FMT == T_Q6_K) {
        if (V == 16 || (lane & 1) == 0) put_group_off(ssc1, qb * V / 16, s16);
      }
      if ((lane & (LPB - 1)) == 0) put_block_scales<FMT>(ssc0, qb / LPB, qb_.d, nan32 ? 0 : s32);
    }
  }
}

template <int FMT, int NT>
__device__ void quantize_to_smem(const float *x, int64_t k, const float *norm_w, double eps, uint8_t *sxq, float *ssc0,
                                 float *ssc1, int warp, int lane) {
  const double rs = norm_w ? rms_scale<NT>(x, k, eps, warp, lane) : 0.0;
  if (k / 8 <= NT) quantize_rounds<FMT, NT, 8>(x, k, norm_w, rs, sxq, ssc0, ssc1, warp, lane);
  else quantize_rounds<FMT, NT, 16>(x, k, norm_w, rs, sxq, ssc0, ssc1, warp, lane);
}

// Stage one token's activation in shared memory (quantized here from f32, or copied when the
// caller quantized it) and return its view.
template <int FMT, int NT>
__device__ __forceinline__ SAct stage_token(const KqArgs &p, uint8_t *base, int warp, int lane, int g) {
  uint8_t *sxq = base;
  float *ssc0 = reinterpret_cast<float *>(sxq + p.k);
  float *ssc1 = FMT == T_Q6_K ? ssc0 + p.k / 32 : nullptr;
  if (p.xq == nullptr) {
    quantize_to_smem<FMT, NT>(p.x, p.k, p.norm_w, p.norm_eps, sxq, ssc0, ssc1, warp, lane);
  } else {
    const uint4 *q4 = reinterpret_cast<const uint4 *>(p.xq);
    for (int i = threadIdx.x; i < p.k / 16; i += NT) {
      const uint4 v = __ldg(q4 + i);
      reinterpret_cast<uint4 *>(sxq)[i] = v;
      if constexpr (FMT == T_Q6_K)
        put_group_off(ssc1, i, __dp4a((int)v.x, 0x01010101, __dp4a((int)v.y, 0x01010101,
                                      __dp4a((int)v.z, 0x01010101, __dp4a((int)v.w, 0x01010101, 0)))));
    }
    for (int i = threadIdx.x; i < p.k / 32; i += NT) put_block_scales<FMT>(ssc0, i, __ldg(p.xd + i), __ldg(p.xs + i));
  }
  SAct sa{};
  sa.xq = smem_u32(sxq); sa.sc0 = smem_u32(ssc0); sa.sc1 = ssc1 ? smem_u32(ssc1) : 0u;
#pragma unroll
  for (int i = 0; i < 8; i++) sa.sel[i] = g == i ? 1u : 0u;
  return sa;
}

// ---------------------------------------------------------------------------- unit registers
// A unit as lane (g, t) needs it: its pieces of rows g and g + 8, loaded straight from HBM; every
// load but the headers and d reads 512 (Q5_K high bits: 256; Q6_K scales: 128) contiguous bytes
// across the warp.  The batch kernel takes the two rows' whole Q6_K scale records (sc16) instead
// of the lane's four scales (sc).
template <int FMT> struct PairRegs;
template <> struct PairRegs<T_Q4_K> { uint4 q[2][2]; uint4 h[2]; };             // quants [row][half], header [row]
template <> struct PairRegs<T_Q5_K> { uint4 q[2][2]; uint4 h[2]; uint2 e[2]; }; // + high bits [row]
template <> struct PairRegs<T_Q6_K> { uint4 l[2][2]; uint4 qh[2]; uint32_t sc[2]; uint4 sc16[2]; uint32_t d[2]; };

// The A operands of chunk c (sub-blocks 2c and 2c + 1) of a Q4_K / Q5_K unit: lo = {row g k 0-3,
// row g+8 k 0-3, row g k 16-19, row g+8 k 16-19} of sub-block 2c, hi the same of sub-block 2c + 1.
template <bool FIVE>
__device__ __forceinline__ void k45_operands(const uint4 (&q)[2][2], uint2 eg, uint2 eh, int c, uint32_t (&lo)[4],
                                             uint32_t (&hi)[4]) {
  const int cp = c >> 1, ci = c & 1;
  const uint4 wq = q[0][cp], vq = q[1][cp];
  const uint32_t wx = ci ? wq.z : wq.x, wy = ci ? wq.w : wq.y, vx = ci ? vq.z : vq.x, vy = ci ? vq.w : vq.y;
  lo[0] = wx & 0x0f0f0f0fu; lo[2] = wy & 0x0f0f0f0fu; lo[1] = vx & 0x0f0f0f0fu; lo[3] = vy & 0x0f0f0f0fu;
  hi[0] = (wx >> 4) & 0x0f0f0f0fu; hi[2] = (wy >> 4) & 0x0f0f0f0fu;
  hi[1] = (vx >> 4) & 0x0f0f0f0fu; hi[3] = (vy >> 4) & 0x0f0f0f0fu;
  if constexpr (FIVE) {
    lo[0] |= ((eg.x >> (2 * c)) & 0x01010101u) << 4; lo[2] |= ((eg.y >> (2 * c)) & 0x01010101u) << 4;
    lo[1] |= ((eh.x >> (2 * c)) & 0x01010101u) << 4; lo[3] |= ((eh.y >> (2 * c)) & 0x01010101u) << 4;
    hi[0] |= ((eg.x >> (2 * c + 1)) & 0x01010101u) << 4; hi[2] |= ((eg.y >> (2 * c + 1)) & 0x01010101u) << 4;
    hi[1] |= ((eh.x >> (2 * c + 1)) & 0x01010101u) << 4; hi[3] |= ((eh.y >> (2 * c + 1)) & 0x01010101u) << 4;
  }
}

// ---------------------------------------------------------------------------- one token, register streaming
// The super-block sums of rows g (p0) and g + 8 (p1) of one unit from registers, in the canonical
// order: the quad tree over lanes t of the pair term of sub-blocks (2t, 2t + 1) (Q6_K: half 0's
// tree plus half 1's tree, each over the pairs of groups 8h + 2t, 8h + 2t + 1).
template <int FMT>
__device__ __forceinline__ void pair_sums(const PairRegs<FMT> &R, int g, int t, const SAct &x, int sb, float &p0,
                                          float &p1) {
  if constexpr (FMT == T_Q6_K) {
    float ph[2][2];
    const float2 xd = lds_f2(x.sc0 + 8 * (sb * 4 + t));               // 32-blocks t, 4 + t
    const uint4 mo = lds128(x.sc1 + 16 * (sb * 4 + t));               // groups 2t, 2t+1, 8+2t, 9+2t
    const float moff[4] = {__uint_as_float(mo.x), __uint_as_float(mo.y), __uint_as_float(mo.z), __uint_as_float(mo.w)};
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const uint32_t lgw[4] = {R.l[0][h].x, R.l[0][h].y, R.l[0][h].z, R.l[0][h].w};
      const uint32_t lhw[4] = {R.l[1][h].x, R.l[1][h].y, R.l[1][h].z, R.l[1][h].w};
      const uint32_t qgw[2] = {h ? R.qh[0].z : R.qh[0].x, h ? R.qh[0].w : R.qh[0].y};
      const uint32_t qhw[2] = {h ? R.qh[1].z : R.qh[1].x, h ? R.qh[1].w : R.qh[1].y};
      const uint32_t xa = lds32(x.xq + sb * 256 + 16 * (8 * h + g) + 4 * t);
      int C[4] = {kBias, kBias, kBias, kBias};
#pragma unroll
      for (int u = 0; u < 2; u++) {
#pragma unroll
        for (int k = 0; k < 4; k++) {
          const uint32_t a0 = q6_unpack(lgw[u * 2], lgw[u * 2 + 1], qgw[u], k);
          const uint32_t a1 = q6_unpack(lhw[u * 2], lhw[u * 2 + 1], qhw[u], k);
          mma_k16(C, a0, a1, xa * x.sel[2 * k + u]);
        }
      }
      const float xdv = h ? xd.y : xd.x;
#pragma unroll
      for (int r = 0; r < 2; r++) {
        const uint32_t scw = R.sc[r] >> (16 * h);
        const float g0 = __fsub_rn(__int_as_float(C[2 * r]), moff[2 * h]);
        const float g1 = __fsub_rn(__int_as_float(C[2 * r + 1]), moff[2 * h + 1]);
        ph[h][r] = quad_tree(q6_pair(xdv, h2f(R.d[r]), sbyte_f(scw, 0), g0, sbyte_f(scw, 1), g1));
      }
    }
    p0 = __fadd_rn(ph[0][0], ph[1][0]);
    p1 = __fadd_rn(ph[0][1], ph[1][1]);
  } else {
    constexpr bool FIVE = FMT == T_Q5_K;
    uint2 eg = make_uint2(0, 0), eh = make_uint2(0, 0);
    if constexpr (FIVE) { eg = R.e[0]; eh = R.e[1]; }
    const uint32_t xa = lds32(x.xq + sb * 256 + 32 * g + 4 * t), xb = lds32(x.xq + sb * 256 + 32 * g + 16 + 4 * t);
    int C0[4] = {kBias, kBias, kBias, kBias}, C1[4] = {0, 0, 0, 0};
#pragma unroll
    for (int c = 0; c < 4; c++) {
      uint32_t lo[4], hi[4];
      k45_operands<FIVE>(R.q, eg, eh, c, lo, hi);
      int(&C)[4] = (c & 1) ? C1 : C0;
      mma_k32(C, lo[0], lo[1], lo[2], lo[3], xa * x.sel[2 * c], xb * x.sel[2 * c]);
      mma_k32(C, hi[0], hi[1], hi[2], hi[3], xa * x.sel[2 * c + 1], xb * x.sel[2 * c + 1]);
    }
    const uint4 xw = lds128(x.sc0 + 16 * (sb * 4 + t));
    const float4 xdm = make_float4(__uint_as_float(xw.x), __uint_as_float(xw.y), __uint_as_float(xw.z), __uint_as_float(xw.w));
#pragma unroll
    for (int r = 0; r < 2; r++) {
      const uint4 hd = R.h[r];
      const K45Sc s = k45_sc(h2f(hd.x & 0xffffu), h2f(hd.x >> 16), k45_field(hd, t));
      const float pr = k45_pair(s, biased_f(C0[2 * r] + C1[2 * r]), biased_f(C0[2 * r + 1] + C1[2 * r + 1]), xdm);
      if (r) p1 = quad_tree(pr); else p0 = quad_tree(pr);
    }
  }
}

// ---------------------------------------------------------------------------- one token, shared-memory ring
// Every warp stages its share of the CTA's units through its own ring of S unit slots in shared
// memory with 16-byte cp.async (lane l copies the unit's 16-byte pieces l, l + 32, ..., the pieces it
// reads back itself, except for the row headers): S units per warp -- for a 4096-row matrix the
// SM's whole share -- are in flight before griddepcontrol.wait, and the registers only ever hold the
// unit being computed.  Sixteen warps (one CTA per SM) keep enough independent work in flight to
// cover the MMA, shared-memory and shuffle latencies of the unit arithmetic; measured on a B200
// against eight warps with two CTAs per SM (the next launch's CTA resident and loading under
// programmatic dependent launch), which was 20-30 % slower.  Waits are cp.async.wait_group (tracked
// by the hardware, no spin loop) and warp / CTA barriers: nothing to bound.
template <int FMT> constexpr int ring_slots() { return FMT == T_Q4_K ? 4 : 3; }
constexpr int kRingWarps = 16;

template <int FMT>
__device__ __forceinline__ void copy_unit(uint32_t dst, const uint8_t *src, int lane) {
  constexpr int CH = unit_bytes<FMT>() / 16;
#pragma unroll
  for (int c = lane; c < CH; c += 32) cp_async16(dst + 16 * c, src + 16 * c);
}

// load_unit's registers from a unit staged in shared memory (same offsets)
template <int FMT>
__device__ __forceinline__ void load_unit_smem(PairRegs<FMT> &R, uint32_t u, int lane, int g) {
#pragma unroll
  for (int r = 0; r < 2; r++) {
    if constexpr (FMT == T_Q6_K) {
      R.l[r][0] = lds128(u + ((2 * r) * 32 + lane) * 16);
      R.l[r][1] = lds128(u + ((2 * r + 1) * 32 + lane) * 16);
      R.qh[r] = lds128(u + kQ6H + (r * 32 + lane) * 16);
      R.sc[r] = lds32(u + kQ6S + (r * 32 + lane) * 4);
      R.d[r] = lds16(u + kQ6D + 2 * (8 * r + g));
    } else {
      R.q[r][0] = lds128(u + ((2 * r) * 32 + lane) * 16);
      R.q[r][1] = lds128(u + ((2 * r + 1) * 32 + lane) * 16);
      R.h[r] = lds128(u + hdr_off<FMT>() + 16 * (8 * r + g));
      if constexpr (FMT == T_Q5_K) R.e[r] = lds64(u + kE5 + (r * 32 + lane) * 8);
    }
  }
}

template <int FMT>
__global__ void __launch_bounds__(kRingWarps * 32, 1) kq_ring_kernel(const KqArgs p) {
  constexpr int NT = kRingWarps * 32, S = ring_slots<FMT>(), US = unit_bytes<FMT>();
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  int T0, T1;
  cta_tiles(p.rows, T0, T1);
  const int nb = p.nb;
  const int npair = (T1 - T0) * nb;
  const int i0 = (int)((int64_t)warp * npair / kRingWarps), i1 = (int)((int64_t)(warp + 1) * npair / kRingWarps);
  const int64_t row0 = (int64_t)T0 * kTile;
  const int nrows = (int)(min((int64_t)T1 * kTile, p.rows) - row0);
  float *sums = reinterpret_cast<float *>(smem + p.part_off);      // [pair][16 rows]
  const uint32_t ring = smem_u32(smem + p.ring_off) + (uint32_t)(warp * S * US);
  const uint8_t *base = p.w + (int64_t)T0 * nb * US;

  // The warp's first unit (two when its run is longer than its ring) streams in before
  // griddepcontrol.wait (the weights are not the previous kernel's output), the rest of its first S
  // only after the activation's loads: loads issued behind a burst of cp.async wait for the burst to
  // drain, and staging the activation behind all S units cost ~8 % of a 4096 x 4096 launch (measured
  // on a B200: 4.61 -> 4.22 us; every unit after the staging 4.92 us; two units before it 4.95 us
  // there, but faster on the long runs of the 8B gate/up and down matrices).
  const int pre = i1 - i0 > S ? 2 : 1;
#pragma unroll
  for (int d = 0; d < 2; d++) {
    if (d < pre) {
      if (i0 + d < i1) copy_unit<FMT>(ring + d * US, base + (int64_t)(i0 + d) * US, lane);
      cp_async_commit();
    }
  }
  pdl_launch_dependents();
  pdl_wait();                                   // the activation is
  const SAct sa = stage_token<FMT, NT>(p, smem + p.x_off, warp, lane, g);
#pragma unroll
  for (int d = 1; d < S; d++) {
    if (d >= pre) {
      if (i0 + d < i1) copy_unit<FMT>(ring + d * US, base + (int64_t)(i0 + d) * US, lane);
      cp_async_commit();
    }
  }
  __syncthreads();

  int sb = nb > 0 ? i0 % nb : 0;                // super-block of unit i
  int slot = 0;
  for (int i = i0; i < i1; i++) {
    cp_async_wait<S - 1>();                     // unit i (the oldest pending group) has landed
    __syncwarp();                               // ... and every lane's pieces of it are visible
    PairRegs<FMT> R;
    load_unit_smem<FMT>(R, ring + slot * US, lane, g);
    float S0, S1;
    pair_sums<FMT>(R, g, t, sa, sb, S0, S1);
    __syncwarp();                               // every lane is done with the slot
    if (i + S < i1) copy_unit<FMT>(ring + slot * US, base + (int64_t)(i + S) * US, lane);
    cp_async_commit();                          // one group per iteration, empty or not
    if (t == 0) { sums[i * kTile + g] = S0; sums[i * kTile + g + 8] = S1; }
    if (++sb == nb) sb = 0;
    if (++slot == S) slot = 0;
  }
  cp_async_wait<0>();
  __syncthreads();

  // one thread per row (per (gate, up) pair with swiglu): the super-block sums in order
  const int step = p.swiglu ? 2 : 1;
  for (int row = step * threadIdx.x; row < nrows; row += step * NT) {
    float o[2] = {0.f, 0.f};
    for (int e = 0; e < step; e++) {
      const int rr = row + e;
      const float *sr = sums + (int64_t)(rr / kTile) * nb * kTile + rr % kTile;
      float tot = 0.f;
      for (int s = 0; s < nb; s++) tot = __fadd_rn(tot, sr[s * kTile]);
      o[e] = tot;
    }
    store_row(p, 0, row0 + row, o[0], o[1]);
  }
}

// ---------------------------------------------------------------------------- 2..16 tokens
// Packed pairs of f32 (Blackwell's f32x2 arithmetic): element x in the low word, y in the high word.
// Each element is rounded exactly as the scalar instruction rounds it, so a packed term is the same
// bits as the scalar formula (k45_pair / q6_pair) of each of its two tokens.
constexpr f2v kBias2 = ((f2v)0x4B400000u << 32) | 0x4B400000u;    // (kBiasF, kBiasF)
// two biased MMA accumulators -> their exact integer values as a pair
__device__ __forceinline__ f2v biased_f2(int a, int b) { return f2sub(f2bits((uint32_t)a, (uint32_t)b), kBias2); }

// Per-warp scale staging of one super-block, token pairs (2u, 2u + 1) packed:
//   Q4_K / Q5_K: [pair u][chunk c] 32 bytes: (xd0, xd0'), (xd1, xd1'), (xm0, xm0'), (xm1, xm1') with
//                xd0 / xd1 the scales of 32-blocks 2c, 2c + 1 and xm = xd * xs (unprimed: token 2u);
//   Q6_K:        [pair u][32-block b] (xd, xd').
template <int FMT, int NTOK> constexpr int batch_sc_bytes() { return FMT == T_Q6_K ? NTOK * 8 * 4 : NTOK * 4 * 16; }

template <int FMT, int NTOK>
__device__ __forceinline__ void stage_batch_scales(const KqArgs &p, int sb, uint8_t *wsc, int lane) {
  const int64_t kb = p.k / 32;
  if constexpr (FMT == T_Q6_K) {
    float2 *o = reinterpret_cast<float2 *>(wsc);
#pragma unroll
    for (int e = lane; e < NTOK / 2 * 8; e += 32) {
      const int u = e >> 3, b = e & 7, t0 = 2 * u, t1 = 2 * u + 1;
      o[e] = make_float2(t0 < p.ntok ? __ldg(p.xd + t0 * kb + sb * 8 + b) : 0.f,
                         t1 < p.ntok ? __ldg(p.xd + t1 * kb + sb * 8 + b) : 0.f);
    }
  } else {
    float4 *o = reinterpret_cast<float4 *>(wsc);
#pragma unroll
    for (int e = lane; e < NTOK / 2 * 4; e += 32) {
      const int u = e >> 2, c = e & 3;
      float v[2][4];
#pragma unroll
      for (int j = 0; j < 2; j++) {
        const int tok = 2 * u + j;
        v[j][0] = v[j][1] = v[j][2] = v[j][3] = 0.f;
        if (tok < p.ntok) {
          const float2 xd = __ldg(reinterpret_cast<const float2 *>(p.xd + tok * kb + sb * 8 + 2 * c));
          const int2 xs = __ldg(reinterpret_cast<const int2 *>(p.xs + tok * kb + sb * 8 + 2 * c));
          v[j][0] = xd.x; v[j][1] = xd.y;
          v[j][2] = __fmul_rn(xd.x, __int2float_rn(xs.x)); v[j][3] = __fmul_rn(xd.y, __int2float_rn(xs.y));
        }
      }
      o[2 * e] = make_float4(v[0][0], v[1][0], v[0][1], v[1][1]);
      o[2 * e + 1] = make_float4(v[0][2], v[1][2], v[0][3], v[1][3]);
    }
  }
}

// B fragments of super-block sb for NG groups of 8 tokens: token 8G + g, words 4m + t (m = 0..15:
// Q4_K / Q5_K sub-block m >> 1, bytes 16 (m & 1) + 4t..; Q6_K group m, bytes 4t..).  Padding tokens
// read zeros.
template <int NG>
__device__ __forceinline__ void load_batch_b(const KqArgs &p, int sb, int g, int t, uint32_t (&B)[NG][16]) {
#pragma unroll
  for (int G = 0; G < NG; G++) {
    const int tok = 8 * G + g;
    const bool live = tok < p.ntok;
    const uint32_t *xw = reinterpret_cast<const uint32_t *>(p.xq + (int64_t)(live ? tok : 0) * p.k + (int64_t)sb * 256);
#pragma unroll
    for (int m = 0; m < 16; m++) B[G][m] = live ? __ldg(xw + 4 * m + t) : 0u;
  }
}

// One Q4_K / Q5_K unit for NG token groups: S[G][r] = the super-block sums of row g + 8r for tokens
// 8G + 2t and 8G + 2t + 1 (packed), in the canonical order: k45_pair per chunk, ((P0 + P1) + (P2 + P3)).
template <int FMT, int NG>
__device__ __forceinline__ void unit_k45_batch(const PairRegs<FMT> &R, const uint32_t (&B)[NG][16], uint32_t wsc, int t,
                                               f2v (&S)[NG][2]) {
  constexpr bool FIVE = FMT == T_Q5_K;
  uint2 eg = make_uint2(0, 0), eh = make_uint2(0, 0);
  if constexpr (FIVE) { eg = R.e[0]; eh = R.e[1]; }
  const float d[2] = {h2f(R.h[0].x & 0xffffu), h2f(R.h[1].x & 0xffffu)};
  const float dm[2] = {h2f(R.h[0].x >> 16), h2f(R.h[1].x >> 16)};
  f2v q01[NG][2];
#pragma unroll
  for (int c = 0; c < 4; c++) {
    uint32_t lo[4], hi[4];
    k45_operands<FIVE>(R.q, eg, eh, c, lo, hi);
    // per row: (d*sc) of both sub-blocks and -(dmin*mn), broadcast to both tokens of a pair
    f2v ds0[2], ds1[2], ndm0[2], ndm1[2];
#pragma unroll
    for (int r = 0; r < 2; r++) {
      const K45Sc s = k45_sc(d[r], dm[r], k45_field(R.h[r], c));
      ds0[r] = f2pack(s.ds0, s.ds0); ds1[r] = f2pack(s.ds1, s.ds1);
      ndm0[r] = f2pack(-s.dm0, -s.dm0); ndm1[r] = f2pack(-s.dm1, -s.dm1);
    }
#pragma unroll
    for (int G = 0; G < NG; G++) {
      int L[4] = {kBias, kBias, kBias, kBias}, U[4] = {kBias, kBias, kBias, kBias};
      mma_k32(L, lo[0], lo[1], lo[2], lo[3], B[G][4 * c], B[G][4 * c + 1]);
      mma_k32(U, hi[0], hi[1], hi[2], hi[3], B[G][4 * c + 2], B[G][4 * c + 3]);
      const uint32_t a = wsc + 32 * ((4 * G + t) * 4 + c);
      const uint4 w0 = lds128(a), w1 = lds128(a + 16);
      const f2v xd0 = f2bits(w0.x, w0.y), xd1 = f2bits(w0.z, w0.w), xm0 = f2bits(w1.x, w1.y), xm1 = f2bits(w1.z, w1.w);
#pragma unroll
      for (int r = 0; r < 2; r++) {
        // k45_pair for both tokens: fma(xd1*ds1, lo1, fma(xd0*ds0, lo0, -(fma(dm1, xm1, dm0*xm0))))
        const f2v nm = f2fma(ndm1[r], xm1, f2mul(ndm0[r], xm0));
        const f2v P = f2fma(f2mul(xd1, ds1[r]), biased_f2(U[2 * r], U[2 * r + 1]),
                            f2fma(f2mul(xd0, ds0[r]), biased_f2(L[2 * r], L[2 * r + 1]), nm));
        if (c == 0 || c == 2) q01[G][r] = P;
        else if (c == 1) S[G][r] = f2add(q01[G][r], P);
        else S[G][r] = f2add(S[G][r], f2add(q01[G][r], P));
      }
    }
  }
}

// One Q6_K unit for NG token groups (same output convention): q6_pair per group pair, the pairs of
// each 128-value half as ((P0 + P1) + (P2 + P3)), then half 0 + half 1.  The terms are scalar here:
// a packed (f32x2) statement of the same formula gave results a few ulps off the one-token kernel's
// on a B200 (measured; the Q4_K / Q5_K packed terms match bit for bit), so Q6_K keeps the scalar
// arithmetic and packs only its sums.
template <int NG>
__device__ __forceinline__ void unit_q6_batch(const PairRegs<T_Q6_K> &R, const uint32_t (&B)[NG][16], uint32_t wsc,
                                              int t, f2v (&Sx)[NG][2]) {
  const float d[2] = {h2f(R.d[0]), h2f(R.d[1])};
  float S[NG][4], part[NG][4];                  // part: the running (P0 + P1) of a half; S holds half 0's tree
#pragma unroll
  for (int h = 0; h < 2; h++) {
    const uint32_t lgw[4] = {R.l[0][h].x, R.l[0][h].y, R.l[0][h].z, R.l[0][h].w};
    const uint32_t lhw[4] = {R.l[1][h].x, R.l[1][h].y, R.l[1][h].z, R.l[1][h].w};
    const uint32_t qgw[2] = {h ? R.qh[0].z : R.qh[0].x, h ? R.qh[0].w : R.qh[0].y};
    const uint32_t qhw[2] = {h ? R.qh[1].z : R.qh[1].x, h ? R.qh[1].w : R.qh[1].y};
    float q[NG][4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      // scales of groups 8h + 2k, 8h + 2k + 1 (word k of the row's record, bytes 2h, 2h + 1)
      const uint32_t w0 = k == 0 ? R.sc16[0].x : k == 1 ? R.sc16[0].y : k == 2 ? R.sc16[0].z : R.sc16[0].w;
      const uint32_t w1 = k == 0 ? R.sc16[1].x : k == 1 ? R.sc16[1].y : k == 2 ? R.sc16[1].z : R.sc16[1].w;
      const float sc[2][2] = {{sbyte_f(w0, 2 * h), sbyte_f(w0, 2 * h + 1)}, {sbyte_f(w1, 2 * h), sbyte_f(w1, 2 * h + 1)}};
      // signed quants q - 32 of groups 8h + 2k + uu (bytes in [0, 63]: + 96 never carries, then flip
      // the top bit), rows g and g + 8
      uint32_t A[2][2];
#pragma unroll
      for (int uu = 0; uu < 2; uu++) {
        A[uu][0] = (q6_unpack(lgw[uu * 2], lgw[uu * 2 + 1], qgw[uu], k) + 0x60606060u) ^ 0x80808080u;
        A[uu][1] = (q6_unpack(lhw[uu * 2], lhw[uu * 2 + 1], qhw[uu], k) + 0x60606060u) ^ 0x80808080u;
      }
#pragma unroll
      for (int G = 0; G < NG; G++) {
        int C0[4] = {kBias, kBias, kBias, kBias}, C1[4] = {kBias, kBias, kBias, kBias};
        mma_k16s(C0, A[0][0], A[0][1], B[G][8 * h + 2 * k]);
        mma_k16s(C1, A[1][0], A[1][1], B[G][8 * h + 2 * k + 1]);
        const uint2 xw = lds64(wsc + 8 * ((4 * G + t) * 8 + 4 * h + k));
        const float xd[2] = {__uint_as_float(xw.x), __uint_as_float(xw.y)};
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const int ri = e >> 1;
          const float P = q6_pair(xd[e & 1], d[ri], sc[ri][0], biased_f(C0[e]), sc[ri][1], biased_f(C1[e]));
          if (k == 0 || k == 2) q[G][e] = P;
          else if (k == 1) part[G][e] = __fadd_rn(q[G][e], P);
          else {
            const float hh = __fadd_rn(part[G][e], __fadd_rn(q[G][e], P));
            S[G][e] = h == 0 ? hh : __fadd_rn(S[G][e], hh);
          }
        }
      }
    }
  }
#pragma unroll
  for (int G = 0; G < NG; G++) {
    Sx[G][0] = f2pack(S[G][0], S[G][1]);
    Sx[G][1] = f2pack(S[G][2], S[G][3]);
  }
}

// 2..16 tokens.  A CTA owns tiles [T0, T1); its units are taken super-block-major (unit i = tile
// i % nt of super-block i / nt) and cut into equal runs, one per warp, so a warp loads the
// activation fragments of a super-block once for all the tiles it takes of it.  Each warp stages its
// units through a ring of kBatchSlots shared-memory slots with 16-byte cp.async (as kq_ring_kernel),
// the first before griddepcontrol.wait; each unit's super-block sums go to shared memory
// [tile][super-block][row][token], and after one CTA barrier a thread per (row, token) adds them in
// super-block order.  The waits are cp.async.wait_group and warp / CTA barriers: nothing to bound.
constexpr int kBatchWarps = 8;
constexpr int kBatchSlots = 2;
constexpr int64_t kBatchBudget = 220 * 1024;

template <int FMT, int NG>
__global__ void __launch_bounds__(kBatchWarps * 32, 1) kq_batch_kernel(const KqArgs p) {
  constexpr int NW = kBatchWarps, NT = NW * 32, NTOK = 8 * NG, S = kBatchSlots, US = unit_bytes<FMT>();
  constexpr int SCB = batch_sc_bytes<FMT, NTOK>();
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  int T0, T1;
  cta_tiles(p.rows, T0, T1);
  const int nb = p.nb, nt = T1 - T0, N = nt * nb;
  const int i0 = (int)((int64_t)warp * N / NW), i1 = (int)((int64_t)(warp + 1) * N / NW);
  const uint32_t ring = smem_u32(smem + p.ring_off) + (uint32_t)(warp * S * US);
  uint8_t *wsc = smem + p.x_off + warp * SCB;
  const uint32_t wsc_a = smem_u32(wsc);
  float *sums = reinterpret_cast<float *>(smem + p.part_off);      // [tile][sb][16 rows][NTOK]
  const uint8_t *base = p.w + (int64_t)T0 * nb * US;
  auto unit_ptr = [&](int i) {
    const int sb = i / nt, tl = i - sb * nt;
    return base + ((int64_t)tl * nb + sb) * US;
  };

#pragma unroll
  for (int d = 0; d < S; d++) {                 // not the previous kernel's output
    if (i0 + d < i1) copy_unit<FMT>(ring + d * US, unit_ptr(i0 + d), lane);
    cp_async_commit();
  }
  pdl_launch_dependents();
  pdl_wait();                                   // the activation is

  uint32_t B[NG][16];
  int cur = -1, slot = 0;
  for (int i = i0; i < i1; i++) {
    const int sb = i / nt, tl = i - sb * nt;
    if (sb != cur) {
      load_batch_b<NG>(p, sb, g, t, B);
      __syncwarp();
      stage_batch_scales<FMT, NTOK>(p, sb, wsc, lane);
      cur = sb;
    }
    cp_async_wait<S - 1>();                     // unit i has landed
    __syncwarp();                               // ... every lane's pieces of it, and the staged scales, are visible
    PairRegs<FMT> R;
    if constexpr (FMT == T_Q6_K) {
      const uint32_t u = ring + slot * US;
#pragma unroll
      for (int r = 0; r < 2; r++) {
        R.l[r][0] = lds128(u + ((2 * r) * 32 + lane) * 16);
        R.l[r][1] = lds128(u + ((2 * r + 1) * 32 + lane) * 16);
        R.qh[r] = lds128(u + kQ6H + (r * 32 + lane) * 16);
        R.sc16[r] = lds128(u + kQ6S + 16 * (8 * r + g));
        R.d[r] = lds16(u + kQ6D + 2 * (8 * r + g));
      }
    } else {
      load_unit_smem<FMT>(R, ring + slot * US, lane, g);
    }
    f2v Sx[NG][2];
    if constexpr (FMT == T_Q6_K) unit_q6_batch<NG>(R, B, wsc_a, t, Sx);
    else unit_k45_batch<FMT, NG>(R, B, wsc_a, t, Sx);
    __syncwarp();                               // every lane is done with the slot and the scales
    if (i + S < i1) copy_unit<FMT>(ring + slot * US, unit_ptr(i + S), lane);
    cp_async_commit();
    float *su = sums + ((int64_t)tl * nb + sb) * kTile * NTOK;
#pragma unroll
    for (int G = 0; G < NG; G++)
#pragma unroll
      for (int r = 0; r < 2; r++) {
        float a, b;
        f2unpack(Sx[G][r], a, b);
        *reinterpret_cast<float2 *>(su + (g + 8 * r) * NTOK + 8 * G + 2 * t) = make_float2(a, b);
      }
    if (++slot == S) slot = 0;
  }
  cp_async_wait<0>();
  __syncthreads();

  // one thread per (row, token) (per (gate, up) pair and token with swiglu): sums in super-block order
  const int step = p.swiglu ? 2 : 1;
  const int64_t row0 = (int64_t)T0 * kTile;
  const int nrows = (int)(min((int64_t)T1 * kTile, p.rows) - row0);
  const int npos = (nrows + step - 1) / step * NTOK;
  for (int idx = threadIdx.x; idx < npos; idx += NT) {
    const int tok = idx % NTOK, row = (idx / NTOK) * step;
    if (tok >= p.ntok) continue;
    float o[2] = {0.f, 0.f};
    for (int e = 0; e < step; e++) {
      const int rr = row + e;
      const float *sr = sums + (int64_t)(rr / kTile) * nb * kTile * NTOK + (rr % kTile) * NTOK + tok;
      float tot = 0.f;
      for (int s = 0; s < nb; s++) tot = __fadd_rn(tot, sr[(int64_t)s * kTile * NTOK]);
      o[e] = tot;
    }
    store_row(p, tok, row0 + row, o[0], o[1]);
  }
}

// ---------------------------------------------------------------------------- host side
int kq_x_bytes(const DevMatrix &m) {
  const int64_t k = m.cols;
  return (int)((k + (m.type == T_Q6_K ? k / 8 + k / 4 : k / 4) + 127) / 128 * 128);
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

// The one-token launches over a matrix (kq_ring_kernel): a CTA per SM, each over whole tiles, at
// most as many per CTA as leave its super-block sums room in shared memory next to the staged
// activation and the weight rings.
constexpr int64_t kRingBudget = 220 * 1024;

int64_t ring_bytes(int type) {
  switch (type) {
    case T_Q4_K: return (int64_t)kRingWarps * ring_slots<T_Q4_K>() * unit_bytes<T_Q4_K>();
    case T_Q5_K: return (int64_t)kRingWarps * ring_slots<T_Q5_K>() * unit_bytes<T_Q5_K>();
    default: return (int64_t)kRingWarps * ring_slots<T_Q6_K>() * unit_bytes<T_Q6_K>();
  }
}

cudaError_t launch_stream(const DevMatrix &m, const ActView &act, float *y, const float *y_add, const GemvFuse &fz,
                          int num_sms, cudaStream_t s, bool pdl, const char **why) {
  const int64_t nb = m.cols / 256;
  const int64_t x_bytes = kq_x_bytes(m), rb = ring_bytes(m.type);
  const int64_t tiles_all = (m.rows + kTile - 1) / kTile;
  const int64_t per_tile = nb * kTile * 4;                                 // super-block sums of one tile
  const int64_t cap = (kRingBudget - rb - x_bytes) / per_tile;              // tiles per CTA
  if (cap < 1) { *why = "k-quant rows too long for the one-token GEMV"; return cudaErrorInvalidValue; }
  const int64_t per_launch = cap * num_sms;
  const int us = kq_unit_bytes(m.type);
  for (int64_t tb = 0; tb < tiles_all; tb += per_launch) {
    const int64_t nt = tiles_all - tb < per_launch ? tiles_all - tb : per_launch;
    const int64_t r0 = tb * kTile;
    const int grid = (int)(nt < num_sms ? nt : num_sms);
    const int64_t tiles_cta = (nt + grid - 1) / grid;
    KqArgs a{};
    a.w = m.data + tb * nb * us;
    a.rows = m.rows - r0 < nt * kTile ? m.rows - r0 : nt * kTile;
    a.nb = (int)nb; a.ntok = 1; a.k = m.cols;
    a.xq = act.xq; a.xd = act.xd; a.xs = act.xs; a.x = act.x;
    a.y = y + (fz.swiglu ? r0 / 2 : r0);
    a.y_add = y_add ? y_add + r0 : nullptr;
    a.norm_w = fz.norm_w; a.norm_eps = fz.eps; a.swiglu = fz.swiglu ? 1 : 0;
    a.ring_off = 0; a.x_off = (int)rb; a.part_off = (int)(rb + x_bytes);
    const int smem = (int)(rb + x_bytes + tiles_cta * per_tile);
    const int block = kRingWarps * 32;
    cudaError_t e;
    switch (m.type) {
      case T_Q4_K: e = launch_ex<kq_ring_kernel<T_Q4_K>>(kRingBudget, a, grid, block, smem, s, pdl); break;
      case T_Q5_K: e = launch_ex<kq_ring_kernel<T_Q5_K>>(kRingBudget, a, grid, block, smem, s, pdl); break;
      default: e = launch_ex<kq_ring_kernel<T_Q6_K>>(kRingBudget, a, grid, block, smem, s, pdl); break;
    }
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

template <int NG>
cudaError_t launch_batch_ng(const KqArgs &a, int type, int grid, int smem, cudaStream_t s, bool pdl) {
  const int block = kBatchWarps * 32;
  switch (type) {
    case T_Q4_K: return launch_ex<kq_batch_kernel<T_Q4_K, NG>>(kBatchBudget, a, grid, block, smem, s, pdl);
    case T_Q5_K: return launch_ex<kq_batch_kernel<T_Q5_K, NG>>(kBatchBudget, a, grid, block, smem, s, pdl);
    default: return launch_ex<kq_batch_kernel<T_Q6_K, NG>>(kBatchBudget, a, grid, block, smem, s, pdl);
  }
}

// 2..n tokens: launches of up to kBatchTok tokens (one or two MMA groups of 8), each over as
// many tiles per CTA as leave the super-block sums room in shared memory beside the weight rings and
// the scale staging.
cudaError_t launch_batch(const DevMatrix &m, const ActView &act, int ntok, float *y, int64_t y_stride,
                         const float *y_add, const GemvFuse &fz, int num_sms, cudaStream_t s, bool pdl,
                         const char **why) {
  if (!act.xq) { *why = "the in-kernel activation quantization takes one token"; return cudaErrorInvalidValue; }
  const int64_t nb = m.cols / 256;
  const int64_t tiles_all = (m.rows + kTile - 1) / kTile;
  const int us = kq_unit_bytes(m.type);
  const int64_t rb = (int64_t)kBatchWarps * kBatchSlots * us;
  for (int t0 = 0; t0 < ntok; t0 += kBatchTok) {
    const int nt_tok = ntok - t0 < kBatchTok ? ntok - t0 : kBatchTok;
    const int ng = nt_tok > 8 ? 2 : 1;
    const int ntokp = 8 * ng;
    const int64_t sc_bytes = (int64_t)kBatchWarps * (m.type == T_Q6_K ? ntokp * 8 * 4 : ntokp * 4 * 16);
    const int64_t per_tile = nb * kTile * ntokp * 4;
    const int64_t cap = (kBatchBudget - rb - sc_bytes) / per_tile;        // tiles per CTA
    if (cap < 1) { *why = "k-quant rows too long for the batched GEMV"; return cudaErrorInvalidValue; }
    const int64_t per_launch = cap * num_sms;
    for (int64_t tb = 0; tb < tiles_all; tb += per_launch) {
      const int64_t nt = tiles_all - tb < per_launch ? tiles_all - tb : per_launch;
      const int64_t r0 = tb * kTile;
      const int grid = (int)(nt < num_sms ? nt : num_sms);
      const int64_t tiles_cta = (nt + grid - 1) / grid;
      KqArgs a{};
      a.w = m.data + tb * nb * us;
      a.rows = m.rows - r0 < nt * kTile ? m.rows - r0 : nt * kTile;
      a.nb = (int)nb; a.ntok = nt_tok; a.k = m.cols;
      a.xq = act.xq + (int64_t)t0 * m.cols;
      a.xd = act.xd + (int64_t)t0 * (m.cols / 32);
      a.xs = act.xs + (int64_t)t0 * (m.cols / 32);
      a.y = y + (int64_t)t0 * y_stride + (fz.swiglu ? r0 / 2 : r0);
      a.y_add = y_add ? y_add + (int64_t)t0 * y_stride + r0 : nullptr;
      a.y_stride = y_stride;
      a.swiglu = fz.swiglu ? 1 : 0;
      a.ring_off = 0; a.x_off = (int)rb; a.part_off = (int)(rb + sc_bytes);
      const int smem = (int)(rb + sc_bytes + tiles_cta * per_tile);
      const cudaError_t e = ng == 2 ? launch_batch_ng<2>(a, m.type, grid, smem, s, pdl)
                                    : launch_batch_ng<1>(a, m.type, grid, smem, s, pdl);
      if (e != cudaSuccess) return e;
    }
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
  (void)status;                                 // these kernels never wait, so they report no timeouts
  if (m.cols % 256 || m.cols < 256) { *why = "k-quant rows must be a whole number of 256-value super-blocks"; return cudaErrorInvalidValue; }
  if (fz.norm_w && (act.xq || !act.x || ntok != 1)) { *why = "the fused RMSNorm takes one f32 token"; return cudaErrorInvalidValue; }
  if (fz.swiglu && (m.rows % 2 || y_add)) { *why = "the SwiGLU epilogue takes (gate, up) row pairs and no residual"; return cudaErrorInvalidValue; }
  if (act.xq == nullptr && (ntok != 1 || act.x == nullptr)) {
    *why = "the in-kernel activation quantization takes one token";
    return cudaErrorInvalidValue;
  }
  if (ntok == 1) return launch_stream(m, act, y, y_add, fz, num_sms, s, pdl, why);
  return launch_batch(m, act, ntok, y, y_stride, y_add, fz, num_sms, s, pdl, why);
}

}  // namespace zllm
