// Decode GEMV for the k-quant formats (Q4_K, Q5_K, Q6_K) with the integer dot products on the
// tensor cores.
//
// Replaces the reference's k-quant matvec kernels: src/compute/ref-kernels.js:196-277 (oracle)
// and the WASM matvec_q4_k / matvec_q5_k / matvec_q6_k and mm_* exports
// (src/compute/wasm/kquant-kernels.js:337-504), dispatched by ggml type as in
// src/compute/worker.js:184-197 / :251-270.
//
// What one launch computes, for up to 8 tokens:  y[t][r] = (y_add) + sum over blocks of
//   Q4_K / Q5_K:  xd * (d*sc*lo - dmin*mn*xs)       per 32-value sub-block (ref-kernels.js:235-236)
//   Q6_K:         xd * d * scale * gsum             per 16-value group     (ref-kernels.js:271)
// where lo / gsum are exact integer dot products of the weight quants with the int8 activation.
//
// Structure.  A CTA owns a contiguous range of rows (the same count for every CTA, within one) and
// walks it in tiles of 16 rows; a tile's rows are streamed HBM -> shared memory in chunks of 16
// (Q6_K: 8) super-blocks by 1D bulk copies (one per row, each issued by its own lane of warp 0,
// completion on an mbarrier), `nst` chunks in flight.  The copies of the first chunks are issued
// before griddepcontrol.wait, so under programmatic dependent launch a matrix streams in while the
// kernel before it is still computing.  Warp w takes super-blocks w and w + 8 of every chunk and
// runs warp-level integer MMAs on them (mma.sync m16n8k32 / m16n8k16, int8 x uint8 -> int32, exact):
//   * one token: the B operand is block-diagonal -- column j carries the activation of sub-block
//     (group) j and is zero elsewhere -- so the 8 MMAs of a super-block leave the 16 rows x 8
//     sub-blocks of integer dots in one accumulator, one value per lane and row pair;
//   * 2..8 tokens: B column j carries token j, one MMA per sub-block (group).
// Each integer dot becomes its block term in IEEE double with the reference's operations and
// rounding (no fused multiply-add where the JS rounds twice), so every block term is bit-identical
// to the oracle's.  Only the order of the final double additions differs from the reference, and
// it is fixed: each super-block's terms are added as a pairwise tree (Q4_K / Q5_K:
// ((T0 + T1) + (T2 + T3)) + ((T4 + T5) + (T6 + T7)); Q6_K: the same over groups 0..7 plus the same
// over 8..15) and the super-block sums are added in super-block order.  That order depends on
// nothing but the row, so a token gets the same bits alone, in a batch, or in any launch shape.
//
// After each chunk one CTA barrier (which also carries the bounded waits' give-up flag to every
// warp) publishes the chunk's super-block sums; one thread per output then adds them in order, and
// warp 0 refills the freed stage.  A one-token launch may take the f32
// activation and quantize it itself (bit-exact with quantize_act_kernel), so a lone matvec is one
// kernel.
#include "common.cuh"
#include "internal.h"
#include "kq_layout.h"

namespace zllm {

namespace {

constexpr int kTile = 16;                    // rows per tile (the MMA's M)
// super-blocks per staged chunk: two per warp for Q4_K / Q5_K (processed together), one per warp for
// Q6_K (its Q6_K SoA groups of 8, and twice the MMAs per super-block)
template <int FMT> constexpr int chunk_sb() { return FMT == T_Q6_K ? 8 : 16; }
__host__ __device__ constexpr int chunk_sb_of(int type) { return type == T_Q6_K ? 8 : 16; }
constexpr int kMaxStages = 8;
constexpr int kMaxTok = 8;                   // tokens per launch (the MMA's N)
constexpr int64_t kSmemBudget = 110 * 1024;  // two CTAs per SM

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

// ---------------------------------------------------------------------------- per super-block, one token
// One warp turns a staged super-block into its sum per row: lane (g, t) holds sub-blocks 2t, 2t+1
// (Q6_K: groups 8h+2t, 8h+2t+1 of half h) of rows g and g+8, forms the pair sum T(2t) + T(2t+1),
// and the quad tree over t gives ((p_0 + p_1) + (p_2 + p_3)) -- the super-block sum (Q6_K: the
// half's tree; super-block = half 0 + half 1).  The token-mode routines build the same trees
// within one lane.
template <bool FIVE>
__device__ __forceinline__ void sb_k45_one(uint32_t blk, int pitch, int g, int t, const SAct &x, int sb, double &p0,
                                           double &p1) {
  constexpr int QS = FIVE ? 48 : 16;
  const uint32_t rg = blk + (uint32_t)(g * pitch), rh = blk + (uint32_t)((g + 8) * pitch);
  uint2 eg = make_uint2(0, 0), eh = make_uint2(0, 0);
  if (FIVE) { eg = lds64(rg + 16 + 8 * t); eh = lds64(rh + 16 + 8 * t); }
  // this lane's activation column: sub-block g, values 4t.. and 16+4t..
  const uint32_t xa = lds32(x.xq + sb * 256 + 32 * g + 4 * t), xb = lds32(x.xq + sb * 256 + 32 * g + 16 + 4 * t);
  int C0[4] = {0, 0, 0, 0}, C1[4] = {0, 0, 0, 0};
#pragma unroll
  for (int cp = 0; cp < 2; cp++) {
    // chunks 2cp, 2cp+1: words (half 0, half 1) of each, rows g and g+8
    const uint4 wq = lds128(rg + QS + 32 * t + 16 * cp), vq = lds128(rh + QS + 32 * t + 16 * cp);
    const uint32_t wg[4] = {wq.x, wq.y, wq.z, wq.w}, wh[4] = {vq.x, vq.y, vq.z, vq.w};
#pragma unroll
    for (int ci = 0; ci < 2; ci++) {
      const int c = 2 * cp + ci;
      uint32_t lg0 = wg[2 * ci] & 0x0f0f0f0fu, lg1 = wg[2 * ci + 1] & 0x0f0f0f0fu;
      uint32_t lh0 = wh[2 * ci] & 0x0f0f0f0fu, lh1 = wh[2 * ci + 1] & 0x0f0f0f0fu;
      uint32_t ug0, ug1, uh0, uh1;
      if (FIVE) {
        lg0 |= ((eg.x >> (2 * c)) & 0x01010101u) << 4; lg1 |= ((eg.y >> (2 * c)) & 0x01010101u) << 4;
        lh0 |= ((eh.x >> (2 * c)) & 0x01010101u) << 4; lh1 |= ((eh.y >> (2 * c)) & 0x01010101u) << 4;
        ug0 = ((wg[2 * ci] >> 4) & 0x0f0f0f0fu) | (((eg.x >> (2 * c + 1)) & 0x01010101u) << 4);
        ug1 = ((wg[2 * ci + 1] >> 4) & 0x0f0f0f0fu) | (((eg.y >> (2 * c + 1)) & 0x01010101u) << 4);
        uh0 = ((wh[2 * ci] >> 4) & 0x0f0f0f0fu) | (((eh.x >> (2 * c + 1)) & 0x01010101u) << 4);
        uh1 = ((wh[2 * ci + 1] >> 4) & 0x0f0f0f0fu) | (((eh.y >> (2 * c + 1)) & 0x01010101u) << 4);
      } else {
        // high nibbles in place (16 x the quant, still an exact uint8): the word minus its low nibbles
        ug0 = wg[2 * ci] - lg0; ug1 = wg[2 * ci + 1] - lg1;
        uh0 = wh[2 * ci] - lh0; uh1 = wh[2 * ci + 1] - lh1;
      }
      int(&C)[4] = (c & 1) ? C1 : C0;
      mma_k32(C, lg0, lh0, lg1, lh1, xa * x.sel[2 * c], xb * x.sel[2 * c]);
      mma_k32(C, ug0, uh0, ug1, uh1, xa * x.sel[2 * c + 1], xb * x.sel[2 * c + 1]);
    }
  }
  // lane (g, t): sub-blocks 2t and 2t+1 of rows g and g+8
  int v0 = C0[0] + C1[0], v1 = C0[1] + C1[1], v2 = C0[2] + C1[2], v3 = C0[3] + C1[3];
  if (!FIVE) { v1 >>= 4; v3 >>= 4; }
  const uint4 xdw = lds128(x.xd + 8 * (sb * 8 + 2 * t));
  const double xd0 = __hiloint2double((int)xdw.y, (int)xdw.x), xd1 = __hiloint2double((int)xdw.w, (int)xdw.z);
  const uint2 xs = lds64(x.xs + 4 * (sb * 8 + 2 * t));
  // d, dmin and this lane's 24-bit scale field (chunk t, bytes 4+3t .. 6+3t of the block)
  const uint32_t fo = 4 + 3 * t, fw = fo & ~3u, fs = (fo & 3) * 8;
#pragma unroll
  for (int r = 0; r < 2; r++) {
    const uint32_t row = r ? rh : rg;
    const uint32_t dw = lds32(row), F = __funnelshift_r(lds32(row + fw), lds32(row + fw + 4), fs);
    const double d = h2d(dw & 0xffffu), dmin = h2d(dw >> 16);
    const double pr = __dadd_rn(k45_term(d, dmin, F & 63, (F >> 12) & 63, r ? v2 : v0, (int)xs.x, xd0),
                                k45_term(d, dmin, (F >> 6) & 63, (F >> 18) & 63, r ? v3 : v1, (int)xs.y, xd1));
    if (r) p1 = quad_tree(pr); else p0 = quad_tree(pr);
  }
}

// Q6_K, half h of super-block j of a staged chunk (group of n super-blocks).
__device__ __forceinline__ void sb_q6_one(uint32_t blk, int pitch, int n, int j, int h, int g, int t, const SAct &x,
                                          int sb, double &p0, double &p1) {
  const uint32_t rg = blk + (uint32_t)(g * pitch), rh = blk + (uint32_t)((g + 8) * pitch);
  const uint32_t qlo = 128 * j + 32 * t + 16 * h, qho = 128 * n + 64 * j + 16 * t + 8 * h,
                 sco = 192 * n + 16 * j + 4 * t + 2 * h, dof = 208 * n + 2 * j;
  // ql words [u][p], qh words [u] of half h
  const uint4 lg = lds128(rg + qlo), lh = lds128(rh + qlo);
  const uint2 qg = lds64(rg + qho), qh = lds64(rh + qho);
  const uint32_t lgw[4] = {lg.x, lg.y, lg.z, lg.w}, lhw[4] = {lh.x, lh.y, lh.z, lh.w};
  const uint32_t qgw[2] = {qg.x, qg.y}, qhw[2] = {qh.x, qh.y};
  // this lane's activation column: group 8h + g, values 4t..4t+3
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
  // lane (g, t): groups 8h+2t, 8h+2t+1 of rows g and g+8
  const uint2 s2 = lds64(x.xs16 + 4 * (sb * 16 + 8 * h + 2 * t));
  const uint2 xdw = lds64(x.xd + 8 * (sb * 8 + 4 * h + t));
  const double xdv = __hiloint2double((int)xdw.y, (int)xdw.x);
#pragma unroll
  for (int r = 0; r < 2; r++) {
    const uint32_t row = r ? rh : rg;
    const uint32_t scw = lds16(row + sco);
    const double xdd = __dmul_rn(xdv, h2d(lds16(row + dof)));
    const double pr = __dadd_rn(q6_term(xdd, (int)(int8_t)(scw & 0xff), C[2 * r] - 32 * (int)s2.x),
                                q6_term(xdd, (int)(int8_t)(scw >> 8), C[2 * r + 1] - 32 * (int)s2.y));
    if (r) p1 = quad_tree(pr); else p0 = quad_tree(pr);
  }
}

// ---------------------------------------------------------------------------- per super-block, 2..8 tokens
// Lane (g, t) supplies token g's activation and owns outputs e = 2*ri + ti: row g + 8*ri, token
// 2t + ti.  It builds the same per-super-block trees as the one-token path from all sub-blocks.
struct GAct {
  const int8_t *xq;     // [ntok][k]
  const float *xd;      // [ntok][k/32]
  const int32_t *xs;    // [ntok][k/32]
  int64_t k;
  int ntok;
};

template <bool FIVE>
__device__ __forceinline__ void sb_k45_tok(uint32_t blk, int pitch, int g, int t, const GAct &x, int sb, double (&S)[4]) {
  constexpr int QS = FIVE ? 48 : 16;
  const uint32_t rg = blk + (uint32_t)(g * pitch), rh = blk + (uint32_t)((g + 8) * pitch);
  const uint4 hdr[2] = {lds128(rg), lds128(rh)};
  const bool live = g < x.ntok;
  const uint32_t *xw = reinterpret_cast<const uint32_t *>(x.xq + (live ? g : 0) * x.k + (int64_t)sb * 256);
  const int t0 = 2 * t < x.ntok ? 2 * t : 0, t1 = 2 * t + 1 < x.ntok ? 2 * t + 1 : 0;   // padding tokens read token 0
  const float *xd0 = x.xd + t0 * (x.k / 32) + sb * 8, *xd1 = x.xd + t1 * (x.k / 32) + sb * 8;
  const int32_t *xs0 = x.xs + t0 * (x.k / 32) + sb * 8, *xs1 = x.xs + t1 * (x.k / 32) + sb * 8;
  double dd[2], dm[2];
#pragma unroll
  for (int ri = 0; ri < 2; ri++) { dd[ri] = h2d(hdr[ri].x & 0xffffu); dm[ri] = h2d(hdr[ri].x >> 16); }
  double q01[4];
#pragma unroll
  for (int c = 0; c < 4; c++) {
    const uint2 wgc = lds64(rg + QS + 32 * t + 8 * c), whc = lds64(rh + QS + 32 * t + 8 * c);
    uint32_t lg0 = wgc.x & 0x0f0f0f0fu, lg1 = wgc.y & 0x0f0f0f0fu, lh0 = whc.x & 0x0f0f0f0fu, lh1 = whc.y & 0x0f0f0f0fu;
    uint32_t ug0, ug1, uh0, uh1;
    if (FIVE) {
      const uint2 eg = lds64(rg + 16 + 8 * t), eh = lds64(rh + 16 + 8 * t);
      lg0 |= ((eg.x >> (2 * c)) & 0x01010101u) << 4; lg1 |= ((eg.y >> (2 * c)) & 0x01010101u) << 4;
      lh0 |= ((eh.x >> (2 * c)) & 0x01010101u) << 4; lh1 |= ((eh.y >> (2 * c)) & 0x01010101u) << 4;
      ug0 = ((wgc.x >> 4) & 0x0f0f0f0fu) | (((eg.x >> (2 * c + 1)) & 0x01010101u) << 4);
      ug1 = ((wgc.y >> 4) & 0x0f0f0f0fu) | (((eg.y >> (2 * c + 1)) & 0x01010101u) << 4);
      uh0 = ((whc.x >> 4) & 0x0f0f0f0fu) | (((eh.x >> (2 * c + 1)) & 0x01010101u) << 4);
      uh1 = ((whc.y >> 4) & 0x0f0f0f0fu) | (((eh.y >> (2 * c + 1)) & 0x01010101u) << 4);
    } else {
      ug0 = wgc.x & 0xf0f0f0f0u; ug1 = wgc.y & 0xf0f0f0f0u; uh0 = whc.x & 0xf0f0f0f0u; uh1 = whc.y & 0xf0f0f0f0u;
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

// Q6_K, 2..8 tokens: Sh[e][h] = tree8 of half h, ((P0 + P1) + (P2 + P3)) with P_k the pair of
// groups 8h + 2k, 8h + 2k + 1 (the pair lane k holds in the one-token path).
__device__ __forceinline__ void sb_q6_tok(uint32_t blk, int pitch, int n, int j, int g, int t, const GAct &x, int sb,
                                          double (&Sh)[4][2]) {
  const uint32_t rg = blk + (uint32_t)(g * pitch), rh = blk + (uint32_t)((g + 8) * pitch);
  const double d[2] = {h2d(lds16(rg + 208 * n + 2 * j)), h2d(lds16(rh + 208 * n + 2 * j))};
  const bool live = g < x.ntok;
  const uint32_t *xw = reinterpret_cast<const uint32_t *>(x.xq + (live ? g : 0) * x.k + (int64_t)sb * 256);
  const int t0 = 2 * t < x.ntok ? 2 * t : 0, t1 = 2 * t + 1 < x.ntok ? 2 * t + 1 : 0;
  const float *xd0 = x.xd + t0 * (x.k / 32) + sb * 8, *xd1 = x.xd + t1 * (x.k / 32) + sb * 8;
#pragma unroll
  for (int h = 0; h < 2; h++) {
    // this lane's quants of half h: ql words [u][p], qh words [u] (values 4t..4t+3 of each group)
    const uint32_t qlo = 128 * j + 32 * t + 16 * h, qho = 128 * n + 64 * j + 16 * t + 8 * h;
    const uint4 lg = lds128(rg + qlo), lh = lds128(rh + qlo);
    const uint2 qg = lds64(rg + qho), qh = lds64(rh + qho);
    const uint32_t gw[4] = {lg.x, lg.y, lg.z, lg.w}, hw[4] = {lh.x, lh.y, lh.z, lh.w};
    const uint32_t gq[2] = {qg.x, qg.y}, hq[2] = {qh.x, qh.y};
    double q[4][2];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      // scales of groups 8h + 2k + u (reordered table: byte 4k + 2h + u) and their 32-block's xd
      const uint32_t sw[2] = {lds16(rg + 192 * n + 16 * j + 4 * k + 2 * h), lds16(rh + 192 * n + 16 * j + 4 * k + 2 * h)};
      const double xdv[2] = {(double)__ldg(xd0 + 4 * h + k), (double)__ldg(xd1 + 4 * h + k)};
      double P[4];
#pragma unroll
      for (int u = 0; u < 2; u++) {
        // signed quants q - 32 (bytes in [0, 63]: + 96 never carries, then flip the top bit)
        const uint32_t a0 = (q6_unpack(gw[u * 2], gw[u * 2 + 1], gq[u], k) + 0x60606060u) ^ 0x80808080u;
        const uint32_t a1 = (q6_unpack(hw[u * 2], hw[u * 2 + 1], hq[u], k) + 0x60606060u) ^ 0x80808080u;
        const uint32_t xa = live ? __ldg(xw + 4 * (8 * h + 2 * k + u) + t) : 0u;
        int Cm[4] = {0, 0, 0, 0};
        mma_k16s(Cm, a0, a1, xa);
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const int ri = e >> 1, ti = e & 1;
          const int scale = (int)(int8_t)((sw[ri] >> (8 * u)) & 0xffu);
          const double T = q6_term(__dmul_rn(xdv[ti], d[ri]), scale, Cm[e]);
          P[e] = u == 0 ? T : __dadd_rn(P[e], T);
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

// ---------------------------------------------------------------------------- kernel
struct KqArgs {
  const uint8_t *w;
  int64_t row_stride;
  int64_t rows;
  int nb;               // super-blocks per row
  int nchunk;           // chunks per row
  int pitch;            // shared-memory bytes per staged row
  int nst;              // stages in the ring
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

// warps per CTA: 16 for one token (latency hiding), 8 for 2..8 tokens (registers)
// A CTA runs NG independent groups of 8 warps.  One token: 2 groups, each taking alternate 16-row
// tiles with its own stage ring, barrier and adder, so one group's waits and barriers overlap the
// other's arithmetic.  2..8 tokens: 1 group (their registers allow no more).
constexpr int kGroupWarps = 8;
template <bool TOK> constexpr int groups_of() { return TOK ? 1 : 2; }

template <int FMT, bool TOK>
__global__ void __launch_bounds__(groups_of<TOK>() * kGroupWarps * 32, 2) kq_gemv_kernel(const KqArgs p) {
  constexpr int BS = FMT == T_Q4_K ? 144 : FMT == T_Q5_K ? 176 : 210;
  constexpr int NTP = TOK ? kMaxTok : 1;
  constexpr int NG = groups_of<TOK>(), NT = NG * kGroupWarps * 32, GT = kGroupWarps * 32;
  constexpr int kChunk = chunk_sb<FMT>();
  constexpr int kSlots = 16;                    // per-chunk slots of super-block sums (Q6_K: 8 x 2 halves)
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int grp = warp / kGroupWarps, gw = warp % kGroupWarps;     // group, warp within the group
  const int nst = p.nst;                        // stages per group
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + p.bar_off) + grp * nst;
  uint8_t *stages = smem + (size_t)grp * nst * kTile * p.pitch;
  double *part = reinterpret_cast<double *>(smem + p.part_off) + (size_t)grp * 2 * kSlots * kTile * NTP;  // [2][slot][row][NTP]

  // row range of this CTA (whole (gate, up) pairs with swiglu)
  const int64_t pr = p.swiglu ? p.rows / 2 : p.rows, rm = p.swiglu ? 2 : 1;
  const int64_t r0 = rm * ((int64_t)blockIdx.x * pr / gridDim.x), r1 = rm * ((int64_t)(blockIdx.x + 1) * pr / gridDim.x);
  const int ntile = (int)((r1 - r0 + kTile - 1) / kTile);
  const int gtiles = (ntile - grp + NG - 1) / NG;   // tiles grp, grp + NG, ...
  const int nunit = gtiles * p.nchunk;              // this group's units: (its k-th tile, chunk)
  const int stage_bytes = kTile * p.pitch;

  // Warp 0 of the group fills stage u % nst with the group's unit u, one bulk copy per row issued
  // by its own lane.
  auto issue = [&](int u) {
    const int s = u % nst, tile = (u / p.nchunk) * NG + grp, c = u % p.nchunk;
    const int64_t row0 = r0 + (int64_t)tile * kTile;
    const int nr = (int)min((int64_t)kTile, r1 - row0);
    const int sb0 = c * kChunk, nsb = min(kChunk, p.nb - sb0);
    const uint32_t bytes = (uint32_t)((nsb * BS + 15) & ~15);
    if (lane == 0) mbar_arrive_expect_tx(&full[s], (uint32_t)nr * bytes);
    __syncwarp();
    if (lane < nr)
      bulk_g2s(stages + (size_t)s * stage_bytes + lane * p.pitch, p.w + (row0 + lane) * p.row_stride + (int64_t)sb0 * BS,
               bytes, &full[s]);
  };

  int issued = 0;                               // units issued so far (tracked by warp 0 of the group)
  if (gw == 0) {
    if (lane == 0) {
      for (int s = 0; s < nst; s++) mbar_init(&full[s], 1);
      fence_mbar_init();
    }
    __syncwarp();
    for (; issued < nunit && issued < nst; issued++) issue(issued);
  }
  pdl_launch_dependents();
  __syncthreads();                              // barriers initialised before anyone waits on them
  pdl_wait();                                   // the activation comes from the previous kernel

  SAct sa{};
  GAct ga{};
  if constexpr (!TOK) {
    uint8_t *sxq = smem + p.x_off;
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
    __syncthreads();
    sa.xq = smem_u32(sxq); sa.xd = smem_u32(sxd); sa.xs = smem_u32(sxs); sa.xs16 = sxs16 ? smem_u32(sxs16) : 0u;
#pragma unroll
    for (int i = 0; i < 8; i++) sa.sel[i] = g == i ? 1u : 0u;
  } else {
    ga.xq = p.xq; ga.xd = p.xd; ga.xs = p.xs; ga.k = p.k; ga.ntok = p.ntok;
  }

  const uint32_t sbase = smem_u32(stages);
  // One thread per output (row, token) of the group's current tile adds the chunk's super-block
  // sums in super-block order: lanes of the group's warp 0 (and 1..3 for 8 tokens).
  const int gtid = threadIdx.x - grp * GT;
  const bool adder = gtid < kTile * NTP;
  double tot = 0.0;
  bool aborted = false;
  for (int u = 0; u < nunit; u++) {
    const int s = u % nst, tile = (u / p.nchunk) * NG + grp, c = u % p.nchunk;
    // after one give-up the warp waits no more: it only passes the barriers until all stop together
    const bool ok = !aborted && mbar_wait_warp(&full[s], (uint32_t)(u / nst) & 1u, lane);
    const int sb0 = c * kChunk, nsb = min(kChunk, p.nb - sb0);
    double *pu = part + (size_t)(u & 1) * kSlots * kTile * NTP;
    if (ok) {
      const uint32_t st = sbase + (uint32_t)(s * stage_bytes);
      if constexpr (!TOK) {
        // warp w of the group: super-blocks w and w + 8 (Q6_K: super-block w, both halves)
#pragma unroll 1
        for (int i = 0; i < 2; i++) {
          const int j = FMT == T_Q6_K ? gw : gw + 8 * i, h = FMT == T_Q6_K ? i : 0;
          const int slot = FMT == T_Q6_K ? gw + 8 * i : j;
          if (j < nsb) {
            double S0, S1;
            if constexpr (FMT == T_Q6_K) sb_q6_one(st, p.pitch, nsb, j, h, g, t, sa, sb0 + j, S0, S1);
            else sb_k45_one<FMT == T_Q5_K>(st + (uint32_t)(j * BS), p.pitch, g, t, sa, sb0 + j, S0, S1);
            if (t == 0) { pu[slot * kTile + g] = S0; pu[slot * kTile + g + 8] = S1; }
          }
        }
      } else {
#pragma unroll
        for (int jj = 0; jj < kChunk / kGroupWarps; jj++) {
          const int j = gw + kGroupWarps * jj;
          if (j >= nsb) break;
          if constexpr (FMT == T_Q6_K) {
            double Sh[4][2];
            sb_q6_tok(st, p.pitch, nsb, j, g, t, ga, sb0 + j, Sh);
#pragma unroll
            for (int e = 0; e < 4; e++)
#pragma unroll
              for (int h = 0; h < 2; h++)
                pu[((j + 8 * h) * kTile + g + 8 * (e >> 1)) * NTP + 2 * t + (e & 1)] = Sh[e][h];
          } else {
            double S[4];
            sb_k45_tok<FMT == T_Q5_K>(st + (uint32_t)(j * BS), p.pitch, g, t, ga, sb0 + j, S);
#pragma unroll
            for (int e = 0; e < 4; e++) pu[(j * kTile + g + 8 * (e >> 1)) * NTP + 2 * t + (e & 1)] = S[e];
          }
        }
      }
    }
    // every warp of the group is done with stage s and has published its sums: one group barrier,
    // which also tells every warp of the group whether any of them gave up waiting
    if (named_sync_or(1 + grp, GT, aborted || !ok)) { aborted = true; break; }
    if (u + nst < nunit && gw == 0) {
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
          v[j] = FMT == T_Q6_K ? __dadd_rn(pu[j * kTile * NTP + gtid], pu[(j + 8) * kTile * NTP + gtid]) : pu[j * kTile * NTP + gtid];
#pragma unroll
      for (int j = 0; j < NJ; j++)
        if (j < nsb) tot = __dadd_rn(tot, v[j]);
      if (c == p.nchunk - 1) {
        const int row = gtid / NTP, tok = gtid % NTP;
        const int64_t r = r0 + (int64_t)tile * kTile + row;
        float out = __double2float_rn(tot);
        if (p.swiglu) {
          // rows r (gate) and r + 1 (up) are the adders gtid and gtid + NTP, in the same warp:
          // silu in double, the product rounded to f32 (src/compute/worker.js:426, ref-kernels.js:322)
          const float up = __shfl_xor_sync(TOK ? 0xffffffffu : 0x0000ffffu, out, NTP);
          if ((row & 1) == 0 && tok < p.ntok && r < r1) {
            const double z = out;
            const double sl = __ddiv_rn(z, __dadd_rn(1.0, exp(-z)));
            p.y[(int64_t)tok * p.y_stride + r / 2] = __double2float_rn(__dmul_rn(sl, (double)up));
          }
        } else if (tok < p.ntok && r < r1) {
          const int64_t o = (int64_t)tok * p.y_stride + r;
          if (p.y_add) out = __fadd_rn(p.y_add[o], out);
          p.y[o] = out;
        }
        tot = 0.0;
      }
    }
  }
  if (aborted) {
    if (lane == 0) atomicOr(p.status, ST_FULL_TIMEOUT);
    if (gw == 0 && lane == 0) {
      // copies still in flight must land before the CTA's shared memory is released
      const uint64_t drain_deadline = globaltimer_ns() + WAIT_DEADLINE_NS;
      for (int v = issued - nst > 0 ? issued - nst : 0; v < issued; v++)
        if (!mbar_wait_bounded(&full[v % nst], (uint32_t)(v / nst) & 1u, drain_deadline))
          atomicOr(p.status, ST_DRAIN_TIMEOUT);
    }
  }
}

struct KqPlan {
  int nchunk, pitch, nst, grid, smem, x_off, part_off, bar_off;
};

bool plan_kq(const DevMatrix &m, int num_sms, bool tok, KqPlan *p, const char **why) {
  const int bs = m.type == T_Q4_K ? 144 : m.type == T_Q5_K ? 176 : 210;
  const int64_t nb = m.cols / 256;
  if (nb < 1 || m.cols % 256) { *why = "k-quant rows must be a whole number of 256-value super-blocks"; return false; }
  if (nb > (1 << 24)) { *why = "k-quant rows too long"; return false; }
  const int kChunk = chunk_sb_of(m.type);
  p->nchunk = (int)((nb + kChunk - 1) / kChunk);
  const int chunk = (int)(((nb < kChunk ? nb : kChunk) * bs + 15) / 16 * 16);
  int pitch = chunk;
  while ((pitch / 4) % 8 != 4) pitch += 16;    // rows g = 0..7 of a tile land on distinct bank groups
  p->pitch = pitch;
  const int64_t grid = m.rows < num_sms ? m.rows : num_sms;
  p->grid = (int)(grid < 1 ? 1 : grid);
  const int64_t rows_cta = (m.rows + p->grid - 1) / p->grid;
  const int ng = tok ? 1 : 2;
  const int64_t units = ((rows_cta + kTile - 1) / kTile + ng - 1) / ng * p->nchunk;   // per group
  const int64_t x_bytes = tok ? 0 : (m.cols + 12 * (m.cols / 32) + (m.type == T_Q6_K ? 4 * (m.cols / 16) : 0) + 127) / 128 * 128;
  const int64_t stage = (int64_t)kTile * pitch;
  const int64_t part_bytes = (int64_t)ng * 2 * 16 * kTile * (tok ? kMaxTok : 1) * 8;
  const int64_t avail = kSmemBudget - x_bytes - part_bytes - 8 * ng * kMaxStages;
  int64_t nst = avail / (stage * ng);
  if (nst > kMaxStages) nst = kMaxStages;
  if (nst > units) nst = units;
  if (nst < 1) { *why = "k-quant rows too long for the shared-memory stages"; return false; }
  p->nst = (int)nst;
  p->x_off = (int)(ng * nst * stage);
  p->part_off = (int)(p->x_off + x_bytes);
  p->bar_off = (int)(p->part_off + part_bytes);
  p->smem = p->bar_off + 8 * ng * p->nst;
  return true;
}

template <int FMT, bool TOK>
cudaError_t launch_kq_t(const KqArgs &a, const KqPlan &pl, cudaStream_t s, bool pdl) {
  auto kern = kq_gemv_kernel<FMT, TOK>;
  static bool granted[64] = {false};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!granted[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBudget + 1024);
    if (e != cudaSuccess) return e;
    granted[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(groups_of<TOK>() * kGroupWarps * 32);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, a);
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
  if (fz.norm_w && (act.xq || !act.x || ntok != 1)) { *why = "the fused RMSNorm takes one f32 token"; return cudaErrorInvalidValue; }
  if (fz.swiglu && (m.rows % 2 || y_add)) { *why = "the SwiGLU epilogue takes (gate, up) row pairs and no residual"; return cudaErrorInvalidValue; }
  KqPlan pl1, plt;
  if (!plan_kq(m, num_sms, false, &pl1, why)) return cudaErrorInvalidValue;
  if (ntok > 1 && !plan_kq(m, num_sms, true, &plt, why)) return cudaErrorInvalidValue;
  if (act.xq == nullptr && (ntok != 1 || act.x == nullptr)) {
    *why = "the in-kernel activation quantization takes one token";
    return cudaErrorInvalidValue;
  }
  for (int t0 = 0; t0 < ntok; t0 += kMaxTok) {
    const int nt = ntok - t0 < kMaxTok ? ntok - t0 : kMaxTok;
    const KqPlan &pl = nt == 1 ? pl1 : plt;
    KqArgs a{};
    a.w = m.data; a.row_stride = m.row_stride; a.rows = m.rows; a.nb = (int)(m.cols / 256);
    a.nchunk = pl.nchunk; a.pitch = pl.pitch; a.nst = pl.nst;
    a.ntok = nt;
    a.k = m.cols;
    a.xq = act.xq ? act.xq + (int64_t)t0 * m.cols : nullptr;
    a.xd = act.xd ? act.xd + (int64_t)t0 * (m.cols / 32) : nullptr;
    a.xs = act.xs ? act.xs + (int64_t)t0 * (m.cols / 32) : nullptr;
    a.x = act.x ? act.x + (int64_t)t0 * m.cols : nullptr;
    a.y = y + (int64_t)t0 * y_stride;
    a.y_add = y_add ? y_add + (int64_t)t0 * y_stride : nullptr;
    a.y_stride = y_stride;
    a.norm_w = fz.norm_w; a.norm_eps = fz.eps; a.swiglu = fz.swiglu ? 1 : 0;
    a.status = status;
    a.x_off = pl.x_off; a.part_off = pl.part_off; a.bar_off = pl.bar_off;
    cudaError_t e;
    const bool tok = nt > 1;
    switch (m.type) {
      case T_Q4_K: e = tok ? launch_kq_t<T_Q4_K, true>(a, pl, s, pdl) : launch_kq_t<T_Q4_K, false>(a, pl, s, pdl); break;
      case T_Q5_K: e = tok ? launch_kq_t<T_Q5_K, true>(a, pl, s, pdl) : launch_kq_t<T_Q5_K, false>(a, pl, s, pdl); break;
      default: e = tok ? launch_kq_t<T_Q6_K, true>(a, pl, s, pdl) : launch_kq_t<T_Q6_K, false>(a, pl, s, pdl); break;
    }
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace zllm
