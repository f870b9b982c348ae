// Prefill / batched GEMM on the 5th-generation tensor cores (tcgen05, accumulators in TMEM).
//
// Replaces the reference's batched k-quant kernels mm_q4_k / mm_q5_k / mm_q6_k
// (src/compute/wasm/kquant-kernels.js:337-504, dispatched by src/compute/worker.js:251-270) for
// passes of 64 or more tokens.  y[t][r] = (y_add) + sum_k W[r][k] * X[t][k], where W is the k-quant
// matrix and X the quantized activation (quantizeAct, ref-kernels.js:44-62).  Expanding the
// reference's block terms, xd * (d*sc*lo - dmin*mn*xs) summed over a row's sub-blocks is exactly
// sum_k (d*sc*q_k - dmin*mn) * (xd * xq_k): the dequantized weight (quant.js:150, :194-197) times the
// dequantized activation, one dense contraction:
//   * A (weights, M = 128 rows per CTA): 8 dequantizing warps, one per 16-row unit of the k-quant
//     layout (kq_layout.h), load their unit's super-block straight into registers (one super-block
//     ahead) and write each 64-value K chunk into shared memory as two f16 tiles, hi = f16(w) and
//     lo = f16(w - hi) (w formed in f32), in the canonical K-major 128-byte-swizzled layout;
//   * B (activations, N = 128 tokens per CTA): prepared once per launch by gemm_bfill_kernel as the
//     same hi / lo pair of xd * xq * 2^-e_t (e_t a per-token power of two that keeps the values in
//     f16's range), pre-tiled and pre-swizzled; 4 producer warps stream each stage's 32 KB with
//     16-byte cp.async (one warp alone issues too slowly to keep up);
//   * three tcgen05.mma kind::f16 per 16-value K slice (hi.hi + hi.lo + lo.hi; lo.lo is below f32's
//     own rounding) into one f32 accumulator in TMEM, issued by one thread, stages released by
//     tcgen05.commit; the epilogue warps read TMEM with tcgen05.ld, scale each token's column by
//     2^e_t (and the matrix's range scale) and write y (plus the residual, or SwiGLU of row pairs).
// Numerics: the hi / lo pairs carry about 22 bits of every weight and activation value, so the
// products summed in f32 agree with the oracle to ~1e-6 of the largest output (the one-token path's
// block terms are exact doubles; the two differ only in rounding).  NaN or infinite block scales
// are rejected on the host and take the exact kernel.
//
// Roles (416 threads): warps 0..3 stream the activation tiles, warp 4 owns TMEM and its lane 0
// issues the MMAs, warps 5..12 dequantize and then run the epilogue.  Every wait is bounded (2 s);
// a give-up sets the status word and an abort flag that ends every loop, the producers let their
// copies land, the MMA thread waits for its MMAs, TMEM is freed.
#include "common.cuh"
#include "internal.h"
#include "kq_layout.h"
#include "tc05.cuh"

namespace zllm {

namespace {

constexpr int GM = 128;            // rows per CTA (MMA M)
constexpr int GN = 128;            // tokens per CTA (MMA N)
constexpr int GK = 64;             // K per stage: one 128-byte swizzle row of f16
constexpr int kAStages = 2;        // dequantized weight tiles (hi, lo): filled from registers, no latency to hide
constexpr int kBStages = 5;        // activation tiles (hi, lo): ~2 us of loaded memory latency to cover
constexpr int kProdWarps = 4;
constexpr int kMmaWarp = kProdWarps;
constexpr int kDqWarp0 = kProdWarps + 1;
constexpr int kDqWarps = 8;
constexpr int kThreads = (kDqWarp0 + kDqWarps) * 32;
constexpr int kTileBytes = GM * GK * 2;   // one 128 x 64 f16 tile: 16 KB (B tiles are the same with GN = GM)
constexpr int kPairBytes = 2 * kTileBytes;   // a hi tile and its lo tile
constexpr int kQ6HOff = 2048, kQ6SOff = 3072, kQ6DOff = 3328;   // Q6_K unit regions (kq_layout.h)
static_assert(GM == GN, "A and B tiles share one size");

__device__ __forceinline__ uint32_t idesc_n(int n) { return idesc_f16(GM, n); }

// ---------------------------------------------------------------------------- dequantization
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t *>(&h);
}
// (hi, lo) f16 pairs of two f32 values: hi = f16(v), lo = f16(v - hi)
__device__ __forceinline__ void split2(float a, float b, uint32_t &hi, uint32_t &lo) {
  const __half2 h = __floats2half2_rn(a, b);
  const float2 f = __half22float2(h);
  hi = *reinterpret_cast<const uint32_t *>(&h);
  lo = pack_h2(a - f.x, b - f.y);
}
// exact int -> f32 for 0 <= v < 2^23 without the conversion pipe
__device__ __forceinline__ float small_f(uint32_t v) { return __int_as_float(0x4B000000 | v) - 8388608.f; }
__device__ __forceinline__ uint32_t word4(const uint4 &v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }

// The 24-bit scale/min field of chunk c from header words 1..3 of a Q4_K / Q5_K block.
__device__ __forceinline__ uint32_t k45_field(const uint4 &h, int c) {
  const uint32_t lo = c < 2 ? h.y : (c == 2 ? h.z : h.w);
  const uint32_t hi = c == 0 ? h.y : (c == 1 ? h.z : (c == 2 ? h.w : 0u));
  return __funnelshift_r(lo, hi, (24 * c) & 31);
}


// A dequantizing thread owns row m of its warp's unit (16 rows) and half of the row's lane pieces
// (t = 2tp, 2tp + 1): 32 of each 64-value K chunk, which land as four 16-byte runs of each swizzled
// A tile.  Raw<FMT> is its share of one super-block of the unit, loaded from HBM into registers a
// super-block ahead; Dq<FMT> holds the current one with its block scales in f32; emit<c> writes chunk
// c's hi / lo runs.  The value is the reference's dequantized weight (quant.js:150:
// d*sc*q - dmin*mn; :194-197: d*scale*q) in f32, times the matrix's power-of-two range scale.
template <int FMT> struct Raw {      // Q4_K, Q5_K
  uint4 q[2][2], e, hd;
  __device__ __forceinline__ void load(const uint8_t *u, int m, int tp) {
    const int r = m >> 3, g = m & 7;
#pragma unroll
    for (int cp = 0; cp < 2; cp++)
#pragma unroll
      for (int tt = 0; tt < 2; tt++) q[cp][tt] = ldg128_now(u + ((2 * r + cp) * 32 + 4 * g + 2 * tp + tt) * 16);
    if constexpr (FMT == T_Q5_K) e = ldg128_now(u + 2048 + 32 * m + 16 * tp);
    hd = ldg128_now(u + (FMT == T_Q4_K ? 2048 : 2560) + 16 * m);
  }
};
template <> struct Raw<T_Q6_K> {
  uint4 ql[2][2], qh[2], sc;
  uint32_t d;
  __device__ __forceinline__ void load(const uint8_t *u, int m, int tp) {
    const int r = m >> 3, g = m & 7;
#pragma unroll
    for (int h = 0; h < 2; h++)
#pragma unroll
      for (int tt = 0; tt < 2; tt++) ql[h][tt] = ldg128_now(u + ((2 * r + h) * 32 + 4 * g + 2 * tp + tt) * 16);
    qh[0] = ldg128_now(u + kQ6HOff + 64 * m + 32 * tp);
    qh[1] = ldg128_now(u + kQ6HOff + 64 * m + 32 * tp + 16);
    sc = ldg128_now(u + kQ6SOff + 16 * m);
    d = __ldg(reinterpret_cast<const unsigned short *>(u + kQ6DOff + 2 * m));
  }
};

template <int FMT> struct Dq {       // Q4_K, Q5_K
  uint4 q[2][2], e;
  float ds[4][2], ndm[4][2];         // per chunk, per nibble (sub-block 2c + nib)
  __device__ __forceinline__ void set(const Raw<FMT> &R, float wsc) {
#pragma unroll
    for (int i = 0; i < 2; i++)
#pragma unroll
      for (int j = 0; j < 2; j++) q[i][j] = R.q[i][j];
    e = R.e;
    const float d = h2f(R.hd.x & 0xffffu) * wsc, dmin = h2f(R.hd.x >> 16) * wsc;
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const uint32_t F = k45_field(R.hd, c);
      ds[c][0] = d * small_f(F & 63u);
      ds[c][1] = d * small_f((F >> 6) & 63u);
      ndm[c][0] = -(dmin * small_f((F >> 12) & 63u));
      ndm[c][1] = -(dmin * small_f((F >> 18) & 63u));
    }
  }
  // chunk c: hi[j] / lo[j] = positions 16j + 8tp .. + 7, j = 2 nib + h
  template <int c>
  __device__ __forceinline__ void emit(uint4 (&hi)[4], uint4 (&lo)[4]) const {
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int nib = j >> 1, h = j & 1;
      uint32_t oh[4], ol[4];
#pragma unroll
      for (int tt = 0; tt < 2; tt++) {
        const uint32_t w = word4(q[c >> 1][tt], 2 * (c & 1) + h);
        uint32_t eb = 0;
        if constexpr (FMT == T_Q5_K) eb = word4(e, 2 * tt + h);
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
          uint32_t qv = (w >> (8 * i + 4 * nib)) & 15u;
          if constexpr (FMT == T_Q5_K) qv |= ((eb >> (8 * i + 2 * c + nib)) & 1u) << 4;
          v[i] = __fmaf_rn(ds[c][nib], small_f(qv), ndm[c][nib]);
        }
        split2(v[0], v[1], oh[2 * tt], ol[2 * tt]);
        split2(v[2], v[3], oh[2 * tt + 1], ol[2 * tt + 1]);
      }
      hi[j] = make_uint4(oh[0], oh[1], oh[2], oh[3]);
      lo[j] = make_uint4(ol[0], ol[1], ol[2], ol[3]);
    }
  }
};
template <> struct Dq<T_Q6_K> {
  uint4 ql[2][2], qh[2];
  float ds[16];                      // d * scale of group G
  __device__ __forceinline__ void set(const Raw<T_Q6_K> &R, float wsc) {
#pragma unroll
    for (int i = 0; i < 2; i++) {
      qh[i] = R.qh[i];
#pragma unroll
      for (int j = 0; j < 2; j++) ql[i][j] = R.ql[i][j];
    }
    const float d = h2f(R.d) * wsc;
#pragma unroll
    for (int G = 0; G < 16; G++) {
      const int o = G < 8 ? 4 * (G >> 1) + (G & 1) : 4 * ((G - 8) >> 1) + 2 + (G & 1);
      ds[G] = d * (float)(int)(int8_t)((word4(R.sc, o >> 2) >> (8 * (o & 3))) & 0xffu);
    }
  }
  // chunk c: hi[j] / lo[j] = positions 16j + 8tp .. + 7, j = 2p + u
  template <int c>
  __device__ __forceinline__ void emit(uint4 (&hi)[4], uint4 (&lo)[4]) const {
    constexpr int half = c >> 1, hb = c & 1;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int p = j >> 1, uu = j & 1, k = 2 * hb + p, G = 8 * half + 2 * k + uu;
      uint32_t oh[4], ol[4];
#pragma unroll
      for (int tt = 0; tt < 2; tt++) {
        const uint32_t w = word4(ql[half][tt], 2 * uu + p), eh = word4(qh[tt], 2 * half + uu);
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const uint32_t lo4 = (w >> (8 * i + 4 * hb)) & 15u, h2 = (eh >> (8 * i + 2 * k)) & 3u;
          v[i] = ds[G] * (small_f(lo4 | (h2 << 4)) - 32.f);
        }
        split2(v[0], v[1], oh[2 * tt], ol[2 * tt]);
        split2(v[2], v[3], oh[2 * tt + 1], ol[2 * tt + 1]);
      }
      hi[j] = make_uint4(oh[0], oh[1], oh[2], oh[3]);
      lo[j] = make_uint4(ol[0], ol[1], ol[2], ol[3]);
    }
  }
};

// FMT: a k-quant type (units dequantized in the kernel, three MMAs per slice: hi*hi, hi*lo, lo*hi);
// 0 -- A already tiled f16, one MMA (A * B hi); T_F16 (1) -- A already tiled f16 against an f32
// activation split into B hi / lo, two MMAs.
template <int FMT> constexpr bool a_tiled() { return FMT == 0 || FMT == T_F16; }
// Ring geometry: dequantized A tiles (hi, lo) come from registers and need little depth; tiled A
// tiles (hi only) stream from HBM like B and get the same depth.
template <int FMT> constexpr int a_stages() { return a_tiled<FMT>() ? 4 : kAStages; }
template <int FMT> constexpr int b_stages() { return a_tiled<FMT>() ? 4 : kBStages; }
template <int FMT> constexpr int a_slot() { return a_tiled<FMT>() ? kTileBytes : kPairBytes; }
template <int FMT> constexpr size_t smem_bytes() {
  return 1024 + (size_t)a_stages<FMT>() * a_slot<FMT>() + (size_t)b_stages<FMT>() * kPairBytes +
         (2 * a_stages<FMT>() + 2 * b_stages<FMT>() + 1) * 8 + 16;
}

struct GemmArgs {
  const uint8_t *w;       // k-quant units of the matrix; or (a_tiled) A tiles [m_tile][K/64][128][64] f16
  const uint8_t *b;       // activation tiles [n_tile][K/64][hi, lo][128][64] f16, 128-byte swizzled
  const float *bscale;    // [n_tiles * 128] per-token multiplier of the accumulators
  float wscale, wscale_inv;   // power of two applied to the dequantized weights, and its inverse
  float *y;
  const float *y_add;
  int64_t y_stride;
  int64_t rows;
  int ntok, nb, kc;       // tokens, super-blocks per row, 64-value chunks per row
  int swiglu;             // rows are (gate, up) pairs: y[t][r / 2] = silu(gate) * up
  unsigned *status;
  // exact-A kernel only: bytes of one activation tile (128 x 64 f16, or fewer rows for a single
  // short token tile), and split-K: nsplit CTAs per output tile (one cluster), sbps super-blocks each
  int btile, nsplit, sbps;
};

// A CTA computes a 128-row x 128-token tile; its MMAs use N = the tile's tokens rounded up to 16,
// and the producers copy only those rows of the activation tiles.
template <int FMT>
__global__ void __launch_bounds__(kThreads, 1) gemm_kq_kernel(const GemmArgs p) {
  constexpr int US = a_tiled<FMT>() ? 0 : FMT == T_Q4_K ? 2304 : FMT == T_Q5_K ? 2816 : 3360;
  constexpr int AS = a_stages<FMT>(), BS = b_stages<FMT>(), ASLOT = a_slot<FMT>();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);   // swizzle atoms need 1024
  uint8_t *a_ring = smem, *b_ring = smem + AS * ASLOT;
  uint64_t *bars = reinterpret_cast<uint64_t *>(b_ring + BS * kPairBytes);
  uint64_t *full_a = bars, *empty_a = bars + AS, *full_b = bars + 2 * AS, *empty_b = full_b + BS;
  uint64_t *acc_full = empty_b + BS;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_full + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  auto a_hi = [&](int s) { return a_ring + (size_t)s * ASLOT; };
  auto a_lo = [&](int s) { return a_ring + (size_t)s * ASLOT + kTileBytes; };   // k-quant A only
  auto b_hi = [&](int s) { return b_ring + (size_t)s * kPairBytes; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tile = blockIdx.x, n_tile = blockIdx.y;
  const int nks = p.kc;                                 // K steps of 64
  const int64_t tiles16 = (p.rows + 15) / 16;
  const int tile0 = m_tile * 8;
  const int ntile = (int)min((int64_t)8, tiles16 - tile0);   // 16-row units present in this M tile
  const Ctl ctl{abort_flag, p.status};
  // each M tile walks K from its own starting super-block, so the CTAs of one token tile do not all
  // ask for the same activation tile at once (the per-output order depends on the tile only)
  const int koff_sb = p.nb > 0 ? (m_tile * 7) % p.nb : 0;
  const int koff = a_tiled<FMT>() ? (m_tile * 28) % nks : 4 * koff_sb;
  const int ntok_tile = min(GN, p.ntok - n_tile * GN);
  const int nmma = (ntok_tile + 15) / 16 * 16;          // MMA N: the tile's tokens, rounded up to 16

  if (threadIdx.x == 0) {
    for (int s = 0; s < AS; s++) {
      mbar_init(&full_a[s], a_tiled<FMT>() ? kProdWarps * 32 : kDqWarps);
      mbar_init(&empty_a[s], 1);
    }
    for (int s = 0; s < BS; s++) {
      mbar_init(&full_b[s], kProdWarps * 32);
      mbar_init(&empty_b[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) tmem_alloc(tmem_slot, GN);     // GN f32 columns x 128 lanes
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < kProdWarps) {
    // ---- activation producers: the 128 producer threads copy the stage's first nmma rows of B hi
    // and lo (and, a_tiled, a quarter of the A tile per warp) with 16-byte cp.async; the stage's
    // barrier counts every lane's completion
    const int pw = warp;
    const int bchunks = nmma * 128 / 16;                // 16-byte chunks of one part's rows [0, nmma)
    for (int k = 0; k < nks; k++) {
      const int s = k % BS;
      if (k >= BS && !waitw(&empty_b[s], (uint32_t)(k / BS - 1) & 1u, ctl, ST_EMPTY_TIMEOUT, lane)) break;
      const int kd = (k + koff) % nks;
      const uint8_t *src = p.b + ((int64_t)n_tile * nks + kd) * 2 * kTileBytes;
      const uint32_t dst = smem_u32(b_hi(s));
#pragma unroll
      for (int part = 0; part < 2; part++) {          // bchunks is a multiple of the 128 producer threads
#pragma unroll 4
        for (int q = threadIdx.x; q < bchunks; q += kProdWarps * 32)
          cp_async16(dst + part * kTileBytes + q * 16, src + part * kTileBytes + q * 16);
      }
      cp_async_arrive(&full_b[s]);
      if constexpr (a_tiled<FMT>()) {
        // the A tile of the same K step goes into its own ring (stage k % AS, after that stage's
        // previous MMAs have released it)
        const int sa = k % AS;
        if (k >= AS && !waitw(&empty_a[sa], (uint32_t)(k / AS - 1) & 1u, ctl, ST_EMPTY_TIMEOUT, lane)) break;
        constexpr int QA = kTileBytes / kProdWarps;
        const uint8_t *asrc = p.w + ((int64_t)m_tile * nks + kd) * kTileBytes + pw * QA;
        const uint32_t adst = smem_u32(a_hi(sa)) + pw * QA;
#pragma unroll 4
        for (int q = lane; q < QA / 16; q += 32) cp_async16(adst + q * 16, asrc + q * 16);
        cp_async_arrive(&full_a[sa]);
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");   // this warp's copies land before it leaves
  } else if (warp == kMmaWarp) {
    // ---- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_n(nmma);
      int issued = 0;
      for (int k = 0; k < nks; k++) {
        const int sb = k % BS, sa = k % AS;
        if (!wait1(&full_b[sb], (uint32_t)(k / BS) & 1u, ctl, ST_FULL_TIMEOUT) ||
            !wait1(&full_a[sa], (uint32_t)(k / AS) & 1u, ctl, ST_FULL_TIMEOUT))
          break;
        fence_async_smem();                             // the generic-proxy stores / cp.async data -> the MMA's reads
        tc_fence_after();
        const uint32_t ah = smem_u32(a_hi(sa)), al = ah + kTileBytes, bh = smem_u32(b_hi(sb)), bl = bh + kTileBytes;
#pragma unroll
        for (int kk = 0; kk < GK / 16; kk++) {
          const uint32_t o = kk * 32;
          mma_f16(tmem, sw128_desc(ah + o), sw128_desc(bh + o), idesc, (k | kk) != 0);
          if constexpr (FMT != 0) mma_f16(tmem, sw128_desc(ah + o), sw128_desc(bl + o), idesc, 1u);
          if constexpr (!a_tiled<FMT>()) mma_f16(tmem, sw128_desc(al + o), sw128_desc(bh + o), idesc, 1u);
        }
        mma_commit(&empty_a[sa]);                       // the stages are free once these MMAs finish
        mma_commit(&empty_b[sb]);
        issued++;
      }
      mma_commit(acc_full);                             // every MMA issued has finished
      if (issued < nks) *abort_flag = 1;
      // TMEM is freed below only after the MMAs have finished, also on the abort path
      if (!mbar_wait_bounded(acc_full, 0u, globaltimer_ns() + WAIT_DEADLINE_NS)) atomicOr(p.status, ST_DRAIN_TIMEOUT);
    }
  } else {
    // ---- dequantizing warps (FMT != 0), then the epilogue
    const int dw = warp - kDqWarp0;
    if constexpr (!a_tiled<FMT>()) {
      // warp dw owns unit dw of the tile (rows 16 dw ..): lane -> row m = (lane & 7) + 8 (lane >> 4)
      // and half tp = (lane >> 3) & 1, so each 8-lane quarter stores 8 rows' runs of one column of
      // 16-byte chunks -- 8 distinct swizzled chunks, no bank conflict
      const int m = (lane & 7) + 8 * (lane >> 4), tp = (lane >> 3) & 1, row = 16 * dw + m;
      const bool present = dw < ntile;
      const uint8_t *ubase = p.w + (int64_t)(tile0 + (present ? dw : 0)) * p.nb * US;
      Raw<FMT> nxt;
      Dq<FMT> cur;
      if (present) nxt.load(ubase + (int64_t)(koff_sb % p.nb) * US, m, tp);
      bool live = true;
      for (int k = 0; k < nks && live; k++) {
        const int s = k % AS, sbi = k >> 2, c = k & 3;
        if (c == 0 && present) {
          cur.set(nxt, p.wscale);
          if (sbi + 1 < p.nb) nxt.load(ubase + (int64_t)((sbi + 1 + koff_sb) % p.nb) * US, m, tp);
        }
        if (k >= AS) live = waitw(&empty_a[s], (uint32_t)(k / AS - 1) & 1u, ctl, ST_EMPTY_TIMEOUT, lane);
        if (!live) break;
        uint4 hi[4], lo[4];
        if (present) {
          // chunk index as a template argument: every register index is a constant
          switch (c) {
            case 0: cur.template emit<0>(hi, lo); break;
            case 1: cur.template emit<1>(hi, lo); break;
            case 2: cur.template emit<2>(hi, lo); break;
            default: cur.template emit<3>(hi, lo); break;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 4; j++) hi[j] = lo[j] = make_uint4(0, 0, 0, 0);
        }
        uint8_t *ah = a_hi(s), *al = a_lo(s);
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const uint32_t o = sw128_off(row, 16 * j + 8 * tp);
          *reinterpret_cast<uint4 *>(ah + o) = hi[j];
          *reinterpret_cast<uint4 *>(al + o) = lo[j];
        }
        fence_async_smem();                             // generic-proxy writes -> the MMA's reads
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_a[s]);
      }
    }
    // epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31; two warps per lane quarter split the columns
    bool ok = waitw(acc_full, 0u, ctl, ST_FULL_TIMEOUT, lane);
    ok = __shfl_sync(0xffffffffu, ok && !*abort_flag, 0);   // warp-uniform: tcgen05.ld is warp-wide
    tc_fence_after();
    if (ok) {
      const int quarter = warp & 3, half = dw >> 2;
      const int64_t row = (int64_t)m_tile * GM + quarter * 32 + lane;
#pragma unroll 1
      for (int cc = 0; cc < GN / 64; cc++) {
        const int col0 = half * (GN / 2) + cc * 32;
        if (col0 >= ntok_tile) break;                  // uniform: no token in these columns
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)col0, v);
        if (p.swiglu) {
          // rows r (gate) and r + 1 (up) sit in adjacent lanes: silu in double, the product rounded
          // to f32 (src/compute/worker.js:426, ref-kernels.js:322), written once per pair
#pragma unroll
          for (int i = 0; i < 32; i++) {
            const int tok = n_tile * GN + col0 + i;
            if (tok < p.ntok) {                     // uniform across the warp
              const float o = v[i] * (p.bscale[tok] * p.wscale_inv);
              const float up = __shfl_xor_sync(0xffffffffu, o, 1);
              if (row < p.rows && (row & 1) == 0) {
                const double z = o;
                const double sl = __ddiv_rn(z, __dadd_rn(1.0, exp(-z)));
                p.y[(int64_t)tok * p.y_stride + row / 2] = __double2float_rn(__dmul_rn(sl, (double)up));
              }
            }
          }
        } else if (row < p.rows) {
#pragma unroll
          for (int i = 0; i < 32; i++) {
            const int tok = n_tile * GN + col0 + i;
            if (tok < p.ntok) {
              float o = v[i] * (p.bscale[tok] * p.wscale_inv);
              const int64_t at = (int64_t)tok * p.y_stride + row;
              if (p.y_add) o = __fadd_rn(p.y_add[at], o);
              p.y[at] = o;
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, GN);
  }
}

// ---------------------------------------------------------------------------- activation tiles
// Per token t: the power of two 2^e_t with every |xd * xq| * 2^-e_t below 2^15 (f16 keeps 11 bits
// down to 2^-14 of it); bscale[t] = 2^e_t multiplies the accumulators back.  Padding tokens get 1.
__global__ void gemm_bscale_kernel(const float *xd, int64_t nblk, int ntok, int npad, float *bscale) {
  const int warp = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  if (warp >= npad) return;
  float amax = 0.f;
  if (warp < ntok)
    for (int64_t b = lane; b < nblk; b += 32) amax = fmaxf(amax, fabsf(xd[(int64_t)warp * nblk + b]));
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  amax *= 127.f;
  float s = 1.f;
  if (amax > 0.f && amax < 3.0e38f) s = exp2f((float)(ilogbf(amax) - 14));
  if (lane == 0) bscale[warp] = s;
}
// Tiles [n_tile][K/64][hi, lo][128][64] f16: thread per 8 consecutive values of one token.
__global__ void gemm_bfill_kernel(const int8_t *xq, const float *xd, int64_t k, int ntok, int npad, const float *bscale,
                                  uint8_t *bt) {
  const int64_t groups = k / 8, total = (int64_t)npad * groups;
  const int kc = (int)(k / 64);
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int n = (int)(e / groups);
    const int64_t g8 = e % groups, k0 = g8 * 8;
    uint32_t h[4] = {0, 0, 0, 0}, l[4] = {0, 0, 0, 0};
    if (n < ntok) {
      const float sc = xd[(int64_t)n * (k / 32) + k0 / 32] / bscale[n];   // exact: bscale is a power of two
      const uint2 q = *reinterpret_cast<const uint2 *>(xq + (int64_t)n * k + k0);
      const int8_t *qb = reinterpret_cast<const int8_t *>(&q);
#pragma unroll
      for (int i = 0; i < 4; i++) split2(sc * (float)qb[2 * i], sc * (float)qb[2 * i + 1], h[i], l[i]);
    }
    const int nt = n / GN, nr = n % GN, c = (int)(k0 / 64), kk = (int)(k0 % 64);
    uint8_t *base = bt + ((int64_t)nt * kc + c) * 2 * kTileBytes + sw128_off(nr, kk);
    *reinterpret_cast<uint4 *>(base) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4 *>(base + kTileBytes) = make_uint4(l[0], l[1], l[2], l[3]);
  }
}
// f32 activations x [ntok][ldx] (the output head's normalized hidden state): per token the power of
// two with every |x| * 2^-e below 2^15, then tiles of hi = f16(x * 2^-e), lo = f16(x * 2^-e - hi).
__global__ void gemm_bscale_f32_kernel(const float *x, int64_t ldx, int64_t k, int ntok, int npad, float *bscale) {
  const int warp = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  if (warp >= npad) return;
  float amax = 0.f;
  if (warp < ntok)
    for (int64_t i = lane; i < k; i += 32) amax = fmaxf(amax, fabsf(x[(int64_t)warp * ldx + i]));
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  float s = 1.f;
  if (amax > 0.f && amax < 3.0e38f) s = exp2f((float)(ilogbf(amax) - 14));
  if (lane == 0) bscale[warp] = s;
}
__global__ void gemm_bfill_f32_kernel(const float *x, int64_t ldx, int64_t k, int ntok, int npad, const float *bscale,
                                      uint8_t *bt) {
  const int64_t groups = k / 8, total = (int64_t)npad * groups;
  const int kc = (int)(k / 64);
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int n = (int)(e / groups);
    const int64_t k0 = (e % groups) * 8;
    uint32_t h[4] = {0, 0, 0, 0}, l[4] = {0, 0, 0, 0};
    if (n < ntok) {
      const float inv = 1.f / bscale[n];                 // exact: a power of two
      const float4 *src = reinterpret_cast<const float4 *>(x + (int64_t)n * ldx + k0);
      const float4 a = src[0], b = src[1];
      split2(a.x * inv, a.y * inv, h[0], l[0]);
      split2(a.z * inv, a.w * inv, h[1], l[1]);
      split2(b.x * inv, b.y * inv, h[2], l[2]);
      split2(b.z * inv, b.w * inv, h[3], l[3]);
    }
    const int nt = n / GN, nr = n % GN, c = (int)(k0 / 64), kk = (int)(k0 % 64);
    uint8_t *base = bt + ((int64_t)nt * kc + c) * 2 * kTileBytes + sw128_off(nr, kk);
    *reinterpret_cast<uint4 *>(base) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4 *>(base + kTileBytes) = make_uint4(l[0], l[1], l[2], l[3]);
  }
}
// Tiles of a plain f16 matrix [rows][k] (row-major, lda elements between rows), rows past the end 0:
// `parts` 1 gives A tiles [m_tile][K/64][128][64]; 2 gives B tiles [n_tile][K/64][hi, lo][128][64]
// with lo = 0.
__global__ void gemm_tile_f16_kernel(const uint16_t *a, int64_t lda, int64_t rows, int64_t k, int64_t mpad, int parts,
                                     uint8_t *at) {
  const int64_t groups = k / 8, total = mpad * groups;
  const int kc = (int)(k / 64);
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = e / groups, k0 = (e % groups) * 8;
    const uint4 v = r < rows ? *reinterpret_cast<const uint4 *>(a + r * lda + k0) : make_uint4(0, 0, 0, 0);
    const int64_t mt = r / GM;
    uint8_t *base = at + (mt * kc + k0 / 64) * parts * kTileBytes + sw128_off((int)(r % GM), (int)(k0 % 64));
    *reinterpret_cast<uint4 *>(base) = v;
    if (parts == 2) *reinterpret_cast<uint4 *>(base + kTileBytes) = make_uint4(0, 0, 0, 0);
  }
}
__global__ void fill_f32_kernel(float *p, int64_t n, float v) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = v;
}

template <int FMT>
cudaError_t launch_t(const GemmArgs &a, dim3 grid, size_t smem, cudaStream_t s) {
  static bool granted[64] = {false};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!granted[dev]) {
    e = cudaFuncSetAttribute(gemm_kq_kernel<FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    granted[dev] = true;
  }
  gemm_kq_kernel<FMT><<<grid, kThreads, smem, s>>>(a);
  return cudaGetLastError();
}

static_assert(smem_bytes<T_Q4_K>() <= 227 * 1024 && smem_bytes<T_F16>() <= 227 * 1024, "shared memory");

// An upper bound of |dequantized value| over a k-quant matrix, as the bits of a non-negative f32
// (atomicMax on the bits orders them); a NaN or infinite scale makes it +inf.
template <int FMT>
__global__ void kq_bound_kernel(const uint8_t *w, int64_t nunits, unsigned *out) {
  constexpr int US = FMT == T_Q4_K ? 2304 : FMT == T_Q5_K ? 2816 : 3360;
  float b = 0.f;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < nunits * 16; e += (int64_t)gridDim.x * blockDim.x) {
    const uint8_t *u = w + (e / 16) * US;
    const int m = (int)(e % 16);
    float v;
    if constexpr (FMT == T_Q6_K) {
      v = fabsf(h2f(*reinterpret_cast<const uint16_t *>(u + kQ6DOff + 2 * m))) * 128.f * 32.f;
    } else {
      const uint32_t h = *reinterpret_cast<const uint32_t *>(u + (FMT == T_Q4_K ? 2048 : 2560) + 16 * m);
      v = fabsf(h2f(h & 0xffffu)) * 63.f * (FMT == T_Q4_K ? 15.f : 31.f) + fabsf(h2f(h >> 16)) * 63.f;
    }
    if (!(v <= 3.0e38f)) v = __int_as_float(0x7f800000);
    b = fmaxf(b, v);
  }
  atomicMax(out, __float_as_uint(b));
}

// ============================================================================ exact-A GEMM (kx)
// The same contraction with the weights dequantized EXACTLY into f16, so only the activation needs a
// hi / lo pair: two MMAs per 16-value K slice (A . B_hi + A . B_lo) instead of three.
//   * A of a super-block is sc * q per sub-block -- Q4_K / Q5_K: 6-bit scale times a 4- or 5-bit
//     quant, at most 63 * 31 = 1953; Q6_K: int8 scale times (q - 32), exact while every |scale| of
//     the matrix is at most 64 (checked once per matrix) -- all integers f16 holds exactly.  The
//     dequantization is byte work: nibbles spread into f16 lanes with prmt, then one f16x2 FMA
//     (1024 + q) * sc - 1024 * sc, whose single rounding is of an exact small integer.
//   * The super-block scale d cannot join an exact f16 operand, so each super-block's MMAs
//     accumulate into one of two TMEM buffers, and four epilogue warps fold d * buffer into a running
//     total in TMEM (tcgen05.ld / st) while the next super-block's MMAs fill the other buffer.
//   * Q4_K / Q5_K's min term -dmin * mn * (sum of the sub-block's activation) rides as one more
//     64-value K step per super-block: A row [-dmin mn hi x8 | same x8 | -dmin mn lo x8 | 0],
//     B row [xsum hi x8 | xsum lo x8 | xsum hi x8 | 0], one MMA over the first 32 columns giving
//     hi.hi + hi.lo + lo.hi, accumulated across super-blocks in a third TMEM region (no d scaling).
//     The min values carry a per-matrix power of two (the mscale argument) and xsum 2^-5 (a 32-value
//     sum of activations each below 2^15) to stay inside f16's range.
// TMEM: buffers [0, 128) and [128, 256), total [256, 384), min term [384, 512).  Roles (448
// threads): lane 0 of warp 0 streams each step's activation tiles with one bulk copy, warp 1 owns
// TMEM and its lane 0 issues the MMAs, warps 2..9 dequantize (each lane holds the next super-block's
// words in registers), warps 10..13 fold the buffers and write y.  Every wait is bounded; the roles
// off the critical path wait with suspending tries.
// The rings move in rounds: a super-block is two rounds, chunks 0 + 1 and chunks 2 + 3 (with Q4_K /
// Q5_K's min step as a third step of the second round), and a stage holds a round's dequantized and
// activation tiles.  A stage has one "full" barrier (the round's bulk-copy bytes and the 8
// dequantizing warps' arrivals) and one "empty" barrier (one MMA commit): one check and one commit
// per round on the MMA lane, whose barrier operations bound the pipeline.  Two stages, so the first
// round of every super-block uses stage 0 (2 slots) and the second stage 1 (2 slots and the min
// step's: a third dequantized tile and one activation hi tile).
constexpr int kXRounds = 2, kXAStages = 2 * kXRounds, kXBStages = kXAStages;
constexpr int kXASlots = kXAStages + 1;                        // + the min step's dequantized tile
constexpr size_t kXBRing = (size_t)kXBStages * kPairBytes + kTileBytes;   // + its activation hi tile
constexpr int kXProdWarp = 0, kXMmaWarp = 1, kXDqWarp0 = 2, kXEpiWarp0 = kXDqWarp0 + kDqWarps, kXEpiWarps = 4;
constexpr int kXThreads = (kXEpiWarp0 + kXEpiWarps) * 32;
constexpr uint32_t kXTmemCols = 512, kXTot = 256, kXMin = 384;
template <int FMT> constexpr int kx_steps_per_sb() { return FMT == T_Q6_K ? 4 : 5; }
constexpr size_t kx_smem_bytes() {
  return 1024 + (size_t)kXASlots * kTileBytes + kXBRing + (2 * kXAStages + 2 * kXBStages + 5) * 8 + 16;
}
static_assert(kx_smem_bytes() <= 232448, "shared memory");

// f16x2 of the low bytes of a word's bytes 0, 1 (sel 0x5140) or 2, 3 (sel 0x7362) as 1024 + b
__device__ __forceinline__ uint32_t bytes_h2(uint32_t t4, uint32_t sel) { return __byte_perm(t4, 0x64646464u, sel); }
__device__ __forceinline__ uint32_t h2fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t h2sub(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t h2mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// f16 bits of a small integer |v| <= 2048, twice (exact)
__device__ __forceinline__ uint32_t int_h2(int v) {
  const uint32_t h = __half_as_ushort(__int2half_rn(v));
  return h | (h << 16);
}

template <int FMT> struct DqX {      // Q4_K, Q5_K: one super-block of one thread's row half
  uint4 q[2][2], e;
  uint32_t F[4];                     // the 24-bit scale / min field of each chunk
  uint32_t hdx;                      // d | dmin << 16 (f16 bits)
  __device__ __forceinline__ void set(const Raw<FMT> &R) {
#pragma unroll
    for (int i = 0; i < 2; i++)
#pragma unroll
      for (int j = 0; j < 2; j++) q[i][j] = R.q[i][j];
    e = R.e;
    hdx = R.hd.x;
#pragma unroll
    for (int c = 0; c < 4; c++) F[c] = k45_field(R.hd, c);
  }
  // chunk c (sub-blocks 2c, 2c + 1): out[j] = positions 16j + 8tp .. + 7 of the step, exact sc * q
  template <int c>
  __device__ __forceinline__ void emit(uint4 (&out)[4]) const {
#pragma unroll
    for (int nib = 0; nib < 2; nib++) {
      const int sc = (int)((F[c] >> (6 * nib)) & 63u);
      const uint32_t s2 = int_h2(sc), nb2 = int_h2(-1024 * sc);
#pragma unroll
      for (int h = 0; h < 2; h++) {
        uint32_t o[4];
#pragma unroll
        for (int tt = 0; tt < 2; tt++) {
          const uint32_t w = word4(q[c >> 1][tt], 2 * (c & 1) + h);
          uint32_t t4 = (w >> (4 * nib)) & 0x0f0f0f0fu;
          if constexpr (FMT == T_Q5_K) t4 |= ((word4(e, 2 * tt + h) >> (2 * c + nib)) & 0x01010101u) << 4;
          o[2 * tt] = h2fma(bytes_h2(t4, 0x5140), s2, nb2);
          o[2 * tt + 1] = h2fma(bytes_h2(t4, 0x7362), s2, nb2);
        }
        out[2 * nib + h] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
  // the min step: position chunk tp + 2j; chunk 0: -dmin*mn hi of sub-blocks 0..7, chunk 1: the same
  // hi, chunk 2: the lo parts, the rest zero
  __device__ __forceinline__ void emit_min(int tp, float mscale, uint4 (&out)[4]) const {
    const float dmin = h2f(hdx >> 16) * mscale;
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      float v[2];
#pragma unroll
      for (int u = 0; u < 2; u++) {
        const int j = 2 * i + u;               // sub-block j: chunk j >> 1, min field j & 1
        v[u] = -(dmin * (float)((F[j >> 1] >> (12 + 6 * (j & 1))) & 63u));
      }
      split2(v[0], v[1], hi[i], lo[i]);
    }
    const uint4 H = make_uint4(hi[0], hi[1], hi[2], hi[3]), Lo = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    const uint4 Z = make_uint4(0, 0, 0, 0);
    out[0] = H;                                // chunk tp: 0 (hi) or 1 (hi again)
    out[1] = tp == 0 ? Lo : Z;                 // chunk tp + 2: 2 (lo) or 3
    out[2] = Z;
    out[3] = Z;
  }
};
template <> struct DqX<T_Q6_K> {
  uint4 ql[2][2], qh[2], sc;
  __device__ __forceinline__ void set(const Raw<T_Q6_K> &R) {
#pragma unroll
    for (int i = 0; i < 2; i++) {
      qh[i] = R.qh[i];
#pragma unroll
      for (int j = 0; j < 2; j++) ql[i][j] = R.ql[i][j];
    }
    sc = R.sc;
  }
  // chunk c (half c >> 1, 32-value run c & 1): out[j] = positions 16j + 8tp .. + 7, (q - 32) * scale
  template <int c>
  __device__ __forceinline__ void emit(uint4 (&out)[4]) const {
    constexpr int half = c >> 1, hb = c & 1;
    const uint32_t k1056 = int_h2(1056);
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int p = j >> 1, uu = j & 1, k = 2 * hb + p, G = 8 * half + 2 * k + uu;
      const int o = G < 8 ? 4 * (G >> 1) + (G & 1) : 4 * ((G - 8) >> 1) + 2 + (G & 1);
      const uint32_t s2 = int_h2((int)(int8_t)((word4(sc, o >> 2) >> (8 * (o & 3))) & 0xffu));
      uint32_t r[4];
#pragma unroll
      for (int tt = 0; tt < 2; tt++) {
        const uint32_t w = word4(ql[half][tt], 2 * uu + p), eh = word4(qh[tt], 2 * half + uu);
        const uint32_t t4 = ((w >> (4 * hb)) & 0x0f0f0f0fu) | (((eh >> (2 * k)) & 0x03030303u) << 4);
        r[2 * tt] = h2mul(h2sub(bytes_h2(t4, 0x5140), k1056), s2);
        r[2 * tt + 1] = h2mul(h2sub(bytes_h2(t4, 0x7362), k1056), s2);
      }
      out[j] = make_uint4(r[0], r[1], r[2], r[3]);
    }
  }
};

// y for 32 tokens from tok0 of one row (a lane): t = output / bscale (kx_store) or the output itself
// (kx_store_scaled); SwiGLU pairs rows 2i, 2i + 1 across neighbouring lanes
__device__ __forceinline__ void kx_store_scaled(const GemmArgs &p, const float (&t)[32], int tok0, int64_t row) {
  if (p.swiglu) {
#pragma unroll
    for (int i = 0; i < 32; i++) {
      const int tok = tok0 + i;
      const float o = t[i];
      const float up = __shfl_xor_sync(0xffffffffu, o, 1);
      if (tok < p.ntok && row < p.rows && (row & 1) == 0) {
        const double z = o;
        const double sl = __ddiv_rn(z, __dadd_rn(1.0, exp(-z)));
        p.y[(int64_t)tok * p.y_stride + row / 2] = __double2float_rn(__dmul_rn(sl, (double)up));
      }
    }
  } else if (row < p.rows) {
#pragma unroll
    for (int i = 0; i < 32; i++) {
      const int tok = tok0 + i;
      if (tok < p.ntok) {
        float o = t[i];
        const int64_t at = (int64_t)tok * p.y_stride + row;
        if (p.y_add) o = __fadd_rn(p.y_add[at], o);
        p.y[at] = o;
      }
    }
  }
}
__device__ __forceinline__ void kx_store(const GemmArgs &p, const float (&t)[32], int tok0, int64_t row) {
  float o[32];
#pragma unroll
  for (int i = 0; i < 32; i++) o[i] = tok0 + i < p.ntok ? t[i] * p.bscale[tok0 + i] : 0.f;
  kx_store_scaled(p, o, tok0, row);
}

template <int FMT>
__global__ void __launch_bounds__(kXThreads, 1) gemm_kx_kernel(const GemmArgs p) {
  constexpr int US = FMT == T_Q4_K ? 2304 : FMT == T_Q5_K ? 2816 : 3360;
  constexpr int AS = kXAStages, BS = kXBStages, SPS = kx_steps_per_sb<FMT>();
  constexpr bool MINS = FMT != T_Q6_K;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t *a_ring = smem, *b_ring = smem + kXASlots * kTileBytes;
  uint64_t *bars = reinterpret_cast<uint64_t *>(b_ring + kXBRing);
  constexpr int RS = kXRounds;
  // steps in the round that starts at step kk of a super-block (0: chunks 0, 1; 2: chunks 2, 3 and,
  // with MINS, the min step); the min step's tiles are dequantized slot AS and the hi tile after the
  // BS activation pairs
  auto round_steps = [](int kk) { return kk == 0 ? 2 : (MINS ? 3 : 2); };
  uint64_t *full_r = bars, *empty_r = bars + RS;                                    // per round stage
  uint64_t *buf_full = bars + 2 * AS + 2 * BS, *buf_free = buf_full + 2, *acc_full = buf_free + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_full + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tile = blockIdx.x, n_tile = blockIdx.y, split = blockIdx.z;
  const int nb = p.nb, nsteps_all = nb * SPS;
  // this CTA's super-blocks: [sb0, sb0 + nsb) of the row (split-K), walked from local index koff_sb
  const int sb0 = split * p.sbps, nsb = min(nb, sb0 + p.sbps) - sb0, nsteps = nsb * SPS;
  const int64_t tiles16 = (p.rows + 15) / 16;
  const int tile0 = m_tile * 8;
  const int ntile = (int)min((int64_t)8, tiles16 - tile0);
  const Ctl ctl{abort_flag, p.status};
  // each M tile starts at its own super-block of the range (spreads the CTAs of one token tile over
  // the activation); the order of the super-block sums then depends on the tile alone
  const int koff_sb = nsb > 0 ? (m_tile * 7) % nsb : 0;
  const int ntok_tile = min(GN, p.ntok - n_tile * GN);
  const int nmma = (ntok_tile + 15) / 16 * 16;

  if (threadIdx.x == 0) {
    for (int s = 0; s < RS; s++) { mbar_init(&full_r[s], kDqWarps + 1); mbar_init(&empty_r[s], 1); }
    for (int b = 0; b < 2; b++) { mbar_init(&buf_full[b], 1); mbar_init(&buf_free[b], kXEpiWarps); }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kXMmaWarp) tmem_alloc(tmem_slot, kXTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kXProdWarp) {
    // ---- activation producer: one lane, one bulk copy per step (the min step: its hi tile alone),
    // a round's copies into its stage's slots (the min step's into the hi tile after them); step s of the walk is step (sb + koff) * SPS + kk
    // of the tiles
    if (lane == 0) {
      pdl_wait();                                      // the activation tiles are the previous kernel's
      const uint32_t part = (uint32_t)nmma * 128;      // the first nmma rows of a tile
      int kk = 0, sbl = koff_sb, r = 0;
      for (int s = 0; s < nsteps; r++) {
        const int n2 = round_steps(kk), st = r % RS;
        if (r >= RS && !wait1(&empty_r[st], (uint32_t)(r / RS - 1) & 1u, ctl, ST_EMPTY_TIMEOUT)) break;
        uint32_t bytes = 0;
        for (int j = 0; j < n2; j++) bytes += MINS && kk + j == 4 ? part : 2 * part;
        mbar_arrive_expect_tx(&full_r[st], bytes);
        for (int j = 0; j < n2; j++) {
          const uint8_t *src = p.b + ((int64_t)n_tile * nsteps_all + (int64_t)(sb0 + sbl) * SPS + kk + j) * 2 * p.btile;
          const bool hi_only = MINS && kk + j == 4;
          uint8_t *dst = hi_only ? b_ring + (size_t)BS * kPairBytes : b_ring + (size_t)(st * 2 + j) * kPairBytes;
          if (!hi_only && part == (uint32_t)kTileBytes) {
            bulk_g2s(dst, src, 2 * kTileBytes, &full_r[st]);
          } else {
            bulk_g2s(dst, src, part, &full_r[st]);
            if (!hi_only) bulk_g2s(dst + kTileBytes, src + p.btile, part, &full_r[st]);
          }
        }
        s += n2;
        kk += n2;
        if (kk == SPS) {
          kk = 0;
          if (++sbl == nsb) sbl = 0;
        }
      }
      // copies still landing in shared memory (an abort) are waited for before the CTA exits
      const uint64_t deadline = globaltimer_ns() + WAIT_DEADLINE_NS;
      for (int q = r > RS ? r - RS : 0; q < r; q++)
        if (!mbar_wait_bounded(&full_r[q % RS], (uint32_t)(q / RS) & 1u, deadline)) atomicOr(p.status, ST_DRAIN_TIMEOUT);
    }
  } else if (warp == kXMmaWarp) {
    // ---- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_n(nmma);
      const uint64_t adesc0 = sw128_desc(smem_u32(a_ring)), bdesc0 = sw128_desc(smem_u32(b_ring));
      int issued = 0, kk = 0, sbi = 0, r = 0;
      // a round: one check of its stage, its 16 MMAs (+ 2 for a min step), one commit
      for (int s = 0; s < nsteps; r++) {
        const int n2 = round_steps(kk), st = r % RS;
        if (kk == 0 && sbi >= 2) {
          // the epilogue's tcgen05.ld / st of this buffer come before the MMAs that overwrite it
          if (!wait1(&buf_free[sbi & 1], (uint32_t)((sbi >> 1) - 1) & 1u, ctl, ST_EMPTY_TIMEOUT)) break;
          tc_fence_after();
        }
        // the tiles' writers fenced their stores into the async proxy before arriving (dequantized
        // tiles) or wrote them through it (bulk copies); the MMAs only read them
        if (!wait1(&full_r[st], (uint32_t)(r / RS) & 1u, ctl, ST_FULL_TIMEOUT)) break;
        for (int j = 0; j < n2; j++) {
          const int kkj = kk + j, slot = MINS && kkj == 4 ? AS : st * 2 + j;
          // descriptor start addresses are in 16-byte units: a byte offset o adds o >> 4 (the min
          // step's activation hi tile follows the BS pairs)
          const uint64_t ad = adesc0 + (uint64_t)(slot * (kTileBytes >> 4));
          const uint64_t bh = bdesc0 + (uint64_t)(slot * (kPairBytes >> 4)), bl = bh + (kTileBytes >> 4);
          if (!MINS || kkj < 4) {
            const uint32_t d = tmem + (uint32_t)((sbi & 1) * GN);
#pragma unroll
            for (int sl = 0; sl < GK / 16; sl++) {
              mma_f16(d, ad + 2 * sl, bh + 2 * sl, idesc, (kkj | sl) != 0);
              mma_f16(d, ad + 2 * sl, bl + 2 * sl, idesc, 1u);
            }
          } else {
#pragma unroll
            for (int sl = 0; sl < 2; sl++)             // columns 0..31 carry the min term
              mma_f16(tmem + kXMin, ad + 2 * sl, bh + 2 * sl, idesc, (sbi | sl) != 0);
          }
        }
        mma_commit(&empty_r[st]);
        if (kk <= 3 && kk + n2 - 1 >= 3) mma_commit(&buf_full[sbi & 1]);
        issued += n2;
        s += n2;
        kk += n2;
        if (kk == SPS) {
          kk = 0;
          sbi++;
        }
      }
      mma_commit(acc_full);
      if (issued < nsteps) *abort_flag = 1;
      if (!mbar_wait_bounded(acc_full, 0u, globaltimer_ns() + WAIT_DEADLINE_NS)) atomicOr(p.status, ST_DRAIN_TIMEOUT);
    }
  } else if (warp < kXEpiWarp0) {
    // ---- dequantizing warps: warp dw owns unit dw of the tile; lane -> row m, half tp (as gemm_kq_kernel)
    const int dw = warp - kXDqWarp0;
    const int m = (lane & 7) + 8 * (lane >> 4), tp = (lane >> 3) & 1, row = 16 * dw + m;
    const bool present = dw < ntile;
    const uint8_t *ubase = p.w + (int64_t)(tile0 + (present ? dw : 0)) * nb * US;
    uint32_t aoff[4];                              // this lane's 16-byte pieces of a swizzled A tile
#pragma unroll
    for (int j = 0; j < 4; j++) aoff[j] = sw128_off(row, 16 * j + 8 * tp);
    // the next super-block's words are loaded into registers while this one is dequantized
    Raw<FMT> nxt;
    DqX<FMT> cur;
    if (present && nsb > 0) nxt.load(ubase + (int64_t)(sb0 + koff_sb) * US, m, tp);
    int kk = 0, sbi = 0, snext = koff_sb + 1 < nsb ? koff_sb + 1 : 0;
    // two K steps per round (chunks 0 + 1, then 2 + 3 with Q4_K / Q5_K's min step): two or three
    // tiles of independent work between the barrier handshakes
    for (int s = 0, r = 0; s < nsteps; r++) {
      const int n2 = round_steps(kk), st = r % RS;
      if (kk == 0) {
        if (present) {
          cur.set(nxt);
          if (sbi + 1 < nsb) nxt.load(ubase + (int64_t)(sb0 + snext) * US, m, tp);
        }
        if (++snext == nsb) snext = 0;
      }
      if (r >= RS && !waitw(&empty_r[st], (uint32_t)(r / RS - 1) & 1u, ctl, ST_EMPTY_TIMEOUT, lane)) break;
      uint4 o0[4], o1[4];
      if (present) {
        if (kk == 0) {
          cur.template emit<0>(o0);
          cur.template emit<1>(o1);
        } else {
          cur.template emit<2>(o0);
          cur.template emit<3>(o1);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 4; j++) o0[j] = o1[j] = make_uint4(0, 0, 0, 0);
      }
      uint8_t *at0 = a_ring + (size_t)(st * 2) * kTileBytes, *at1 = at0 + kTileBytes;
#pragma unroll
      for (int j = 0; j < 4; j++) *reinterpret_cast<uint4 *>(at0 + aoff[j]) = o0[j];
#pragma unroll
      for (int j = 0; j < 4; j++) *reinterpret_cast<uint4 *>(at1 + aoff[j]) = o1[j];
      if (n2 == 3) {                               // the min step: dequantized slot AS
        if constexpr (MINS) {
          if (present) cur.emit_min(tp, p.wscale, o0);
          else
#pragma unroll
            for (int j = 0; j < 4; j++) o0[j] = make_uint4(0, 0, 0, 0);
          uint8_t *at2 = a_ring + (size_t)AS * kTileBytes;
#pragma unroll
          for (int j = 0; j < 4; j++) *reinterpret_cast<uint4 *>(at2 + aoff[j]) = o0[j];
        }
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&full_r[st]);
      s += n2;
      kk += n2;
      if (kk == SPS) {
        kk = 0;
        sbi++;
      }
    }
  } else {
    // ---- epilogue: warp w owns TMEM lanes 32 (w % 4) ..; per super-block total += d * buffer
    pdl_wait();                                        // bscale, the tile counters and y_add
    const int quarter = warp & 3;
    const int64_t row = (int64_t)m_tile * GM + quarter * 32 + lane;
    const int64_t t16 = row / 16;
    const bool rv = row < p.rows && t16 < tiles16;
    const uint8_t *urow = p.w + t16 * nb * US;
    const uint32_t lanes = (uint32_t)(quarter * 32) << 16;
    const int nch = (nmma + 31) / 32;
    const int mrow = (int)(row & 15);
    const unsigned short *dptr = reinterpret_cast<const unsigned short *>(
        urow + (FMT == T_Q6_K ? kQ6DOff + 2 * mrow : (FMT == T_Q4_K ? 2048 : 2560) + 16 * mrow));
    bool ok = true;
    int sbl = koff_sb;
    for (int sbi = 0; sbi < nsb && ok; sbi++) {
      const float d = rv ? h2f(__ldg(dptr + (int64_t)(sb0 + sbl) * (US / 2))) : 0.f;
      if (++sbl == nsb) sbl = 0;
      ok = waitw<true>(&buf_full[sbi & 1], (uint32_t)(sbi >> 1) & 1u, ctl, ST_FULL_TIMEOUT, lane);
      ok = __shfl_sync(0xffffffffu, ok && !*abort_flag, 0);
      if (!ok) break;
      tc_fence_after();
      const uint32_t buf = tmem + lanes + (uint32_t)((sbi & 1) * GN);
      for (int c = 0; c < nch; c++) {
        float v[32], t[32];
        tmem_ld32(buf + c * 32, v);
        if (sbi > 0) {
          tmem_ld32(tmem + lanes + kXTot + c * 32, t);
#pragma unroll
          for (int i = 0; i < 32; i++) t[i] = __fmaf_rn(d, v[i], t[i]);
        } else {
#pragma unroll
          for (int i = 0; i < 32; i++) t[i] = __fmul_rn(d, v[i]);
        }
        tmem_st32(tmem + lanes + kXTot + c * 32, t);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&buf_free[sbi & 1]);
    }
    if (ok) ok = waitw<true>(acc_full, 0u, ctl, ST_FULL_TIMEOUT, lane);
    ok = __shfl_sync(0xffffffffu, ok && !*abort_flag, 0);
    tc_fence_after();
    if (ok) {
      for (int c = 0; c < nch; c++) {
        const int col0 = c * 32;
        if (col0 >= ntok_tile) break;
        float t[32], mv[32];
        tmem_ld32(tmem + lanes + kXTot + col0, t);
        if constexpr (MINS) {
          tmem_ld32(tmem + lanes + kXMin + col0, mv);
#pragma unroll
          for (int i = 0; i < 32; i++) t[i] = __fmaf_rn(mv[i], p.wscale_inv, t[i]);
        }
        if (p.nsplit > 1) {
          // this split's partial sums, [token][row] in its own shared memory (the A ring: every MMA
          // that read it has completed); the cluster adds them up after the kernel's roles end
          float *ps = reinterpret_cast<float *>(smem);
#pragma unroll
          for (int i = 0; i < 32; i++) {
            const int tok = n_tile * GN + col0 + i;
            ps[(col0 + i) * GM + quarter * 32 + lane] = tok < p.ntok ? t[i] * p.bscale[tok] : 0.f;
          }
        } else {
          kx_store(p, t, n_tile * GN + col0, row);
        }
      }
    }
  }
  if (p.nsplit > 1) {
    // split-K: the nsplit CTAs of an output tile form a cluster; after every partial is in its CTA's
    // shared memory, CTA z adds the partials of token chunks z, z + nsplit, .. in split order
    // through distributed shared memory (the bits of a one-CTA sum of the same order) and writes
    // them; the second barrier keeps every CTA's shared memory alive until the others have read it
    cluster_sync_all();
    if (warp >= kXEpiWarp0) {
      const int quarter = warp & 3, rowl = quarter * 32 + lane;
      const int64_t row = (int64_t)m_tile * GM + rowl;
      const float *ps = reinterpret_cast<const float *>(smem);
      for (int c = split; c * 32 < ntok_tile; c += p.nsplit) {
        float t[32];
#pragma unroll
        for (int i = 0; i < 32; i++) t[i] = 0.f;
        for (int z = 0; z < p.nsplit; z++) {
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; i++) v[i] = ld_dsmem_f32(ps + (c * 32 + i) * GM + rowl, (uint32_t)z);
#pragma unroll
          for (int i = 0; i < 32; i++) t[i] = __fadd_rn(t[i], v[i]);
        }
        kx_store_scaled(p, t, n_tile * GN + c * 32, row);
      }
    }
    cluster_sync_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kXMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kXTmemCols);
  }
}

// Activation tiles of the kx walk: [n_tile][step][hi, lo][rows][64] f16 (rows = 128, or the 16-row
// rounding of the tokens when there is one short tile; btile = rows * 128 bytes), steps kk < 4 of
// super-block sb are values 256 sb + 64 kk .. as gemm_bfill_kernel writes them; Q4_K / Q5_K's step 4
// is the min step: xsum of sub-block j (xd * xs, the sum of its dequantized activation) * 2^-5 /
// bscale as [hi x8 | lo x8 | hi x8 | 0] in the hi tile.  nrows tokens are filled (zeros past ntok).
__global__ void gemm_bfill_kx_kernel(const int8_t *xq, const float *xd, int64_t k, int ntok, int nrows,
                                     const float *bscale, int sps, int btile, uint8_t *bt) {
  pdl_launch_dependents();                      // the GEMM after it may start its weight work
  const int64_t groups = k / 8, total = (int64_t)nrows * groups;
  const int nsteps = (int)(k / 256) * sps;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int n = (int)(e / groups);
    const int64_t g8 = e % groups, k0 = g8 * 8;
    uint32_t h[4] = {0, 0, 0, 0}, l[4] = {0, 0, 0, 0};
    if (n < ntok) {
      const float sc = xd[(int64_t)n * (k / 32) + k0 / 32] / bscale[n];
      const uint2 q = *reinterpret_cast<const uint2 *>(xq + (int64_t)n * k + k0);
      const int8_t *qb = reinterpret_cast<const int8_t *>(&q);
#pragma unroll
      for (int i = 0; i < 4; i++) split2(sc * (float)qb[2 * i], sc * (float)qb[2 * i + 1], h[i], l[i]);
    }
    const int nt = n / GN, nr = n % GN, c = (int)(k0 / 64), kk = (int)(k0 % 64);
    const int step = (c >> 2) * sps + (c & 3);
    uint8_t *base = bt + ((int64_t)nt * nsteps + step) * 2 * btile + sw128_off(nr, kk);
    *reinterpret_cast<uint4 *>(base) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4 *>(base + btile) = make_uint4(l[0], l[1], l[2], l[3]);
  }
}
__global__ void gemm_bfill_kx_min_kernel(const float *xd, const int32_t *xs, int64_t k, int ntok, int nrows,
                                         const float *bscale, int btile, uint8_t *bt) {
  pdl_launch_dependents();                      // the GEMM after it may start its weight work
  const int nb = (int)(k / 256), nsteps = nb * 5;
  const int64_t total = (int64_t)nrows * nb * 8;        // (token, super-block, 16-byte chunk)
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int n = (int)(e / (nb * 8)), sb = (int)((e / 8) % nb), ch = (int)(e % 8);
    uint32_t hi[4] = {0, 0, 0, 0}, lo[4] = {0, 0, 0, 0};
    if (n < ntok && ch < 3) {
      const float inv = 0.03125f / bscale[n];          // 2^-5 / 2^e: exact
#pragma unroll
      for (int i = 0; i < 4; i++) {
        float v[2];
#pragma unroll
        for (int u = 0; u < 2; u++) {
          const int64_t b = (int64_t)n * (k / 32) + sb * 8 + 2 * i + u;
          v[u] = __fmul_rn(xd[b], (float)xs[b]) * inv;
        }
        split2(v[0], v[1], hi[i], lo[i]);
      }
    }
    const int nt = n / GN, nr = n % GN;
    uint8_t *base = bt + ((int64_t)nt * nsteps + sb * 5 + 4) * 2 * btile;
    const uint4 val = ch == 0 || ch == 2 ? make_uint4(hi[0], hi[1], hi[2], hi[3])
                      : ch == 1           ? make_uint4(lo[0], lo[1], lo[2], lo[3])
                                          : make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4 *>(base + sw128_off(nr, 8 * ch)) = val;
  }
}

// Per matrix, for the kx path: bits of max |dmin| * 63 (Q4_K / Q5_K: the min values' range) and, for
// Q6_K, the largest |scale| (exact only up to 64).
template <int FMT>
__global__ void kx_info_kernel(const uint8_t *w, int64_t nunits, unsigned *out) {
  constexpr int US = FMT == T_Q4_K ? 2304 : FMT == T_Q5_K ? 2816 : 3360;
  float b = 0.f;
  unsigned scmax = 0;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < nunits * 16; e += (int64_t)gridDim.x * blockDim.x) {
    const uint8_t *u = w + (e / 16) * US;
    const int m = (int)(e % 16);
    if constexpr (FMT == T_Q6_K) {
      for (int i = 0; i < 16; i++) {
        const int v = (int)(int8_t)u[kQ6SOff + 16 * m + i];
        scmax = max(scmax, (unsigned)(v < 0 ? -v : v));
      }
    } else {
      const uint32_t h = *reinterpret_cast<const uint32_t *>(u + (FMT == T_Q4_K ? 2048 : 2560) + 16 * m);
      float v = fabsf(h2f(h >> 16)) * 63.f;
      if (!(v <= 3.0e38f)) v = __int_as_float(0x7f800000);
      b = fmaxf(b, v);
    }
  }
  atomicMax(out, __float_as_uint(b));
  atomicMax(out + 1, scmax);
}

}  // namespace

cudaError_t launch_kq_bound(const DevMatrix &m, unsigned *out, cudaStream_t s) {
  const int64_t nunits = (m.rows + 15) / 16 * (m.cols / 256);
  const int64_t grid = (nunits * 16 + 255) / 256 < 1024 ? (nunits * 16 + 255) / 256 : 1024;
  cudaError_t e = cudaMemsetAsync(out, 0, 4, s);
  if (e != cudaSuccess) return e;
  switch (m.type) {
    case T_Q4_K: kq_bound_kernel<T_Q4_K><<<(unsigned)grid, 256, 0, s>>>(m.data, nunits, out); break;
    case T_Q5_K: kq_bound_kernel<T_Q5_K><<<(unsigned)grid, 256, 0, s>>>(m.data, nunits, out); break;
    default: kq_bound_kernel<T_Q6_K><<<(unsigned)grid, 256, 0, s>>>(m.data, nunits, out); break;
  }
  return cudaGetLastError();
}


int64_t gemm_tokens_pad(int ntok) { return ((int64_t)ntok + GN - 1) / GN * GN; }

size_t gemm_b_bytes(int64_t k, int ntok) { return (size_t)gemm_tokens_pad(ntok) * (size_t)k * 4 + (size_t)gemm_tokens_pad(ntok) * 4; }

bool gemm_kq_supported(const DevMatrix &m) {
  return kq_type(m.type) && m.cols % 256 == 0 && m.rows > 0;
}

cudaError_t launch_gemm_prep(const ActView &act, int ntok, void *bbuf, cudaStream_t s) {
  const int64_t npad = gemm_tokens_pad(ntok);
  uint8_t *bt = reinterpret_cast<uint8_t *>(bbuf);
  float *bscale = reinterpret_cast<float *>(bt + npad * act.k * 4);
  const int threads = 256;
  gemm_bscale_kernel<<<(unsigned)((npad * 32 + threads - 1) / threads), threads, 0, s>>>(act.xd, act.k / 32, ntok, (int)npad,
                                                                                         bscale);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int64_t total = npad * (act.k / 8);
  const int64_t grid = (total + threads - 1) / threads < 148 * 16 ? (total + threads - 1) / threads : 148 * 16;
  gemm_bfill_kernel<<<(unsigned)grid, threads, 0, s>>>(act.xq, act.xd, act.k, ntok, (int)npad, bscale, bt);
  return cudaGetLastError();
}

float gemm_weight_scale(float bound) {
  if (!(bound > 0.f) || !(bound < 3.0e38f)) return 1.f;
  return ldexpf(1.f, 14 - ilogbf(bound));
}

cudaError_t launch_gemm_kq(const DevMatrix &m, const void *bbuf, int ntok, float *y, int64_t y_stride, const float *y_add,
                           float wscale, unsigned *status, cudaStream_t s, bool swiglu) {
  if (!gemm_kq_supported(m) || (swiglu && (m.rows % 2 || y_add))) return cudaErrorInvalidValue;
  const int64_t npad = gemm_tokens_pad(ntok);
  GemmArgs a{};
  a.w = m.data;
  a.b = reinterpret_cast<const uint8_t *>(bbuf);
  a.bscale = reinterpret_cast<const float *>(a.b + npad * m.cols * 4);
  a.y = y; a.y_add = y_add; a.y_stride = y_stride;
  a.wscale = wscale; a.wscale_inv = 1.f / wscale; a.swiglu = swiglu ? 1 : 0;
  a.rows = m.rows; a.ntok = ntok; a.nb = (int)(m.cols / 256); a.kc = (int)(m.cols / 64);
  a.status = status;
  const dim3 grid((unsigned)((m.rows + GM - 1) / GM), (unsigned)(npad / GN));
  switch (m.type) {
    case T_Q4_K: return launch_t<T_Q4_K>(a, grid, smem_bytes<T_Q4_K>(), s);
    case T_Q5_K: return launch_t<T_Q5_K>(a, grid, smem_bytes<T_Q5_K>(), s);
    default: return launch_t<T_Q6_K>(a, grid, smem_bytes<T_Q6_K>(), s);
  }
}

size_t gemm_f16_scratch_bytes(int64_t m, int64_t n, int64_t k) {
  const int64_t mpad = (m + GM - 1) / GM * GM;
  return (size_t)mpad * k * 2 + gemm_b_bytes(k, (int)n);
}

cudaError_t launch_gemm_f16(const uint16_t *A, const uint16_t *B, int64_t m, int64_t n, int64_t k, float *D, void *scratch,
                            unsigned *status, cudaStream_t s) {
  const int64_t mpad = (m + GM - 1) / GM * GM, npad = gemm_tokens_pad((int)n);
  uint8_t *at = reinterpret_cast<uint8_t *>(scratch), *bt = at + mpad * k * 2;
  float *bscale = reinterpret_cast<float *>(bt + npad * k * 4);
  const int threads = 256;
  int64_t tot = mpad * (k / 8);
  gemm_tile_f16_kernel<<<(unsigned)((tot + threads - 1) / threads < 4096 ? (tot + threads - 1) / threads : 4096), threads, 0, s>>>(
      A, k, m, k, mpad, 1, at);
  tot = npad * (k / 8);
  gemm_tile_f16_kernel<<<(unsigned)((tot + threads - 1) / threads < 4096 ? (tot + threads - 1) / threads : 4096), threads, 0, s>>>(
      B, k, n, k, npad, 2, bt);
  fill_f32_kernel<<<(unsigned)((npad + 255) / 256), 256, 0, s>>>(bscale, npad, 1.f);   // unit scales
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  GemmArgs a{};
  a.w = at; a.b = bt; a.bscale = bscale; a.y = D; a.y_stride = m; a.rows = m; a.ntok = (int)n;
  a.wscale = 1.f; a.wscale_inv = 1.f;
  a.nb = (int)(k / 256); a.kc = (int)(k / 64); a.status = status;
  return launch_t<0>(a, dim3((unsigned)(mpad / GM), (unsigned)(npad / GN)), smem_bytes<0>(), s);
}


size_t gemm_f16_tiles_bytes(int64_t rows, int64_t k) { return (size_t)((rows + GM - 1) / GM * GM) * (size_t)k * 2; }

cudaError_t launch_gemm_tile_f16(const DevMatrix &m, void *tiles, cudaStream_t s) {
  if (m.type != T_F16 || m.cols % 64 || m.row_stride % 2) return cudaErrorInvalidValue;
  const int64_t mpad = (m.rows + GM - 1) / GM * GM, tot = mpad * (m.cols / 8);
  const int threads = 256;
  gemm_tile_f16_kernel<<<(unsigned)((tot + threads - 1) / threads < 8192 ? (tot + threads - 1) / threads : 8192), threads, 0, s>>>(
      reinterpret_cast<const uint16_t *>(m.data), m.row_stride / 2, m.rows, m.cols, mpad, 1, reinterpret_cast<uint8_t *>(tiles));
  return cudaGetLastError();
}

cudaError_t launch_gemm_prep_f32(const float *x, int64_t ldx, int64_t k, int ntok, void *bbuf, cudaStream_t s) {
  if (k % 64 || ldx % 4 || (uintptr_t)x % 16) return cudaErrorInvalidValue;
  const int64_t npad = gemm_tokens_pad(ntok);
  uint8_t *bt = reinterpret_cast<uint8_t *>(bbuf);
  float *bscale = reinterpret_cast<float *>(bt + npad * k * 4);
  const int threads = 256;
  gemm_bscale_f32_kernel<<<(unsigned)((npad * 32 + threads - 1) / threads), threads, 0, s>>>(x, ldx, k, ntok, (int)npad, bscale);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int64_t total = npad * (k / 8);
  const int64_t grid = (total + threads - 1) / threads < 148 * 16 ? (total + threads - 1) / threads : 148 * 16;
  gemm_bfill_f32_kernel<<<(unsigned)grid, threads, 0, s>>>(x, ldx, k, ntok, (int)npad, bscale, bt);
  return cudaGetLastError();
}

cudaError_t launch_gemm_f16_tiled(const void *tiles, int64_t rows, int64_t k, const void *bbuf, int ntok, float *y,
                                  int64_t y_stride, unsigned *status, cudaStream_t s) {
  if (k % 64 || ntok < 1) return cudaErrorInvalidValue;
  const int64_t mpad = (rows + GM - 1) / GM * GM, npad = gemm_tokens_pad(ntok);
  GemmArgs a{};
  a.w = reinterpret_cast<const uint8_t *>(tiles);
  a.b = reinterpret_cast<const uint8_t *>(bbuf);
  a.bscale = reinterpret_cast<const float *>(a.b + npad * k * 4);
  a.y = y; a.y_stride = y_stride; a.rows = rows; a.ntok = ntok;
  a.wscale = 1.f; a.wscale_inv = 1.f;
  a.nb = (int)(k / 256); a.kc = (int)(k / 64); a.status = status;
  return launch_t<T_F16>(a, dim3((unsigned)(mpad / GM), (unsigned)(npad / GN)), smem_bytes<T_F16>(), s);
}

// ---------------------------------------------------------------------------- exact-A GEMM host side
cudaError_t launch_kx_info(const DevMatrix &m, unsigned *out, cudaStream_t s) {
  const int64_t nunits = (m.rows + 15) / 16 * (m.cols / 256);
  const int64_t grid = (nunits * 16 + 255) / 256 < 1024 ? (nunits * 16 + 255) / 256 : 1024;
  cudaError_t e = cudaMemsetAsync(out, 0, 8, s);
  if (e != cudaSuccess) return e;
  switch (m.type) {
    case T_Q4_K: kx_info_kernel<T_Q4_K><<<(unsigned)grid, 256, 0, s>>>(m.data, nunits, out); break;
    case T_Q5_K: kx_info_kernel<T_Q5_K><<<(unsigned)grid, 256, 0, s>>>(m.data, nunits, out); break;
    case T_Q6_K: kx_info_kernel<T_Q6_K><<<(unsigned)grid, 256, 0, s>>>(m.data, nunits, out); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

int kx_steps(int type) { return type == T_Q6_K ? kx_steps_per_sb<T_Q6_K>() : kx_steps_per_sb<T_Q4_K>(); }

// Token tiles: 128 rows each; a single short tile keeps the 16-row rounding of its tokens.
static int kx_tile_rows(int ntok) { return ntok < GN ? (ntok + 15) / 16 * 16 : GN; }
static int kx_sms() {
  static int sms[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!sms[dev] && cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) sms[dev] = 148;
  return sms[dev];
}
// Split-K, only where the output tiles alone would leave more than half of the SMs idle (a split
// CTA pays a pipeline fill, its partial sums and a share of the reduction): as many splits as fit
// one wave, at least 4 super-blocks each.
int kx_splits(int64_t rows, int ntok, int64_t k) {
  const int64_t tiles = (rows + GM - 1) / GM * (gemm_tokens_pad(ntok) / GN);
  const int nb = (int)(k / 256), sms = kx_sms();
  if (tiles * 2 > sms || nb < 8) return 1;
  int sp = (int)(sms / tiles);
  if (sp > nb / 4) sp = nb / 4;
  if (sp > 8) sp = 8;                                  // the splits of a tile are one (portable) cluster
  const int sbps = (nb + sp - 1) / sp;
  return (nb + sbps - 1) / sbps;
}

// [activation tiles][bscale: npad floats]
static size_t kx_tiles_bytes(int64_t k, int ntok, int type) {
  return (size_t)(gemm_tokens_pad(ntok) / GN) * (size_t)(k / 256) * kx_steps(type) * 2 * kx_tile_rows(ntok) * 128;
}
size_t gemm_bx_bytes(int64_t k, int ntok, int type, int64_t rows) {
  (void)rows;                                          // split-K partials stay in the clusters' shared memory
  const size_t b = kx_tiles_bytes(k, ntok, type) + (size_t)gemm_tokens_pad(ntok) * 4;
  return (b + 255) / 256 * 256;
}

cudaError_t launch_gemm_prep_kx(const ActView &act, int ntok, int type, int64_t rows, void *bbuf, cudaStream_t s) {
  const int64_t npad = gemm_tokens_pad(ntok), k = act.k;
  const int sps = kx_steps(type), tr = kx_tile_rows(ntok), nrows = ntok < GN ? tr : (int)npad;
  (void)rows;
  uint8_t *bt = reinterpret_cast<uint8_t *>(bbuf);
  float *bscale = reinterpret_cast<float *>(bt + kx_tiles_bytes(k, ntok, type));
  const int threads = 256;
  gemm_bscale_kernel<<<(unsigned)((npad * 32 + threads - 1) / threads), threads, 0, s>>>(act.xd, k / 32, ntok, (int)npad,
                                                                                         bscale);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  int64_t total = (int64_t)nrows * (k / 8);
  int64_t grid = (total + threads - 1) / threads < 148 * 16 ? (total + threads - 1) / threads : 148 * 16;
  gemm_bfill_kx_kernel<<<(unsigned)grid, threads, 0, s>>>(act.xq, act.xd, k, ntok, nrows, bscale, sps, tr * 128, bt);
  e = cudaGetLastError();
  if (e != cudaSuccess || sps == 4) return e;
  total = (int64_t)nrows * (k / 256) * 8;
  grid = (total + threads - 1) / threads < 148 * 8 ? (total + threads - 1) / threads : 148 * 8;
  gemm_bfill_kx_min_kernel<<<(unsigned)grid, threads, 0, s>>>(act.xd, act.xs, k, ntok, nrows, bscale, tr * 128, bt);
  return cudaGetLastError();
}

template <int FMT>
static cudaError_t launch_kx_t(const GemmArgs &a, dim3 grid, cudaStream_t s) {
  static bool granted[64] = {false};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!granted[dev]) {
    e = cudaFuncSetAttribute(gemm_kx_kernel<FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kx_smem_bytes());
    if (e != cudaSuccess) return e;
    granted[dev] = true;
  }
  // chained to the activation preparation with programmatic dependent launch: the dequantizing
  // warps and the MMA lane start on the weights while the preparation finishes; the activation
  // producer and the epilogue warps wait for it (griddepcontrol.wait) before touching its output
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kXThreads);
  cfg.dynamicSmemBytes = kx_smem_bytes();
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (s != nullptr && s != cudaStreamLegacy && s != cudaStreamPerThread) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na++].val.programmaticStreamSerializationAllowed = 1;
  }
  if (grid.z > 1) {                                 // split-K: a tile's splits are one cluster
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = 1;
    attr[na++].val.clusterDim.z = grid.z;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, gemm_kx_kernel<FMT>, a);
}

cudaError_t launch_gemm_kx(const DevMatrix &m, void *bbuf, int ntok, float *y, int64_t y_stride, const float *y_add,
                           float mscale, unsigned *status, cudaStream_t s, bool swiglu) {
  if (!gemm_kq_supported(m) || (swiglu && (m.rows % 2 || y_add))) return cudaErrorInvalidValue;
  const int64_t npad = gemm_tokens_pad(ntok);
  const int nb = (int)(m.cols / 256), sp = kx_splits(m.rows, ntok, m.cols);
  uint8_t *base = reinterpret_cast<uint8_t *>(bbuf);
  const size_t tb = kx_tiles_bytes(m.cols, ntok, m.type);
  GemmArgs a{};
  a.w = m.data;
  a.b = base;
  a.bscale = reinterpret_cast<const float *>(base + tb);
  a.y = y; a.y_add = y_add; a.y_stride = y_stride;
  // the min values carry mscale and xsum 2^-5: their accumulator comes back with 2^5 / mscale
  a.wscale = mscale; a.wscale_inv = 32.f / mscale; a.swiglu = swiglu ? 1 : 0;
  a.rows = m.rows; a.ntok = ntok; a.nb = nb; a.kc = (int)(m.cols / 64);
  a.btile = kx_tile_rows(ntok) * 128;
  a.nsplit = sp;
  a.sbps = (nb + sp - 1) / sp;
  a.status = status;
  const dim3 grid((unsigned)((m.rows + GM - 1) / GM), (unsigned)(npad / GN), (unsigned)sp);
  switch (m.type) {
    case T_Q4_K: return launch_kx_t<T_Q4_K>(a, grid, s);
    case T_Q5_K: return launch_kx_t<T_Q5_K>(a, grid, s);
    default: return launch_kx_t<T_Q6_K>(a, grid, s);
  }
}

}  // namespace zllm
