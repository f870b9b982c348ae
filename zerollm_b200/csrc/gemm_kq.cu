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

// ---------------------------------------------------------------------------- tcgen05 wrappers
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 16-byte global -> shared copy through L2 (LDGSTS); completion tracked per thread
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
// arrive on `bar` once this thread's earlier cp.async copies have landed (no pending-count increment:
// the barrier's expected count includes these arrivals)
__device__ __forceinline__ void cp_async_arrive(uint64_t *bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// D[tmem] (+)= A[smem] . B[smem]^T, both K-major f16, f32 accumulation
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(acc)
      : "memory");
}
// arrive on `bar` once every tcgen05 operation this thread issued before has completed
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// 32 lanes x 32 consecutive f32 columns: thread i gets lane (base lane + i), columns col..col+31
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu)      // start address
         | ((uint64_t)1 << 16)                   // leading byte offset (unused for swizzled K-major)
         | ((uint64_t)(1024 >> 4) << 32)         // stride byte offset: 8 rows x 128 B
         | ((uint64_t)1 << 46)                   // descriptor version
         | ((uint64_t)2 << 61);                  // 128-byte swizzle
}
// Instruction descriptor of kind::f16: f16 A and B, f32 D, both K-major, M x N.
// instruction descriptor of kind::f16 with f32 accumulation, M = GM; N (a multiple of 16, at most
// GN) goes in bits 17..22 as N / 8
constexpr uint32_t kIdescM = (1u << 4) | ((uint32_t)(GM >> 4) << 24);
__device__ __forceinline__ uint32_t idesc_n(int n) { return kIdescM | ((uint32_t)(n >> 3) << 17); }

// byte offset of element (row, k) of a [rows][64] f16 tile in the 128-byte-swizzled layout
__host__ __device__ __forceinline__ uint32_t sw128_off(int row, int k) {
  return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((((k >> 3) ^ (row & 7)) & 7) << 4) + (k & 7) * 2);
}

// ---------------------------------------------------------------------------- bounded waits
// try_wait without a suspend-time hint: the thread polls instead of sleeping between tries, which
// keeps the reaction to a completed phase short in these tightly coupled pipelines
__device__ __forceinline__ bool try_wait_spin(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
struct Ctl {
  volatile int *abort;
  unsigned *status;
};
// one thread; false after a give-up (sets the status bit and the abort flag) or when aborted
__device__ __forceinline__ bool wait1(uint64_t *bar, uint32_t parity, const Ctl &c, uint32_t bit) {
  if (*c.abort) return false;
  for (int i = 0; i < 64; i++)
    if (try_wait_spin(bar, parity)) return true;
  const uint64_t deadline = globaltimer_ns() + WAIT_DEADLINE_NS;
  uint32_t n = 0;
  while (!try_wait_spin(bar, parity)) {
    if (*c.abort) return false;
    if ((++n & 63u) == 0 && globaltimer_ns() > deadline) {
      atomicOr(c.status, bit);
      *c.abort = 1;
      return false;
    }
  }
  return true;
}
// a warp: lane 0 waits, the verdict is broadcast
__device__ __forceinline__ bool waitw(uint64_t *bar, uint32_t parity, const Ctl &c, uint32_t bit, int lane) {
  bool ok = true;
  if (lane == 0) ok = wait1(bar, parity, c, bit);
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  return ok;
}

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
      for (int tt = 0; tt < 2; tt++) q[cp][tt] = ldg128(u + ((2 * r + cp) * 32 + 4 * g + 2 * tp + tt) * 16);
    if constexpr (FMT == T_Q5_K) e = ldg128(u + 2048 + 32 * m + 16 * tp);
    hd = ldg128(u + (FMT == T_Q4_K ? 2048 : 2560) + 16 * m);
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
      for (int tt = 0; tt < 2; tt++) ql[h][tt] = ldg128(u + ((2 * r + h) * 32 + 4 * g + 2 * tp + tt) * 16);
    qh[0] = ldg128(u + kQ6HOff + 64 * m + 32 * tp);
    qh[1] = ldg128(u + kQ6HOff + 64 * m + 32 * tp + 16);
    sc = ldg128(u + kQ6SOff + 16 * m);
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

}  // namespace zllm
