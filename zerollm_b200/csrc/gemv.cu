// Decode GEMV (one activation vector x one weight matrix) for the legacy quant types (Q8_0, Q4_0,
// Q5_0), the dispatch by ggml type (k-quants go to gemv_kq.cu, float types to gemv_float.cu), and
// the load-time repack of raw GGUF rows into the layout the kernels read.
//
// Replaces the reference's per-type matvec kernels: src/compute/ref-kernels.js:127-195 (oracle)
// and the WASM `matvec_*` exports (src/compute/wasm/kernels.js:30-114), dispatched by ggml type as
// in src/compute/worker.js:184-197 / :251-270.
//
// Structure (one persistent CTA per SM):
//   * a producer thread streams whole chunks of consecutive rows HBM -> shared memory with 1D bulk
//     copies (cp.async.bulk, completion on an mbarrier), up to `ns` chunks in flight per SM; the
//     copies are issued before griddepcontrol.wait, so under programmatic dependent launch the
//     weights of this matrix stream while the previous kernel is still finishing;
//   * consumer threads each own a fixed set of "units" of the row (64 values of a k-quant, one
//     32-block of a legacy quant, 8 / 4 values of a float row) and keep that unit's activation in
//     registers for the whole launch; every weight byte is read from shared memory exactly once;
//   * integer block dots use dp4a (exact, like the reference's integer sums); the per-block
//     scale arithmetic is done in IEEE double with the reference's operation order and no fused
//     multiply-add (src/compute/ref-kernels.js:146, :235-236, :271), so each per-block term is
//     bit-identical to the oracle's and only the order of the final double summation differs;
//   * a row's partial sums are reduced across lanes (shuffles) and across the warps of its row
//     group (shared memory) in a fixed order, so results are deterministic.
#include "common.cuh"
#include "internal.h"
#include "kq_layout.h"

namespace zllm {

// ============================================================================ helpers
// 4 bits -> bit 0 of each of 4 bytes
__device__ __forceinline__ uint32_t spread4(uint32_t t) { return (t * 0x00204081u) & 0x01010101u; }

// ============================================================================ formats
// Each format: Acc (partial sum type), units(K), Act (per-unit activation registers),
// load(Act&, ActView, u) and dot(Act, row_in_smem, u, nb, Acc&) which adds the unit's terms.

// ---- Q8_0 / Q4_0 / Q5_0: unit = one 32-value block.  acc += s * d * xd  (ref-kernels.js:132-195)
// Device layouts per row: Q8_0 qs[32*nb] | d[2*nb];  Q4_0 qs[16*nb] | d[2*nb];  Q5_0 qs[16*nb] | qh[4*nb] | d[2*nb].
template <int T>
struct FmtQ0 {
  using Acc = double;
  static constexpr bool QACT = true;
  struct Act { uint32_t x[8]; double xd; int xs; };
  static __host__ __device__ int units(int64_t k) { return (int)(k / 32); }
  __device__ static void load(Act &a, const ActView &v, int u) {
    const uint8_t *q = reinterpret_cast<const uint8_t *>(v.xq) + (int64_t)u * 32;
    uint4 t0 = ldg128(q), t1 = ldg128(q + 16);
    a.x[0] = t0.x; a.x[1] = t0.y; a.x[2] = t0.z; a.x[3] = t0.w;
    a.x[4] = t1.x; a.x[5] = t1.y; a.x[6] = t1.z; a.x[7] = t1.w;
    a.xd = (double)__ldg(v.xd + u);
    a.xs = __ldg(v.xs + u);
  }
  __device__ static void dot(const Act &a, uint32_t row, int u, int nb, Acc &acc) {
    int s = 0;
    float d;
    if (T == T_Q8_0) {
      const uint4 q0 = lds128(row + u * 32), q1 = lds128(row + u * 32 + 16);
      const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
      for (int i = 0; i < 8; i++) s = __dp4a((int)w[i], (int)a.x[i], s);
      d = h2f(lds16(row + 32 * nb + u * 2));
    } else {
      const uint4 q = lds128(row + u * 16);
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
      uint32_t qh = 0;
      if (T == T_Q5_0) qh = lds32(row + 16 * nb + u * 4);
#pragma unroll
      for (int i = 0; i < 4; i++) {
        uint32_t vl = w[i] & 0x0f0f0f0fu, vh = (w[i] >> 4) & 0x0f0f0f0fu;
        if (T == T_Q5_0) {
          vl |= spread4((qh >> (4 * i)) & 15u) << 4;
          vh |= spread4((qh >> (16 + 4 * i)) & 15u) << 4;
        }
        s = __dp4a((int)vl, (int)a.x[i], s);
        s = __dp4a((int)vh, (int)a.x[4 + i], s);
      }
      s -= (T == T_Q5_0 ? 16 : 8) * a.xs;                    // sum((q - offset) * x), exact
      d = h2f(lds16(row + (T == T_Q5_0 ? 20 : 16) * nb + u * 2));
    }
    // acc += s * d * xd (ref-kernels.js:146): s*d is exact in double, the product by xd rounds once
    acc = __dadd_rn(acc, __dmul_rn(__dmul_rn(i2d_exact(s), (double)d), a.xd));
  }
};

__device__ __forceinline__ double acc_add(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ float acc_add(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ void warp_sum2(double &a, double &b) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a = __dadd_rn(a, __shfl_xor_sync(0xffffffffu, a, o));
    b = __dadd_rn(b, __shfl_xor_sync(0xffffffffu, b, o));
  }
}
__device__ __forceinline__ void warp_sum2(float &a, float &b) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, o));
    b = __fadd_rn(b, __shfl_xor_sync(0xffffffffu, b, o));
  }
}
// Butterfly reduction of RB per-lane partials (RB = 2 or 4) across the 32 lanes: the first log2(RB)
// steps exchange half of the remaining values with the partner lane, the rest add one value; lane
// k*32/RB ends with row k's total.  The order of additions is fixed, so results are deterministic.
template <int RB, class T>
__device__ __forceinline__ T reduce_rows(T (&v)[RB], int lane) {
  if (RB == 4) {
    const bool b4 = lane & 16;
    T w0 = acc_add(b4 ? v[2] : v[0], __shfl_xor_sync(0xffffffffu, b4 ? v[0] : v[2], 16));
    T w1 = acc_add(b4 ? v[3] : v[1], __shfl_xor_sync(0xffffffffu, b4 ? v[1] : v[3], 16));
    const bool b3 = lane & 8;
    T z = acc_add(b3 ? w1 : w0, __shfl_xor_sync(0xffffffffu, b3 ? w0 : w1, 8));
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) z = acc_add(z, __shfl_xor_sync(0xffffffffu, z, o));
    return z;
  } else {
    const bool b4 = lane & 16;
    T z = acc_add(b4 ? v[1] : v[0], __shfl_xor_sync(0xffffffffu, b4 ? v[0] : v[1], 16));
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) z = acc_add(z, __shfl_xor_sync(0xffffffffu, z, o));
    return z;
  }
}
__device__ __forceinline__ double warp_sum(double v) { return warp_sum_f64(v); }
__device__ __forceinline__ float warp_sum(float v) { return warp_sum_f32(v); }

// ============================================================================ kernel
// One CTA = 8 warps split into row groups of G warps (G = 1, 2, 4 or 8).  A row group owns a
// contiguous range of the CTA's rows and its own ring of shared-memory stages; each warp of the
// group owns a contiguous slice of every row's units (with its activation in registers).  Lane 0
// of the group's first warp issues the group's bulk copies.  Warps wait on mbarriers only: there
// is no CTA-wide barrier until the very end, where rows with G > 1 add their G warp partials in
// warp order.
struct GemvArgs {
  const uint8_t *w;
  int64_t row_stride;
  int64_t rows;
  int nb;            // super-blocks (k-quants) or blocks (legacy quants) per row
  ActView act;
  float *y;
  const float *y_add;
  unsigned *status;
  int units;         // units per row
  int g;             // warps per row group
  int uw;            // units per warp (slice width)
  int cr;            // rows per chunk (one bulk copy)
  int nsg;           // stages per row group
  int stage_bytes;
  int ntok;          // activations processed against each staged chunk (weights read once for all)
  int64_t y_stride;  // floats between consecutive tokens' outputs (and y_add rows)
};

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxStagesPerGroup = 16;
constexpr int kMaxTok = 64;                  // tokens per launch (the reference's MAX_BATCH, src/compute/layout.js:23)

template <class F, int UPT, int MINB>
__global__ void __launch_bounds__(kThreads, MINB) gemv_kernel(const GemvArgs p) {
  constexpr int RB = UPT == 1 ? 4 : 2;           // rows per reduction batch
  using Acc = typename F::Acc;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ngroups = kWarps / p.g;
  const int gi = warp / p.g, wi = warp % p.g;
  const bool leader = wi == 0 && lane == 0;

  uint8_t *stages = smem + (size_t)gi * p.nsg * p.stage_bytes;
  const size_t stage_area = (size_t)kWarps / p.g * p.nsg * p.stage_bytes;
  // partial sums of multi-warp row groups: [group][stage][token][chunk row][warp of group]
  const size_t part_per_group = (size_t)p.nsg * p.ntok * p.cr * p.g;
  Acc *part_tab = reinterpret_cast<Acc *>(smem + stage_area) + (size_t)gi * part_per_group;
  const size_t part_bytes = p.g > 1 ? ((size_t)ngroups * part_per_group * sizeof(Acc) + 15) / 16 * 16 : 0;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + stage_area + part_bytes);
  uint64_t *full = bars + (size_t)gi * 2 * p.nsg;
  uint64_t *empty = full + p.nsg;

  // row partition (32-bit arithmetic: rows * grid < 2^31 is checked on the host)
  const uint32_t G = gridDim.x, R = (uint32_t)p.rows;
  const int64_t c0 = (blockIdx.x * R) / G, c1 = ((blockIdx.x + 1) * R) / G;
  const uint32_t cta_rows = (uint32_t)(c1 - c0);
  const int64_t r0 = c0 + (gi * cta_rows) / (uint32_t)ngroups, r1 = c0 + ((gi + 1) * cta_rows) / (uint32_t)ngroups;
  const int nrows = (int)(r1 - r0);
  const int nchunks = (nrows + p.cr - 1) / p.cr;

  // ---- set-up: the group leader initialises its barriers and starts its first copies at once
  //      (weights never depend on the previous kernel, so this runs before griddepcontrol.wait)
  int issued = min(nchunks, p.nsg);                 // tracked identically by every lane
  if (leader) {
    for (int i = 0; i < p.nsg; i++) { mbar_init(&full[i], 1); mbar_init(&empty[i], p.g); }
    fence_mbar_init();
    for (int i = 0; i < issued; i++) {
      const int nr = min(p.cr, nrows - i * p.cr);
      const uint32_t bytes = (uint32_t)(nr * p.row_stride);
      mbar_arrive_expect_tx(&full[i], bytes);
      bulk_g2s(stages + (size_t)i * p.stage_bytes, p.w + (r0 + (int64_t)i * p.cr) * p.row_stride, bytes, &full[i]);
    }
  }
  __syncthreads();                                   // barriers initialised before anyone waits on them
  pdl_launch_dependents();
  pdl_wait();                                        // the activation comes from the previous kernel

  typename F::Act act[UPT];
  const int u0 = wi * p.uw, u1 = min(p.units, u0 + p.uw);
  // lanes past the end of the slice load (and later compute) a duplicate unit whose result is
  // discarded: the inner loop stays branch-free
  bool valid[UPT];
#pragma unroll
  for (int j = 0; j < UPT; j++) {
    const int u = u0 + lane + 32 * j;
    valid[j] = u < u1;
    F::load(act[j], p.act, valid[j] ? u : u1 - 1);
  }
  const uint32_t stages_s = smem_u32(stages);

  const uint64_t deadline = globaltimer_ns() + WAIT_DEADLINE_NS;
  bool aborted = false;
  for (int i = 0; i < nchunks; i++) {
    const int s = i % p.nsg;
    // warp-uniform decision: every lane waits (bounded), then the warp agrees
    const bool ok = mbar_wait_bounded(&full[s], (i / p.nsg) & 1, deadline);
    if (!__all_sync(0xffffffffu, ok)) { aborted = true; break; }
    const uint32_t st = stages_s + (uint32_t)(s * p.stage_bytes);
    const int nr = min(p.cr, nrows - i * p.cr);
    for (int t = 0; t < p.ntok; t++) {
      if (p.ntok > 1) {
        // the staged rows are reused for every token: reload this token's activation slice
        ActView at = p.act;
        if (at.xq) at.xq += (int64_t)t * at.k;
        if (at.xd) at.xd += (int64_t)t * (at.k / 32);
        if (at.xs) at.xs += (int64_t)t * (at.k / 32);
        if (at.x) at.x += (int64_t)t * at.k;
#pragma unroll
        for (int j = 0; j < UPT; j++) F::load(act[j], at, valid[j] ? u0 + lane + 32 * j : u1 - 1);
      }
      // RB rows at a time, one accumulator per (row, unit): independent dependency chains for the
      // scheduler; then one butterfly reduction across the warp leaves row k's total in lane k*32/RB
      for (int rr = 0; rr < nr; rr += RB) {
        Acc v[RB];
#pragma unroll
        for (int k = 0; k < RB; k++) {
          const int rk = min(rr + k, nr - 1);            // the tail repeats the last row (result unused)
          const uint32_t row = st + (uint32_t)(rk * p.row_stride);
          Acc part[UPT];
#pragma unroll
          for (int j = 0; j < UPT; j++) {
            part[j] = 0;
            const int u = valid[j] ? u0 + lane + 32 * j : u1 - 1;
            F::dot(act[j], row, u, p.nb, part[j]);
            part[j] = valid[j] ? part[j] : (Acc)0;
          }
          v[k] = part[0];
#pragma unroll
          for (int j = 1; j < UPT; j++) v[k] = acc_add(v[k], part[j]);
        }
        const Acc tot = reduce_rows<RB>(v, lane);
        constexpr int SPAN = 32 / RB;
        const int k = lane / SPAN;
        if (lane % SPAN == 0 && rr + k < nr) {
          if (p.g == 1) {
            const int64_t r = r0 + (int64_t)i * p.cr + rr + k;
            float out = (float)tot;
            if (p.y_add) out = __fadd_rn(p.y_add[t * p.y_stride + r], out);
            p.y[t * p.y_stride + r] = out;
          } else {
            part_tab[(((size_t)s * p.ntok + t) * p.cr + rr + k) * p.g + wi] = tot;
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    // the group's first warp waits until every warp of the group released the stage, then adds the
    // group's partial sums of this chunk in warp order and refills the stage with chunk i + nsg
    if (wi == 0 && (p.g > 1 || issued < nchunks)) {
      bool fine = true;
      if (lane == 0) fine = mbar_wait_bounded(&empty[s], (i / p.nsg) & 1, deadline);
      if (!__shfl_sync(0xffffffffu, fine, 0)) { aborted = true; break; }
      if (p.g > 1) {
        for (int e = lane; e < p.ntok * nr; e += 32) {
          const int t = e / nr, rr = e % nr;
          const Acc *pp = part_tab + (((size_t)s * p.ntok + t) * p.cr + rr) * p.g;
          Acc acc = pp[0];
          for (int w = 1; w < p.g; w++) acc = acc_add(acc, pp[w]);
          const int64_t r = r0 + (int64_t)i * p.cr + rr;
          float out = (float)acc;
          if (p.y_add) out = __fadd_rn(p.y_add[t * p.y_stride + r], out);
          p.y[t * p.y_stride + r] = out;
        }
        __syncwarp();
      }
      if (issued < nchunks) {
        if (lane == 0) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          const int nr2 = min(p.cr, nrows - issued * p.cr);
          const uint32_t bytes = (uint32_t)(nr2 * p.row_stride);
          mbar_arrive_expect_tx(&full[s], bytes);
          bulk_g2s(stages + (size_t)s * p.stage_bytes, p.w + (r0 + (int64_t)issued * p.cr) * p.row_stride, bytes,
                   &full[s]);
        }
        issued++;
      }
    }
  }
  if (aborted && lane == 0) atomicOr(p.status, ST_FULL_TIMEOUT);
  if (leader) {
    // every copy this group started must land before the CTA exits (only pending after an abort)
    const uint64_t drain_deadline = globaltimer_ns() + WAIT_DEADLINE_NS;
    for (int s = 0; s < p.nsg && s < issued; s++) {
      const int last = s + ((issued - 1 - s) / p.nsg) * p.nsg;
      if (!mbar_wait_bounded(&full[s], (last / p.nsg) & 1, drain_deadline)) atomicOr(p.status, ST_DRAIN_TIMEOUT);
    }
  }
}

// ============================================================================ repack (load time)
__global__ void repack_kernel(int type, const uint8_t *raw, int64_t raw_row, uint8_t *dst, int64_t stride,
                              int64_t rows, int nb) {
  const bool kq = type == T_Q4_K || type == T_Q5_K || type == T_Q6_K;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const uint8_t *s = raw + r * raw_row;
    if (kq) {
      // the k-quants: each byte to its place in the (tile, super-block) units (kq_layout.h)
      for (int64_t i = threadIdx.x; i < raw_row; i += blockDim.x) {
        uint8_t v = s[i];
        if (type != T_Q6_K) {
          const int bs = type == T_Q4_K ? 144 : 176;
          const int e = (int)(i % bs);
          if (e >= 4 && e < 16) {
            // byte e of the 12-byte scale table: rebuilt from the whole table (quant.js:109-118)
            const uint8_t *q = s + (i - e) + 4;
            const int j = (e - 4) / 3, k = (e - 4) % 3;      // chunk j, byte k of its 24-bit field
            auto scale = [&](int t) { return t < 4 ? q[t] & 63 : (q[t + 4] & 15) | ((q[t - 4] >> 6) << 4); };
            auto minv = [&](int t) { return t < 4 ? q[t + 4] & 63 : (q[t + 4] >> 4) | ((q[t] >> 6) << 4); };
            const uint32_t f = scale(2 * j) | (scale(2 * j + 1) << 6) | (minv(2 * j) << 12) | (minv(2 * j + 1) << 18);
            v = (uint8_t)(f >> (8 * k));
          }
        }
        dst[kq_dev_pos(type, r, i, nb)] = v;
      }
      continue;
    }
    uint8_t *d = dst + r * stride;
    for (int64_t i = threadIdx.x; i < raw_row; i += blockDim.x) {
      int64_t o = i;
      if (type == T_Q8_0) {
        const int b = (int)(i / 34), e = (int)(i % 34);
        o = e < 2 ? 32LL * nb + b * 2 + e : b * 32 + (e - 2);
      } else if (type == T_Q4_0) {
        const int b = (int)(i / 18), e = (int)(i % 18);
        o = e < 2 ? 16LL * nb + b * 2 + e : b * 16 + (e - 2);
      } else if (type == T_Q5_0) {
        const int b = (int)(i / 22), e = (int)(i % 22);
        o = e < 2 ? 20LL * nb + b * 2 + e : e < 6 ? 16LL * nb + b * 4 + (e - 2) : b * 16 + (e - 6);
      }
      d[o] = s[i];
    }
    for (int64_t i = raw_row + threadIdx.x; i < stride; i += blockDim.x) d[i] = 0;
  }
}

// Rows src[0 .. nrows) of a k-quant matrix to rows dst_row0 + i * dst_step of another of the same
// type and width (both in the unit layout): the concatenations of model.cu.
__global__ void kq_copy_rows_kernel(int type, int nb, uint8_t *dst, int64_t dst_row0, int64_t dst_step,
                                    const uint8_t *src, int64_t nrows) {
  const int64_t rb = (int64_t)nb * kq_block_bytes(type);
  for (int64_t r = blockIdx.x; r < nrows; r += gridDim.x) {
    const int64_t rd = dst_row0 + r * dst_step;
    for (int64_t i = threadIdx.x; i < rb; i += blockDim.x) dst[kq_dev_pos(type, rd, i, nb)] = src[kq_dev_pos(type, r, i, nb)];
  }
}

// ============================================================================ host side
bool type_supported(int t) {
  switch (t) {
    case T_F32: case T_F16: case T_BF16: case T_Q4_0: case T_Q5_0: case T_Q8_0: case T_Q4_K: case T_Q5_K: case T_Q6_K:
      return true;
    default: return false;
  }
}
bool type_quantized(int t) { return type_supported(t) && t != T_F32 && t != T_F16 && t != T_BF16; }

int64_t raw_row_bytes(int t, int64_t cols) {
  switch (t) {
    case T_F32: return cols * 4;
    case T_F16: case T_BF16: return cols * 2;
    case T_Q8_0: return cols % 32 ? -1 : cols / 32 * 34;
    case T_Q4_0: return cols % 32 ? -1 : cols / 32 * 18;
    case T_Q5_0: return cols % 32 ? -1 : cols / 32 * 22;
    case T_Q4_K: return cols % 256 ? -1 : cols / 256 * 144;
    case T_Q5_K: return cols % 256 ? -1 : cols / 256 * 176;
    case T_Q6_K: return cols % 256 ? -1 : cols / 256 * 210;
    default: return -1;
  }
}

int64_t dev_row_stride(int t, int64_t cols) {
  const int64_t rb = raw_row_bytes(t, cols);
  return rb < 0 ? -1 : (rb + 15) / 16 * 16;
}

int64_t dev_matrix_bytes(int t, int64_t rows, int64_t cols) {
  if (t == T_Q4_K || t == T_Q5_K || t == T_Q6_K) return cols % 256 ? -1 : kq_matrix_bytes(t, rows, cols / 256);
  const int64_t rs = dev_row_stride(t, cols);
  return rs < 0 ? -1 : rs * rows;
}

cudaError_t repack_upload(const DevMatrix &m, const void *raw_dev, cudaStream_t s) {
  const int64_t rb = raw_row_bytes(m.type, m.cols);
  const bool kq = m.type == T_Q4_K || m.type == T_Q5_K || m.type == T_Q6_K;
  const int nb = (int)(kq ? m.cols / 256 : m.cols / 32);
  if (kq && m.rows % kKqTile) {
    // the rows that pad the last tile read as zeros
    const cudaError_t e = cudaMemsetAsync(m.data, 0, (size_t)kq_matrix_bytes(m.type, m.rows, nb), s);
    if (e != cudaSuccess) return e;
  }
  const int64_t grid = m.rows < 65535 ? m.rows : 65535;
  repack_kernel<<<(unsigned)grid, 256, 0, s>>>(m.type, (const uint8_t *)raw_dev, rb, m.data, m.row_stride, m.rows, nb);
  return cudaGetLastError();
}

cudaError_t launch_kq_copy_rows(const DevMatrix &dst, int64_t dst_row0, int64_t dst_step, const DevMatrix &src,
                                cudaStream_t s) {
  if (dst.type != src.type || dst.cols != src.cols || !kq_type(src.type)) return cudaErrorInvalidValue;
  const int64_t grid = src.rows < 65535 ? src.rows : 65535;
  kq_copy_rows_kernel<<<(unsigned)grid, 256, 0, s>>>(src.type, (int)(src.cols / 256), dst.data, dst_row0, dst_step,
                                                     src.data, src.rows);
  return cudaGetLastError();
}

static int units_of(int t, int64_t k) {
  switch (t) {
    case T_Q4_K: case T_Q5_K: case T_Q6_K: return (int)(k / 64);
    case T_Q8_0: case T_Q4_0: case T_Q5_0: return (int)(k / 32);
    case T_F16: case T_BF16: return (int)(k / 8);
    case T_F32: return (int)(k / 4);
  }
  return 0;
}

static size_t acc_bytes(int t) { return type_quantized(t) ? 8 : 4; }

// Shared memory one CTA may use for stages: two CTAs fit per SM, so the next kernel of the stream
// can become resident (and start its own weight copies) while this one finishes.
constexpr int64_t kStageBudget = 96 * 1024;

bool plan_gemv(const DevMatrix &m, int num_sms, GemvPlan *p, const char **why) {
  if (!type_supported(m.type)) { *why = "unsupported tensor type"; return false; }
  if ((m.type == T_F16 || m.type == T_BF16) && m.cols % 8) { *why = "F16/BF16 rows must be a multiple of 8 values"; return false; }
  if (m.type == T_F32 && m.cols % 4) { *why = "F32 rows must be a multiple of 4 values"; return false; }
  const int U = units_of(m.type, m.cols);
  if (U <= 0) { *why = "empty row"; return false; }
  p->units = U;
  // warps per row group: as few as possible while each lane holds at most 2 units (else 4)
  // one unit per lane when the row splits evenly over whole warps (4-row batches fit in registers),
  // else as few warps as keep each lane at <= 2 (then <= 4) units
  int g = 0;
  for (int c = 1; c <= kWarps && !g; c *= 2) if ((U + c - 1) / c <= 32 && U >= 24 * c) g = c;
  for (int c = 1; c <= kWarps && !g; c *= 2) if ((U + c - 1) / c <= 64) g = c;
  for (int c = 1; c <= kWarps && !g; c *= 2) if ((U + c - 1) / c <= 128) g = c;
  if (!g) { *why = "row too long for the decode GEMV"; return false; }
  p->g = g;
  p->uw = (U + g - 1) / g;
  p->upt = (p->uw + 31) / 32;
  if (p->upt == 3) p->upt = 4;
  const int ngroups = kWarps / g;
  int64_t grid = m.rows < num_sms ? m.rows : num_sms;
  if (grid < 1) grid = 1;
  if ((m.rows + 1) * grid >= (1LL << 32)) { *why = "too many rows for the decode GEMV"; return false; }
  p->grid = (int)grid;
  const int64_t rows_cta = (m.rows + grid - 1) / grid;
  const int64_t rows_grp = (rows_cta + ngroups - 1) / ngroups;
  // ~8 KB chunks: the compute left after the last chunk lands stays short
  int64_t cr = (8192 + m.row_stride / 2) / m.row_stride;
  if (cr < 1) cr = 1;
  if (cr > rows_grp) cr = rows_grp;
  if (cr < 1) cr = 1;
  p->cr = (int)cr;
  const int64_t stage = (cr * m.row_stride + 127) / 128 * 128;
  if (stage > 110 * 1024) { *why = "row too long for a shared-memory stage"; return false; }
  p->stage_bytes = (int)stage;
  const int64_t chunks = (rows_grp + cr - 1) / cr;
  int64_t nsg = kStageBudget / ngroups / stage;
  if (nsg > kMaxStagesPerGroup) nsg = kMaxStagesPerGroup;
  if (nsg > chunks) nsg = chunks;
  if (nsg < 1) nsg = 1;
  p->nsg = (int)nsg;
  p->max_rows = (int)rows_cta + 1;
  return true;
}

// shared memory of one launch over `ntok` tokens
static size_t gemv_smem(const DevMatrix &m, const GemvPlan &pl, int ntok) {
  const int ngroups = kWarps / pl.g;
  const size_t part = pl.g > 1 ? ((size_t)ngroups * pl.nsg * ntok * pl.cr * pl.g * acc_bytes(m.type) + 15) / 16 * 16 : 0;
  return (size_t)ngroups * pl.nsg * pl.stage_bytes + part + (size_t)ngroups * 2 * pl.nsg * 8;
}

template <class F, int UPT>
static cudaError_t launch_one(const GemvArgs &a, const GemvPlan &pl, cudaStream_t s, bool pdl) {
  constexpr int MINB = UPT <= 2 ? 2 : 1;
  auto kern = gemv_kernel<F, UPT, MINB>;
  // the opt-in shared-memory size is a per-device function attribute: set it once per device so
  // that launches inside stream capture make no attribute calls
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
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = pl.smem_bytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <class F>
static cudaError_t launch_fmt(const GemvArgs &a, const GemvPlan &pl, cudaStream_t s, bool pdl) {
  switch (pl.upt) {
    case 1: return launch_one<F, 1>(a, pl, s, pdl);
    case 2: return launch_one<F, 2>(a, pl, s, pdl);
    default: return launch_one<F, 4>(a, pl, s, pdl);
  }
}

cudaError_t launch_gemv(const DevMatrix &m, const ActView &act, int ntok, float *y, int64_t y_stride,
                        const float *y_add, unsigned *status, int num_sms, cudaStream_t s, bool pdl, const char **why) {
  if (kq_type(m.type)) return launch_gemv_kq(m, act, ntok, y, y_stride, y_add, status, num_sms, s, pdl, why);
  if (float_type(m.type)) return launch_gemv_float(m, act, ntok, y, y_stride, y_add, num_sms, s, pdl, why);
  GemvPlan pl;
  if (!plan_gemv(m, num_sms, &pl, why)) return cudaErrorInvalidValue;
  const int64_t nbk = (m.type == T_Q4_K || m.type == T_Q5_K || m.type == T_Q6_K) ? m.cols / 256 : m.cols / 32;
  // up to kMaxTok tokens share one pass over the weights
  for (int t0 = 0; t0 < ntok; t0 += kMaxTok) {
    const int nt = ntok - t0 < kMaxTok ? ntok - t0 : kMaxTok;
    pl.smem_bytes = (int)gemv_smem(m, pl, nt);
    GemvArgs a;
    a.w = m.data;
    a.row_stride = m.row_stride;
    a.rows = m.rows;
    a.nb = (int)nbk;
    a.act.k = act.k;
    a.act.xq = act.xq ? act.xq + (int64_t)t0 * act.k : nullptr;
    a.act.xd = act.xd ? act.xd + (int64_t)t0 * (act.k / 32) : nullptr;
    a.act.xs = act.xs ? act.xs + (int64_t)t0 * (act.k / 32) : nullptr;
    a.act.x = act.x ? act.x + (int64_t)t0 * act.k : nullptr;
    a.y = y + (int64_t)t0 * y_stride;
    a.y_add = y_add ? y_add + (int64_t)t0 * y_stride : nullptr;
    a.ntok = nt;
    a.y_stride = y_stride;
    a.status = status;
    a.units = pl.units; a.g = pl.g; a.uw = pl.uw; a.cr = pl.cr; a.nsg = pl.nsg; a.stage_bytes = pl.stage_bytes;
    cudaError_t e;
    switch (m.type) {
      case T_Q8_0: e = launch_fmt<FmtQ0<T_Q8_0>>(a, pl, s, pdl); break;
      case T_Q4_0: e = launch_fmt<FmtQ0<T_Q4_0>>(a, pl, s, pdl); break;
      case T_Q5_0: e = launch_fmt<FmtQ0<T_Q5_0>>(a, pl, s, pdl); break;
      default: *why = "unsupported tensor type"; return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace zllm
