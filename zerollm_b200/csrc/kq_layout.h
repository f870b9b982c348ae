// Device layout of the k-quant formats (Q4_K, Q5_K, Q6_K): where each byte of a raw GGUF row goes
// when a matrix is uploaded.  Shared by the load-time repack (gemv.cu), the tensor-core GEMV
// (gemv_kq.cu) and the row dequantization of the embedding lookup (ops.cu).
//
// The layout serves the warp-level integer MMAs of the GEMV: lane (g, t) of a warp (g = lane / 4,
// t = lane % 4) feeds rows g and g + 8 of a 16-row tile at value positions 4t..4t+3 (and
// 16 + 4t..16 + 4t+3) of each 32-value sub-block (Q4_K / Q5_K) or each 16-value group (Q6_K).  The
// bytes one lane needs from one row of one super-block are made contiguous, so it fetches them with
// one or two 16-byte shared-memory loads.  Nothing is added or dropped: a device row holds exactly
// the raw row's bytes (plus padding to 16), so HBM traffic equals the GGUF size.
//
//  * Q4_K (144 B per 256 values) and Q5_K (176 B): block order unchanged.  Bytes 0..3 (d, dmin)
//    unchanged; bytes 4..15 (the packed 6-bit scales and mins, src/compute/quant.js:103-118) are
//    rewritten as four 24-bit fields, one per 64-value chunk c, at bit 24c:
//    sc(2c) | sc(2c+1) << 6 | mn(2c) << 12 | mn(2c+1) << 18.
//    The quants (raw word w = 8c + 4h + t of qs: bytes 32c + 16h + 4t.., low nibbles = sub-block 2c,
//    high nibbles = sub-block 2c + 1) move to word t*8 + c*2 + h, so lane t reads its 32 bytes at
//    qs + 32t.  Q5_K's high bits (raw word w = 4h + t of qh) move to word t*2 + h (8 bytes at
//    qh + 8t).
//  * Q6_K (210 B per 256 values): super-blocks are grouped by 8 (the last group of a row may be
//    shorter); a group of n super-blocks stores ql[n][128] | qh[n][64] | scales[n][16] | d[n][2],
//    so every region starts 16-byte aligned.  Within a super-block, raw ql word
//    w = 16h + 8p + 4u + t (half h, part p, 16-value half u of the 32-value run) moves to word
//    t*8 + h*4 + u*2 + p; raw qh word w = 8h + 4u + t moves to word t*4 + h*2 + u; the 16 int8
//    scales are reordered so lane t's four (groups 2t, 2t+1, 8+2t, 9+2t) are bytes 4t..4t+3.
#pragma once
#include <stdint.h>

#ifdef __CUDACC__
#define ZLLM_HD __host__ __device__ __forceinline__
#else
#define ZLLM_HD inline
#endif

namespace zllm {

constexpr int kQ6Group = 8;          // Q6_K super-blocks per SoA group

// Byte offset within a device row of raw byte `i` of a row of `nb` super-blocks.  For Q4_K / Q5_K
// bytes 4..15 of a block (the scale table) are rebuilt rather than moved; the offset returned
// for them is their own position.
ZLLM_HD int64_t kq_dev_offset(int type, int64_t i, int64_t nb) {
  if (type == 12 || type == 13) {                       // Q4_K, Q5_K
    const int bs = type == 12 ? 144 : 176, qs = type == 12 ? 16 : 48;
    const int64_t b = i / bs;
    const int e = (int)(i % bs);
    int o = e;
    if (e >= qs) {
      const int q = e - qs, w = q >> 2, c = w >> 3, h = (w >> 2) & 1, t = w & 3;
      o = qs + 4 * (t * 8 + c * 2 + h) + (q & 3);
    } else if (type == 13 && e >= 16) {
      const int q = e - 16, w = q >> 2, h = w >> 2, t = w & 3;
      o = 16 + 4 * (t * 2 + h) + (q & 3);
    }
    return b * bs + o;
  }
  // Q6_K
  const int64_t b = i / 210;
  const int e = (int)(i % 210);
  const int64_t grp = b / kQ6Group;
  const int j = (int)(b % kQ6Group);
  const int64_t left = nb - grp * kQ6Group;
  const int n = left < kQ6Group ? (int)left : kQ6Group;
  const int64_t base = grp * kQ6Group * 210;
  if (e < 128) {
    const int w = e >> 2, h = w >> 4, p = (w >> 3) & 1, u = (w >> 2) & 1, t = w & 3;
    return base + 128 * j + 4 * (t * 8 + h * 4 + u * 2 + p) + (e & 3);
  }
  if (e < 192) {
    const int q = e - 128, w = q >> 2, h = w >> 3, u = (w >> 2) & 1, t = w & 3;
    return base + 128 * n + 64 * j + 4 * (t * 4 + h * 2 + u) + (q & 3);
  }
  if (e < 208) {
    const int G = e - 192;
    const int o = G < 8 ? 4 * (G >> 1) + (G & 1) : 4 * ((G - 8) >> 1) + 2 + (G & 1);
    return base + 192 * n + 16 * j + o;
  }
  return base + 208 * n + 2 * j + (e - 208);
}

}  // namespace zllm
