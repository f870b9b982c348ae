// Device layout of the k-quant formats (Q4_K, Q5_K, Q6_K): where each byte of a raw GGUF matrix
// goes when it is uploaded.  Shared by the load-time repack and row copies (gemv.cu), the GEMV
// kernels (gemv_kq.cu) and the row dequantization of the embedding lookup (ops.cu).
//
// The GEMVs run warp-level integer MMAs on tiles of 16 rows: lane (g, t) of a warp (g = lane / 4,
// t = lane % 4) feeds rows g and g + 8 of the tile at value positions 4t..4t+3 (and 16 + 4t..)
// of each 32-value sub-block (Q4_K / Q5_K) or each 16-value group (Q6_K).  The matrix is stored
// as UNITS, one per (tile of 16 rows, super-block), in the order (tile, super-block): unit
// (T, s) holds super-block s of rows 16T .. 16T + 15, and the units of a tile follow one another,
// so a run of super-blocks of one tile is one contiguous range.  Inside a unit every region that
// a lane reads is laid out so that the 32 lanes' pieces are consecutive: one warp-wide 16-byte
// load reads 512 contiguous bytes.  Row m of the unit is written m = 8r + g (r = 0: row g,
// r = 1: row g + 8).  Nothing is added or dropped except whole zero rows that pad the last tile:
// HBM traffic equals the GGUF size.
//
// First, each super-block is permuted in place (the "lane order"):
//  * Q4_K (144 B per 256 values) and Q5_K (176 B): bytes 0..3 (d, dmin) unchanged; bytes 4..15
//    (the packed 6-bit scales and mins, src/compute/quant.js:103-118) rewritten as four 24-bit
//    fields, one per 64-value chunk c, at bit 24c: sc(2c) | sc(2c+1) << 6 | mn(2c) << 12 |
//    mn(2c+1) << 18.  The quants (raw word w = 8c + 4h + t of qs: bytes 32c + 16h + 4t..,
//    low nibbles = sub-block 2c, high nibbles = sub-block 2c + 1) move to word t*8 + c*2 + h, so
//    lane t's 32 bytes are qs bytes 32t..32t+31.  Q5_K's high bits (raw word w = 4h + t of qh)
//    move to word t*2 + h (lane t's 8 bytes at 8t).
//  * Q6_K (210 B per 256 values): raw ql word w = 16h + 8p + 4u + t (half h, part p, 16-value
//    half u of the 32-value run) moves to word t*8 + h*4 + u*2 + p (lane t's 32 bytes at 32t, half
//    h at 32t + 16h); raw qh word w = 8h + 4u + t moves to word t*4 + h*2 + u (lane t's 16 bytes at
//    16t); the 16 int8 scales are reordered so lane t's four (groups 2t, 2t+1, 8+2t, 9+2t) are
//    bytes 4t..4t+3.
// Then the 16 rows' permuted super-blocks are spread over the unit's regions:
//  * Q4_K, 2304 B: Q [0, 2048): byte 16j + e of lane t's 32 quant bytes of row 8r + g at
//    ((2r + j) * 32 + 4g + t) * 16 + e (four 512-byte slabs: row g low/high 16 bytes, row g + 8
//    low/high); H [2048, 2304): the 16-byte header (d, dmin, fields) of row m at 2048 + 16m.
//  * Q5_K, 2816 B: Q as Q4_K; E [2048, 2560): the 8 high-bit bytes of row m at 2048 + 32m + 8t
//    (lane t's piece); H [2560, 2816): header of row m at 2560 + 16m.
//  * Q6_K, 3360 B: L [0, 2048): lane t's ql half h of row 8r + g at ((2r + h) * 32 + 4g + t) * 16;
//    QH [2048, 3072): the 64 qh bytes of row m at 2048 + 64m (lane t's 16 at + 16t); SC [3072,
//    3328): the 16 scales of row m at 3072 + 16m (lane t's 4 at + 4t); D [3328, 3360): d of row m
//    at 3328 + 2m.
#pragma once
#include <stdint.h>

#ifdef __CUDACC__
#define ZLLM_HD __host__ __device__ __forceinline__
#else
#define ZLLM_HD inline
#endif

namespace zllm {

constexpr int kKqTile = 16;          // rows per unit

ZLLM_HD int kq_block_bytes(int type) { return type == 12 ? 144 : type == 13 ? 176 : 210; }
ZLLM_HD int kq_unit_bytes(int type) { return kKqTile * kq_block_bytes(type); }
// device bytes of a rows x (256 nb) k-quant matrix (the last tile padded with zero rows)
ZLLM_HD int64_t kq_matrix_bytes(int type, int64_t rows, int64_t nb) {
  return (rows + kKqTile - 1) / kKqTile * nb * kq_unit_bytes(type);
}

// Byte offset in the device matrix of raw byte `i` of row `row` (of `nb` super-blocks).  For
// Q4_K / Q5_K bytes 4..15 of a block (the scale table) are rebuilt rather than moved; the offset
// returned for raw byte e of the table is where rebuilt byte e goes.
ZLLM_HD int64_t kq_dev_pos(int type, int64_t row, int64_t i, int64_t nb) {
  const int bs = kq_block_bytes(type);
  const int64_t sb = i / bs;
  const int e = (int)(i % bs);
  const int m = (int)(row % kKqTile), r = m >> 3, g = m & 7;
  const int64_t unit = ((row / kKqTile) * nb + sb) * (int64_t)kq_unit_bytes(type);
  if (type == 12 || type == 13) {                       // Q4_K, Q5_K
    const int qs = type == 12 ? 16 : 48, hreg = type == 12 ? 2048 : 2560;
    if (e < 16) return unit + hreg + 16 * m + e;       // d, dmin, scale fields
    if (e < qs) {                                       // Q5_K high bits
      const int q = e - 16, w = q >> 2, h = w >> 2, t = w & 3;
      return unit + 2048 + 32 * m + 4 * (t * 2 + h) + (q & 3);
    }
    const int q = e - qs, w = q >> 2, c = w >> 3, h = (w >> 2) & 1, t = w & 3;
    const int b = 4 * (c * 2 + h) + (q & 3);           // byte within lane t's 32
    return unit + ((2 * r + (b >> 4)) * 32 + 4 * g + t) * 16 + (b & 15);
  }
  // Q6_K
  if (e < 128) {
    const int w = e >> 2, h = w >> 4, p = (w >> 3) & 1, u = (w >> 2) & 1, t = w & 3;
    const int b = 4 * (h * 4 + u * 2 + p) + (e & 3);   // byte within lane t's 32 (half h = b >> 4)
    return unit + ((2 * r + (b >> 4)) * 32 + 4 * g + t) * 16 + (b & 15);
  }
  if (e < 192) {
    const int q = e - 128, w = q >> 2, h = w >> 3, u = (w >> 2) & 1, t = w & 3;
    return unit + 2048 + 64 * m + 4 * (t * 4 + h * 2 + u) + (q & 3);
  }
  if (e < 208) {
    const int G = e - 192;
    const int o = G < 8 ? 4 * (G >> 1) + (G & 1) : 4 * ((G - 8) >> 1) + 2 + (G & 1);
    return unit + 3072 + 16 * m + o;
  }
  return unit + 3328 + 2 * m + (e - 208);
}

}  // namespace zllm
