// Host-side declarations shared by the .cu files of libzllm_cuda.so (not part of the C ABI).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

namespace zllm {

// ggml type ids (src/gguf/types.js:10-15)
enum GgmlType : int {
  T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q5_0 = 6, T_Q8_0 = 8, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14, T_BF16 = 30
};

bool type_supported(int type);
bool type_quantized(int type);
// bytes of one raw GGUF row; -1 when cols is not a whole number of blocks
int64_t raw_row_bytes(int type, int64_t cols);
// bytes of one device row (repacked layout, padded to 16); for the k-quants, whose rows are
// interleaved in units of 16 (kq_layout.h), the raw row length rounded up to 16
int64_t dev_row_stride(int type, int64_t cols);
// device bytes of a whole matrix
int64_t dev_matrix_bytes(int type, int64_t rows, int64_t cols);

// A device-resident matrix in the kernels' layout (see repack in gemv.cu).
struct DevMatrix {
  int type;
  int64_t rows, cols;
  int64_t row_stride;   // bytes, multiple of 16
  uint8_t *data;        // 256-byte aligned (cudaMalloc)
};

// Activation of `ntok` tokens: quantized (xq int8 [ntok][K], xd f32 [ntok][K/32], xs int32
// [ntok][K/32]) for quantized weights, plain f32 x [ntok][K] for F16/BF16/F32 weights.
struct ActView {
  const int8_t *xq;
  const float *xd;
  const int32_t *xs;
  const float *x;
  int64_t k;
};

// Launch geometry of one GEMV (computed on the host, see plan_gemv).
struct GemvPlan {
  int units, g, uw, upt, cr, nsg, stage_bytes, grid, smem_bytes, max_rows;
};

// Paged KV caches: a layer's K (and V) pool holds num_pages pages of [n_kv][1 << page_log2][head_dim]
// elements; row s of table lists sequence s's pages in position order (max_pages entries), so
// position p of sequence s lives at row p & (page size - 1) of page table[s * max_pages + (p >> page_log2)].
struct KvPages {
  const int32_t *table;            // device [nseq][max_pages]; NULL: contiguous caches
  int max_pages, num_pages, page_log2;
};
// element offset of position p's row of KV head kh of sequence row `srow` in a page pool; a position
// past the row's max_pages pages or an entry outside [0, num_pages) reads page 0 and reports
// ST_BAD_ARGS (the table lives on the device, where the host does not look)
__device__ __forceinline__ int64_t kv_page_row(const KvPages &pg, int64_t srow, int n_kv, int kh, int p, int hd,
                                               unsigned *status) {
  const int slot = p >> pg.page_log2;
  int page = slot < pg.max_pages ? __ldg(pg.table + srow * pg.max_pages + slot) : -1;
  if (page < 0 || page >= pg.num_pages) {
    if (status) atomicOr(status, 8u);   // ST_BAD_ARGS (common.cuh)
    page = 0;
  }
  return ((((int64_t)page * n_kv + kh) << pg.page_log2) + (p & ((1 << pg.page_log2) - 1))) * hd;
}

// q/k/v post-processing of `ntok` tokens (biases, q/k RMSNorm, RoPE) and the K/V append.
struct QkvPostArgs {
  const float *q, *k, *v;          // [ntok][q_stride] / [ntok][kv_stride] f32 projections
  int64_t q_stride, kv_stride;
  const float *bq, *bk, *bv;       // optional biases
  const float *q_norm, *k_norm;    // optional per-head RMSNorm weights [head_dim]
  const float *rope_cos, *rope_sin;  // [ctx][n_rot/2]
  const int *pos, *seq;            // per token: position and sequence index
  float *q_out;                    // [ntok][q_out_stride] roped queries
  int64_t q_out_stride;
  void *kcache, *vcache;           // caches, element f16 or f32
  int64_t seq_stride, head_stride; // elements between sequences / KV heads (positions are head_dim apart)
  int n_head, n_kv, head_dim, n_rot, neox, kv_f16, ntok;
  double eps;
  KvPages pages;                   // paged caches (pages.table != NULL): kcache / vcache are page pools
  unsigned *status;                // device status word (a bad page index), may be NULL
};

// decode attention: a sequence of n positions is cut into context splits whose number and length
// depend on n and the layer's geometry alone (so a query's partition, and its bits, do not depend on
// the batch around it).  A split is processed by attn_warps(n_kv) warps: 8, or 16 when a layer has at
// most 2 KV heads (a tensor-parallel rank's share of a GQA model), where the few (KV head, split)
// CTAs of a short batch would otherwise each walk long chains of positions.  At least kAttnMinSplit
// positions per split, at most a cap of splits (37 CTAs of 8 warps per KV head: two per SM over 8 KV
// heads; 18 of 16 warps: one per SM) until the splits reach a maximum length.  Measured on B200
// (config 2 and the 8B decode), 256 positions per split beat 128 (more work per warp, fewer partials
// to merge: +30 % at 2048 x 64 sequences and 8192 x 1, +5 % at 32-sequence decode) and 512 (which
// starves one short sequence of CTAs: -26 % at 2048 x 1); 16 warps everywhere gained 23-26 % at one
// sequence but lost 4-28 % at 64 (one CTA per SM idles at CTA boundaries), hence only for few KV heads.
// attn_nsplit is non-decreasing in n, so a launch sized for the longest sequence fits every other.
constexpr int kAttnMinSplit = 256;
__host__ __device__ constexpr int attn_warps(int n_kv) { return n_kv <= 2 ? 16 : 8; }
__host__ __device__ inline int attn_nsplit(int n, int warps) {
  const int cap = warps == 16 ? 18 : 37, max_len = warps == 16 ? 2048 : 1024;
  int ns = (n + kAttnMinSplit - 1) / kAttnMinSplit;
  if (ns > cap) ns = cap;
  const int big = (n + max_len - 1) / max_len;
  if (ns < big) ns = big;
  return ns < 1 ? 1 : ns;
}
// positions per warp of a split (the split is `warps` times that)
__host__ __device__ inline int attn_warp_len(int n, int warps) {
  const int ns = attn_nsplit(n, warps);
  const int per = (n + ns - 1) / ns;
  return (per + warps - 1) / warps;
}

struct AttnArgs {
  const float *q;                  // [nseq][n_head][head_dim]
  const int *seq;                  // cache sequence of query b (NULL: b)
  const void *kcache, *vcache;
  int64_t seq_stride, head_stride;
  const int *npos;                 // positions to attend per sequence (device)
  float *out;                      // [nseq][n_head][head_dim]
  float *partial;                  // [nseq * n_kv][nsplit][group * (head_dim + 2)] scratch (nsplit >= attn_nsplit(npos))
  int *counters;                   // [nseq * n_kv], zero between launches
  unsigned *status;
  float scale;
  int n_head, n_kv, head_dim, nseq, nsplit;
  // fused decode (every query a different sequence, at its position npos - 1): the kernel does the
  // q/k/v post-processing of `post` itself (q is then unused) -- the roped queries stay in shared
  // memory and the last context split appends the key / value row before reading it
  int fused;
  QkvPostArgs post;
  KvPages pages;                   // paged caches (pages.table != NULL; not with `fused`): row b of the table is query b's
};

cudaError_t launch_qkv_post(const QkvPostArgs &a, cudaStream_t s, bool pdl);
bool attn_supported(int head_dim, int group);
cudaError_t launch_attn(const AttnArgs &a, bool f16, cudaStream_t s, bool pdl);
cudaError_t launch_kv_block_copy(void *dst, int64_t dst_row, int64_t dst_blk, const void *src, int64_t src_row,
                                 int64_t src_blk, int64_t row_bytes, int rows, int nblk, int num_sms, cudaStream_t s);
cudaError_t launch_kv_convert(float *stage, void *cache, int n, int n_kv, int hd, int64_t head_stride, bool f16, int dir,
                              cudaStream_t s);

cudaError_t launch_rmsnorm_quant(const float *x, const float *w, int n, int ntok, double eps, float *xb, int8_t *xq, float *xd,
                                 int32_t *xs, cudaStream_t s, bool pdl);
cudaError_t launch_swiglu_quant(const float *gate, const float *up, int n, int ntok, int64_t stride, float *hb, int8_t *xq,
                                float *xd, int32_t *xs, cudaStream_t s, bool pdl);
cudaError_t launch_embed(const DevMatrix &m, const int32_t *tokens, int ntok, float *x, cudaStream_t s, bool pdl);
// argmax in two stages over kArgmaxChunks chunks per token; pv / pi: [ntok][kArgmaxChunks] scratch
constexpr int kArgmaxChunks = 64;
cudaError_t launch_argmax(const float *logits, int64_t n, int64_t stride, int ntok, int32_t *out, float *pv, int *pi,
                          cudaStream_t s, bool pdl);
// the k best logits per row (sample.cu): kTopkChunks chunks of at most kTopkSmem bytes (value + index) each, k <= kTopkMax,
// at most kTopkMaxPen penalised tokens; pv / pi: [ntok][kTopkChunks][k] scratch; out: [ntok][k]
constexpr int kTopkChunks = 64;              // <= 64: the merge warp owns two lists per lane
constexpr int kTopkMax = 256;
constexpr int kTopkMaxPen = 4096;
constexpr int64_t kTopkSmem = 40 * 1024;
cudaError_t launch_topk(const float *logits, int64_t n, int64_t stride, int ntok, int k, const int32_t *pen_tok,
                        const int32_t *pen_cnt, int n_pen, double rp, double freq, double pres, float *pv, int *pi,
                        float *out_v, int32_t *out_i, cudaStream_t s);
cudaError_t launch_advance(const int32_t *arg, int n, int32_t *tok, int32_t *pos, int32_t *npos, int32_t *out,
                           int32_t *step, cudaStream_t s, bool pdl);

cudaError_t repack_upload(const DevMatrix &m, const void *raw_dev, cudaStream_t s);

// Tensor-core GEMM for k-quant matrices and 64 or more tokens (gemm_kq.cu).  The activation is
// first turned into f16 tiles (launch_gemm_prep, gemm_b_bytes of scratch), then launch_gemm_kq
// computes y[t][r] (+ y_add) for all tokens.  launch_kq_bound writes an upper bound of the
// matrix's |dequantized value| (as f32 bits); a finite bound qualifies the matrix, and
// gemm_weight_scale(bound) is the power of two that brings its values just under 2^15 in f16.
// Below kGemmMinTokens (zllm_mm and model passes alike) the batched GEMV streams the weights faster
// and keeps every token's bits equal to a single-token pass.
constexpr int kGemmMinTokens = 64;
// An F16 output head of 16 or more logit rows runs on the tensor-core GEMM (f32 activation as f16
// hi / lo, ~1e-6 of the largest logit from the CUDA-core GEMV, whose f32 FMA chain it replaces).
constexpr int kHeadGemmMinRows = 16;
float gemm_weight_scale(float bound);
int64_t gemm_tokens_pad(int ntok);
size_t gemm_b_bytes(int64_t k, int ntok);
bool gemm_kq_supported(const DevMatrix &m);
cudaError_t launch_kq_bound(const DevMatrix &m, unsigned *out, cudaStream_t s);
cudaError_t launch_gemm_prep(const ActView &act, int ntok, void *bbuf, cudaStream_t s);
cudaError_t launch_gemm_kq(const DevMatrix &m, const void *bbuf, int ntok, float *y, int64_t y_stride, const float *y_add,
                           float wscale, unsigned *status, cudaStream_t s, bool swiglu = false);
// The exact-A variant of the same GEMM (weights dequantized exactly into f16, two MMAs per slice,
// per-super-block scaling in TMEM): launch_kx_info writes (bits of max |dmin| * 63, max |Q6_K scale|)
// of a matrix; Q4_K / Q5_K with finite scales always qualify, Q6_K when every |scale| <= 64.  The
// activation goes through launch_gemm_prep_kx (gemm_bx_bytes of scratch, which also holds the
// split-K partial sums: kx_splits CTAs share an output tile when the tiles alone would leave SMs
// idle); mscale is the power of two gemm_weight_scale gives for the dmin bound.
cudaError_t launch_kx_info(const DevMatrix &m, unsigned *out, cudaStream_t s);
int kx_splits(int64_t rows, int ntok, int64_t k);
size_t gemm_bx_bytes(int64_t k, int ntok, int type, int64_t rows);
cudaError_t launch_gemm_prep_kx(const ActView &act, int ntok, int type, int64_t rows, void *bbuf, cudaStream_t s);
cudaError_t launch_gemm_kx(const DevMatrix &m, void *bbuf, int ntok, float *y, int64_t y_stride, const float *y_add,
                           float mscale, unsigned *status, cudaStream_t s, bool swiglu = false);
// Tensor-parallel collectives (tp.cu): NCCL opened at run time.  Return 0 / cudaSuccess, else set *why.
size_t tp_unique_id_bytes();
int tp_unique_id(void *out, size_t bytes, const char **why);
int tp_comm_init(void **comm, int rank, int size, const void *unique_id, const char **why);
void tp_comm_destroy(void *comm);
cudaError_t tp_allreduce_sum(void *comm, float *buf, size_t count, cudaStream_t s, const char **why);
// One-shot all-reduce over NVLink peer memory (CUDA IPC between the ranks' processes), for vectors
// of at most `cap` floats; tp_ar_setup returns -1 (and every rank keeps NCCL) when a peer cannot be
// mapped.  Collective: every rank calls setup and destroy.
struct TpAr;
int tp_ar_setup(void *comm, int rank, int size, int64_t cap, cudaStream_t s, TpAr **out, const char **why);
cudaError_t tp_ar_sum(TpAr *ar, float *x, int64_t n, unsigned *status, cudaStream_t s, bool pdl = false);
void tp_ar_destroy(TpAr *ar, void *comm, cudaStream_t s);
// Vocab-split output head: every rank's logits slice (padded to vpad columns) to every rank, then
// the slices in vocab order (rank r holds rows [r V / size, (r + 1) V / size)).
cudaError_t tp_allgather(void *comm, const float *send, float *recv, size_t count, cudaStream_t s, const char **why);
cudaError_t launch_vocab_gather(const float *recv, int nl, int64_t vpad, int64_t V, int size, float *logits,
                                cudaStream_t s);
// The all-reduce kernel against a phantom peer that never stamps: its bounded wait expires.
int tp_ar_phantom_wait(unsigned *status, cudaStream_t s, const char **why);

// An F16 matrix (the output head) pre-tiled once for the same kernel, against f32 activations
// x [ntok][ldx] split into f16 hi / lo tiles (two MMAs, f32 accumulation): y[t][r] = W[r] . x_t.
size_t gemm_f16_tiles_bytes(int64_t rows, int64_t k);
cudaError_t launch_gemm_tile_f16(const DevMatrix &m, void *tiles, cudaStream_t s);
cudaError_t launch_gemm_prep_f32(const float *x, int64_t ldx, int64_t k, int ntok, void *bbuf, cudaStream_t s);
cudaError_t launch_gemm_f16_tiled(const void *tiles, int64_t rows, int64_t k, const void *bbuf, int ntok, float *y,
                                  int64_t y_stride, unsigned *status, cudaStream_t s);
// f16 x f16 -> f32 on the same kernel: D[j][i] = sum_k A[i][k] B[j][k] (row-major, k % 64 == 0)
size_t gemm_f16_scratch_bytes(int64_t m, int64_t n, int64_t k);
cudaError_t launch_gemm_f16(const uint16_t *A, const uint16_t *B, int64_t m, int64_t n, int64_t k, float *D, void *scratch,
                            unsigned *status, cudaStream_t s);
// k-quant rows src[i] -> dst row dst_row0 + i * dst_step (same type and width)
cudaError_t launch_kq_copy_rows(const DevMatrix &dst, int64_t dst_row0, int64_t dst_step, const DevMatrix &src,
                                cudaStream_t s);
cudaError_t launch_quantize(const float *x, int64_t k, int ntok, int8_t *xq, float *xd, int32_t *xs, unsigned *status,
                            cudaStream_t s, bool pdl);
// y[t*y_stride + r] = (y_add ? y_add[t*y_stride + r] : 0) + W[r] . act_t   for t < ntok
cudaError_t launch_gemv(const DevMatrix &m, const ActView &a, int ntok, float *y, int64_t y_stride, const float *y_add,
                        unsigned *status, int num_sms, cudaStream_t s, bool pdl, const char **why);
bool plan_gemv(const DevMatrix &m, int num_sms, GemvPlan *p, const char **why);
// k-quant (Q4_K / Q5_K / Q6_K) GEMV on the tensor cores (gemv_kq.cu).  With one token, act.xq may be
// NULL and act.x the f32 activation: the kernel quantizes it itself.
bool kq_type(int type);
// F16 / BF16 / F32 GEMV (gemv_float.cu)
bool float_type(int type);
cudaError_t launch_gemv_float(const DevMatrix &m, const ActView &a, int ntok, float *y, int64_t y_stride,
                              const float *y_add, int num_sms, cudaStream_t s, bool pdl, const char **why);
cudaError_t launch_gemv_kq(const DevMatrix &m, const ActView &a, int ntok, float *y, int64_t y_stride,
                           const float *y_add, unsigned *status, int num_sms, cudaStream_t s, bool pdl, const char **why);
// Work fused into a k-quant GEMV: norm_w -- RMSNorm of the f32 activation before the in-kernel
// quantization (one token); swiglu -- rows are interleaved (gate, up) pairs and y receives
// f32(silu(gate) * up) per pair.
struct GemvFuse {
  const float *norm_w = nullptr;
  double eps = 0.0;
  bool swiglu = false;
};
cudaError_t launch_gemv_kq_ex(const DevMatrix &m, const ActView &a, int ntok, float *y, int64_t y_stride,
                              const float *y_add, const GemvFuse &fz, unsigned *status, int num_sms, cudaStream_t s,
                              bool pdl, const char **why);

}  // namespace zllm
