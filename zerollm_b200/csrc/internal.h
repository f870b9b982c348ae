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
// bytes of one device row (repacked layout, padded to 16)
int64_t dev_row_stride(int type, int64_t cols);

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

cudaError_t repack_upload(const DevMatrix &m, const void *raw_dev, cudaStream_t s);
cudaError_t launch_quantize(const float *x, int64_t k, int ntok, int8_t *xq, float *xd, int32_t *xs, unsigned *status,
                            cudaStream_t s, bool pdl);
// y[t*y_stride + r] = (y_add ? y_add[t*y_stride + r] : 0) + W[r] . act_t   for t < ntok
cudaError_t launch_gemv(const DevMatrix &m, const ActView &a, int ntok, float *y, int64_t y_stride, const float *y_add,
                        unsigned *status, int num_sms, cudaStream_t s, bool pdl, const char **why);
bool plan_gemv(const DevMatrix &m, int num_sms, GemvPlan *p, const char **why);

}  // namespace zllm
