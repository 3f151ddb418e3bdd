// Weight preparation: fp32 master weights -> bf16 tensor-core operands.
//
// A LayerNorm followed by a projection, W (gamma * xhat + beta), is applied to the RAW
// activation x as  rstd * (W' x - mean * wsum) + bias  with
//   W'   = bf16(W diag(gamma))       the MMA operand,
//   wsum = sum_k W'[n, k]            (of the bf16-rounded W', so the subtraction is exact
//                                     with respect to what the tensor core multiplied),
//   bias = W beta                    (fp32),
// so the kernels feed raw bf16 activations straight from TMA to the tensor core and the
// normalisation costs two FMAs per output in the epilogue.
//
// The operand is written in the shared-memory image the kernels use: K-major, 64-column
// (128-byte) blocks of `rows` rows each, 16-byte chunks XOR-swizzled by (row % 8). A
// kernel copies the image linearly into 1024-byte aligned shared memory.
#include "common.cuh"
#include "kernels.h"

namespace ffb {
namespace {

__global__ void pack_weight_kernel(const float* __restrict__ w, int rows, int k, const float* __restrict__ gamma,
                                   const float* __restrict__ beta, uint8_t* __restrict__ image, int row_offset,
                                   int image_rows, float* __restrict__ wsum, float* __restrict__ bias, float scale) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const float* wr = w + static_cast<int64_t>(r) * k;
  float s = 0.f, bsum = 0.f;
  const int dst_row = row_offset + r;
  for (int c = 0; c < k; ++c) {
    const float g = gamma ? gamma[c] : 1.0f;
    const __nv_bfloat16 q = __float2bfloat16_rn(wr[c] * g * scale);
    s += __bfloat162float(q);
    if (beta) bsum += wr[c] * beta[c];
    const int kb = c / 64;
    uint8_t* block = image + static_cast<int64_t>(kb) * image_rows * 128;
    *reinterpret_cast<__nv_bfloat16*>(block + sw128_offset(dst_row, c % 64)) = q;
  }
  if (wsum) wsum[dst_row] = s;
  if (bias) bias[dst_row] = bsum * scale;
}

}  // namespace

int launch_pack_weight(const float* w, int rows, int k, const float* gamma, const float* beta, uint8_t* image,
                       int row_offset, int image_rows, float* wsum, float* bias, cudaStream_t stream, float scale) {
  pack_weight_kernel<<<(rows + 127) / 128, 128, 0, stream>>>(w, rows, k, gamma, beta, image, row_offset, image_rows,
                                                             wsum, bias, scale);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace ffb
