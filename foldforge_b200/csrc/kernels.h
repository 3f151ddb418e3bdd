// Internal launch interface between the C-ABI layer (abi.cu) and the kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ffb {

enum GemmEpilogue : int {
  kEpiStore = 0,     // D = acc (+ bias[n])
  kEpiResidual = 1,  // D = R + (acc (+ bias[n])) * row_mask[m]
  kEpiSwiGLU = 2,    // D[:, h] = silu(a_h) * b_h from an a/b-interleaved weight
};

struct GemmParams {
  int M, N, K, batch;
  void* D;
  int64_t ldd;
  int64_t batch_stride_d;
  int d_is_f32;
  int epilogue;
  const float* bias;
  const void* residual;
  const uint8_t* row_mask;
  int* err;
  int tma_store;  // set by launch_gemm_nt: the bf16 store epilogue goes through TMA stores
  const float* row_scale = nullptr;  // (acc + bias) times row_scale[m] (store and residual epilogues)
  // residual epilogue only: acc times sigmoid(col_gate[(m % gate_rows) * N + n]) before the add
  const float* col_gate = nullptr;
  int gate_rows = 0;
  // two-level batch: batch index b = outer * batch_inner + inner; the operand maps are then 4-D
  // ({K, rows, inner, outer}) and D's offset is inner * batch_stride_d + outer * batch_stride_d2
  int batch_inner = 0;
  int64_t batch_stride_d2 = 0;
};

size_t gemm_smem_bytes(int bn);
int launch_gemm_nt(const CUtensorMap& map_a, const CUtensorMap& map_b, const GemmParams& p, int bn, int num_sms,
                   cudaStream_t stream);

// LayerNorm over the last axis of `rows` rows of `c` channels.
int launch_layernorm(const void* x, void* y, const float* gamma, const float* beta, int64_t rows, int c, float eps,
                     int is_f32, int num_sms, cudaStream_t stream);

// Packs an fp32 [rows, k] weight (optionally times diag(gamma)) into the K-major SW128
// shared-memory image at row offset `row_offset` of an image with `image_rows` rows;
// writes wsum / bias (W beta) per row when the pointers are non-null.
int launch_pack_weight(const float* w, int rows, int k, const float* gamma, const float* beta, uint8_t* image,
                       int row_offset, int image_rows, float* wsum, float* bias, cudaStream_t stream,
                       float scale = 1.0f);

struct DeviceInfo;

// ---- triangle multiplication (c_z = hidden = 128)
struct TriMulWeights {
  const float *ln_w, *ln_b, *ln_out_w, *ln_out_b;
  const float *to_left, *to_right, *to_left_gate, *to_right_gate, *to_out, *to_gate;
};
size_t trimul_packed_bytes();
size_t trimul_workspace_bytes(int B, int N);
int trimul_prepare(const TriMulWeights& w, void* packed, cudaStream_t stream);
int trimul_forward(const void* z, const uint8_t* mask, const void* packed, void* out, void* workspace, int B, int N,
                   int outgoing, int masked_zero, int stages, const DeviceInfo& info, cudaStream_t stream);
int trimul_shard_proj(const void* z, const uint8_t* mask, const void* packed, void* left, void* right, void* zstats,
                      int R, int N, int row0, const DeviceInfo& info, cudaStream_t stream);
int trimul_channel_contract(const void* left, const void* right, void* u, int C, int N, const DeviceInfo& info,
                            cudaStream_t stream);
int trimul_shard_contract(const void* left, const void* right_all, void* u, int R, int N, const DeviceInfo& info,
                          cudaStream_t stream);
int trimul_shard_out(const void* z, const uint8_t* mask, const void* packed, const void* u, const void* zstats,
                     void* ustats, void* out, int R, int N, int row0, int masked_zero, const DeviceInfo& info,
                     cudaStream_t stream);

// ---- triangle attention (c_z = 128, 4 heads x 32)
struct TriAttnWeights {
  const float *ln_w, *ln_b, *to_bias, *to_query, *to_key, *to_value, *to_gate, *to_out;
};
size_t triattn_packed_bytes();
size_t triattn_workspace_bytes(int B, int N);
int triattn_prepare(const TriAttnWeights& w, void* packed, cudaStream_t stream);
int triattn_forward(const void* z, const uint8_t* mask, const void* packed, void* out, void* workspace, int B, int N,
                    int starting, int masked_zero, int stages, const DeviceInfo& info, cudaStream_t stream);
int triattn_shard_proj(const void* z, const void* packed, void* q, void* k, void* vt, void* bias_rows, int R, int N,
                       const DeviceInfo& info, cudaStream_t stream);
int triattn_shard_attn(const void* q, const void* k, const void* vt, const void* bias_all, const uint8_t* mask, void* o,
                       int R, int N, int row0, const DeviceInfo& info, cudaStream_t stream);
int triattn_shard_out(const void* z, const uint8_t* mask, const void* packed, const void* o, void* out, int R, int N,
                      int row0, int masked_zero, const DeviceInfo& info, cudaStream_t stream);

// ---- pair transition (c_z = 128, n = 4)
struct TransitionWeights {
  const float *ln_w, *ln_b, *expand_a, *expand_b, *squeeze;
};
size_t transition_packed_bytes();
int transition_prepare(const TransitionWeights& w, void* packed, cudaStream_t stream);
int transition_forward(const void* z, const uint8_t* mask, const void* packed, void* out, int B, int N,
                       int masked_zero, const DeviceInfo& info, cudaStream_t stream);

// ---- single track (c_s = 384, 16 heads x 24, c_z = 128)
struct ApbWeights {
  const float *ln_single_w, *ln_single_b, *to_query, *query_bias, *to_key, *to_value, *to_gate, *to_out;
  const float *ln_pair_w, *to_bias;
};
size_t apb_packed_bytes();
size_t apb_workspace_bytes(int B, int N);
int apb_prepare(const ApbWeights& w, void* packed, cudaStream_t stream);
int apb_forward(const void* s, const void* z, const uint8_t* mask, const void* packed, const void* extra,
                int extra_f32, float gate_bias, void* out, void* workspace, int B, int N, int masked_zero,
                const DeviceInfo& info, cudaStream_t stream);
int apb_shard_pair_bias(const void* z, const void* packed, void* pb_rows, int R, int N, const DeviceInfo& info,
                        cudaStream_t stream);
// The 16-head pair bias pb[h * pb_h + row * pb_r + col] = W'[h] . z[pair] - folded LayerNorm,
// for the `rows` x N pairs of z (bf16, 128 channels), from a weight image w_img (the SW128
// image of W diag(gamma), 16 rows x 128) and its row sums wsum.
int pair_bias16(const void* z, const uint8_t* w_img, const float* wsum, float* pb, int64_t rows, int N, int64_t pb_h,
                int64_t pb_r, const DeviceInfo& info, cudaStream_t stream);
size_t apb_single_workspace_bytes(int N);
int apb_shard_single_rows(const void* s, const uint8_t* mask, const void* packed, const void* pb_rows, float gate_bias,
                          void* out_rows, void* workspace, int N, int row0, int R, int masked_zero,
                          const DeviceInfo& info, cudaStream_t stream);
int apb_shard_single(const void* s, const uint8_t* mask, const void* packed, const void* pb_all, const void* extra,
                     int extra_f32, float gate_bias, void* out, void* workspace, int N, int masked_zero,
                     const DeviceInfo& info, cudaStream_t stream);
int transition_shard_forward(const void* z, const uint8_t* mask, const void* packed, void* out, int R, int N, int row0,
                             int masked_zero, const DeviceInfo& info, cudaStream_t stream);
size_t single_transition_packed_bytes();
size_t single_transition_workspace_bytes(int B, int N);
int single_transition_prepare(const TransitionWeights& w, void* packed, cudaStream_t stream);
int single_transition_forward(const void* s, const uint8_t* mask, const void* packed, void* out, void* workspace,
                              int B, int N, int masked_zero, const DeviceInfo& info, cudaStream_t stream);

// ---- the fp32 / any-width path (generic.cu); weights in the engine's [out, in] layout
struct GenericTriMulWeights {
  const float *ln_w, *ln_b, *ln_out_w, *ln_out_b, *to_left, *to_right, *to_left_gate, *to_right_gate, *to_out,
      *to_gate;
};
struct GenericTriAttnWeights {
  const float *ln_w, *ln_b, *to_bias, *to_query, *to_key, *to_value, *to_gate, *to_out;
};
struct GenericTransitionWeights {
  const float *ln_w, *ln_b, *expand_a, *expand_b, *squeeze;
};
struct GenericApbWeights {
  const float *ln_single_w, *ln_single_b, *to_query, *to_query_b, *to_key, *to_value, *to_gate, *to_out, *ln_pair_w,
      *to_bias;
};
size_t generic_trimul_workspace(int B, int N, int c, int h);
int generic_trimul(const float* z, const uint8_t* mask, const GenericTriMulWeights& w, float* out, void* workspace,
                   int B, int N, int c, int h, int outgoing, int masked_zero, cudaStream_t stream);
size_t generic_triattn_workspace(int B, int N, int c, int H, int d);
int generic_triattn(const float* z, const uint8_t* mask, const GenericTriAttnWeights& w, float* out, void* workspace,
                    int B, int N, int c, int H, int d, int starting, int masked_zero, cudaStream_t stream);
size_t generic_transition_workspace(int64_t rows, int c, int n);
int generic_transition(const float* x, const uint8_t* mask, const GenericTransitionWeights& w, float* out,
                       void* workspace, int64_t rows, int c, int n, int mask_kind, int mask_n, cudaStream_t stream);
size_t generic_apb_workspace(int B, int N, int cs, int cz, int H);
int generic_apb(const float* s, const float* z, const uint8_t* mask, const GenericApbWeights& w, const float* extra,
                float* out, void* workspace, int B, int N, int cs, int cz, int H, float gate_bias, int masked_zero,
                cudaStream_t stream);

}  // namespace ffb

