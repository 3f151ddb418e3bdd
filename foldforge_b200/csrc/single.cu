// Single track of the Pairformer block: attention with pair bias and the single
// transition (c_s = 384, 16 heads x 24, factor 4). Both are small next to the pair ops
// (about 1% of a block's flops at N = 512) and are composed from the library's tcgen05
// GEMM and LayerNorm launchers plus one attention kernel:
//
// attention with pair bias (legacy/pairformer.py:204-226, legacy/transformer.py:88-133):
//   pb[h, b, i, j] = W_pb (gamma_pair * LNhat(z[b, i, j]))     LayerNorm + GEMM (16 rows)
//   y = LN(s);  [q | k | v | g] = y W^T + [b_q | 0 | 0 | 0]     GEMM (N = 1536)
//   o = softmax_j(q_i . k_j / sqrt(24) + pb[i, j, h] (+ extra[h, i, j]), key mask) v_j
//   s' = s + W_o (sigmoid(g + gate_bias) * o)                    GEMM with residual epilogue
// single transition: s' = s + W_sq (silu(W_a LN(s)) * W_b LN(s))  (SwiGLU GEMM epilogue)
#include "abi_util.h"
#include "common.cuh"
#include "kernels.h"

namespace ffb {
namespace {

constexpr int kCs = 384;
constexpr int kHs = 16;
constexpr int kDs = 24;
constexpr int kCz = 128;

// ---------------------------------------------------------------- weight conversion
// dst[r, :] = bf16(src[perm(r), :]); perm interleaves a / b halves in blocks of 16 rows
// when `interleave` is set (the SwiGLU epilogue layout), identity otherwise.
__global__ void to_bf16_rows_kernel(const float* __restrict__ a, const float* __restrict__ b, int rows_each, int cols,
                                    int interleave, __nv_bfloat16* __restrict__ dst) {
  const int64_t total = static_cast<int64_t>(interleave ? 2 * rows_each : rows_each) * cols;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / cols);
    const int c = static_cast<int>(i % cols);
    float v;
    if (interleave) {
      const int blk = r / 32, within = r % 32;
      const int src_row = blk * 16 + (within % 16);
      v = (within < 16 ? a : b)[static_cast<int64_t>(src_row) * cols + c];
    } else {
      v = a[static_cast<int64_t>(r) * cols + c];
    }
    dst[i] = __float2bfloat16_rn(v);
  }
}

int to_bf16(const float* a, const float* b, int rows_each, int cols, int interleave, void* dst, cudaStream_t st) {
  to_bf16_rows_kernel<<<256, 256, 0, st>>>(a, b, rows_each, cols, interleave, static_cast<__nv_bfloat16*>(dst));
  return static_cast<int>(cudaGetLastError());
}

// ---------------------------------------------------------------- attention kernel
// A CTA per (batch, head, 32 queries), 4 warps. Lane = query; warp w takes keys w*16 ..
// w*16+15 of every 64-key chunk, which is staged once per CTA in shared memory: keys and
// values (fp32) and the pair-bias tile [32 q][64 k] (head-major bias, coalesced rows, padded
// rows so that lanes reading one key hit distinct banks). Each warp keeps a private exact
// online softmax per query; the four partial states are merged at the end. Masked keys get
// the reference's REPLACED logit -1e9, so a row whose keys are all masked averages
// uniformly; keys past N do not exist.
constexpr int kQ = 32;        // queries per CTA
constexpr int kKC = 64;       // keys per staged chunk
constexpr int kWarps = 4;
constexpr int kKPW = kKC / kWarps;

__global__ void __launch_bounds__(kQ * kWarps) single_attention_kernel(
    const __nv_bfloat16* __restrict__ qkvg, const float* __restrict__ pair_bias_hm, const void* __restrict__ extra,
    int extra_f32, const uint8_t* __restrict__ mask, float gate_bias, __nv_bfloat16* __restrict__ out, int B, int N) {
  __shared__ float ks[kKC][kDs];
  __shared__ float vs[kKC][kDs];
  __shared__ float bias[kQ][kKC + 1];
  __shared__ float keep[kKC];
  __shared__ float part[kWarps][kQ][kDs + 2];
  const int qblocks = (N + kQ - 1) / kQ;
  const int h = blockIdx.x % kHs;
  const int qb = (blockIdx.x / kHs) % qblocks;
  const int b = blockIdx.x / (kHs * qblocks);
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  const int i = qb * kQ + lane;
  const int row = i < N ? i : N - 1;
  const __nv_bfloat16* row_i = qkvg + (static_cast<int64_t>(b) * N + row) * (4 * kCs);
  const float scale = rsqrtf(static_cast<float>(kDs));
  float q[kDs];
#pragma unroll
  for (int d = 0; d < kDs; ++d) q[d] = __bfloat162float(row_i[h * kDs + d]) * scale;
  float m = -1.0e30f, l = 0.f;
  float o[kDs];
#pragma unroll
  for (int d = 0; d < kDs; ++d) o[d] = 0.f;
  // head-major bias: [h][b][i][j]
  const float* pb = pair_bias_hm + (static_cast<int64_t>(h) * B + b) * static_cast<int64_t>(N) * N;
  for (int j0 = 0; j0 < N; j0 += kKC) {
    const int nk = N - j0 < kKC ? N - j0 : kKC;
    __syncthreads();
    for (int e = threadIdx.x; e < kKC * kDs; e += kQ * kWarps) {
      const int j = e / kDs, d = e % kDs;
      float kv = 0.f, vv = 0.f;
      if (j < nk) {
        const __nv_bfloat16* rj = qkvg + (static_cast<int64_t>(b) * N + j0 + j) * (4 * kCs) + h * kDs + d;
        kv = __bfloat162float(rj[kCs]);
        vv = __bfloat162float(rj[2 * kCs]);
      }
      ks[j][d] = kv;
      vs[j][d] = vv;
    }
    for (int e = threadIdx.x; e < kQ * kKC; e += kQ * kWarps) {
      const int qq = e / kKC, j = e % kKC;
      const int ii = qb * kQ + qq;
      float v = 0.f;
      if (ii < N && j < nk) {
        v = pb[static_cast<int64_t>(ii) * N + j0 + j];
        if (extra != nullptr) {
          const int64_t x = ((static_cast<int64_t>(b) * kHs + h) * N + ii) * N + j0 + j;
          v += extra_f32 ? static_cast<const float*>(extra)[x]
                         : __bfloat162float(static_cast<const __nv_bfloat16*>(extra)[x]);
        }
      }
      bias[qq][j] = v;
    }
    for (int j = threadIdx.x; j < kKC; j += kQ * kWarps)
      keep[j] = (j < nk) ? (mask[static_cast<int64_t>(b) * N + j0 + j] ? 1.f : 0.f) : -1.f;
    __syncthreads();
#pragma unroll 2
    for (int jj = 0; jj < kKPW; ++jj) {
      const int j = warp * kKPW + jj;
      const float kp = keep[j];
      if (kp < 0.f) continue;  // past N (uniform across the warp)
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
      for (int d = 0; d < kDs; d += 4) {
        a0 += q[d] * ks[j][d];
        a1 += q[d + 1] * ks[j][d + 1];
        a2 += q[d + 2] * ks[j][d + 2];
        a3 += q[d + 3] * ks[j][d + 3];
      }
      float x = (a0 + a1) + (a2 + a3) + bias[lane][j];
      if (kp == 0.f) x = -1.0e9f;
      if (x > m) {
        const float alpha = __expf(m - x);
        l *= alpha;
#pragma unroll
        for (int d = 0; d < kDs; ++d) o[d] *= alpha;
        m = x;
      }
      const float p = __expf(x - m);
      l += p;
#pragma unroll
      for (int d = 0; d < kDs; ++d) o[d] += p * vs[j][d];
    }
  }
  // merge the four warps' partial softmax states per query
#pragma unroll
  for (int d = 0; d < kDs; ++d) part[warp][lane][d] = o[d];
  part[warp][lane][kDs] = m;
  part[warp][lane][kDs + 1] = l;
  __syncthreads();
  if (warp != 0 || i >= N) return;
  float mm = -1.0e30f;
  for (int w = 0; w < kWarps; ++w)
    if (part[w][lane][kDs + 1] > 0.f) mm = fmaxf(mm, part[w][lane][kDs]);
  float ll = 0.f, acc[kDs];
#pragma unroll
  for (int d = 0; d < kDs; ++d) acc[d] = 0.f;
  for (int w = 0; w < kWarps; ++w) {
    const float lw = part[w][lane][kDs + 1];
    if (lw <= 0.f) continue;
    const float f = __expf(part[w][lane][kDs] - mm);
    ll += lw * f;
#pragma unroll
    for (int d = 0; d < kDs; ++d) acc[d] += part[w][lane][d] * f;
  }
  const float inv = 1.0f / ll;
  __nv_bfloat16* dst = out + (static_cast<int64_t>(b) * N + i) * kCs + h * kDs;
#pragma unroll
  for (int d = 0; d < kDs; ++d) {
    const float g = __bfloat162float(row_i[3 * kCs + h * kDs + d]) + gate_bias;
    dst[d] = __float2bfloat16_rn(acc[d] * inv * sigmoidf_(g));
  }
}

// ---------------------------------------------------------------- helpers
int gemm(const void* a, const void* w, void* d, int m, int n, int k, int d_f32, const float* bias, int epilogue,
         const void* residual, const uint8_t* row_mask, const DeviceInfo& info, cudaStream_t stream) {
  const int bn = n >= 256 ? 256 : 128;
  CUtensorMap ma, mb;
  const uint64_t adims[3] = {static_cast<uint64_t>(k), static_cast<uint64_t>(m), 1};
  const uint64_t astr[2] = {static_cast<uint64_t>(k) * 2, static_cast<uint64_t>(k) * m * 2};
  const uint32_t abox[3] = {64, 128, 1};
  int st = make_map(&ma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a, adims, astr, abox, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  const uint64_t bdims[3] = {static_cast<uint64_t>(k), static_cast<uint64_t>(n), 1};
  const uint64_t bstr[2] = {static_cast<uint64_t>(k) * 2, static_cast<uint64_t>(k) * n * 2};
  const uint32_t bbox[3] = {64, static_cast<uint32_t>(bn), 1};
  st = make_map(&mb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, w, bdims, bstr, bbox, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  GemmParams p;
  p.M = m;
  p.N = n;
  p.K = k;
  p.batch = 1;
  p.D = d;
  p.ldd = epilogue == kEpiSwiGLU ? n / 2 : n;
  p.batch_stride_d = 0;
  p.d_is_f32 = d_f32;
  p.epilogue = epilogue;
  p.bias = bias;
  p.residual = residual;
  p.row_mask = row_mask;
  p.err = info.err;
  return cuda_status(launch_gemm_nt(ma, mb, p, bn, info.num_sms, stream), "single-track gemm");
}

size_t a256(size_t x) { return (x + 255) / 256 * 256; }

// packed attention-with-pair-bias image
struct ApbLayout {
  size_t w_qkvg, b_qkvg, w_o, w_pb, ln_s_w, ln_s_b, ln_p_w, total;
};
ApbLayout apb_layout() {
  ApbLayout L;
  size_t o = 0;
  L.w_qkvg = o;  o = a256(o + static_cast<size_t>(4 * kCs) * kCs * 2);
  L.b_qkvg = o;  o = a256(o + 4 * kCs * 4);
  L.w_o = o;     o = a256(o + static_cast<size_t>(kCs) * kCs * 2);
  L.w_pb = o;    o = a256(o + kHs * kCz * 2);
  L.ln_s_w = o;  o = a256(o + kCs * 4);
  L.ln_s_b = o;  o = a256(o + kCs * 4);
  L.ln_p_w = o;  o = a256(o + kCz * 4);
  L.total = o;
  return L;
}

struct StLayout {
  size_t w_ab, w_sq, ln_w, ln_b, total;
};
StLayout st_layout() {
  StLayout L;
  size_t o = 0;
  L.w_ab = o;  o = a256(o + static_cast<size_t>(8 * kCs) * kCs * 2);
  L.w_sq = o;  o = a256(o + static_cast<size_t>(kCs) * 4 * kCs * 2);
  L.ln_w = o;  o = a256(o + kCs * 4);
  L.ln_b = o;  o = a256(o + kCs * 4);
  L.total = o;
  return L;
}

}  // namespace

size_t apb_packed_bytes() { return apb_layout().total; }

size_t apb_workspace_bytes(int B, int N) {
  const size_t P = static_cast<size_t>(B) * N * N, T = static_cast<size_t>(B) * N;
  return a256(P * kCz * 2) + a256(P * kHs * 4) + a256(T * kCs * 2) + a256(T * 4 * kCs * 2) + a256(T * kCs * 2);
}

int apb_prepare(const ApbWeights& w, void* packed, cudaStream_t stream) {
  const ApbLayout L = apb_layout();
  uint8_t* img = static_cast<uint8_t*>(packed);
  int rc = static_cast<int>(cudaMemsetAsync(packed, 0, L.total, stream));
  const float* mats[4] = {w.to_query, w.to_key, w.to_value, w.to_gate};
  for (int i = 0; i < 4 && rc == 0; ++i)
    rc = to_bf16(mats[i], nullptr, kCs, kCs, 0, img + L.w_qkvg + static_cast<size_t>(i) * kCs * kCs * 2, stream);
  if (rc == 0) rc = static_cast<int>(cudaMemcpyAsync(img + L.b_qkvg, w.query_bias, kCs * 4, cudaMemcpyDeviceToDevice, stream));
  if (rc == 0) rc = to_bf16(w.to_out, nullptr, kCs, kCs, 0, img + L.w_o, stream);
  if (rc == 0) rc = to_bf16(w.to_bias, nullptr, kHs, kCz, 0, img + L.w_pb, stream);
  if (rc == 0) rc = static_cast<int>(cudaMemcpyAsync(img + L.ln_s_w, w.ln_single_w, kCs * 4, cudaMemcpyDeviceToDevice, stream));
  if (rc == 0) rc = static_cast<int>(cudaMemcpyAsync(img + L.ln_s_b, w.ln_single_b, kCs * 4, cudaMemcpyDeviceToDevice, stream));
  if (rc == 0) rc = static_cast<int>(cudaMemcpyAsync(img + L.ln_p_w, w.ln_pair_w, kCz * 4, cudaMemcpyDeviceToDevice, stream));
  return rc;
}

int apb_forward(const void* s, const void* z, const uint8_t* mask, const void* packed, const void* extra,
                int extra_f32, float gate_bias, void* out, void* workspace, int B, int N, int masked_zero,
                const DeviceInfo& info, cudaStream_t stream) {
  const ApbLayout L = apb_layout();
  const uint8_t* img = static_cast<const uint8_t*>(packed);
  const size_t P = static_cast<size_t>(B) * N * N, T = static_cast<size_t>(B) * N;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* zn = ws;
  float* pb = reinterpret_cast<float*>(ws + a256(P * kCz * 2));
  void* y = ws + a256(P * kCz * 2) + a256(P * kHs * 4);
  void* qkvg = static_cast<uint8_t*>(y) + a256(T * kCs * 2);
  void* gated = static_cast<uint8_t*>(qkvg) + a256(T * 4 * kCs * 2);
  int st = cuda_status(launch_layernorm(z, zn, reinterpret_cast<const float*>(img + L.ln_p_w), nullptr,
                                        static_cast<int64_t>(P), kCz, 1e-5f, 0, info.num_sms, stream),
                       "apb pair layernorm");
  if (st) return st;
  // head-major pair bias pb[h][p] = W_pb[h] . zn[p]: the weight is the A operand (16 rows;
  // the tile's other rows are zero-filled by TMA), the pairs are the N dimension
  st = gemm(img + L.w_pb, zn, pb, kHs, static_cast<int>(P), kCz, 1, nullptr, kEpiStore, nullptr, nullptr, info, stream);
  if (st) return st;
  st = cuda_status(launch_layernorm(s, y, reinterpret_cast<const float*>(img + L.ln_s_w),
                                    reinterpret_cast<const float*>(img + L.ln_s_b), static_cast<int64_t>(T), kCs,
                                    1e-5f, 0, info.num_sms, stream),
                   "apb single layernorm");
  if (st) return st;
  st = gemm(y, img + L.w_qkvg, qkvg, static_cast<int>(T), 4 * kCs, kCs, 0,
            reinterpret_cast<const float*>(img + L.b_qkvg), kEpiStore, nullptr, nullptr, info, stream);
  if (st) return st;
  const int ctas = B * kHs * ((N + kQ - 1) / kQ);
  single_attention_kernel<<<ctas, kQ * kWarps, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(qkvg), pb, extra, extra_f32, mask, gate_bias,
      static_cast<__nv_bfloat16*>(gated), B, N);
  st = cuda_status(static_cast<int>(cudaGetLastError()), "single attention launch");
  if (st) return st;
  return gemm(gated, img + L.w_o, out, static_cast<int>(T), kCs, kCs, 0, nullptr, kEpiResidual, s,
              masked_zero ? mask : nullptr, info, stream);
}

size_t single_transition_packed_bytes() { return st_layout().total; }

size_t single_transition_workspace_bytes(int B, int N) {
  const size_t T = static_cast<size_t>(B) * N;
  return a256(T * kCs * 2) + a256(T * 4 * kCs * 2);
}

int single_transition_prepare(const TransitionWeights& w, void* packed, cudaStream_t stream) {
  const StLayout L = st_layout();
  uint8_t* img = static_cast<uint8_t*>(packed);
  int rc = to_bf16(w.expand_a, w.expand_b, 4 * kCs, kCs, 1, img + L.w_ab, stream);
  if (rc == 0) rc = to_bf16(w.squeeze, nullptr, kCs, 4 * kCs, 0, img + L.w_sq, stream);
  if (rc == 0) rc = static_cast<int>(cudaMemcpyAsync(img + L.ln_w, w.ln_w, kCs * 4, cudaMemcpyDeviceToDevice, stream));
  if (rc == 0) rc = static_cast<int>(cudaMemcpyAsync(img + L.ln_b, w.ln_b, kCs * 4, cudaMemcpyDeviceToDevice, stream));
  return rc;
}

int single_transition_forward(const void* s, const uint8_t* mask, const void* packed, void* out, void* workspace,
                              int B, int N, int masked_zero, const DeviceInfo& info, cudaStream_t stream) {
  const StLayout L = st_layout();
  const uint8_t* img = static_cast<const uint8_t*>(packed);
  const size_t T = static_cast<size_t>(B) * N;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* y = ws;
  void* hid = ws + a256(T * kCs * 2);
  int st = cuda_status(launch_layernorm(s, y, reinterpret_cast<const float*>(img + L.ln_w),
                                        reinterpret_cast<const float*>(img + L.ln_b), static_cast<int64_t>(T), kCs,
                                        1e-5f, 0, info.num_sms, stream),
                       "single transition layernorm");
  if (st) return st;
  st = gemm(y, img + L.w_ab, hid, static_cast<int>(T), 8 * kCs, kCs, 0, nullptr, kEpiSwiGLU, nullptr, nullptr, info,
            stream);
  if (st) return st;
  return gemm(hid, img + L.w_sq, out, static_cast<int>(T), kCs, 4 * kCs, 0, nullptr, kEpiResidual, s,
              masked_zero ? mask : nullptr, info, stream);
}

}  // namespace ffb
