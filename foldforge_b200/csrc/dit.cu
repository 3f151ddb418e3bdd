// AF3's token diffusion transformer block (TokenDiT: c = 768, 16 heads x 48, conditioning 384,
// pair 128, SwiGLU factor 2), bf16 activations, fp32 accumulation
// (legacy/transformer.py:28-294, modules/dense/diffusion_transformer.py:47-404):
//   a  = sigmoid(W_s1 LN_c1(cond) + b_s1) * LN(x) + W_b1 LN_c1(cond)
//   o  = softmax_k(q_i . k_k / sqrt(48) + P_h[i, k], masked keys -> -1e9) v_k,  [q|k|v] = W a (+ b_q)
//   x += sigmoid(W_z1 cond + b_z1) * W_o (sigmoid(W_g a) * o)
//   a2 = sigmoid(W_s2 LN_c2(cond) + b_s2) * LN(x) + W_b2 LN_c2(cond)
//   x += sigmoid(W_z2 cond + b_z2) * W_sq (silu(W_a a2) * W_b a2)
// with P_h = W_pb LN(pair) the block's pair logits.
//
// Everything that reads only the conditioning is the same at every sampler step of a fold,
// so it is computed once per fold (ffb_dit_condition): the two AdaLN scale / shift tables, the
// two output-gate tables ([L][768] each, the gates as logits) and the pair logits [16][L][Lp]
// (the pair-bias kernel of the single track with this block's weights; Lp = L rounded up to
// 8). A step (ffb_dit_fwd) on x [S][L][768] is: the AdaLN kernel, the [q|k|v|g] GEMM, the
// attention (Q K^T batched over samples x heads, the softmax kernel with the pair logits and
// the key mask, V transposed, P V batched likewise, the gate kernel), the output GEMM whose
// epilogue applies the gate table and the residual, the second AdaLN, the SwiGLU GEMM, and the
// squeeze GEMM with the second gate and residual. GEMMs are the library's tcgen05 GEMM.
#include "../../include/foldforge_b200.h"
#include "abi_util.h"
#include "common.cuh"
#include "kernels.h"

namespace ffb {
namespace {

constexpr int kC = 768;
constexpr int kH = 16;
constexpr int kD = 48;
constexpr int kCc = 384;
constexpr int kCp = 128;
constexpr int kHid = 1536;

size_t a256(size_t x) { return (x + 255) / 256 * 256; }

// packed image of one block
struct DitLayout {
  size_t w_qkvg, b_qkvg, w_o, w_ab, w_sq, w_c1, b_c1, w_c2, b_c2, w_z, b_z, ln_c1, ln_c2, w_pb, pb_wsum, total;
};

DitLayout dit_layout() {
  DitLayout L;
  size_t o = 0;
  L.w_qkvg = o;  o = a256(o + static_cast<size_t>(4 * kC) * kC * 2);   // [q; k; v; g] rows
  L.b_qkvg = o;  o = a256(o + 4 * kC * 4);                              // b_q, then zeros
  L.w_o = o;     o = a256(o + static_cast<size_t>(kC) * kC * 2);
  L.w_ab = o;    o = a256(o + static_cast<size_t>(2 * kHid) * kC * 2);  // a / b interleaved per 16 rows
  L.w_sq = o;    o = a256(o + static_cast<size_t>(kC) * kHid * 2);
  L.w_c1 = o;    o = a256(o + static_cast<size_t>(2 * kC) * kCc * 2);   // [W_s1; W_b1] diag(ln_c1)
  L.b_c1 = o;    o = a256(o + 2 * kC * 4);                              // b_s1, then zeros
  L.w_c2 = o;    o = a256(o + static_cast<size_t>(2 * kC) * kCc * 2);
  L.b_c2 = o;    o = a256(o + 2 * kC * 4);
  L.w_z = o;     o = a256(o + static_cast<size_t>(2 * kC) * kCc * 2);   // [W_z1; W_z2]
  L.b_z = o;     o = a256(o + 2 * kC * 4);
  L.ln_c1 = o;   o = a256(o + kCc * 4);
  L.ln_c2 = o;   o = a256(o + kCc * 4);
  L.w_pb = o;    o = a256(o + 2 * kH * 128);                            // SW128 image of W_pb diag(ln_pair)
  L.pb_wsum = o; o = a256(o + kH * 4);
  L.total = o;
  return L;
}

// dst[r][c] = bf16(src[perm(r)][c] * (col_scale ? col_scale[c] : 1)); perm interleaves the
// rows of a and b in blocks of 16 (the SwiGLU epilogue's layout) when b is given
__global__ void dit_pack_kernel(const float* __restrict__ a, const float* __restrict__ b, int rows_each, int cols,
                                const float* __restrict__ col_scale, __nv_bfloat16* __restrict__ dst) {
  const int64_t total = static_cast<int64_t>(b ? 2 * rows_each : rows_each) * cols;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / cols), c = static_cast<int>(i % cols);
    float v;
    if (b) {
      const int blk = r / 32, within = r % 32;
      v = (within < 16 ? a : b)[static_cast<int64_t>(blk * 16 + within % 16) * cols + c];
    } else {
      v = a[static_cast<int64_t>(r) * cols + c];
    }
    dst[i] = __float2bfloat16_rn(col_scale ? v * col_scale[c] : v);
  }
}

int pack(const float* a, const float* b, int rows_each, int cols, const float* col_scale, void* dst, cudaStream_t st) {
  dit_pack_kernel<<<256, 256, 0, st>>>(a, b, rows_each, cols, col_scale, static_cast<__nv_bfloat16*>(dst));
  return static_cast<int>(cudaGetLastError());
}

int copy_f32(void* dst, const float* src, int n, cudaStream_t st) {
  return static_cast<int>(cudaMemcpyAsync(dst, src, static_cast<size_t>(n) * 4, cudaMemcpyDeviceToDevice, st));
}

// ---------------------------------------------------------------- AdaLN
// y[r] = sigmoid(tab[t][0:768]) * LN(x[r]) + tab[t][768:1536], t = r % L (the table rows are
// tokens; the samples share them). One warp per row: 24 channels per lane held in registers,
// two-pass variance. rows = S * L.
constexpr int kLnWarps = 8;

__global__ void __launch_bounds__(kLnWarps * 32) dit_adaln_kernel(const __nv_bfloat16* __restrict__ x,
                                                                  const float* __restrict__ tab,
                                                                  __nv_bfloat16* __restrict__ y, int64_t rows, int L) {
  const int lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * kLnWarps + (threadIdx.x >> 5);
  if (r >= rows) return;
  // lane owns channels 8 (lane + 32 j) .. + 7, j = 0..2: three 16-byte vectors
  const uint4* xr = reinterpret_cast<const uint4*>(x + r * kC);
  float v[24];
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const uint4 u = xr[lane + 32 * j];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      v[8 * j + 2 * e] = bf16_lo(w[e]);
      v[8 * j + 2 * e + 1] = bf16_hi(w[e]);
      s += v[8 * j + 2 * e] + v[8 * j + 2 * e + 1];
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
  const float mean = s * (1.0f / kC);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < 24; ++i) {
    const float d = v[i] - mean;
    q += d * d;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) q += __shfl_xor_sync(0xFFFFFFFFu, q, o);
  const float rstd = rsqrtf(q * (1.0f / kC) + 1e-5f);
  const float* tr = tab + static_cast<int64_t>(r % L) * (2 * kC);
  uint4* yr = reinterpret_cast<uint4*>(y + r * kC);
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int c0 = 8 * (lane + 32 * j);
    const float4 s0 = *reinterpret_cast<const float4*>(tr + c0), s1 = *reinterpret_cast<const float4*>(tr + c0 + 4);
    const float4 b0 = *reinterpret_cast<const float4*>(tr + kC + c0);
    const float4 b1 = *reinterpret_cast<const float4*>(tr + kC + c0 + 4);
    const float sc[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    const float sh[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    float o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = (v[8 * j + e] - mean) * rstd / (1.0f + __expf(-sc[e])) + sh[e];
    yr[lane + 32 * j] = make_uint4(pack_bf16(o[0], o[1]), pack_bf16(o[2], o[3]), pack_bf16(o[4], o[5]),
                                   pack_bf16(o[6], o[7]));
  }
}

// ---------------------------------------------------------------- attention on the tensor cores
// For each sample: S[h] = Q_h K_h^T (a tcgen05 GEMM batched over the 16 heads, straight from the
// [q|k|v|g] rows; K = 48 zero-filled to 64 by TMA), then one warp per row (s, h, i) takes
// x_j = S[i][j] / sqrt(48) + P_h[i][j] (masked keys REPLACED by -1e9), the softmax in fp32,
// and writes the normalised row as bf16 (keys past L: 0), then O_h = P_h V_h (a second
// batched GEMM, V transposed to [48][Lp] first) lands in the [token][768] layout, and the gate
// kernel multiplies by sigmoid(g). Rows of keys are padded to Lp (a multiple of 8) for TMA.
// One warp per row; rows of up to kSmKeys keys are held in registers, four keys per lane per
// step read as 16-byte vectors (S and the pair-logit rows have Lp columns, a multiple of 8, so
// rows are 32-byte aligned); longer rows take three passes over global memory.
constexpr int kSmKeys = 1024;

__global__ void __launch_bounds__(256) dit_softmax_kernel(const float* __restrict__ S, const float* __restrict__ logits,
                                                          const uint8_t* __restrict__ mask, __nv_bfloat16* __restrict__ P,
                                                          int64_t rows, int L, int Lp) {
  const int lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int i = static_cast<int>(r % L);
  const int h = static_cast<int>((r / L) % kH);
  const float* srow = S + r * Lp;
  const float* brow = logits + (static_cast<int64_t>(h) * L + i) * Lp;
  __nv_bfloat16* prow = P + r * Lp;
  const float scale = rsqrtf(static_cast<float>(kD));
  if (Lp <= kSmKeys) {
    constexpr int kSteps = kSmKeys / 128;
    float x[kSteps][4];
    float m = -INFINITY;
#pragma unroll
    for (int t = 0; t < kSteps; ++t) {
      const int j0 = 4 * lane + 128 * t;
#pragma unroll
      for (int e = 0; e < 4; ++e) x[t][e] = -INFINITY;
      if (j0 < Lp) {
        const float4 sv = *reinterpret_cast<const float4*>(srow + j0);
        const float4 bv = *reinterpret_cast<const float4*>(brow + j0);
        const float sa[4] = {sv.x, sv.y, sv.z, sv.w}, ba[4] = {bv.x, bv.y, bv.z, bv.w};
        uint32_t mk;
        if (j0 + 4 <= L && (reinterpret_cast<uintptr_t>(mask + j0) & 3u) == 0) {
          mk = *reinterpret_cast<const uint32_t*>(mask + j0);
        } else {
          mk = 0;
          for (int e = 0; e < 4; ++e)
            if (j0 + e < L && mask[j0 + e]) mk |= 1u << (8 * e);
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if (j0 + e < L) x[t][e] = ((mk >> (8 * e)) & 0xFFu) ? fmaf(sa[e], scale, ba[e]) : -1.0e9f;
          m = fmaxf(m, x[t][e]);
        }
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    float sum = 0.f;
#pragma unroll
    for (int t = 0; t < kSteps; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        x[t][e] = __expf(x[t][e] - m);  // keys past L: exp(-inf) = 0
        sum += x[t][e];
      }
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
    const float inv = 1.0f / sum;
#pragma unroll
    for (int t = 0; t < kSteps; ++t) {
      const int j0 = 4 * lane + 128 * t;
      if (j0 < Lp)
        *reinterpret_cast<uint2*>(prow + j0) =
            make_uint2(pack_bf16(x[t][0] * inv, x[t][1] * inv), pack_bf16(x[t][2] * inv, x[t][3] * inv));
    }
    return;
  }
  auto logit = [&](int j) { return mask[j] ? fmaf(srow[j], scale, brow[j]) : -1.0e9f; };
  float m = -INFINITY;
  for (int j = lane; j < L; j += 32) m = fmaxf(m, logit(j));
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
  float sum = 0.f;
  for (int j = lane; j < L; j += 32) sum += __expf(logit(j) - m);
#pragma unroll
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
  const float inv = 1.0f / sum;
  for (int j = lane; j < Lp; j += 32) prow[j] = __float2bfloat16_rn(j < L ? __expf(logit(j) - m) * inv : 0.f);
}

// VT[s][h][d][j] = v[s L + j][h 48 + d] (keys j >= L: 0)
__global__ void dit_vt_kernel(const __nv_bfloat16* __restrict__ qkvg, __nv_bfloat16* __restrict__ vt, int S, int L,
                              int Lp) {
  const int64_t total = static_cast<int64_t>(S) * kH * kD * Lp;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int j = static_cast<int>(e % Lp);
    const int64_t rest = e / Lp;
    const int d = static_cast<int>(rest % kD);
    const int h = static_cast<int>((rest / kD) % kH);
    const int s = static_cast<int>(rest / (kD * kH));
    vt[e] = j < L ? qkvg[(static_cast<int64_t>(s) * L + j) * (4 * kC) + 2 * kC + h * kD + d] : __float2bfloat16_rn(0.f);
  }
}

// o[r][c] *= sigmoid(g[r][c]), g = qkvg[r][3 * 768 + c]; 8 channels per thread
__global__ void dit_gate_kernel(__nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ qkvg, int64_t rows) {
  const int64_t total = rows * (kC / 8);
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = e / (kC / 8);
    const int c8 = static_cast<int>(e % (kC / 8));
    uint4* op = reinterpret_cast<uint4*>(o + r * kC) + c8;
    const uint4 ov = *op;
    const uint4 gv = *(reinterpret_cast<const uint4*>(qkvg + r * (4 * kC) + 3 * kC) + c8);
    const uint32_t ow[4] = {ov.x, ov.y, ov.z, ov.w}, gw[4] = {gv.x, gv.y, gv.z, gv.w};
    uint32_t res[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
      res[k] = pack_bf16(bf16_lo(ow[k]) / (1.0f + __expf(-bf16_lo(gw[k]))),
                         bf16_hi(ow[k]) / (1.0f + __expf(-bf16_hi(gw[k]))));
    *op = make_uint4(res[0], res[1], res[2], res[3]);
  }
}

// ---------------------------------------------------------------- host side
// tables of one block for L tokens: AdaLN 1 and 2 ([L][scale 768 | shift 768] fp32), the two
// output gates ([L][768] fp32 logits), the pair logits [16][L][L] fp32
struct DitTables {
  float *ada1, *ada2, *gate1, *gate2, *logits;
};

int pad8(int x) { return (x + 7) / 8 * 8; }

size_t tables_bytes(int L) {
  const size_t l = static_cast<size_t>(L);
  return 2 * a256(l * 2 * kC * 4) + 2 * a256(l * kC * 4) + a256(static_cast<size_t>(kH) * l * pad8(L) * 4);
}

DitTables carve_tables(void* base, int L) {
  const size_t l = static_cast<size_t>(L);
  uint8_t* p = static_cast<uint8_t*>(base);
  DitTables t;
  t.ada1 = reinterpret_cast<float*>(p);  p += a256(l * 2 * kC * 4);
  t.ada2 = reinterpret_cast<float*>(p);  p += a256(l * 2 * kC * 4);
  t.gate1 = reinterpret_cast<float*>(p); p += a256(l * kC * 4);
  t.gate2 = reinterpret_cast<float*>(p); p += a256(l * kC * 4);
  t.logits = reinterpret_cast<float*>(p);
  return t;
}

size_t condition_workspace_bytes(int L) { return a256(static_cast<size_t>(L) * kCc * 2); }

size_t forward_workspace_bytes(int S, int L) {
  const size_t m = static_cast<size_t>(S) * L;
  const size_t sl = static_cast<size_t>(S) * kH * L * pad8(L);
  return a256(m * kC * 2) + a256(m * 4 * kC * 2) + a256(sl * 4) + a256(sl * 2) +
         a256(static_cast<size_t>(S) * kH * kD * pad8(L) * 2);
}

// D[m][n] = A[m][:] . W[n][:] on the tcgen05 GEMM (A, W bf16 K-major); the residual epilogue
// optionally scales acc by sigmoid(gate[m % gate_rows][n]) first
int dgemm(const void* a, const void* w, void* d, int m, int n, int k, int d_f32, const float* bias, int epilogue,
          const void* residual, const float* gate, int gate_rows, const DeviceInfo& info, cudaStream_t stream) {
  const int tiles256 = ((m + 127) / 128) * ((n + 255) / 256);
  const int bn = (n >= 256 && tiles256 >= info.num_sms) ? 256 : 128;
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
  p.row_mask = nullptr;
  p.err = info.err;
  p.col_gate = gate;
  p.gate_rows = gate_rows;
  return cuda_status(launch_gemm_nt(ma, mb, p, bn, info.num_sms, stream), "diffusion transformer gemm");
}

// D[s][h][m][n] = A[s][h][m][:] . W[s][h][n][:] for `heads` x `samples` batches (bf16 operands
// with element strides: rows ld, heads hs, samples ss; K zero-filled past k to the 64-wide K
// block by TMA); D's batch offset is h * d_hs + s * d_ss
int bgemm(const void* a, int64_t a_ld, int64_t a_hs, int64_t a_ss, const void* w, int64_t w_ld, int64_t w_hs,
          int64_t w_ss, void* d, int64_t ldd, int64_t d_hs, int64_t d_ss, int m, int n, int k, int heads, int samples,
          int d_f32, const DeviceInfo& info, cudaStream_t stream) {
  const int bn = n >= 256 ? 256 : 128;
  CUtensorMap ma, mb;
  const uint64_t adims[4] = {static_cast<uint64_t>(k), static_cast<uint64_t>(m), static_cast<uint64_t>(heads),
                             static_cast<uint64_t>(samples)};
  const uint64_t astr[3] = {static_cast<uint64_t>(a_ld) * 2, static_cast<uint64_t>(a_hs) * 2,
                            static_cast<uint64_t>(a_ss) * 2};
  const uint32_t abox[4] = {64, 128, 1, 1};
  int st = make_map(&ma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, a, adims, astr, abox, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  const uint64_t bdims[4] = {static_cast<uint64_t>(k), static_cast<uint64_t>(n), static_cast<uint64_t>(heads),
                             static_cast<uint64_t>(samples)};
  const uint64_t bstr[3] = {static_cast<uint64_t>(w_ld) * 2, static_cast<uint64_t>(w_hs) * 2,
                            static_cast<uint64_t>(w_ss) * 2};
  const uint32_t bbox[4] = {64, static_cast<uint32_t>(bn), 1, 1};
  st = make_map(&mb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, w, bdims, bstr, bbox, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  GemmParams p;
  p.M = m;
  p.N = n;
  p.K = k;
  p.batch = heads * samples;
  p.D = d;
  p.ldd = ldd;
  p.batch_stride_d = d_hs;
  p.d_is_f32 = d_f32;
  p.epilogue = kEpiStore;
  p.bias = nullptr;
  p.residual = nullptr;
  p.row_mask = nullptr;
  p.err = info.err;
  p.batch_inner = heads;
  p.batch_stride_d2 = d_ss;
  return cuda_status(launch_gemm_nt(ma, mb, p, bn, info.num_sms, stream), "diffusion transformer attention gemm");
}

int adaln(const void* x, const float* tab, void* y, int64_t rows, int L, cudaStream_t stream) {
  const int grid = static_cast<int>((rows + kLnWarps - 1) / kLnWarps);
  dit_adaln_kernel<<<grid, kLnWarps * 32, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), tab,
                                                       static_cast<__nv_bfloat16*>(y), rows, L);
  return cuda_status(static_cast<int>(cudaGetLastError()), "diffusion transformer adaln");
}

}  // namespace

size_t dit_packed_bytes() { return dit_layout().total; }
size_t dit_tables_bytes(int L) { return tables_bytes(L); }
size_t dit_condition_workspace_bytes(int L) { return condition_workspace_bytes(L); }
size_t dit_workspace_bytes(int S, int L) { return forward_workspace_bytes(S, L); }

// weights: the 23 fp32 tensors of one block in the engine schema's order (see the header)
int dit_prepare(const float* const* w, void* packed, cudaStream_t stream) {
  const DitLayout L = dit_layout();
  uint8_t* img = static_cast<uint8_t*>(packed);
  enum { A1_LN, A1_SW, A1_SB, A1_BW, WQ, BQ, WK, WV, WG, AT_ZW, AT_ZB, WO, LN_PAIR, W_PB,
         A2_LN, A2_SW, A2_SB, A2_BW, WA, WB, WSQ, TR_ZW, TR_ZB };
  int rc = static_cast<int>(cudaMemsetAsync(packed, 0, L.total, stream));
  const int qkvg[4] = {WQ, WK, WV, WG};
  for (int i = 0; i < 4 && rc == 0; ++i)
    rc = pack(w[qkvg[i]], nullptr, kC, kC, nullptr, img + L.w_qkvg + static_cast<size_t>(i) * kC * kC * 2, stream);
  if (rc == 0) rc = copy_f32(img + L.b_qkvg, w[BQ], kC, stream);
  if (rc == 0) rc = pack(w[WO], nullptr, kC, kC, nullptr, img + L.w_o, stream);
  if (rc == 0) rc = pack(w[WA], w[WB], kHid, kC, nullptr, img + L.w_ab, stream);
  if (rc == 0) rc = pack(w[WSQ], nullptr, kC, kHid, nullptr, img + L.w_sq, stream);
  // AdaLN projections act on LN(cond) without its weight: the weight is folded into their columns
  if (rc == 0) rc = pack(w[A1_SW], nullptr, kC, kCc, w[A1_LN], img + L.w_c1, stream);
  if (rc == 0) rc = pack(w[A1_BW], nullptr, kC, kCc, w[A1_LN], img + L.w_c1 + static_cast<size_t>(kC) * kCc * 2, stream);
  if (rc == 0) rc = copy_f32(img + L.b_c1, w[A1_SB], kC, stream);
  if (rc == 0) rc = pack(w[A2_SW], nullptr, kC, kCc, w[A2_LN], img + L.w_c2, stream);
  if (rc == 0) rc = pack(w[A2_BW], nullptr, kC, kCc, w[A2_LN], img + L.w_c2 + static_cast<size_t>(kC) * kCc * 2, stream);
  if (rc == 0) rc = copy_f32(img + L.b_c2, w[A2_SB], kC, stream);
  if (rc == 0) rc = pack(w[AT_ZW], nullptr, kC, kCc, nullptr, img + L.w_z, stream);
  if (rc == 0) rc = pack(w[TR_ZW], nullptr, kC, kCc, nullptr, img + L.w_z + static_cast<size_t>(kC) * kCc * 2, stream);
  if (rc == 0) rc = copy_f32(img + L.b_z, w[AT_ZB], kC, stream);
  if (rc == 0) rc = copy_f32(img + L.b_z + kC * 4, w[TR_ZB], kC, stream);
  if (rc == 0)
    rc = launch_pack_weight(w[W_PB], kH, kCp, w[LN_PAIR], nullptr, img + L.w_pb, 0, kH,
                            reinterpret_cast<float*>(img + L.pb_wsum), nullptr, stream);
  return rc;
}

int dit_condition(const void* cond, const void* pair, const void* packed, void* tables, void* workspace, int L,
                  const DeviceInfo& info, cudaStream_t stream) {
  const DitLayout Ly = dit_layout();
  const uint8_t* img = static_cast<const uint8_t*>(packed);
  const DitTables t = carve_tables(tables, L);
  int st = cuda_status(launch_layernorm(cond, workspace, nullptr, nullptr, L, kCc, 1e-5f, 0, info.num_sms, stream),
                       "diffusion transformer conditioning layernorm");
  if (st) return st;
  st = dgemm(workspace, img + Ly.w_c1, t.ada1, L, 2 * kC, kCc, 1, reinterpret_cast<const float*>(img + Ly.b_c1),
             kEpiStore, nullptr, nullptr, 0, info, stream);
  if (st) return st;
  st = dgemm(workspace, img + Ly.w_c2, t.ada2, L, 2 * kC, kCc, 1, reinterpret_cast<const float*>(img + Ly.b_c2),
             kEpiStore, nullptr, nullptr, 0, info, stream);
  if (st) return st;
  st = dgemm(cond, img + Ly.w_z, t.gate1, L, kC, kCc, 1, reinterpret_cast<const float*>(img + Ly.b_z), kEpiStore,
             nullptr, nullptr, 0, info, stream);
  if (st) return st;
  st = dgemm(cond, img + Ly.w_z + static_cast<size_t>(kC) * kCc * 2, t.gate2, L, kC, kCc, 1,
             reinterpret_cast<const float*>(img + Ly.b_z) + kC, kEpiStore, nullptr, nullptr, 0, info, stream);
  if (st) return st;
  // pair logits [16][L][Lp] (rows padded to Lp columns for the softmax's vector loads)
  return pair_bias16(pair, img + Ly.w_pb, reinterpret_cast<const float*>(img + Ly.pb_wsum), t.logits, L, L,
                     static_cast<int64_t>(L) * pad8(L), pad8(L), info, stream);
}

int dit_forward(const void* x, const uint8_t* mask, const void* packed, const void* tables, void* out, void* workspace,
                int S, int L, const DeviceInfo& info, cudaStream_t stream) {
  const DitLayout Ly = dit_layout();
  const uint8_t* img = static_cast<const uint8_t*>(packed);
  const DitTables t = carve_tables(const_cast<void*>(tables), L);
  const int m = S * L;
  uint8_t* a = static_cast<uint8_t*>(workspace);                     // [m][768]: a, then sigmoid(g) o, then a2
  uint8_t* big = a + a256(static_cast<size_t>(m) * kC * 2);          // [m][3072] q|k|v|g, then h [m][1536]
  int st = adaln(x, t.ada1, a, m, L, stream);
  if (st) return st;
  st = dgemm(a, img + Ly.w_qkvg, big, m, 4 * kC, kC, 0, reinterpret_cast<const float*>(img + Ly.b_qkvg), kEpiStore,
             nullptr, nullptr, 0, info, stream);
  if (st) return st;
  // attention: S = Q K^T and O = P V on the tensor cores, the softmax (with the pair logits and
  // the key mask) and the gate in between
  const int Lp = pad8(L);
  const int64_t sl = static_cast<int64_t>(S) * kH * L * Lp;
  float* sbuf = reinterpret_cast<float*>(big + a256(static_cast<size_t>(m) * 4 * kC * 2));
  __nv_bfloat16* pbuf = reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<uint8_t*>(sbuf) + a256(sl * 4));
  __nv_bfloat16* vt = reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<uint8_t*>(pbuf) + a256(sl * 2));
  const __nv_bfloat16* qk = reinterpret_cast<const __nv_bfloat16*>(big);
  st = bgemm(qk, 4 * kC, kD, static_cast<int64_t>(L) * 4 * kC, qk + kC, 4 * kC, kD, static_cast<int64_t>(L) * 4 * kC,
             sbuf, Lp, static_cast<int64_t>(L) * Lp, static_cast<int64_t>(kH) * L * Lp, L, L, kD, kH, S, 1, info, stream);
  if (st) return st;
  dit_softmax_kernel<<<static_cast<int>((static_cast<int64_t>(S) * kH * L + 7) / 8), 256, 0, stream>>>(
      sbuf, t.logits, mask, pbuf, static_cast<int64_t>(S) * kH * L, L, Lp);
  dit_vt_kernel<<<4 * info.num_sms, 256, 0, stream>>>(qk, vt, S, L, Lp);
  st = cuda_status(static_cast<int>(cudaGetLastError()), "diffusion transformer softmax launch");
  if (st) return st;
  st = bgemm(pbuf, Lp, static_cast<int64_t>(L) * Lp, static_cast<int64_t>(kH) * L * Lp, vt, Lp,
             static_cast<int64_t>(kD) * Lp, static_cast<int64_t>(kH) * kD * Lp, a, kC, kD, static_cast<int64_t>(L) * kC,
             L, kD, Lp, kH, S, 0, info, stream);
  if (st) return st;
  dit_gate_kernel<<<4 * info.num_sms, 256, 0, stream>>>(reinterpret_cast<__nv_bfloat16*>(a), qk, m);
  st = cuda_status(static_cast<int>(cudaGetLastError()), "diffusion transformer gate launch");
  if (st) return st;
  st = dgemm(a, img + Ly.w_o, out, m, kC, kC, 0, nullptr, kEpiResidual, x, t.gate1, L, info, stream);
  if (st) return st;
  st = adaln(out, t.ada2, a, m, L, stream);
  if (st) return st;
  st = dgemm(a, img + Ly.w_ab, big, m, 2 * kHid, kC, 0, nullptr, kEpiSwiGLU, nullptr, nullptr, 0, info, stream);
  if (st) return st;
  return dgemm(big, img + Ly.w_sq, out, m, kC, kHid, 0, nullptr, kEpiResidual, out, t.gate2, L, info, stream);
}

}  // namespace ffb

// ---------------------------------------------------------------- C ABI
extern "C" {

size_t ffb_dit_packed_bytes(void) { return ffb::dit_packed_bytes(); }
size_t ffb_dit_tables_bytes(int L) { return L > 0 ? ffb::dit_tables_bytes(L) : 0; }
size_t ffb_dit_condition_workspace_bytes(int L) { return L > 0 ? ffb::dit_condition_workspace_bytes(L) : 0; }
size_t ffb_dit_workspace_bytes(int S, int L) { return (S > 0 && L > 0) ? ffb::dit_workspace_bytes(S, L) : 0; }

int ffb_dit_prepare(const float* const* weights, void* packed, void* stream) {
  if (!weights || !packed) return ffb::fail(FFB_ERR_ARG, "dit_prepare: null pointer");
  for (int i = 0; i < 23; ++i)
    if (!weights[i]) return ffb::fail(FFB_ERR_ARG, "dit_prepare: weight %d is null", i);
  if (reinterpret_cast<uintptr_t>(packed) & 255u) return ffb::fail(FFB_ERR_ARG, "dit_prepare: packed not 256-aligned");
  return ffb::cuda_status(ffb::dit_prepare(weights, packed, static_cast<cudaStream_t>(stream)), "dit_prepare");
}

int ffb_dit_condition(const void* cond, const void* pair, const void* packed, void* tables, void* workspace,
                      size_t workspace_bytes, int L, void* stream) {
  if (L <= 0 || static_cast<int64_t>(L) * L >= (int64_t{1} << 31)) return ffb::fail(FFB_ERR_ARG, "dit_condition: L=%d", L);
  if (!cond || !pair || !packed || !tables || !workspace) return ffb::fail(FFB_ERR_ARG, "dit_condition: null pointer");
  if (workspace_bytes < ffb::dit_condition_workspace_bytes(L))
    return ffb::fail(FFB_ERR_ARG, "dit_condition: workspace %zu < %zu bytes", workspace_bytes,
                     ffb::dit_condition_workspace_bytes(L));
  if (((reinterpret_cast<uintptr_t>(cond) | reinterpret_cast<uintptr_t>(pair)) & 15u) ||
      ((reinterpret_cast<uintptr_t>(packed) | reinterpret_cast<uintptr_t>(tables) |
        reinterpret_cast<uintptr_t>(workspace)) & 255u))
    return ffb::fail(FFB_ERR_ARG, "dit_condition: misaligned pointer");
  ffb::DeviceInfo info;
  int st = ffb::device_info(&info);
  if (st != FFB_OK) return st;
  return ffb::dit_condition(cond, pair, packed, tables, workspace, L, info, static_cast<cudaStream_t>(stream));
}

int ffb_dit_fwd(const void* x, const uint8_t* mask, const void* packed, const void* tables, void* out, void* workspace,
                size_t workspace_bytes, int S, int L, void* stream) {
  if (S <= 0 || L <= 0) return ffb::fail(FFB_ERR_ARG, "dit_fwd: S=%d L=%d", S, L);
  if (!x || !mask || !packed || !tables || !out || !workspace) return ffb::fail(FFB_ERR_ARG, "dit_fwd: null pointer");
  if (x == out) return ffb::fail(FFB_ERR_ARG, "dit_fwd: out must not alias x");
  if (workspace_bytes < ffb::dit_workspace_bytes(S, L))
    return ffb::fail(FFB_ERR_ARG, "dit_fwd: workspace %zu < %zu bytes", workspace_bytes, ffb::dit_workspace_bytes(S, L));
  if (((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15u) ||
      ((reinterpret_cast<uintptr_t>(packed) | reinterpret_cast<uintptr_t>(tables) |
        reinterpret_cast<uintptr_t>(workspace)) & 255u))
    return ffb::fail(FFB_ERR_ARG, "dit_fwd: misaligned pointer");
  ffb::DeviceInfo info;
  int st = ffb::device_info(&info);
  if (st != FFB_OK) return st;
  return ffb::dit_forward(x, mask, packed, tables, out, workspace, S, L, info, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
