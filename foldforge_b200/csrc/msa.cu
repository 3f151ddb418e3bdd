// The MSA module's ops (AF3's MSA-stack block): outer product mean, MSA pair-weighted
// averaging, and a tensor-core transition for any width (the MSA transition, c_m = 64).
// bf16 activations, fp32 accumulation; the heavy products run on the tcgen05 GEMM (gemm.cu).
//
// Outer product mean (legacy/reference/attention.py:57-74, legacy/primitives.py:40-136, AF3
// form: no projection bias, the output bias added before the divide):
//   x = LN(m);  L[s,i,:] = m_si W_l x[s,i];  R[s,j,:] = m_sj W_r x[s,j]            (32 channels)
//   delta[i,j,f] = (sum_{c,e} (sum_s L[s,i,c] R[s,j,e]) W_o[f, c 32 + e] + b_o[f]) / d(n_ij)
//   n_ij = sum_s m_si m_sj,  d(n) = n + offset (AF3: 1e-3) or max(n, 1) (offset < 0)
// Launches: opm_proj (LN + both projections + mask, written transposed as K-major GEMM
// operands L^T, R^T [(i, c)][s] and the mask M^T [i][s]); GEMM n = M^T M^T^T (pair counts,
// fp32); opm_scale (1 / d(n)); GEMM D = L^T R^T^T [(i, c)][(j, e)] (the contraction over MSA
// rows, tensor cores); opm_relayout (D -> P [(i, j)][(c, e)]); GEMM delta = P W_o^T + b_o
// scaled per pair row by 1 / d(n).
//
// MSA pair-weighted averaging (legacy/attention.py:174-229, engine weights of
// legacy/released.py:253-281):
//   w_h[i, :] = softmax_j(W_b LN_z(z)[i, j] (LN offset dropped: softmax-invariant)
//                         - 1e9 where no MSA row has column j)               (added, as the reference)
//   o[s, i, h] = sum_j w_h[i, j] v[s, j, h],  v = W_v LN(m),  g = W_g LN(m)
//   m' = m + W_o (sigmoid(g) * o)
// Launches: pwa_logits (LN_z + 8 head projections per pair); pwa_softmax (per head and row,
// weights written as K-major GEMM operands [h][i][j]); LayerNorm of m; GEMM [v | g] = LN(m)
// [W_v; W_g]^T; pwa_values (v -> [h][(s, e)][j]); batched GEMM over the 8 heads o_h = w_h v_h;
// pwa_gate (sigmoid(g) * o, back to [(s, i)][(h, e)]); GEMM m' = m + G W_o^T.
#include <math.h>

#include "../../include/foldforge_b200.h"
#include "abi_util.h"
#include "common.cuh"
#include "kernels.h"

namespace ffb {
namespace {

constexpr int kCm = 64;    // MSA channels
constexpr int kOc = 32;    // outer-product channels a side
constexpr int kCz = 128;   // pair channels
constexpr int kPh = 8;     // pair-weighted averaging heads
constexpr int kPd = 8;     // value width per head

size_t a256(size_t x) { return (x + 255) / 256 * 256; }
int round_up(int x, int m) { return (x + m - 1) / m * m; }

// ------------------------------------------------------------------ GEMM helper
// D[b] = A[b] B[b]^T on the tcgen05 GEMM: A [m, k] (row stride lda), B [n, k] (ldb), D [m, n]
// (ldd), batch strides in elements; epilogue as gemm.cu; row_scale optional.
struct Gemm {
  const void* a;
  const void* b;
  void* d;
  int batch = 1, m = 0, n = 0, k = 0;
  int64_t lda = 0, ldb = 0, ldd = 0, sa = 0, sb = 0, sd = 0;
  int d_f32 = 0;
  const float* bias = nullptr;
  int epilogue = kEpiStore;
  const void* residual = nullptr;
  const float* row_scale = nullptr;
};

int run_gemm(const Gemm& g, const DeviceInfo& info, cudaStream_t stream) {
  const int bn = g.n >= 256 ? 256 : 128;
  CUtensorMap ma, mb;
  const uint64_t adims[3] = {static_cast<uint64_t>(g.k), static_cast<uint64_t>(g.m), static_cast<uint64_t>(g.batch)};
  const uint64_t astr[2] = {static_cast<uint64_t>(g.lda) * 2,
                            static_cast<uint64_t>(g.batch > 1 ? g.sa : g.lda * g.m) * 2};
  const uint32_t abox[3] = {64, 128, 1};
  int st = make_map(&ma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, g.a, adims, astr, abox, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  const uint64_t bdims[3] = {static_cast<uint64_t>(g.k), static_cast<uint64_t>(g.n), static_cast<uint64_t>(g.batch)};
  const uint64_t bstr[2] = {static_cast<uint64_t>(g.ldb) * 2,
                            static_cast<uint64_t>(g.batch > 1 ? g.sb : g.ldb * g.n) * 2};
  const uint32_t bbox[3] = {64, static_cast<uint32_t>(bn), 1};
  st = make_map(&mb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, g.b, bdims, bstr, bbox, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  GemmParams p;
  p.M = g.m;
  p.N = g.n;
  p.K = g.k;
  p.batch = g.batch;
  p.D = g.d;
  p.ldd = g.ldd;
  p.batch_stride_d = g.sd;
  p.d_is_f32 = g.d_f32;
  p.epilogue = g.epilogue;
  p.bias = g.bias;
  p.residual = g.residual;
  p.row_mask = nullptr;
  p.row_scale = g.row_scale;
  p.err = info.err;
  return cuda_status(launch_gemm_nt(ma, mb, p, bn, info.num_sms, stream), "msa gemm launch");
}

int launched(const char* what) { return cuda_status(static_cast<int>(cudaGetLastError()), what); }

// fp32 [rows, cols] -> bf16; with `interleave`, a and b ([rows, cols] each) become the SwiGLU
// operand of gemm.cu: blocks of 16 rows of a, then 16 of b.
__global__ void to_bf16_kernel(const float* __restrict__ a, const float* __restrict__ b, int rows, int cols,
                               int interleave, __nv_bfloat16* __restrict__ dst) {
  const int64_t total = static_cast<int64_t>(interleave ? 2 * rows : rows) * cols;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(t / cols), col = static_cast<int>(t % cols);
    float v;
    if (!interleave) {
      v = a[t];
    } else {
      const int blk = row / 32, r = row % 32;
      v = (r < 16 ? a : b)[static_cast<int64_t>(blk * 16 + (r % 16)) * cols + col];
    }
    dst[t] = __float2bfloat16_rn(v);
  }
}

// ================================================================== outer product mean
// Packed image: W_o bf16 [128][1024] | fp32 ln_w[64] ln_b[64] w_l[32][64] w_r[32][64] b_o[128]
constexpr size_t kOpmWo = static_cast<size_t>(kCz) * kOc * kOc * 2;
constexpr size_t kOpmVec = kCm + kCm + 2 * kOc * kCm + kCz;
constexpr size_t kOpmPacked = kOpmWo + kOpmVec * 4;

constexpr int kOpmRows = 64;  // MSA rows per opm_proj block

// One block per (token i, 64 MSA rows): LayerNorm of the 64 rows' channels, the left and
// right projections times the row mask, written transposed ([(i, c)][s], s contiguous) with
// the mask M^T [i][s]. Rows past S are written as zeros (the contraction runs over Sp).
__global__ void __launch_bounds__(128) opm_proj_kernel(const __nv_bfloat16* __restrict__ m,
                                                       const uint8_t* __restrict__ mask, const float* __restrict__ vec,
                                                       __nv_bfloat16* __restrict__ lt, __nv_bfloat16* __restrict__ rt,
                                                       __nv_bfloat16* __restrict__ mt, int S, int N, int Sp) {
  __shared__ float x[kOpmRows][kCm + 1];
  __shared__ float w[2][kOc][kCm + 1];
  __shared__ float keep[kOpmRows];
  const int i = blockIdx.x;
  const int s0 = blockIdx.y * kOpmRows;
  const float* ln_w = vec;
  const float* ln_b = vec + kCm;
  const float* wl = vec + 2 * kCm;
  for (int t = threadIdx.x; t < 2 * kOc * kCm; t += blockDim.x) w[t / (kOc * kCm)][(t / kCm) % kOc][t % kCm] = wl[t];
  for (int t = threadIdx.x; t < kOpmRows * kCm; t += blockDim.x) {
    const int r = t / kCm, c = t % kCm, s = s0 + r;
    x[r][c] = s < S ? __bfloat162float(m[(static_cast<int64_t>(s) * N + i) * kCm + c]) : 0.0f;
  }
  if (threadIdx.x < kOpmRows) {
    const int s = s0 + threadIdx.x;
    keep[threadIdx.x] = (s < S && mask[static_cast<int64_t>(s) * N + i]) ? 1.0f : 0.0f;
  }
  __syncthreads();
  if (threadIdx.x < kOpmRows) {  // LayerNorm of row r in place (two-pass)
    const int r = threadIdx.x;
    float sum = 0.f;
    for (int c = 0; c < kCm; ++c) sum += x[r][c];
    const float mean = sum / kCm;
    float q = 0.f;
    for (int c = 0; c < kCm; ++c) {
      const float d = x[r][c] - mean;
      q += d * d;
    }
    const float rstd = rsqrtf(q / kCm + 1e-5f);
    for (int c = 0; c < kCm; ++c) x[r][c] = (x[r][c] - mean) * rstd * ln_w[c] + ln_b[c];
  }
  __syncthreads();
  // thread: side (L / R), channel c; 64 rows -> one contiguous run of s
  const int side = threadIdx.x / kOc, c = threadIdx.x % kOc;
  if (side < 2) {
    uint32_t packed[kOpmRows / 2];
#pragma unroll 4
    for (int r = 0; r < kOpmRows; r += 2) {
      float acc0 = 0.f, acc1 = 0.f;
#pragma unroll 8
      for (int k = 0; k < kCm; ++k) {
        acc0 = fmaf(x[r][k], w[side][c][k], acc0);
        acc1 = fmaf(x[r + 1][k], w[side][c][k], acc1);
      }
      packed[r / 2] = pack_bf16(acc0 * keep[r], acc1 * keep[r + 1]);
    }
    uint4* dst = reinterpret_cast<uint4*>((side == 0 ? lt : rt) + (static_cast<int64_t>(i) * kOc + c) * Sp + s0);
#pragma unroll
    for (int q = 0; q < kOpmRows / 8; ++q)
      dst[q] = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
  } else if (threadIdx.x - 2 * kOc < kOpmRows / 2) {
    const int r = 2 * (threadIdx.x - 2 * kOc);
    reinterpret_cast<uint32_t*>(mt + static_cast<int64_t>(i) * Sp + s0)[r / 2] = pack_bf16(keep[r], keep[r + 1]);
  }
}

// scale[p] = 1 / (n + offset) (offset >= 0) or 1 / max(n, 1) (offset < 0), in place on n.
__global__ void opm_scale_kernel(float* __restrict__ n, int64_t count, float offset) {
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < count;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float v = n[t];
    n[t] = 1.0f / (offset >= 0.0f ? v + offset : fmaxf(v, 1.0f));
  }
}

// D [(i, c)][(j, e)] -> P [(i, j)][(c, e)], 16 bytes (8 e) per thread and step.
__global__ void opm_relayout_kernel(const uint4* __restrict__ d, uint4* __restrict__ p, int N) {
  const int64_t total = static_cast<int64_t>(N) * kOc * N * (kOc / 8);
  const int64_t row_words = static_cast<int64_t>(N) * kOc / 8;  // one D row (i, c) in 16-byte words
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t ic = t / row_words, w = t % row_words;  // D row and word in it
    const int64_t i = ic / kOc, c = ic % kOc;
    const int64_t j = w / (kOc / 8), e8 = w % (kOc / 8);
    p[((i * N + j) * kOc + c) * (kOc / 8) + e8] = d[t];
  }
}

int grid_of(int64_t n, int threads, const DeviceInfo& info) {
  const int64_t g = (n + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(info.num_sms) * 16;
  return static_cast<int>(g < 1 ? 1 : (g > cap ? cap : g));
}

struct OpmWs {
  __nv_bfloat16 *lt, *rt, *mt, *d, *p;
  float* n;
};

OpmWs opm_carve(void* ws, int S, int N) {
  const int Sp = round_up(S, kOpmRows);
  uint8_t* q = static_cast<uint8_t*>(ws);
  OpmWs w;
  const size_t side = a256(static_cast<size_t>(N) * kOc * Sp * 2);
  w.lt = reinterpret_cast<__nv_bfloat16*>(q);
  w.rt = reinterpret_cast<__nv_bfloat16*>(q + side);
  q += 2 * side;
  w.mt = reinterpret_cast<__nv_bfloat16*>(q);
  q += a256(static_cast<size_t>(N) * Sp * 2);
  w.n = reinterpret_cast<float*>(q);
  q += a256(static_cast<size_t>(N) * N * 4);
  w.d = reinterpret_cast<__nv_bfloat16*>(q);
  q += a256(static_cast<size_t>(N) * kOc * N * kOc * 2);
  w.p = reinterpret_cast<__nv_bfloat16*>(q);
  return w;
}

size_t opm_workspace(int S, int N) {
  const size_t Sp = round_up(S, kOpmRows);
  return 2 * a256(static_cast<size_t>(N) * kOc * Sp * 2) + a256(static_cast<size_t>(N) * Sp * 2) +
         a256(static_cast<size_t>(N) * N * 4) + 2 * a256(static_cast<size_t>(N) * kOc * N * kOc * 2);
}

int opm_forward(const void* m, const uint8_t* mask, const void* packed, void* delta, void* workspace, int S, int N,
                float offset, const DeviceInfo& info, cudaStream_t stream) {
  const int Sp = round_up(S, kOpmRows);
  OpmWs w = opm_carve(workspace, S, N);
  const uint8_t* img = static_cast<const uint8_t*>(packed);
  const float* vec = reinterpret_cast<const float*>(img + kOpmWo);
  opm_proj_kernel<<<dim3(N, Sp / kOpmRows), 128, 0, stream>>>(static_cast<const __nv_bfloat16*>(m), mask, vec, w.lt,
                                                              w.rt, w.mt, S, N, Sp);
  int st = launched("opm_proj launch");
  if (st) return st;
  Gemm cnt;  // n_ij = sum_s m_si m_sj (0 / 1 operands, exact in fp32)
  cnt.a = w.mt;
  cnt.b = w.mt;
  cnt.d = w.n;
  cnt.m = N;
  cnt.n = N;
  cnt.k = Sp;
  cnt.lda = cnt.ldb = Sp;
  cnt.ldd = N;
  cnt.d_f32 = 1;
  st = run_gemm(cnt, info, stream);
  if (st) return st;
  opm_scale_kernel<<<grid_of(static_cast<int64_t>(N) * N, 256, info), 256, 0, stream>>>(
      w.n, static_cast<int64_t>(N) * N, offset);
  st = launched("opm_scale launch");
  if (st) return st;
  Gemm con;  // the contraction over MSA rows
  con.a = w.lt;
  con.b = w.rt;
  con.d = w.d;
  con.m = con.n = N * kOc;
  con.k = Sp;
  con.lda = con.ldb = Sp;
  con.ldd = static_cast<int64_t>(N) * kOc;
  st = run_gemm(con, info, stream);
  if (st) return st;
  const int64_t words = static_cast<int64_t>(N) * kOc * N * (kOc / 8);
  opm_relayout_kernel<<<grid_of(words, 256, info), 256, 0, stream>>>(reinterpret_cast<const uint4*>(w.d),
                                                                     reinterpret_cast<uint4*>(w.p), N);
  st = launched("opm_relayout launch");
  if (st) return st;
  Gemm proj;  // (P W_o^T + b_o) / d(n), one pair per row
  proj.a = w.p;
  proj.b = img;
  proj.d = delta;
  proj.m = N * N;
  proj.n = kCz;
  proj.k = kOc * kOc;
  proj.lda = proj.ldb = kOc * kOc;
  proj.ldd = kCz;
  proj.bias = vec + 2 * kCm + 2 * kOc * kCm;
  proj.row_scale = w.n;
  return run_gemm(proj, info, stream);
}

// ================================================================== pair-weighted averaging
// Packed image: [W_v; W_g] bf16 [128][64] | W_o bf16 [64][64] | fp32 ln_m_w[64] ln_m_b[64]
// ln_z_w[128] w_b[8][128]
constexpr size_t kPwaVg = static_cast<size_t>(2 * kCm) * kCm * 2;
constexpr size_t kPwaWo = static_cast<size_t>(kCm) * kCm * 2;
constexpr size_t kPwaVec = kCm + kCm + kCz + kPh * kCz;
constexpr size_t kPwaPacked = kPwaVg + kPwaWo + kPwaVec * 4;

// logits[h][i][j] = W_b[h] . (gamma * LNhat(z[i, j])): one warp per pair, 4 channels a lane.
__global__ void __launch_bounds__(256) pwa_logits_kernel(const __nv_bfloat16* __restrict__ z,
                                                         const float* __restrict__ vec, float* __restrict__ logits,
                                                         int N) {
  __shared__ float wb[kPh][kCz];
  __shared__ float g[kCz];
  const float* ln_z = vec + 2 * kCm;
  for (int t = threadIdx.x; t < kPh * kCz; t += blockDim.x) wb[t / kCz][t % kCz] = ln_z[kCz + t];
  for (int t = threadIdx.x; t < kCz; t += blockDim.x) g[t] = ln_z[t];
  __syncthreads();
  const int lane = threadIdx.x % 32;
  const int64_t pairs = static_cast<int64_t>(N) * N;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  for (int64_t p = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32; p < pairs; p += warps) {
    const uint2 raw = reinterpret_cast<const uint2*>(z + p * kCz)[lane];
    float v[4] = {bf16_lo(raw.x), bf16_hi(raw.x), bf16_lo(raw.y), bf16_hi(raw.y)};
    const float mean = warp_sum(v[0] + v[1] + v[2] + v[3]) * (1.0f / kCz);
    float q = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      v[k] -= mean;
      q += v[k] * v[k];
    }
    const float rstd = rsqrtf(warp_sum(q) * (1.0f / kCz) + 1e-5f);
    float acc[kPh];
#pragma unroll
    for (int h = 0; h < kPh; ++h) {
      float a = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) a = fmaf(v[k] * g[4 * lane + k], wb[h][4 * lane + k], a);
      acc[h] = warp_sum(a) * rstd;
    }
    if (lane < kPh) {
      float mine = acc[0];
#pragma unroll
      for (int h = 1; h < kPh; ++h)
        if (lane == h) mine = acc[h];
      logits[static_cast<int64_t>(lane) * pairs + p] = mine;
    }
  }
}

// weights[h][i][j] = softmax_j(logits[h][i][j] - 1e9 (1 - keys[j])), bf16, zero for N <= j < Np.
// One warp per (h, i) row.
__global__ void __launch_bounds__(256) pwa_softmax_kernel(const float* __restrict__ logits,
                                                          const uint8_t* __restrict__ keys,
                                                          __nv_bfloat16* __restrict__ weights, int N, int Np) {
  const int lane = threadIdx.x % 32;
  const int64_t rows = static_cast<int64_t>(kPh) * N;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32; r < rows; r += warps) {
    const float* row = logits + r * N;
    float mx = -INFINITY;
    for (int j = lane; j < N; j += 32) mx = fmaxf(mx, row[j] + (keys[j] ? 0.0f : -1.0e9f));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    float sum = 0.f;
    for (int j = lane; j < N; j += 32) sum += __expf(row[j] + (keys[j] ? 0.0f : -1.0e9f) - mx);
    const float inv = 1.0f / warp_sum(sum);
    __nv_bfloat16* out = weights + r * Np;
    for (int j = lane; j < Np; j += 32)
      out[j] = __float2bfloat16_rn(j < N ? __expf(row[j] + (keys[j] ? 0.0f : -1.0e9f) - mx) * inv : 0.0f);
  }
}

// vg [(s, j)][h 8 + e] (v part, the first 64 columns of 128) -> vt[h][(s, e)][j], zero for N <= j < Np.
__global__ void pwa_values_kernel(const __nv_bfloat16* __restrict__ vg, __nv_bfloat16* __restrict__ vt, int S, int N,
                                  int Np) {
  const int64_t total = static_cast<int64_t>(kPh) * S * kPd * Np;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int j = static_cast<int>(t % Np);
    const int64_t hse = t / Np;
    const int e = static_cast<int>(hse % kPd);
    const int64_t hs = hse / kPd;
    const int s = static_cast<int>(hs % S), h = static_cast<int>(hs / S);
    vt[t] = j < N ? vg[(static_cast<int64_t>(s) * N + j) * (2 * kCm) + h * kPd + e] : __float2bfloat16_rn(0.0f);
  }
}

// G[(s, i)][h 8 + e] = sigmoid(g[(s, i)][h 8 + e]) * o[h][i][s 8 + e]
__global__ void pwa_gate_kernel(const __nv_bfloat16* __restrict__ vg, const __nv_bfloat16* __restrict__ o,
                                __nv_bfloat16* __restrict__ gated, int S, int N) {
  const int64_t total = static_cast<int64_t>(S) * N * kCm;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int he = static_cast<int>(t % kCm);
    const int64_t si = t / kCm;
    const int i = static_cast<int>(si % N), s = static_cast<int>(si / N);
    const int h = he / kPd, e = he % kPd;
    const float gv = __bfloat162float(vg[si * (2 * kCm) + kCm + he]);
    const float ov = __bfloat162float(o[(static_cast<int64_t>(h) * N + i) * (static_cast<int64_t>(S) * kPd) + s * kPd + e]);
    gated[t] = __float2bfloat16_rn(ov / (1.0f + __expf(-gv)));
  }
}

struct PwaWs {
  float* logits;
  __nv_bfloat16 *weights, *x, *vg, *vt, *o, *gated;
};

PwaWs pwa_carve(void* ws, int S, int N) {
  const int Np = round_up(N, 8);
  uint8_t* q = static_cast<uint8_t*>(ws);
  PwaWs w;
  const size_t sn = static_cast<size_t>(S) * N;
  w.logits = reinterpret_cast<float*>(q);
  q += a256(static_cast<size_t>(kPh) * N * N * 4);
  w.weights = reinterpret_cast<__nv_bfloat16*>(q);
  q += a256(static_cast<size_t>(kPh) * N * Np * 2);
  w.x = reinterpret_cast<__nv_bfloat16*>(q);
  q += a256(sn * kCm * 2);
  w.vg = reinterpret_cast<__nv_bfloat16*>(q);
  q += a256(sn * 2 * kCm * 2);
  w.vt = reinterpret_cast<__nv_bfloat16*>(q);
  q += a256(static_cast<size_t>(kPh) * S * kPd * Np * 2);
  w.o = reinterpret_cast<__nv_bfloat16*>(q);
  q += a256(sn * kCm * 2);
  w.gated = reinterpret_cast<__nv_bfloat16*>(q);
  return w;
}

size_t pwa_workspace(int S, int N) {
  const size_t Np = round_up(N, 8);
  const size_t sn = static_cast<size_t>(S) * N;
  return a256(static_cast<size_t>(kPh) * N * N * 4) + a256(static_cast<size_t>(kPh) * N * Np * 2) + a256(sn * kCm * 2) +
         a256(sn * 2 * kCm * 2) + a256(static_cast<size_t>(kPh) * S * kPd * Np * 2) + 2 * a256(sn * kCm * 2);
}

int pwa_forward(const void* m, const void* z, const uint8_t* keys, const void* packed, void* out, void* workspace,
                int S, int N, const DeviceInfo& info, cudaStream_t stream) {
  const int Np = round_up(N, 8);
  PwaWs w = pwa_carve(workspace, S, N);
  const uint8_t* img = static_cast<const uint8_t*>(packed);
  const float* vec = reinterpret_cast<const float*>(img + kPwaVg + kPwaWo);
  const int64_t sn = static_cast<int64_t>(S) * N;
  pwa_logits_kernel<<<grid_of(static_cast<int64_t>(N) * N * 32, 256, info), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(z), vec, w.logits, N);
  int st = launched("pwa_logits launch");
  if (st) return st;
  pwa_softmax_kernel<<<grid_of(static_cast<int64_t>(kPh) * N * 32, 256, info), 256, 0, stream>>>(w.logits, keys,
                                                                                                  w.weights, N, Np);
  st = launched("pwa_softmax launch");
  if (st) return st;
  st = cuda_status(launch_layernorm(m, w.x, vec, vec + kCm, sn, kCm, 1e-5f, 0, info.num_sms, stream),
                   "pwa layernorm launch");
  if (st) return st;
  Gemm vgp;  // [v | g] = LN(m) [W_v; W_g]^T
  vgp.a = w.x;
  vgp.b = img;
  vgp.d = w.vg;
  vgp.m = static_cast<int>(sn);
  vgp.n = 2 * kCm;
  vgp.k = kCm;
  vgp.lda = vgp.ldb = kCm;
  vgp.ldd = 2 * kCm;
  st = run_gemm(vgp, info, stream);
  if (st) return st;
  pwa_values_kernel<<<grid_of(static_cast<int64_t>(kPh) * S * kPd * Np, 256, info), 256, 0, stream>>>(w.vg, w.vt, S,
                                                                                                       N, Np);
  st = launched("pwa_values launch");
  if (st) return st;
  Gemm avg;  // o_h = w_h v_h for the 8 heads: [N(i)] x [(s, e)] over j
  avg.a = w.weights;
  avg.b = w.vt;
  avg.d = w.o;
  avg.batch = kPh;
  avg.m = N;
  avg.n = S * kPd;
  avg.k = Np;
  avg.lda = avg.ldb = Np;
  avg.ldd = static_cast<int64_t>(S) * kPd;
  avg.sa = static_cast<int64_t>(N) * Np;
  avg.sb = static_cast<int64_t>(S) * kPd * Np;
  avg.sd = static_cast<int64_t>(N) * S * kPd;
  st = run_gemm(avg, info, stream);
  if (st) return st;
  pwa_gate_kernel<<<grid_of(sn * kCm, 256, info), 256, 0, stream>>>(w.vg, w.o, w.gated, S, N);
  st = launched("pwa_gate launch");
  if (st) return st;
  Gemm outp;  // m' = m + G W_o^T
  outp.a = w.gated;
  outp.b = img + kPwaVg;
  outp.d = out;
  outp.m = static_cast<int>(sn);
  outp.n = kCm;
  outp.k = kCm;
  outp.lda = outp.ldb = kCm;
  outp.ldd = kCm;
  outp.epilogue = kEpiResidual;
  outp.residual = m;
  return run_gemm(outp, info, stream);
}

// ================================================================== transition on tensor cores
// x + W_sq(silu(W_a LN(x)) * W_b LN(x)) for rows of any width c (a multiple of 8) and factor
// n: LayerNorm, one GEMM with the SwiGLU epilogue (a / b interleaved in blocks of 16 rows),
// one GEMM with the residual epilogue. Packed: W_ab bf16 [2 n c][c] | W_sq bf16 [c][n c] |
// fp32 ln_w[c] ln_b[c].
struct TgLayout {
  size_t w_ab, w_sq, ln_w, ln_b, total;
};

TgLayout tg_layout(int c, int n) {
  TgLayout L;
  size_t o = 0;
  L.w_ab = o;
  o = a256(o + static_cast<size_t>(2 * n * c) * c * 2);
  L.w_sq = o;
  o = a256(o + static_cast<size_t>(c) * n * c * 2);
  L.ln_w = o;
  o = a256(o + static_cast<size_t>(c) * 4);
  L.ln_b = o;
  o = a256(o + static_cast<size_t>(c) * 4);
  L.total = o;
  return L;
}

size_t tg_workspace(int64_t rows, int c, int n) {
  return a256(static_cast<size_t>(rows) * c * 2) + a256(static_cast<size_t>(rows) * n * c * 2);
}

int tg_forward(const void* x, const void* packed, void* out, void* workspace, int64_t rows, int c, int n,
               const DeviceInfo& info, cudaStream_t stream) {
  const TgLayout L = tg_layout(c, n);
  const uint8_t* img = static_cast<const uint8_t*>(packed);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* y = ws;
  void* hid = ws + a256(static_cast<size_t>(rows) * c * 2);
  int st = cuda_status(launch_layernorm(x, y, reinterpret_cast<const float*>(img + L.ln_w),
                                        reinterpret_cast<const float*>(img + L.ln_b), rows, c, 1e-5f, 0, info.num_sms,
                                        stream),
                       "transition layernorm launch");
  if (st) return st;
  Gemm up;
  up.a = y;
  up.b = img + L.w_ab;
  up.d = hid;
  up.m = static_cast<int>(rows);
  up.n = 2 * n * c;
  up.k = c;
  up.lda = up.ldb = c;
  up.ldd = static_cast<int64_t>(n) * c;
  up.epilogue = kEpiSwiGLU;
  st = run_gemm(up, info, stream);
  if (st) return st;
  Gemm down;
  down.a = hid;
  down.b = img + L.w_sq;
  down.d = out;
  down.m = static_cast<int>(rows);
  down.n = c;
  down.k = n * c;
  down.lda = down.ldb = static_cast<int64_t>(n) * c;
  down.ldd = c;
  down.epilogue = kEpiResidual;
  down.residual = x;
  return run_gemm(down, info, stream);
}

int to_bf16(const float* a, const float* b, int rows, int cols, int interleave, void* dst, cudaStream_t stream) {
  to_bf16_kernel<<<256, 256, 0, stream>>>(a, b, rows, cols, interleave, static_cast<__nv_bfloat16*>(dst));
  return static_cast<int>(cudaGetLastError());
}

int copy_f32(void* dst, const float* src, size_t count, cudaStream_t stream) {
  return static_cast<int>(cudaMemcpyAsync(dst, src, count * 4, cudaMemcpyDeviceToDevice, stream));
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

}  // namespace
}  // namespace ffb

using namespace ffb;

extern "C" {

size_t ffb_opm_packed_bytes(void) { return kOpmPacked; }

size_t ffb_opm_workspace_bytes(int S, int N) { return (S > 0 && N > 0) ? opm_workspace(S, N) : 0; }

int ffb_opm_prepare(const float* ln_w, const float* ln_b, const float* to_left, const float* to_right,
                    const float* to_out_w, const float* to_out_b, void* packed, void* stream) {
  if (!ln_w || !ln_b || !to_left || !to_right || !to_out_w || !to_out_b || !packed)
    return fail(FFB_ERR_ARG, "opm_prepare: null pointer");
  if (!aligned(packed, 16)) return fail(FFB_ERR_ARG, "opm_prepare: packed not 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* img = static_cast<uint8_t*>(packed);
  float* vec = reinterpret_cast<float*>(img + kOpmWo);
  int rc = to_bf16(to_out_w, nullptr, kCz, kOc * kOc, 0, img, s);
  if (rc == 0) rc = copy_f32(vec, ln_w, kCm, s);
  if (rc == 0) rc = copy_f32(vec + kCm, ln_b, kCm, s);
  if (rc == 0) rc = copy_f32(vec + 2 * kCm, to_left, kOc * kCm, s);
  if (rc == 0) rc = copy_f32(vec + 2 * kCm + kOc * kCm, to_right, kOc * kCm, s);
  if (rc == 0) rc = copy_f32(vec + 2 * kCm + 2 * kOc * kCm, to_out_b, kCz, s);
  return cuda_status(rc, "opm_prepare");
}

int ffb_opm_fwd(const void* msa, const uint8_t* row_mask, const void* packed, void* delta, void* workspace,
                size_t workspace_bytes, int B, int S, int N, float count_offset, void* stream) {
  if (B <= 0 || S <= 0 || N <= 0) return fail(FFB_ERR_ARG, "opm: B=%d S=%d N=%d", B, S, N);
  if (!msa || !row_mask || !packed || !delta || !workspace) return fail(FFB_ERR_ARG, "opm: null pointer");
  if (workspace_bytes < opm_workspace(S, N)) return fail(FFB_ERR_ARG, "opm: workspace of %zu bytes, %zu needed",
                                                         workspace_bytes, opm_workspace(S, N));
  if (!aligned(workspace, 256) || !aligned(packed, 16) || !aligned(delta, 16) || !aligned(msa, 16))
    return fail(FFB_ERR_ARG, "opm: misaligned pointer");
  DeviceInfo info;
  int st = device_info(&info);
  if (st) return st;
  for (int b = 0; b < B && st == 0; ++b)
    st = opm_forward(static_cast<const __nv_bfloat16*>(msa) + static_cast<int64_t>(b) * S * N * kCm,
                     row_mask + static_cast<int64_t>(b) * S * N, packed,
                     static_cast<__nv_bfloat16*>(delta) + static_cast<int64_t>(b) * N * N * kCz, workspace, S, N,
                     count_offset, info, static_cast<cudaStream_t>(stream));
  return st;
}

size_t ffb_pwa_packed_bytes(void) { return kPwaPacked; }

size_t ffb_pwa_workspace_bytes(int S, int N) { return (S > 0 && N > 0) ? pwa_workspace(S, N) : 0; }

int ffb_pwa_prepare(const float* ln_msa_w, const float* ln_msa_b, const float* ln_pair_w, const float* to_bias,
                    const float* to_value, const float* to_gate, const float* to_out, void* packed, void* stream) {
  if (!ln_msa_w || !ln_msa_b || !ln_pair_w || !to_bias || !to_value || !to_gate || !to_out || !packed)
    return fail(FFB_ERR_ARG, "pwa_prepare: null pointer");
  if (!aligned(packed, 16)) return fail(FFB_ERR_ARG, "pwa_prepare: packed not 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* img = static_cast<uint8_t*>(packed);
  float* vec = reinterpret_cast<float*>(img + kPwaVg + kPwaWo);
  int rc = to_bf16(to_value, nullptr, kCm, kCm, 0, img, s);
  if (rc == 0) rc = to_bf16(to_gate, nullptr, kCm, kCm, 0, img + kPwaVg / 2, s);
  if (rc == 0) rc = to_bf16(to_out, nullptr, kCm, kCm, 0, img + kPwaVg, s);
  if (rc == 0) rc = copy_f32(vec, ln_msa_w, kCm, s);
  if (rc == 0) rc = copy_f32(vec + kCm, ln_msa_b, kCm, s);
  if (rc == 0) rc = copy_f32(vec + 2 * kCm, ln_pair_w, kCz, s);
  if (rc == 0) rc = copy_f32(vec + 2 * kCm + kCz, to_bias, kPh * kCz, s);
  return cuda_status(rc, "pwa_prepare");
}

int ffb_pwa_fwd(const void* msa, const void* pair, const uint8_t* key_mask, const void* packed, void* out,
                void* workspace, size_t workspace_bytes, int B, int S, int N, void* stream) {
  if (B <= 0 || S <= 0 || N <= 0) return fail(FFB_ERR_ARG, "pwa: B=%d S=%d N=%d", B, S, N);
  if (!msa || !pair || !key_mask || !packed || !out || !workspace) return fail(FFB_ERR_ARG, "pwa: null pointer");
  if (msa == out) return fail(FFB_ERR_ARG, "pwa: out must not alias the MSA");
  if (workspace_bytes < pwa_workspace(S, N))
    return fail(FFB_ERR_ARG, "pwa: workspace of %zu bytes, %zu needed", workspace_bytes, pwa_workspace(S, N));
  if (!aligned(workspace, 256) || !aligned(packed, 16) || !aligned(out, 16) || !aligned(msa, 16) || !aligned(pair, 16))
    return fail(FFB_ERR_ARG, "pwa: misaligned pointer");
  DeviceInfo info;
  int st = device_info(&info);
  if (st) return st;
  for (int b = 0; b < B && st == 0; ++b)
    st = pwa_forward(static_cast<const __nv_bfloat16*>(msa) + static_cast<int64_t>(b) * S * N * kCm,
                     static_cast<const __nv_bfloat16*>(pair) + static_cast<int64_t>(b) * N * N * kCz,
                     key_mask + static_cast<int64_t>(b) * N, packed,
                     static_cast<__nv_bfloat16*>(out) + static_cast<int64_t>(b) * S * N * kCm, workspace, S, N, info,
                     static_cast<cudaStream_t>(stream));
  return st;
}

size_t ffb_transition_gemm_packed_bytes(int c, int n) { return (c > 0 && n > 0) ? tg_layout(c, n).total : 0; }

size_t ffb_transition_gemm_workspace_bytes(int64_t rows, int c, int n) {
  return (rows > 0 && c > 0 && n > 0) ? tg_workspace(rows, c, n) : 0;
}

int ffb_transition_gemm_prepare(const float* ln_w, const float* ln_b, const float* expand_a, const float* expand_b,
                                const float* squeeze, int c, int n, void* packed, void* stream) {
  if (!ln_w || !ln_b || !expand_a || !expand_b || !squeeze || !packed)
    return fail(FFB_ERR_ARG, "transition_gemm_prepare: null pointer");
  if (c <= 0 || n <= 0 || c % 8 != 0 || (n * c) % 16 != 0)
    return fail(FFB_ERR_UNSUPPORTED, "transition_gemm: c=%d n=%d (c a multiple of 8, n c of 16)", c, n);
  if (!aligned(packed, 256)) return fail(FFB_ERR_ARG, "transition_gemm_prepare: packed not 256-byte aligned");
  const TgLayout L = tg_layout(c, n);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* img = static_cast<uint8_t*>(packed);
  int rc = to_bf16(expand_a, expand_b, n * c, c, 1, img + L.w_ab, s);
  if (rc == 0) rc = to_bf16(squeeze, nullptr, c, n * c, 0, img + L.w_sq, s);
  if (rc == 0) rc = copy_f32(img + L.ln_w, ln_w, c, s);
  if (rc == 0) rc = copy_f32(img + L.ln_b, ln_b, c, s);
  return cuda_status(rc, "transition_gemm_prepare");
}

int ffb_transition_gemm_fwd(const void* x, const void* packed, void* out, void* workspace, size_t workspace_bytes,
                            int64_t rows, int c, int n, void* stream) {
  if (rows <= 0 || c <= 0 || n <= 0 || c % 8 != 0 || (n * c) % 16 != 0 || rows > (1ll << 31) - 1)
    return fail(FFB_ERR_UNSUPPORTED, "transition_gemm: rows=%lld c=%d n=%d", static_cast<long long>(rows), c, n);
  if (!x || !packed || !out || !workspace) return fail(FFB_ERR_ARG, "transition_gemm: null pointer");
  if (x == out) return fail(FFB_ERR_ARG, "transition_gemm: out must not alias x");
  if (workspace_bytes < tg_workspace(rows, c, n))
    return fail(FFB_ERR_ARG, "transition_gemm: workspace of %zu bytes, %zu needed", workspace_bytes,
                tg_workspace(rows, c, n));
  if (!aligned(workspace, 256) || !aligned(packed, 256) || !aligned(x, 16) || !aligned(out, 16))
    return fail(FFB_ERR_ARG, "transition_gemm: misaligned pointer");
  DeviceInfo info;
  int st = device_info(&info);
  if (st) return st;
  return tg_forward(x, packed, out, workspace, rows, c, n, info, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
