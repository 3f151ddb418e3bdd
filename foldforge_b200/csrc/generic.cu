// The fp32 ("fp32" precision) path of the Pairformer ops, and the path for widths the
// tcgen05 kernels are not built for (e.g. the template stack's c_z = 64), on FP32 SIMT cores.
//
// Every op runs in fp32 end to end: LayerNorms with a two-pass variance, matrix products as
// register-blocked FFMA GEMMs with fp32 accumulation, softmax with `expf`. The equations are
// the reference block's (legacy/reference/triangle.py:19-50, legacy/attention.py:108-171,
// legacy/reference/attention.py:14-100, legacy/transformer.py:88-133,
// legacy/reference/transition.py:28-59); weights are the engine's fp32 matrices in their
// natural [out, in] layout (no packing). This path exists for accuracy (the north star's
// fp32 mode) and generality, not speed: the bf16 tcgen05 kernels serve the AF3 widths in
// master precision.
//
// Building blocks (all launched on the caller's stream, scratch from the caller's workspace):
//   sgemm_nt_kernel        C[b] = A[b] B[b]^T (+ bias) with a fused epilogue (store, masked
//                          residual, sigmoid-gated masked residual)
//   ln_rows_kernel         LayerNorm over the last axis (any width), fp32
//   trimul_gate_kernel     L / R = P * sigmoid(P_gate) * m_i m_k, written channel-major (the
//                          incoming direction transposed) for the per-channel contraction
//   channel_ln_kernel      LayerNorm over the channels of a channel-major U, written pair-major
//   attention_f32_kernel   softmax(q k^T / sqrt(d) + bias, mask -> -1e9) v per query thread with an
//                          online softmax, optional sigmoid gate on the output
//   swiglu_kernel          H = silu(A) * B
#include <math.h>

#include "../../include/foldforge_b200.h"
#include "abi_util.h"
#include "common.cuh"
#include "kernels.h"

namespace ffb {
namespace {

// ------------------------------------------------------------------ GEMM
enum GenericEpi : int {
  kGStore = 0,         // C = acc + bias[n]
  kGResidual = 1,      // C = R + (acc + bias[n]) * rowmask(m)
  kGGatedResidual = 2  // C = R + (acc + bias[n]) * sigmoid(G[m, n]) * rowmask(m)
};

// rowmask(m): 1 (kind 0); mask[m] (kind 1, token rows); mask[b N + i] mask[b N + j] for
// m = (b N + i) N + j (kind 2, pair rows).
struct RowMask {
  const uint8_t* mask;
  int kind;
  int N;
  __device__ __forceinline__ float operator()(int64_t m) const {
    if (kind == 0 || mask == nullptr) return 1.0f;
    if (kind == 1) return mask[m] ? 1.0f : 0.0f;
    const int64_t j = m % N;
    const int64_t bi = m / N;
    const int64_t b = bi / N;
    return (mask[bi] && mask[b * N + j]) ? 1.0f : 0.0f;
  }
};

struct SgemmArgs {
  const float* A;
  const float* B;
  float* C;
  int M, N, K;
  int64_t lda, ldb, ldc;
  int64_t sa, sb, sc;  // batch strides (elements)
  const float* bias;   // [N] or null
  int epi;
  const float* R;      // residual, layout of C
  const float* G;      // gate, layout of C
  RowMask rm;
};

constexpr int kBM = 64, kBN = 64, kBK = 16, kGThreads = 256;

// 64 x 64 tile per CTA, 4 x 4 per thread, K staged in 16-wide slices (transposed in shared
// memory so that the inner product reads contiguous rows).
__global__ void __launch_bounds__(kGThreads) sgemm_nt_kernel(SgemmArgs g) {
  __shared__ float As[kBK][kBM + 4];
  __shared__ float Bs[kBK][kBN + 4];
  const int b = blockIdx.z;
  const float* A = g.A + b * g.sa;
  const float* B = g.B + b * g.sb;
  const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * kBN;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float acc[4][4] = {};
  // loader: each thread moves 4 elements of A and 4 of B per slice
  const int lr = threadIdx.x / 4;        // row 0..63 of the tile
  const int lk = (threadIdx.x % 4) * 4;  // k 0, 4, 8, 12
  for (int k0 = 0; k0 < g.K; k0 += kBK) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int k = k0 + lk + e;
      const int am = m0 + lr, bn = n0 + lr;
      As[lk + e][lr] = (am < g.M && k < g.K) ? A[am * g.lda + k] : 0.0f;
      Bs[lk + e][lr] = (bn < g.N && k < g.K) ? B[bn * g.ldb + k] : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kBK; ++kk) {
      float a[4], bb[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bb[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], bb[j], acc[i][j]);
    }
    __syncthreads();
  }
  float* C = g.C + b * g.sc;
  const float* R = g.R ? g.R + b * g.sc : nullptr;
  const float* G = g.G ? g.G + b * g.sc : nullptr;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= g.M) continue;
    const float rmv = g.epi == kGStore ? 1.0f : g.rm(static_cast<int64_t>(b) * g.M + m);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n >= g.N) continue;
      float v = acc[i][j] + (g.bias ? g.bias[n] : 0.0f);
      const int64_t at = m * g.ldc + n;
      if (g.epi == kGResidual) {
        v = R[at] + v * rmv;
      } else if (g.epi == kGGatedResidual) {
        v = R[at] + v * (1.0f / (1.0f + expf(-G[at]))) * rmv;
      }
      C[at] = v;
    }
  }
}

int sgemm(const SgemmArgs& g, int batch, cudaStream_t stream) {
  if (g.M <= 0 || g.N <= 0 || batch <= 0) return 0;
  dim3 grid((g.N + kBN - 1) / kBN, (g.M + kBM - 1) / kBM, batch);
  sgemm_nt_kernel<<<grid, kGThreads, 0, stream>>>(g);
  return static_cast<int>(cudaGetLastError());
}

SgemmArgs plain_gemm(const float* A, const float* W, float* C, int64_t M, int N, int K) {
  SgemmArgs g{};
  g.A = A;
  g.B = W;
  g.C = C;
  g.M = static_cast<int>(M);
  g.N = N;
  g.K = K;
  g.lda = K;
  g.ldb = K;
  g.ldc = N;
  g.epi = kGStore;
  return g;
}

// ------------------------------------------------------------------ LayerNorm (any width)
// One warp per row, two-pass variance from global memory (rows stay in L1 / L2).
__global__ void ln_rows_kernel(const float* __restrict__ x, float* __restrict__ y, const float* __restrict__ gamma,
                               const float* __restrict__ beta, int64_t rows, int c, float eps) {
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;
  const float* xr = x + row * c;
  float s = 0.f;
  for (int i = lane; i < c; i += 32) s += xr[i];
  const float mean = warp_sum(s) / static_cast<float>(c);
  float q = 0.f;
  for (int i = lane; i < c; i += 32) {
    const float d = xr[i] - mean;
    q += d * d;
  }
  const float rstd = 1.0f / sqrtf(warp_sum(q) / static_cast<float>(c) + eps);
  float* yr = y + row * c;
  for (int i = lane; i < c; i += 32) {
    float v = (xr[i] - mean) * rstd;
    if (gamma) v *= gamma[i];
    if (beta) v += beta[i];
    yr[i] = v;
  }
}

int ln_rows(const float* x, float* y, const float* gamma, const float* beta, int64_t rows, int c, cudaStream_t stream) {
  if (rows <= 0) return 0;
  const int threads = 256;
  const int64_t blocks = (rows * 32 + threads - 1) / threads;
  ln_rows_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(x, y, gamma, beta, rows, c, 1e-5f);
  return static_cast<int>(cudaGetLastError());
}

// ------------------------------------------------------------------ triangle multiplication pieces
__device__ __forceinline__ float sigm(float x) { return 1.0f / (1.0f + expf(-x)); }

// P [B, N, N, 4h] holds (left, right, left gate, right gate) per pair. Writes, for channel c,
// L_c[a][k] and R_c[a][k] ([B, h, N, N]) so that u_c = L_c R_c^T:
//   outgoing: L_c[a][k] = left[a, k]      incoming: L_c[a][k] = left[k, a]
__global__ void trimul_gate_kernel(const float* __restrict__ P, const uint8_t* __restrict__ mask,
                                   float* __restrict__ Lc, float* __restrict__ Rc, int B, int N, int h,
                                   int outgoing) {
  const int64_t total = static_cast<int64_t>(B) * h * N * N;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int k = static_cast<int>(t % N);
    const int a = static_cast<int>((t / N) % N);
    const int c = static_cast<int>((t / (static_cast<int64_t>(N) * N)) % h);
    const int b = static_cast<int>(t / (static_cast<int64_t>(N) * N * h));
    const int i = outgoing ? a : k, j = outgoing ? k : a;  // the pair (i, j) read
    const float m = (mask[b * N + i] && mask[b * N + j]) ? 1.0f : 0.0f;
    const float* pp = P + ((static_cast<int64_t>(b) * N + i) * N + j) * (4 * h);
    Lc[t] = pp[c] * m * sigm(pp[2 * h + c]);
    Rc[t] = pp[h + c] * m * sigm(pp[3 * h + c]);
  }
}

// U [B, h, N, N] channel-major -> u [B, N, N, h] = LN over the h channels of each pair.
__global__ void channel_ln_kernel(const float* __restrict__ U, float* __restrict__ u, const float* __restrict__ gamma,
                                  const float* __restrict__ beta, int B, int N, int h) {
  const int64_t pairs = static_cast<int64_t>(B) * N * N;
  const int64_t nn = static_cast<int64_t>(N) * N;
  for (int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; p < pairs;
       p += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t b = p / nn, ij = p % nn;
    const float* src = U + b * h * nn + ij;
    float s = 0.f;
    for (int c = 0; c < h; ++c) s += src[c * nn];
    const float mean = s / static_cast<float>(h);
    float q = 0.f;
    for (int c = 0; c < h; ++c) {
      const float d = src[c * nn] - mean;
      q += d * d;
    }
    const float rstd = 1.0f / sqrtf(q / static_cast<float>(h) + 1e-5f);
    float* dst = u + p * h;
    for (int c = 0; c < h; ++c) dst[c] = (src[c * nn] - mean) * rstd * gamma[c] + beta[c];
  }
}

__global__ void swiglu_kernel(const float* __restrict__ A, const float* __restrict__ Bm, float* __restrict__ H,
                              int64_t n) {
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < n;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float a = A[t];
    H[t] = a * sigm(a) * Bm[t];
  }
}

int grid_for(int64_t n, int threads = 256) {
  const int64_t g = (n + threads - 1) / threads;
  return static_cast<int>(g < 148 * 32 ? (g > 0 ? g : 1) : 148 * 32);
}

// ------------------------------------------------------------------ attention
// One thread per query of one (batch, problem row, head). Element (b, r, q, e) of head h of
// Q / K / V / G / O is at base + b*s_b + r*s_r + q*s_q + h*d + e. Logits:
//   (q * d^-1/2) . k + bias[b, h, q, k] (+ bias2[b, h, q, k]);
// keys with mask[b, k] == 0, or every key when row_mask and mask[b, row0 + r] == 0, get the
// logit REPLACED by -1e9 (a fully masked row averages uniformly). O = softmax . V, times
// sigmoid(G + gate_bias) when G is given.
struct AttnArgs {
  const float *q, *k, *v, *g;
  float* o;
  int64_t s_b, s_r, s_q;
  const float* bias;
  int64_t bb, bh, bq, bk;
  const float* bias2;
  int64_t cb, ch, cq, ck;
  const uint8_t* mask;
  int row_mask, row0;
  int B, R, N, H, d;
  float gate_bias;
};

constexpr int kAQ = 128;   // queries per CTA
constexpr int kAK = 32;    // keys per shared-memory chunk
constexpr int kADmax = 64;

// kD: a bound on the head width d (registers hold q and the output accumulator)
template <int kD>
__global__ void __launch_bounds__(kAQ) attention_f32_kernel(AttnArgs a) {
  __shared__ float ks[kAK][kADmax];
  __shared__ float vs[kAK][kADmax];
  __shared__ float kmask[kAK];
  const int prob = blockIdx.y;  // (b, r, h)
  const int h = prob % a.H;
  const int r = (prob / a.H) % a.R;
  const int b = prob / (a.H * a.R);
  const int q = blockIdx.x * kAQ + threadIdx.x;
  const bool active = q < a.N;
  const int d = a.d;
  const int64_t base = b * a.s_b + r * a.s_r + h * d;
  const float scale = rsqrtf(static_cast<float>(d));
  float qv[kD], acc[kD];
#pragma unroll
  for (int e = 0; e < kD; ++e) {
    qv[e] = (active && e < d) ? a.q[base + q * a.s_q + e] * scale : 0.0f;
    acc[e] = 0.0f;
  }
  const bool row_on = !a.row_mask || a.mask[static_cast<int64_t>(b) * a.N + a.row0 + r] != 0;
  float m = -INFINITY, l = 0.0f;
  for (int k0 = 0; k0 < a.N; k0 += kAK) {
    const int nk = a.N - k0 < kAK ? a.N - k0 : kAK;
    __syncthreads();
    for (int t = threadIdx.x; t < nk * d; t += kAQ) {
      const int kk = t / d, e = t % d;
      const int64_t at = base + static_cast<int64_t>(k0 + kk) * a.s_q + e;
      ks[kk][e] = a.k[at];
      vs[kk][e] = a.v[at];
    }
    for (int t = threadIdx.x; t < nk; t += kAQ)
      kmask[t] = (row_on && a.mask[static_cast<int64_t>(b) * a.N + k0 + t]) ? 1.0f : 0.0f;
    __syncthreads();
    if (!active) continue;
    for (int kk = 0; kk < nk; ++kk) {
      float s = 0.0f;
#pragma unroll
      for (int e = 0; e < kD; ++e)
        if (e < d) s = fmaf(qv[e], ks[kk][e], s);
      const int key = k0 + kk;
      if (a.bias) s += a.bias[b * a.bb + h * a.bh + q * a.bq + key * a.bk];
      if (a.bias2) s += a.bias2[b * a.cb + h * a.ch + q * a.cq + key * a.ck];
      if (kmask[kk] == 0.0f) s = -1.0e9f;
      if (s > m) {
        const float corr = expf(m - s);  // 0 for the first key (m = -inf)
        l *= corr;
#pragma unroll
        for (int e = 0; e < kD; ++e) acc[e] *= corr;
        m = s;
      }
      const float p = expf(s - m);
      l += p;
#pragma unroll
      for (int e = 0; e < kD; ++e)
        if (e < d) acc[e] = fmaf(p, vs[kk][e], acc[e]);
    }
  }
  if (!active) return;
  const float inv = 1.0f / l;
  const int64_t at = base + q * a.s_q;
#pragma unroll
  for (int e = 0; e < kD; ++e) {
    if (e >= d) break;
    float v = acc[e] * inv;
    if (a.g) v *= sigm(a.g[at + e] + a.gate_bias);
    a.o[at + e] = v;
  }
}

int attention(const AttnArgs& a, cudaStream_t stream) {
  if (a.d > kADmax || a.d <= 0) return static_cast<int>(cudaErrorInvalidValue);
  dim3 grid((a.N + kAQ - 1) / kAQ, a.B * a.R * a.H);
  if (a.d <= 8)
    attention_f32_kernel<8><<<grid, kAQ, 0, stream>>>(a);
  else if (a.d <= 32)
    attention_f32_kernel<32><<<grid, kAQ, 0, stream>>>(a);
  else
    attention_f32_kernel<kADmax><<<grid, kAQ, 0, stream>>>(a);
  return static_cast<int>(cudaGetLastError());
}

// ------------------------------------------------------------------ workspace carving
struct Carver {
  uint8_t* p;
  size_t used = 0;
  float* take(int64_t floats) {
    float* out = reinterpret_cast<float*>(p + used);
    used += (static_cast<size_t>(floats) * 4 + 255) / 256 * 256;
    return out;
  }
};

int64_t up256(int64_t floats) { return (floats * 4 + 255) / 256 * 256; }

}  // namespace

// ================================================================== ops
size_t generic_trimul_workspace(int B, int N, int c, int h) {
  const int64_t M = static_cast<int64_t>(B) * N * N;
  return up256(M * c) + up256(M * 4 * h) + 3 * up256(static_cast<int64_t>(B) * h * N * N) + up256(M * h) +
         up256(M * c);
}

int generic_trimul(const float* z, const uint8_t* mask, const GenericTriMulWeights& w, float* out, void* workspace,
                   int B, int N, int c, int h, int outgoing, int masked_zero, cudaStream_t stream) {
  const int64_t M = static_cast<int64_t>(B) * N * N;
  Carver ws{static_cast<uint8_t*>(workspace)};
  float* x = ws.take(M * c);
  float* P = ws.take(M * 4 * h);
  float* Lc = ws.take(static_cast<int64_t>(B) * h * N * N);
  float* Rc = ws.take(static_cast<int64_t>(B) * h * N * N);
  float* U = ws.take(static_cast<int64_t>(B) * h * N * N);
  float* u = ws.take(M * h);
  float* G = ws.take(M * c);
  int rc = ln_rows(z, x, w.ln_w, w.ln_b, M, c, stream);
  // P = x [W_l; W_r; W_lg; W_rg]^T, one product per weight into its column block
  const float* ws4[4] = {w.to_left, w.to_right, w.to_left_gate, w.to_right_gate};
  for (int t = 0; t < 4 && rc == 0; ++t) {
    SgemmArgs g = plain_gemm(x, ws4[t], P + t * h, M, h, c);
    g.ldc = 4 * h;
    rc = sgemm(g, 1, stream);
  }
  if (rc == 0) {
    trimul_gate_kernel<<<grid_for(static_cast<int64_t>(B) * h * N * N), 256, 0, stream>>>(P, mask, Lc, Rc, B, N, h,
                                                                                          outgoing);
    rc = static_cast<int>(cudaGetLastError());
  }
  if (rc == 0) {  // U_c = L_c R_c^T for every (batch, channel)
    SgemmArgs g = plain_gemm(Lc, Rc, U, N, N, N);
    g.sa = g.sb = g.sc = static_cast<int64_t>(N) * N;
    rc = sgemm(g, B * h, stream);
  }
  if (rc == 0) {
    channel_ln_kernel<<<grid_for(M), 256, 0, stream>>>(U, u, w.ln_out_w, w.ln_out_b, B, N, h);
    rc = static_cast<int>(cudaGetLastError());
  }
  if (rc == 0) rc = sgemm(plain_gemm(x, w.to_gate, G, M, c, c), 1, stream);
  if (rc == 0) {
    SgemmArgs g = plain_gemm(u, w.to_out, out, M, c, h);
    g.epi = kGGatedResidual;
    g.R = z;
    g.G = G;
    g.rm = RowMask{mask, masked_zero ? 2 : 0, N};
    rc = sgemm(g, 1, stream);
  }
  return rc;
}

size_t generic_triattn_workspace(int B, int N, int c, int H, int d) {
  const int64_t M = static_cast<int64_t>(B) * N * N;
  const int64_t hd = static_cast<int64_t>(H) * d;
  return up256(M * c) + 5 * up256(M * hd) + up256(M * H);
}

int generic_triattn(const float* z, const uint8_t* mask, const GenericTriAttnWeights& w, float* out, void* workspace,
                    int B, int N, int c, int H, int d, int starting, int masked_zero, cudaStream_t stream) {
  const int64_t M = static_cast<int64_t>(B) * N * N;
  const int hd = H * d;
  Carver ws{static_cast<uint8_t*>(workspace)};
  float* x = ws.take(M * c);
  float* Q = ws.take(M * hd);
  float* K = ws.take(M * hd);
  float* V = ws.take(M * hd);
  float* Gt = ws.take(M * hd);
  float* O = ws.take(M * hd);
  float* Bp = ws.take(M * H);
  int rc = ln_rows(z, x, w.ln_w, w.ln_b, M, c, stream);
  const float* wm[4] = {w.to_query, w.to_key, w.to_value, w.to_gate};
  float* dst[4] = {Q, K, V, Gt};
  for (int t = 0; t < 4 && rc == 0; ++t) rc = sgemm(plain_gemm(x, wm[t], dst[t], M, hd, c), 1, stream);
  if (rc == 0) rc = sgemm(plain_gemm(x, w.to_bias, Bp, M, H, c), 1, stream);
  if (rc == 0) {
    // pair (i, j) of batch b at ((b N + i) N + j) * hd. Starting: problem row r = i, query /
    // key = j. Ending: r = j, query / key = i. The bias is b_h[query][key] = Bp[b, q, k, h]
    // in both directions (untransposed, AF3).
    AttnArgs a{};
    a.q = Q;
    a.k = K;
    a.v = V;
    a.g = Gt;
    a.o = O;
    a.s_b = static_cast<int64_t>(N) * N * hd;
    a.s_r = starting ? static_cast<int64_t>(N) * hd : hd;
    a.s_q = starting ? hd : static_cast<int64_t>(N) * hd;
    a.bias = Bp;
    a.bb = static_cast<int64_t>(N) * N * H;
    a.bh = 1;
    a.bq = static_cast<int64_t>(N) * H;
    a.bk = H;
    a.mask = mask;
    a.row_mask = 1;
    a.row0 = 0;
    a.B = B;
    a.R = N;
    a.N = N;
    a.H = H;
    a.d = d;
    rc = attention(a, stream);
  }
  if (rc == 0) {
    SgemmArgs g = plain_gemm(O, w.to_out, out, M, c, hd);
    g.epi = kGResidual;
    g.R = z;
    g.rm = RowMask{mask, masked_zero ? 2 : 0, N};
    rc = sgemm(g, 1, stream);
  }
  return rc;
}

size_t generic_transition_workspace(int64_t rows, int c, int n) {
  return up256(rows * c) + 3 * up256(rows * static_cast<int64_t>(n) * c);
}

int generic_transition(const float* x, const uint8_t* mask, const GenericTransitionWeights& w, float* out,
                       void* workspace, int64_t rows, int c, int n, int mask_kind, int mask_n, cudaStream_t stream) {
  Carver ws{static_cast<uint8_t*>(workspace)};
  const int f = n * c;
  float* y = ws.take(rows * c);
  float* A = ws.take(rows * f);
  float* Bm = ws.take(rows * f);
  float* Hd = ws.take(rows * f);
  int rc = ln_rows(x, y, w.ln_w, w.ln_b, rows, c, stream);
  if (rc == 0) rc = sgemm(plain_gemm(y, w.expand_a, A, rows, f, c), 1, stream);
  if (rc == 0) rc = sgemm(plain_gemm(y, w.expand_b, Bm, rows, f, c), 1, stream);
  if (rc == 0) {
    swiglu_kernel<<<grid_for(rows * f), 256, 0, stream>>>(A, Bm, Hd, rows * f);
    rc = static_cast<int>(cudaGetLastError());
  }
  if (rc == 0) {
    SgemmArgs g = plain_gemm(Hd, w.squeeze, out, rows, c, f);
    g.epi = kGResidual;
    g.R = x;
    g.rm = RowMask{mask, mask_kind, mask_n};
    rc = sgemm(g, 1, stream);
  }
  return rc;
}

size_t generic_apb_workspace(int B, int N, int cs, int cz, int H) {
  const int64_t M = static_cast<int64_t>(B) * N * N;
  const int64_t T = static_cast<int64_t>(B) * N;
  return up256(M * cz) + up256(M * H) + 6 * up256(T * cs);
}

int generic_apb(const float* s, const float* z, const uint8_t* mask, const GenericApbWeights& w, const float* extra,
                float* out, void* workspace, int B, int N, int cs, int cz, int H, float gate_bias, int masked_zero,
                cudaStream_t stream) {
  const int64_t M = static_cast<int64_t>(B) * N * N;
  const int64_t T = static_cast<int64_t>(B) * N;
  const int d = cs / H;
  Carver ws{static_cast<uint8_t*>(workspace)};
  float* zl = ws.take(M * cz);
  float* Bp = ws.take(M * H);
  float* y = ws.take(T * cs);
  float* Q = ws.take(T * cs);
  float* K = ws.take(T * cs);
  float* V = ws.take(T * cs);
  float* Gt = ws.take(T * cs);
  float* O = ws.take(T * cs);
  int rc = ln_rows(z, zl, w.ln_pair_w, nullptr, M, cz, stream);  // offset discarded (softmax-invariant)
  if (rc == 0) rc = sgemm(plain_gemm(zl, w.to_bias, Bp, M, H, cz), 1, stream);
  if (rc == 0) rc = ln_rows(s, y, w.ln_single_w, w.ln_single_b, T, cs, stream);
  if (rc == 0) {
    SgemmArgs g = plain_gemm(y, w.to_query, Q, T, cs, cs);
    g.bias = w.to_query_b;
    rc = sgemm(g, 1, stream);
  }
  if (rc == 0) rc = sgemm(plain_gemm(y, w.to_key, K, T, cs, cs), 1, stream);
  if (rc == 0) rc = sgemm(plain_gemm(y, w.to_value, V, T, cs, cs), 1, stream);
  if (rc == 0) rc = sgemm(plain_gemm(y, w.to_gate, Gt, T, cs, cs), 1, stream);
  if (rc == 0) {
    AttnArgs a{};
    a.q = Q;
    a.k = K;
    a.v = V;
    a.g = Gt;
    a.o = O;
    a.s_b = static_cast<int64_t>(N) * cs;
    a.s_r = 0;
    a.s_q = cs;
    a.bias = Bp;  // [B, q, k, H]
    a.bb = static_cast<int64_t>(N) * N * H;
    a.bh = 1;
    a.bq = static_cast<int64_t>(N) * H;
    a.bk = H;
    a.bias2 = extra;  // [B, H, q, k] or null
    a.cb = static_cast<int64_t>(H) * N * N;
    a.ch = static_cast<int64_t>(N) * N;
    a.cq = N;
    a.ck = 1;
    a.mask = mask;
    a.row_mask = 0;
    a.B = B;
    a.R = 1;
    a.N = N;
    a.H = H;
    a.d = d;
    a.gate_bias = gate_bias;
    rc = attention(a, stream);
  }
  if (rc == 0) {
    SgemmArgs g = plain_gemm(O, w.to_out, out, T, cs, cs);
    g.epi = kGResidual;
    g.R = s;
    g.rm = RowMask{mask, masked_zero ? 1 : 0, N};
    rc = sgemm(g, 1, stream);
  }
  return rc;
}

}  // namespace ffb

using namespace ffb;

namespace {

int check_common(const void* x, const uint8_t* mask, const float* const* weights, const void* out,
                 const void* workspace, size_t ws_bytes, size_t need, const char* what) {
  if (!x || !mask || !weights || !out) return fail(FFB_ERR_ARG, "%s: null pointer", what);
  if (need > 0 && (!workspace || ws_bytes < need))
    return fail(FFB_ERR_ARG, "%s: workspace of %zu bytes, %zu needed", what, ws_bytes, need);
  if (reinterpret_cast<uintptr_t>(workspace) & 255u) return fail(FFB_ERR_ARG, "%s: workspace not 256-byte aligned", what);
  if (x == out) return fail(FFB_ERR_ARG, "%s: out must not alias the input", what);
  return FFB_OK;
}

int finish(int rc, const char* what) { return cuda_status(rc, what); }

}  // namespace

extern "C" {

size_t ffb_trimul_f32_workspace_bytes(int B, int N, int c, int h) {
  return (B > 0 && N > 0 && c > 0 && h > 0) ? generic_trimul_workspace(B, N, c, h) : 0;
}

int ffb_trimul_fwd_f32(const float* z, const uint8_t* mask, const float* const* weights, float* out, void* workspace,
                       size_t workspace_bytes, int B, int N, int c, int h, int outgoing, int masked, void* stream) {
  if (B <= 0 || N <= 0 || c <= 0 || h <= 0) return fail(FFB_ERR_ARG, "trimul_f32: B=%d N=%d c=%d h=%d", B, N, c, h);
  if (masked != FFB_MASKED_COMPUTE && masked != FFB_MASKED_ZERO) return fail(FFB_ERR_ARG, "trimul_f32: masked=%d", masked);
  int st = check_common(z, mask, weights, out, workspace, workspace_bytes, generic_trimul_workspace(B, N, c, h),
                        "trimul_f32");
  if (st) return st;
  for (int i = 0; i < 10; ++i)
    if (!weights[i]) return fail(FFB_ERR_ARG, "trimul_f32: weight %d is null", i);
  DeviceInfo info;
  st = device_info(&info);
  if (st) return st;
  GenericTriMulWeights w{weights[0], weights[1], weights[2], weights[3], weights[4],
                         weights[5], weights[6], weights[7], weights[8], weights[9]};
  return finish(generic_trimul(z, mask, w, out, workspace, B, N, c, h, outgoing != 0, masked == FFB_MASKED_ZERO,
                               static_cast<cudaStream_t>(stream)),
                "trimul_f32 launch");
}

size_t ffb_triattn_f32_workspace_bytes(int B, int N, int c, int H, int d) {
  return (B > 0 && N > 0 && c > 0 && H > 0 && d > 0) ? generic_triattn_workspace(B, N, c, H, d) : 0;
}

int ffb_triattn_fwd_f32(const float* z, const uint8_t* mask, const float* const* weights, float* out, void* workspace,
                        size_t workspace_bytes, int B, int N, int c, int H, int d, int starting, int masked,
                        void* stream) {
  if (B <= 0 || N <= 0 || c <= 0 || H <= 0 || d <= 0 || d > 64)
    return fail(FFB_ERR_ARG, "triattn_f32: B=%d N=%d c=%d H=%d d=%d (d <= 64)", B, N, c, H, d);
  if (masked != FFB_MASKED_COMPUTE && masked != FFB_MASKED_ZERO) return fail(FFB_ERR_ARG, "triattn_f32: masked=%d", masked);
  int st = check_common(z, mask, weights, out, workspace, workspace_bytes, generic_triattn_workspace(B, N, c, H, d),
                        "triattn_f32");
  if (st) return st;
  for (int i = 0; i < 8; ++i)
    if (!weights[i]) return fail(FFB_ERR_ARG, "triattn_f32: weight %d is null", i);
  DeviceInfo info;
  st = device_info(&info);
  if (st) return st;
  GenericTriAttnWeights w{weights[0], weights[1], weights[2], weights[3], weights[4], weights[5], weights[6], weights[7]};
  return finish(generic_triattn(z, mask, w, out, workspace, B, N, c, H, d, starting != 0, masked == FFB_MASKED_ZERO,
                                static_cast<cudaStream_t>(stream)),
                "triattn_f32 launch");
}

size_t ffb_transition_f32_workspace_bytes(int64_t rows, int c, int n) {
  return (rows > 0 && c > 0 && n > 0) ? generic_transition_workspace(rows, c, n) : 0;
}

int ffb_transition_fwd_f32(const float* x, const uint8_t* mask, const float* const* weights, float* out,
                           void* workspace, size_t workspace_bytes, int B, int N, int c, int n, int pair, int masked,
                           void* stream) {
  if (B <= 0 || N <= 0 || c <= 0 || n <= 0) return fail(FFB_ERR_ARG, "transition_f32: B=%d N=%d c=%d n=%d", B, N, c, n);
  if (masked != FFB_MASKED_COMPUTE && masked != FFB_MASKED_ZERO)
    return fail(FFB_ERR_ARG, "transition_f32: masked=%d", masked);
  const int64_t rows = static_cast<int64_t>(B) * N * (pair ? N : 1);
  int st = check_common(x, mask, weights, out, workspace, workspace_bytes, generic_transition_workspace(rows, c, n),
                        "transition_f32");
  if (st) return st;
  for (int i = 0; i < 5; ++i)
    if (!weights[i]) return fail(FFB_ERR_ARG, "transition_f32: weight %d is null", i);
  DeviceInfo info;
  st = device_info(&info);
  if (st) return st;
  GenericTransitionWeights w{weights[0], weights[1], weights[2], weights[3], weights[4]};
  const int kind = masked == FFB_MASKED_ZERO ? (pair ? 2 : 1) : 0;
  return finish(generic_transition(x, mask, w, out, workspace, rows, c, n, kind, N, static_cast<cudaStream_t>(stream)),
                "transition_f32 launch");
}

size_t ffb_apb_f32_workspace_bytes(int B, int N, int cs, int cz, int H) {
  return (B > 0 && N > 0 && cs > 0 && cz > 0 && H > 0) ? generic_apb_workspace(B, N, cs, cz, H) : 0;
}

int ffb_apb_fwd_f32(const float* s, const float* z, const uint8_t* mask, const float* const* weights,
                    const float* extra_bias, float gate_bias, float* out, void* workspace, size_t workspace_bytes,
                    int B, int N, int cs, int cz, int H, int masked, void* stream) {
  if (B <= 0 || N <= 0 || cs <= 0 || cz <= 0 || H <= 0 || cs % H != 0 || cs / H > 64)
    return fail(FFB_ERR_ARG, "apb_f32: B=%d N=%d c_s=%d c_z=%d H=%d", B, N, cs, cz, H);
  if (masked != FFB_MASKED_COMPUTE && masked != FFB_MASKED_ZERO) return fail(FFB_ERR_ARG, "apb_f32: masked=%d", masked);
  if (!z) return fail(FFB_ERR_ARG, "apb_f32: null pair");
  int st = check_common(s, mask, weights, out, workspace, workspace_bytes, generic_apb_workspace(B, N, cs, cz, H),
                        "apb_f32");
  if (st) return st;
  for (int i = 0; i < 10; ++i)
    if (!weights[i]) return fail(FFB_ERR_ARG, "apb_f32: weight %d is null", i);
  DeviceInfo info;
  st = device_info(&info);
  if (st) return st;
  GenericApbWeights w{weights[0], weights[1], weights[2], weights[3], weights[4],
                      weights[5], weights[6], weights[7], weights[8], weights[9]};
  return finish(generic_apb(s, z, mask, w, extra_bias, out, workspace, B, N, cs, cz, H, gate_bias,
                            masked == FFB_MASKED_ZERO, static_cast<cudaStream_t>(stream)),
                "apb_f32 launch");
}

}  // extern "C"
