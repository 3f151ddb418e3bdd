// Single track of the Pairformer block: attention with pair bias and the single
// transition (c_s = 384, 16 heads x 24, factor 4). Both are small next to the pair ops
// (about 1% of a block's flops at N = 512) and are composed from the library's tcgen05
// GEMM and LayerNorm launchers plus two kernels of their own:
//
// attention with pair bias (legacy/pairformer.py:204-226, legacy/transformer.py:88-133):
//   pb[h, b, i, j] = W_pb (gamma_pair * LNhat(z[b, i, j]))     pair_bias_kernel (tcgen05,
//                                                              LayerNorm folded, reads z once)
//   y = LN(s);  [q | k | v | g] = y W^T + [b_q | 0 | 0 | 0]     GEMM (N = 1536)
//   o = softmax_j(q_i . k_j / sqrt(24) + pb[i, j, h] (+ extra[h, i, j]), key mask) v_j
//   s' = s + W_o (sigmoid(g + gate_bias) * o)                    GEMM with residual epilogue
// single transition: s' = s + W_sq (silu(W_a LN(s)) * W_b LN(s))  (SwiGLU GEMM epilogue)
#include "../../include/foldforge_b200.h"
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

// ---------------------------------------------------------------- pair bias
// pb[h][p] = W_pb[h] . (gamma * LNhat(z[p])) for every pair p of the B * N * N rows of z,
// head-major ([h][b][i][j]). The LayerNorm is folded: W' = bf16(W_pb diag gamma) and
// wsum[h] = sum_c W'[h][c], so pb = rstd * (W' z - mean * wsum) on RAW z (the LayerNorm
// offset beta adds one constant per head to every logit of a row, which the softmax
// cancels). Persistent, warp-specialised, 128-pair tiles, two CTAs per SM (eight
// statistics / epilogue warps per SM hide the staged-tile and TMEM latencies):
//   warp 0      TMA: z tiles (two 64-channel SW128 blocks) through a 3-stage ring
//   warp 1      MMA: acc[p][h] = z[p] . W'[h] (M = 128 pairs, N = 16 heads, K = 128),
//               double-buffered in TMEM
//   warps 2-5   lane = pair: LayerNorm statistics from the staged tile, then the epilogue;
//               a warp's 32 pairs of one head are one coalesced 128-byte store
constexpr int kPbTile = 128;
constexpr int kPbStages = 3;  // three stages keep the CTA under half the SM's shared memory: two CTAs per SM
constexpr int kPbThreads = 192;
constexpr uint32_t kPbWBytes = 2 * kHs * 128;  // W' image: two 64-channel blocks of 16 rows

struct PbSmem {
  alignas(1024) uint8_t z[kPbStages][2][kPbTile * 128];
  alignas(1024) uint8_t w[kPbWBytes];
  float wsum[kHs];
  uint64_t full[kPbStages];
  uint64_t empty[kPbStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t wbar;
  uint32_t tmem_base;
};

__global__ void __launch_bounds__(kPbThreads, 2)
    pair_bias_kernel(const __grid_constant__ CUtensorMap map_z, const uint8_t* __restrict__ w_img,
                     const float* __restrict__ wsum, float* __restrict__ pb, int64_t P, int N, int64_t pb_h,
                     int64_t pb_r, int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  PbSmem& s = *reinterpret_cast<PbSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                         ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t tiles = (P + kPbTile - 1) / kPbTile;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kPbStages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1 + 4);  // the MMA commit and the four statistics warps
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.acc_full[i], 1);
      mbar_init(&s.acc_empty[i], 4);
    }
    mbar_init(&s.wbar, 1);
    fence_mbar_init();
  }
  if (threadIdx.x < kHs) s.wsum[threadIdx.x] = wsum[threadIdx.x];
  if (warp == 1) {
    tmem_alloc(&s.tmem_base, 32);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) tma_prefetch_map(&map_z);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(&s.wbar, kPbWBytes);
      bulk_load(s.w, w_img, kPbWBytes, &s.wbar);
      int it = 0;
      for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x, ++it) {
        const int st = it % kPbStages;
        if (!mbar_wait(&s.empty[st], ((it / kPbStages) & 1) ^ 1, err, kErrTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&s.full[st], 2 * kPbTile * 128);
        const int y = static_cast<int>(t * kPbTile);
        tma_load_2d(s.z[st][0], &map_z, &s.full[st], 0, y);
        tma_load_2d(s.z[st][1], &map_z, &s.full[st], 64, y);
      }
      // every issued copy lands before the CTA may exit
      mbar_wait(&s.wbar, 0, err, kErrTimeoutLoad);
      for (int k = 0; k < kPbStages && k < it; ++k) {
        const int j = it - 1 - k;
        mbar_wait(&s.full[j % kPbStages], (j / kPbStages) & 1, err, kErrTimeoutLoad);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && mbar_wait(&s.wbar, 0, err, kErrTimeoutLoad)) {
      const uint32_t idesc = idesc_bf16_f32(kPbTile, kHs);
      int it = 0;
      for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x, ++it) {
        const int st = it % kPbStages, acc = it & 1;
        if (!mbar_wait(&s.acc_empty[acc], ((it >> 1) & 1) ^ 1, err, kErrTimeoutEmpty)) break;
        if (!mbar_wait(&s.full[st], (it / kPbStages) & 1, err, kErrTimeoutLoad)) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * kHs;
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
          const uint64_t da = desc_kmajor_sw128(smem_u32(s.z[st][kb]));
          const uint64_t db = desc_kmajor_sw128(smem_u32(s.w + kb * kHs * 128));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) mma_bf16(d, da + 2 * kk, db + 2 * kk, idesc, (kb | kk) != 0);
        }
        mma_commit(&s.empty[st]);
        mma_commit(&s.acc_full[acc]);
      }
    }
  } else {
    const int quarter = warp & 3;  // TMEM lane quarter this warp may read
    const int row = quarter * 32 + lane;
    int it = 0;
    for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x, ++it) {
      const int st = it % kPbStages, acc = it & 1;
      bool ok = mbar_wait(&s.full[st], (it / kPbStages) & 1, err, kErrTimeoutLoad);
      if (!__all_sync(0xFFFFFFFFu, ok)) break;
      float mean, rstd;
      ln_stats_c128(s.z[st][0], kPbTile * 128, row, mean, rstd);
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.empty[st]);
      ok = mbar_wait(&s.acc_full[acc], (it >> 1) & 1, err, kErrTimeoutMma);
      if (!__all_sync(0xFFFFFFFFu, ok)) break;
      tc_fence_after();
      uint32_t v[16];
      tmem_ld16(tmem + (static_cast<uint32_t>(quarter * 32) << 16) + acc * kHs, v);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.acc_empty[acc]);
      const int64_t p = t * kPbTile + row;
      if (p < P) {
        // pair p = row * N + col of the rows held: pb[h * pb_h + row * pb_r + col]
        float* dst = pb + (p / N) * pb_r + (p % N);
#pragma unroll
        for (int h = 0; h < kHs; ++h) dst[h * pb_h] = rstd * (__uint_as_float(v[h]) - mean * s.wsum[h]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 32);
  }
}

// ---------------------------------------------------------------- attention kernel
// A CTA per (batch, head, 32 queries), 8 warps. Lane = query; warp w takes keys w*8 ..
// w*8+7 of every 64-key chunk. Chunks are staged in shared memory (keys and values as fp32,
// the pair-bias tile [32 q][64 k] from the head-major bias with padded rows so lanes
// reading one key hit distinct banks) through two buffers: the global loads of chunk c + 1
// are issued before the warps work on chunk c and land in the other buffer afterwards, one
// barrier per chunk. Each warp keeps an exact online softmax per query, updated once per 8
// keys; the eight partial states are merged at the end. Masked keys get the reference's
// REPLACED logit -1e9, so a row whose keys are all masked averages uniformly; keys past N
// do not exist.
constexpr int kQ = 32;        // queries per CTA
constexpr int kKC = 64;       // keys per staged chunk
constexpr int kWarps = 8;
constexpr int kKPW = kKC / kWarps;
constexpr int kAttnThreads = kQ * kWarps;
constexpr int kBiasPitch = kKC + 1;
constexpr int kBufFloats = 2 * kKC * kDs + kQ * kBiasPitch + kKC;  // keys, values, bias, keep
constexpr int kPartPitch = kDs + 2;
static_assert(kWarps * kQ * kPartPitch <= 2 * kBufFloats, "merge scratch must fit the chunk buffers");
static_assert(kKC * 6 <= 2 * kAttnThreads && kQ * kKC / 4 == 2 * kAttnThreads, "staging assignment");

struct ChunkRegs {
  uint4 kv[2];     // key / value vectors (8 bf16 each)
  float4 bias[2];  // four bias values each
  float keep;
};

__device__ __forceinline__ void attn_load_chunk(ChunkRegs& r, const __nv_bfloat16* __restrict__ qkvg,
                                                const float* __restrict__ pb, int64_t pb_r, const void* __restrict__ extra,
                                                int extra_f32, const uint8_t* __restrict__ mask, int b, int h,
                                                int qb, int N, int j0, int q0, int nq) {
  const int t = threadIdx.x;
  const int nk = N - j0 < kKC ? N - j0 : kKC;
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int e = t + u * kAttnThreads;
    r.kv[u] = make_uint4(0u, 0u, 0u, 0u);
    if (e < kKC * 6) {
      const int j = e / 6, part = e % 6;  // part 0-2: key vectors, 3-5: value vectors
      if (j < nk)
        r.kv[u] = *reinterpret_cast<const uint4*>(qkvg + (static_cast<int64_t>(b) * N + j0 + j) * (4 * kCs) +
                                                  (part < 3 ? kCs : 2 * kCs) + h * kDs + (part % 3) * 8);
    }
  }
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int e = t + u * kAttnThreads;
    const int qq = e / (kKC / 4), j = (e % (kKC / 4)) * 4;
    const int ii = qb * kQ + qq;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (ii < nq) {
      const float* src = pb + static_cast<int64_t>(ii) * pb_r + j0 + j;
      if (j + 4 <= nk && (reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
        const float4 f = *reinterpret_cast<const float4*>(src);
        v[0] = f.x;
        v[1] = f.y;
        v[2] = f.z;
        v[3] = f.w;
      } else {
        for (int i = 0; i < 4; ++i)
          if (j + i < nk) v[i] = src[i];
      }
      if (extra != nullptr) {
        for (int i = 0; i < 4 && j + i < nk; ++i) {
          const int64_t x = ((static_cast<int64_t>(b) * kHs + h) * N + q0 + ii) * N + j0 + j + i;
          v[i] += extra_f32 ? static_cast<const float*>(extra)[x]
                            : __bfloat162float(static_cast<const __nv_bfloat16*>(extra)[x]);
        }
      }
    }
    r.bias[u] = make_float4(v[0], v[1], v[2], v[3]);
  }
  r.keep = 0.f;
  if (t < kKC) r.keep = (t < nk) ? (mask[static_cast<int64_t>(b) * N + j0 + t] ? 1.f : 0.f) : -1.f;
}

__device__ __forceinline__ void attn_store_chunk(const ChunkRegs& r, float* buf) {
  float* ks = buf;
  float* vs = buf + kKC * kDs;
  float* bias = vs + kKC * kDs;
  float* keep = bias + kQ * kBiasPitch;
  const int t = threadIdx.x;
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int e = t + u * kAttnThreads;
    if (e < kKC * 6) {
      const int j = e / 6, part = e % 6;
      float* dst = (part < 3 ? ks : vs) + j * kDs + (part % 3) * 8;
      const uint32_t w[4] = {r.kv[u].x, r.kv[u].y, r.kv[u].z, r.kv[u].w};
      float4 lo, hi;
      lo.x = bf16_lo(w[0]); lo.y = bf16_hi(w[0]); lo.z = bf16_lo(w[1]); lo.w = bf16_hi(w[1]);
      hi.x = bf16_lo(w[2]); hi.y = bf16_hi(w[2]); hi.z = bf16_lo(w[3]); hi.w = bf16_hi(w[3]);
      reinterpret_cast<float4*>(dst)[0] = lo;
      reinterpret_cast<float4*>(dst)[1] = hi;
    }
  }
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int e = t + u * kAttnThreads;
    const int qq = e / (kKC / 4), j = (e % (kKC / 4)) * 4;
    float* dst = bias + qq * kBiasPitch + j;
    dst[0] = r.bias[u].x;
    dst[1] = r.bias[u].y;
    dst[2] = r.bias[u].z;
    dst[3] = r.bias[u].w;
  }
  if (t < kKC) keep[t] = r.keep;
}

// Queries [q0, q0 + nq) of each batch entry (local index i = query - q0) against all N keys:
// the pair-bias row of local query i is pair_bias + h * pb_h + (b * nq + i) * pb_r and the
// output row is out + (b * nq + i) * 384, so a rank passes only its own rows of both.
__global__ void __launch_bounds__(kAttnThreads, 2) single_attention_kernel(
    const __nv_bfloat16* __restrict__ qkvg, const float* __restrict__ pair_bias, int64_t pb_h, int64_t pb_r,
    const void* __restrict__ extra,
    int extra_f32, const uint8_t* __restrict__ mask, float gate_bias, __nv_bfloat16* __restrict__ out, int B, int N,
    int q0, int nq) {
  __shared__ __align__(16) float smem[2 * kBufFloats];
  const int qblocks = (nq + kQ - 1) / kQ;
  const int h = blockIdx.x % kHs;
  const int qb = (blockIdx.x / kHs) % qblocks;
  const int b = blockIdx.x / (kHs * qblocks);
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  const int i = qb * kQ + lane;
  const int row = q0 + (i < nq ? i : nq - 1);
  const __nv_bfloat16* row_i = qkvg + (static_cast<int64_t>(b) * N + row) * (4 * kCs);
  const float scale = rsqrtf(static_cast<float>(kDs));
  float q[kDs];
#pragma unroll
  for (int u = 0; u < 3; ++u) {
    const uint4 v = *reinterpret_cast<const uint4*>(row_i + h * kDs + u * 8);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      q[u * 8 + 2 * k] = bf16_lo(w[k]) * scale;
      q[u * 8 + 2 * k + 1] = bf16_hi(w[k]) * scale;
    }
  }
  float m = -1.0e30f, l = 0.f;
  float o[kDs];
#pragma unroll
  for (int d = 0; d < kDs; ++d) o[d] = 0.f;
  // bias row i of head h: pair_bias + h * pb_h + (b * nq + i) * pb_r
  const float* pb = pair_bias + h * pb_h + static_cast<int64_t>(b) * nq * pb_r;
  const int chunks = (N + kKC - 1) / kKC;
  {
    ChunkRegs r;
    attn_load_chunk(r, qkvg, pb, pb_r, extra, extra_f32, mask, b, h, qb, N, 0, q0, nq);
    attn_store_chunk(r, smem);
  }
  __syncthreads();
  for (int c = 0; c < chunks; ++c) {
    const bool next = c + 1 < chunks;
    ChunkRegs r;
    if (next) attn_load_chunk(r, qkvg, pb, pb_r, extra, extra_f32, mask, b, h, qb, N, (c + 1) * kKC, q0, nq);
    const float* buf = smem + (c & 1) * kBufFloats;
    const float* ks = buf;
    const float* vs = buf + kKC * kDs;
    const float* bias = vs + kKC * kDs;
    const float* keep = bias + kQ * kBiasPitch;
    float x[kKPW];
    float mx = -INFINITY;
#pragma unroll
    for (int jj = 0; jj < kKPW; ++jj) {
      const int j = warp * kKPW + jj;
      const float4* kr = reinterpret_cast<const float4*>(ks + j * kDs);
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
      for (int u = 0; u < kDs / 4; ++u) {
        const float4 kk = kr[u];
        a0 = fmaf(q[4 * u], kk.x, a0);
        a1 = fmaf(q[4 * u + 1], kk.y, a1);
        a2 = fmaf(q[4 * u + 2], kk.z, a2);
        a3 = fmaf(q[4 * u + 3], kk.w, a3);
      }
      const float kp = keep[j];
      float xv = (a0 + a1) + (a2 + a3) + bias[lane * kBiasPitch + j];
      if (kp == 0.f) xv = -1.0e9f;
      if (kp < 0.f) xv = -INFINITY;  // past N
      x[jj] = xv;
      mx = fmaxf(mx, xv);
    }
    const float m_new = fmaxf(m, mx);
    const float alpha = __expf(m - m_new);
    l *= alpha;
#pragma unroll
    for (int d = 0; d < kDs; ++d) o[d] *= alpha;
#pragma unroll
    for (int jj = 0; jj < kKPW; ++jj) {
      const int j = warp * kKPW + jj;
      const float p = __expf(x[jj] - m_new);
      l += p;
      const float4* vr = reinterpret_cast<const float4*>(vs + j * kDs);
#pragma unroll
      for (int u = 0; u < kDs / 4; ++u) {
        const float4 vv = vr[u];
        o[4 * u] = fmaf(p, vv.x, o[4 * u]);
        o[4 * u + 1] = fmaf(p, vv.y, o[4 * u + 1]);
        o[4 * u + 2] = fmaf(p, vv.z, o[4 * u + 2]);
        o[4 * u + 3] = fmaf(p, vv.w, o[4 * u + 3]);
      }
    }
    m = m_new;
    if (next) attn_store_chunk(r, smem + ((c + 1) & 1) * kBufFloats);
    __syncthreads();
  }
  // merge the warps' partial softmax states per query (scratch aliases the chunk buffers;
  // the loop's last barrier ended every read of them)
  float* part = smem;
#pragma unroll
  for (int d = 0; d < kDs; ++d) part[(warp * kQ + lane) * kPartPitch + d] = o[d];
  part[(warp * kQ + lane) * kPartPitch + kDs] = m;
  part[(warp * kQ + lane) * kPartPitch + kDs + 1] = l;
  __syncthreads();
  if (warp != 0 || i >= nq) return;
  float mm = -1.0e30f;
  for (int w = 0; w < kWarps; ++w) {
    const float* pw = part + (w * kQ + lane) * kPartPitch;
    if (pw[kDs + 1] > 0.f) mm = fmaxf(mm, pw[kDs]);
  }
  float ll = 0.f, acc[kDs];
#pragma unroll
  for (int d = 0; d < kDs; ++d) acc[d] = 0.f;
  for (int w = 0; w < kWarps; ++w) {
    const float* pw = part + (w * kQ + lane) * kPartPitch;
    const float lw = pw[kDs + 1];
    if (lw <= 0.f) continue;
    const float f = __expf(pw[kDs] - mm);
    ll += lw * f;
#pragma unroll
    for (int d = 0; d < kDs; ++d) acc[d] = fmaf(pw[d], f, acc[d]);
  }
  const float inv = 1.0f / ll;
  __nv_bfloat16* dst = out + (static_cast<int64_t>(b) * nq + i) * kCs + h * kDs;
#pragma unroll
  for (int u = 0; u < 3; ++u) {
    const uint4 gv = *reinterpret_cast<const uint4*>(row_i + 3 * kCs + h * kDs + u * 8);
    const uint32_t w[4] = {gv.x, gv.y, gv.z, gv.w};
    uint32_t ov[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int d = u * 8 + 2 * k;
      ov[k] = pack_bf16(acc[d] * inv * sigmoidf_(bf16_lo(w[k]) + gate_bias),
                        acc[d + 1] * inv * sigmoidf_(bf16_hi(w[k]) + gate_bias));
    }
    reinterpret_cast<uint4*>(dst)[u] = make_uint4(ov[0], ov[1], ov[2], ov[3]);
  }
}

// ---------------------------------------------------------------- helpers
int gemm(const void* a, const void* w, void* d, int m, int n, int k, int d_f32, const float* bias, int epilogue,
         const void* residual, const uint8_t* row_mask, const DeviceInfo& info, cudaStream_t stream) {
  // 128-wide tiles unless 256-wide ones already give every SM a tile: the single track's
  // GEMMs are small (M = B * N tokens), so more CTAs beat wider tiles
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
  p.row_mask = row_mask;
  p.err = info.err;
  return cuda_status(launch_gemm_nt(ma, mb, p, bn, info.num_sms, stream), "single-track gemm");
}

size_t a256(size_t x) { return (x + 255) / 256 * 256; }

// packed attention-with-pair-bias image
struct ApbLayout {
  size_t w_qkvg, b_qkvg, w_o, w_pb, pb_wsum, ln_s_w, ln_s_b, total;
};
ApbLayout apb_layout() {
  ApbLayout L;
  size_t o = 0;
  L.w_qkvg = o;  o = a256(o + static_cast<size_t>(4 * kCs) * kCs * 2);
  L.b_qkvg = o;  o = a256(o + 4 * kCs * 4);
  L.w_o = o;     o = a256(o + static_cast<size_t>(kCs) * kCs * 2);
  L.w_pb = o;    o = a256(o + kPbWBytes);  // W_pb diag(gamma_pair), SW128 image
  L.pb_wsum = o; o = a256(o + kHs * 4);
  L.ln_s_w = o;  o = a256(o + kCs * 4);
  L.ln_s_b = o;  o = a256(o + kCs * 4);
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
  return a256(P * kHs * 4) + a256(T * kCs * 2) + a256(T * 4 * kCs * 2) + a256(T * kCs * 2);
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
  if (rc == 0)
    rc = launch_pack_weight(w.to_bias, kHs, kCz, w.ln_pair_w, nullptr, img + L.w_pb, 0, kHs,
                            reinterpret_cast<float*>(img + L.pb_wsum), nullptr, stream);
  if (rc == 0) rc = static_cast<int>(cudaMemcpyAsync(img + L.ln_s_w, w.ln_single_w, kCs * 4, cudaMemcpyDeviceToDevice, stream));
  if (rc == 0) rc = static_cast<int>(cudaMemcpyAsync(img + L.ln_s_b, w.ln_single_b, kCs * 4, cudaMemcpyDeviceToDevice, stream));
  return rc;
}

namespace {

// pb[h * pb_h + row * pb_r + col] for the `rows` pair rows of N pairs of z
int launch_pair_bias(const void* z, const uint8_t* img, float* pb, int64_t rows, int N, int64_t pb_h, int64_t pb_r,
                     const DeviceInfo& info, cudaStream_t stream) {
  const ApbLayout L = apb_layout();
  return pair_bias16(z, img + L.w_pb, reinterpret_cast<const float*>(img + L.pb_wsum), pb, rows, N, pb_h, pb_r, info,
                     stream);
}

}  // namespace

int pair_bias16(const void* z, const uint8_t* w_img, const float* wsum, float* pb, int64_t rows, int N, int64_t pb_h,
                int64_t pb_r, const DeviceInfo& info, cudaStream_t stream) {
  const size_t P = static_cast<size_t>(rows) * N;
  if (P >= (static_cast<size_t>(1) << 31))
    return fail(FFB_ERR_UNSUPPORTED, "attention_pair_bias: %zu pairs exceed the 2^31 TMA row range", P);
  CUtensorMap mz;
  const uint64_t zdims[2] = {static_cast<uint64_t>(kCz), static_cast<uint64_t>(P)};
  const uint64_t zstr[1] = {static_cast<uint64_t>(kCz) * 2};
  const uint32_t zbox[2] = {64, kPbTile};
  int st = make_map(&mz, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, z, zdims, zstr, zbox, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  const int64_t tiles = static_cast<int64_t>((P + kPbTile - 1) / kPbTile);
  const int grid = static_cast<int>(tiles < 2 * info.num_sms ? tiles : 2 * info.num_sms);
  const size_t smem = sizeof(PbSmem) + 1024;
  cudaFuncSetAttribute(pair_bias_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  pair_bias_kernel<<<grid, kPbThreads, smem, stream>>>(mz, w_img, wsum, pb, static_cast<int64_t>(P), N, pb_h, pb_r,
                                                       info.err);
  return cuda_status(static_cast<int>(cudaGetLastError()), "pair bias launch");
}

namespace {

// the single track of attention with pair bias, given the pair bias (strides pb_h, pb_r)
int launch_single_attention(const void* s, const uint8_t* mask, const uint8_t* img, const float* pb, int64_t pb_h,
                            int64_t pb_r, const void* extra, int extra_f32, float gate_bias, void* out, uint8_t* ws,
                            int B, int N, int masked_zero, const DeviceInfo& info, cudaStream_t stream) {
  const ApbLayout L = apb_layout();
  const size_t T = static_cast<size_t>(B) * N;
  void* y = ws;
  void* qkvg = static_cast<uint8_t*>(y) + a256(T * kCs * 2);
  void* gated = static_cast<uint8_t*>(qkvg) + a256(T * 4 * kCs * 2);
  int st = cuda_status(launch_layernorm(s, y, reinterpret_cast<const float*>(img + L.ln_s_w),
                                        reinterpret_cast<const float*>(img + L.ln_s_b), static_cast<int64_t>(T), kCs,
                                        1e-5f, 0, info.num_sms, stream),
                       "apb single layernorm");
  if (st) return st;
  st = gemm(y, img + L.w_qkvg, qkvg, static_cast<int>(T), 4 * kCs, kCs, 0,
            reinterpret_cast<const float*>(img + L.b_qkvg), kEpiStore, nullptr, nullptr, info, stream);
  if (st) return st;
  const int ctas = B * kHs * ((N + kQ - 1) / kQ);
  single_attention_kernel<<<ctas, kAttnThreads, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(qkvg), pb, pb_h, pb_r, extra, extra_f32, mask, gate_bias,
      static_cast<__nv_bfloat16*>(gated), B, N, 0, N);
  st = cuda_status(static_cast<int>(cudaGetLastError()), "single attention launch");
  if (st) return st;
  return gemm(gated, img + L.w_o, out, static_cast<int>(T), kCs, kCs, 0, nullptr, kEpiResidual, s,
              masked_zero ? mask : nullptr, info, stream);
}

}  // namespace

int apb_forward(const void* s, const void* z, const uint8_t* mask, const void* packed, const void* extra,
                int extra_f32, float gate_bias, void* out, void* workspace, int B, int N, int masked_zero,
                const DeviceInfo& info, cudaStream_t stream) {
  const uint8_t* img = static_cast<const uint8_t*>(packed);
  const size_t P = static_cast<size_t>(B) * N * N;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* pb = reinterpret_cast<float*>(ws);
  // head-major pair bias [16][B][N][N] from raw z (LayerNorm folded into the epilogue)
  int st = launch_pair_bias(z, img, pb, static_cast<int64_t>(B) * N, N, static_cast<int64_t>(P), N, info, stream);
  if (st) return st;
  return launch_single_attention(s, mask, img, pb, static_cast<int64_t>(P), N, extra, extra_f32, gate_bias, out,
                                 ws + a256(P * kHs * 4), B, N, masked_zero, info, stream);
}

// ---- row-sharded pieces (B = 1). The rank's pair-bias rows [R][16][N] (fp32) concatenate
// under an all-gather into the [N][16][N] bias the single track reads; the single track is
// replicated on every rank (workspace: apb_single_workspace_bytes).
int apb_shard_pair_bias(const void* z, const void* packed, void* pb_rows, int R, int N, const DeviceInfo& info,
                        cudaStream_t stream) {
  return launch_pair_bias(z, static_cast<const uint8_t*>(packed), static_cast<float*>(pb_rows), R, N, N,
                          static_cast<int64_t>(kHs) * N, info, stream);
}

size_t apb_single_workspace_bytes(int N) {
  const size_t T = static_cast<size_t>(N);
  return a256(T * kCs * 2) + a256(T * 4 * kCs * 2) + a256(T * kCs * 2);
}

int apb_shard_single(const void* s, const uint8_t* mask, const void* packed, const void* pb_all, const void* extra,
                     int extra_f32, float gate_bias, void* out, void* workspace, int N, int masked_zero,
                     const DeviceInfo& info, cudaStream_t stream) {
  return launch_single_attention(s, mask, static_cast<const uint8_t*>(packed), static_cast<const float*>(pb_all), N,
                                 static_cast<int64_t>(kHs) * N, extra, extra_f32, gate_bias, out,
                                 static_cast<uint8_t*>(workspace), 1, N, masked_zero, info, stream);
}

// The rank's rows [row0, row0 + R) of the single track's attention with pair bias, from its
// own pair-bias rows pb_rows [R][16][N] (fp32, as apb_shard_pair_bias writes them): LayerNorm
// and the [q | k | v | g] projection over all N tokens (s is replicated; the keys and values
// need every token), the attention for the R queries only, and the output projection with
// the residual s[row0 + r] (masked rows zeroed under masked_zero). out_rows is [R][384].
int apb_shard_single_rows(const void* s, const uint8_t* mask, const void* packed, const void* pb_rows, float gate_bias,
                          void* out_rows, void* workspace, int N, int row0, int R, int masked_zero,
                          const DeviceInfo& info, cudaStream_t stream) {
  const uint8_t* img = static_cast<const uint8_t*>(packed);
  const ApbLayout L = apb_layout();
  const size_t T = static_cast<size_t>(N);
  uint8_t* y = static_cast<uint8_t*>(workspace);
  uint8_t* qkvg = y + a256(T * kCs * 2);
  uint8_t* gated = qkvg + a256(T * 4 * kCs * 2);
  int st = cuda_status(launch_layernorm(s, y, reinterpret_cast<const float*>(img + L.ln_s_w),
                                        reinterpret_cast<const float*>(img + L.ln_s_b), static_cast<int64_t>(T), kCs,
                                        1e-5f, 0, info.num_sms, stream),
                       "apb rows layernorm");
  if (st) return st;
  st = gemm(y, img + L.w_qkvg, qkvg, N, 4 * kCs, kCs, 0, reinterpret_cast<const float*>(img + L.b_qkvg), kEpiStore,
            nullptr, nullptr, info, stream);
  if (st) return st;
  const int ctas = kHs * ((R + kQ - 1) / kQ);
  single_attention_kernel<<<ctas, kAttnThreads, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkvg), static_cast<const float*>(pb_rows), N,
      static_cast<int64_t>(kHs) * N, nullptr, 0, mask, gate_bias, reinterpret_cast<__nv_bfloat16*>(gated), 1, N, row0, R);
  st = cuda_status(static_cast<int>(cudaGetLastError()), "single attention (rows) launch");
  if (st) return st;
  return gemm(gated, img + L.w_o, out_rows, R, kCs, kCs, 0, nullptr, kEpiResidual,
              static_cast<const __nv_bfloat16*>(s) + static_cast<int64_t>(row0) * kCs,
              masked_zero ? mask + row0 : nullptr, info, stream);
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
