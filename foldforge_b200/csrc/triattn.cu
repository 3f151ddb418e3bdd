// Triangle attention around the starting / ending node, bf16 activations, c_z = 128,
// 4 heads x 32 (AF3: untransposed pair bias, no projection biases).
//
//   x = LN(z);  b_h[q, k] = W_b x[q, k];  per problem row r:
//   o[r, q] = sum_k softmax_k(q[r,q] . k[r,k] / sqrt(32) + b_h[q, k], key mask m_r m_k) v[r, k]
//   z' = z + W_o (sigmoid(W_g x) * o)
// The starting node's problem row r is pair row i (q, k index columns); the ending node's
// is pair column j (q, k index rows) and its output is written back transposed
// (legacy/attention.py:108-171 with spec.py:125,437,470; masked logits are REPLACED by
// -1e9, legacy/reference/attention.py:14-54, so a fully masked row averages uniformly).
//
// Three launches:
//  1. triattn_proj: 128-pair tiles of raw z (row tiles for the starting node, column
//     tiles for the ending node, so the Q / K / V^T writes are contiguous) x the resident
//     packed [W_q; W_k; W_v; W_b] with the input LayerNorm folded into the epilogue; V is
//     computed transposed (W_v z^T) and leaves through TMA stores. W_q carries
//     log2(e)/sqrt(32) and W_b log2(e), so the softmax works in base 2. Writes
//     Q, K [B, N(r), H, N(n), 32], V^T [B, N(r), H, 32, Np(n)] and the bias
//     [B, H, N, Np] in the natural pair layout, which both nodes read as [query][key] rows
//     (the ending node's column tiles write it with a stride).
//  2. triattn_attn: flash attention on tcgen05. A CTA owns 256 queries (two groups of
//     128, one per softmax warpgroup) of one (row, head) and streams 64-key blocks of K,
//     V^T and the bias through a 3-stage TMA ring shared by both groups. S = Q K^T and
//     P V run on the tensor cores with fp32 accumulators in TMEM (double-buffered);
//     each softmax thread owns one query row (exact online softmax, running max) and
//     accumulates the P V partials in registers.
//  3. triattn_out: per 128-pair tile (natural layout for both nodes), the gate GEMM on
//     raw z (folded LayerNorm), sigmoid(gate) * o written back as a K-major operand, the
//     output GEMM, mask and residual, TMA store.
#include "abi_util.h"
#include "common.cuh"
#include "kernels.h"

namespace ffb {
namespace {

constexpr int kC = 128;
constexpr int kHeads = 4;
constexpr int kD = 32;
constexpr int kTile = 128;
constexpr int kGroups = 2;
constexpr int kProjRows = 400;  // Q 128 | K 128 | V 128 | bias 16 (4 used)
constexpr float kLog2e = 1.4426950408889634f;

constexpr size_t kProjBytes = static_cast<size_t>(kProjRows) * kC * 2;  // 102400
constexpr size_t kGateBytes = kC * kC * 2;
constexpr size_t kOutBytes = kC * kC * 2;
constexpr size_t kVecFloats = 2 * kProjRows + 2 * 128;
constexpr size_t kPackedBytes = kProjBytes + kGateBytes + kOutBytes + kVecFloats * 4;

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// LayerNorm statistics of row `row` of a 128-row tile stored as two SW128 channel blocks.
__device__ __forceinline__ void tile_stats(const uint8_t* tile, int row, float& mean, float& rstd) {
  ln_stats_c128(tile, 16384, row, mean, rstd);
}

// ====================================================================== 1. projection
// Warp-specialised, persistent, 128-pair tiles. Per tile three products on the resident
// weights, all reading the same z tile from shared memory:
//   X[pair][256]   = z . [W_q; W_k]^T     (TMEM lane = pair)     Q, K
//   X[pair][16]    = z . W_b^T            (lane = pair)          pair bias (4 heads used)
//   Y[channel][128] = W_v . z^T           (lane = V channel)     V^T, computed transposed
// so every thread's output run is contiguous: a pair's 32 channels of Q / K per head, a
// channel's 128 pairs of V^T (staged 128-byte-swizzled, written by TMA stores).
//   warp 0      TMA: the weights once, z tiles into a 2-stage ring
//   warp 1      MMA: X (QK + bias, 272 columns) and Y (V^T, 128 columns), one buffer each
//   warps 2-5   thread = pair: LayerNorm statistics (-> shared memory for warps 6-9), then
//               Q, K and bias from X with the LayerNorm folded in
//   warps 6-9   thread = V channel: V^T from Y with the pair statistics folded in
constexpr int kProjThreads = 320;
constexpr int kProjStages = 2;
constexpr uint32_t kColX = 0;    // QK 0..255, bias 256..271
constexpr uint32_t kColY = 384;  // V^T 384..511

struct ProjSmem {
  alignas(1024) uint8_t w[kProjBytes];
  alignas(1024) uint8_t z[kProjStages][kTile * kC * 2];
  alignas(1024) uint8_t vt[2][kC * 64 * 2];  // V^T staging: [128 channels][pairs 0..63 | 64..127], SW128
  float wsum[kProjRows];
  float bias[kProjRows];
  float4 stats[2][kTile / 2];  // pair couple (j, j + 1): rstd x2, -rstd mean x2; by tile parity
  float4 wb[kProjRows / 2];      // channel couple (c, c + 1): wsum x2, bias x2
  uint64_t wbar;
  uint64_t z_full[kProjStages], z_empty[kProjStages];
  uint64_t x_full, x_free, y_full, y_free;
  uint64_t st_full[2], st_free[2];
  uint32_t tmem_base;
};

static_assert(sizeof(ProjSmem) + 1024 <= 232448, "projection shared memory exceeds the per-CTA limit");

struct ProjParams {
  const uint8_t* packed;
  __nv_bfloat16* q;     // [B, N, H, N, 32]
  __nv_bfloat16* k;     // [B, N, H, N, 32]
  __nv_bfloat16* bias;  // natural pair layout, element strides below
  int B, N, Np;
  int R, row0;          // problem rows held (N unless row-sharded) and the first one's global index
  int64_t bias_b, bias_h, bias_r;  // bias strides of batch, head and pair row (pair column: 1)
  int starting;
  int* err;
};

__global__ void __launch_bounds__(kProjThreads, 1)
    triattn_proj_kernel(const __grid_constant__ CUtensorMap map_z, const __grid_constant__ CUtensorMap map_vt,
                        ProjParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  ProjSmem& s = *reinterpret_cast<ProjSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int tiles_per_row = (p.N + kTile - 1) / kTile;
  const int total = p.B * p.R * tiles_per_row;

  if (threadIdx.x == 0) {
    mbar_init(&s.wbar, 1);
    for (int i = 0; i < kProjStages; ++i) {
      mbar_init(&s.z_full[i], 1);
      mbar_init(&s.z_empty[i], 1 + 4);  // MMA commit + the four statistics warps
    }
    mbar_init(&s.x_full, 1);
    mbar_init(&s.x_free, 4);
    mbar_init(&s.y_full, 1);
    mbar_init(&s.y_free, 4);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.st_full[i], 4);
      mbar_init(&s.st_free[i], 4);
    }
    fence_mbar_init();
  }
  {
    const float* v = reinterpret_cast<const float*>(p.packed + kProjBytes + kGateBytes + kOutBytes);
    for (int i = threadIdx.x; i < kProjRows; i += kProjThreads) {
      s.wsum[i] = v[i];
      s.bias[i] = v[kProjRows + i];
    }
    for (int i = threadIdx.x; i < kProjRows / 2; i += kProjThreads)
      s.wb[i] = make_float4(v[2 * i], v[2 * i + 1], v[kProjRows + 2 * i], v[kProjRows + 2 * i + 1]);
  }
  if (warp == 0) {
    tmem_alloc(&s.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem0 = s.tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_map(&map_z);
      tma_prefetch_map(&map_vt);
      mbar_arrive_expect_tx(&s.wbar, kProjBytes);
      for (int off = 0; off < static_cast<int>(kProjBytes); off += 25600)
        bulk_load(s.w + off, p.packed + off, 25600, &s.wbar);
      int it = 0;
      for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++it) {
        const int st = it % kProjStages;
        if (!mbar_wait(&s.z_empty[st], ((it / kProjStages) & 1) ^ 1, p.err, kErrTimeoutEmpty)) break;
        const int c0 = (tile % tiles_per_row) * kTile;
        const int rr = tile / tiles_per_row;
        const int b = rr / p.R, r = rr - b * p.R;
        mbar_arrive_expect_tx(&s.z_full[st], kTile * kC * 2);
        for (int kb = 0; kb < 2; ++kb) {
          uint8_t* dst = s.z[st] + kb * (kTile * 128);
          if (p.starting)
            tma_load_3d(dst, &map_z, &s.z_full[st], kb * 64, c0, rr);          // z[b, r, c0 + t]
          else
            tma_load_3d(dst, &map_z, &s.z_full[st], kb * 64, r, b * p.N + c0);  // z[b, c0 + t, r]
        }
      }
      // every issued load has landed before the CTA can exit
      mbar_wait(&s.wbar, 0, p.err, kErrTimeoutLoad);
      if (it > 0) mbar_wait(&s.z_full[(it - 1) % kProjStages], ((it - 1) / kProjStages) & 1, p.err, kErrTimeoutLoad);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc_qk = idesc_bf16_f32(128, 256);
      const uint32_t idesc_b = idesc_bf16_f32(128, 16);
      const uint32_t idesc_v = idesc_bf16_f32(128, kTile);
      const uint32_t wa = smem_u32(s.w);
      constexpr uint32_t kWBlock = kProjRows * 128;  // one 64-channel K block of the weights
      bool ok = mbar_wait(&s.wbar, 0, p.err, kErrTimeoutLoad);
      int it = 0;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, ++it) {
        const int st = it % kProjStages;
        const uint32_t za = smem_u32(s.z[st]);
        if (!mbar_wait(&s.z_full[st], (it / kProjStages) & 1, p.err, kErrTimeoutLoad)) break;
        if (!mbar_wait(&s.x_free, (it & 1) ^ 1, p.err, kErrTimeoutEmpty)) break;
        tc_fence_after();
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t dz = desc_kmajor_sw128(za + kb * (kTile * 128)) + 2 * kk;
            mma_bf16(tmem0 + kColX, dz, desc_kmajor_sw128(wa + kb * kWBlock) + 2 * kk, idesc_qk, (kb | kk) != 0);
            mma_bf16(tmem0 + kColX + 256, dz, desc_kmajor_sw128(wa + kb * kWBlock + 384 * 128) + 2 * kk, idesc_b,
                     (kb | kk) != 0);
          }
        mma_commit(&s.x_full);
        if (!mbar_wait(&s.y_free, (it & 1) ^ 1, p.err, kErrTimeoutEmpty)) break;
        tc_fence_after();
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_bf16(tmem0 + kColY, desc_kmajor_sw128(wa + kb * kWBlock + 256 * 128) + 2 * kk,
                     desc_kmajor_sw128(za + kb * (kTile * 128)) + 2 * kk, idesc_v, (kb | kk) != 0);
        mma_commit(&s.y_full);
        mma_commit(&s.z_empty[st]);
      }
    }
  } else if (warp < 6) {
    // thread = pair t of the tile (TMEM lanes of warp w are 32 (w % 4) ...)
    const int t = (warp & 3) * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    int it = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++it) {
      const int st = it % kProjStages, sb = it & 1;
      bool w1 = mbar_wait(&s.z_full[st], (it / kProjStages) & 1, p.err, kErrTimeoutLoad);
      bool w2 = mbar_wait(&s.st_free[sb], ((it >> 1) & 1) ^ 1, p.err, kErrTimeoutEmpty);
      if (!__all_sync(0xFFFFFFFFu, w1 && w2)) break;
      float mean, rstd;
      tile_stats(s.z[st], t, mean, rstd);
      {
        float* st4 = reinterpret_cast<float*>(&s.stats[sb][t >> 1]);
        st4[t & 1] = rstd;
        st4[2 + (t & 1)] = -rstd * mean;
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&s.st_full[sb]);
        mbar_arrive(&s.z_empty[st]);
      }
      const int c0 = (tile % tiles_per_row) * kTile;
      const int rr = tile / tiles_per_row;
      const int b = rr / p.R, r = rr - b * p.R;
      const int n = c0 + t;
      const bool valid = n < p.N;
      if (!__all_sync(0xFFFFFFFFu, mbar_wait(&s.x_full, it & 1, p.err, kErrTimeoutMma))) break;
      tc_fence_after();
      const int64_t row_base = (static_cast<int64_t>(b) * p.R + r) * kHeads;  // (b, r) -> head 0
      const uint64_t rs2 = f32x2(rstd, rstd), nrm2 = f32x2(-rstd * mean, -rstd * mean);
      // Q (columns 0..127) and K (128..255): one head = 32 columns = 64 contiguous bytes.
      // Double-buffered TMEM loads: chunk cc + 32 is in flight while chunk cc is written.
      auto qk_chunk = [&](int cc, const uint32_t (&v)[32]) {
        if (!valid) return;
        // channels (c, c + 1): rstd v - rstd mean wsum + bias
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float4 wb = s.wb[(cc >> 1) + i];
          float a, bb;
          f32x2_split(fma_f32x2(rs2, f32x2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1])),
                                fma_f32x2(nrm2, f32x2(wb.x, wb.y), f32x2(wb.z, wb.w))),
                      a, bb);
          w[i] = pack_bf16(a, bb);
        }
        const int head = (cc % 128) / 32;
        uint4* dst = reinterpret_cast<uint4*>((cc < 128 ? p.q : p.k) + ((row_base + head) * p.N + n) * kD);
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
      };
      uint32_t va[32], vb[32];
      tmem_ld32(tmem0 + lane_off + kColX, va);
#pragma unroll 1
      for (int cc = 0; cc < 256; cc += 64) {
        tmem_ld_wait();
        tmem_ld32(tmem0 + lane_off + kColX + cc + 32, vb);
        qk_chunk(cc, va);
        tmem_ld_wait();
        if (cc + 64 < 256) tmem_ld32(tmem0 + lane_off + kColX + cc + 64, va);
        qk_chunk(cc + 32, vb);
      }
      {
        uint32_t v[16];
        tmem_ld16(tmem0 + lane_off + kColX + 256, v);
        tmem_ld_wait();
        if (valid) {
#pragma unroll
          for (int h = 0; h < kHeads; ++h) {
            const int c = 384 + h;
            // natural pair layout [b, h, i, j] for both nodes (starting: i = r, j = n;
            // ending: i = n, j = r), so the attention reads rows of queries x keys
            const int64_t bi = p.starting ? r : n, bj = p.starting ? n : r;
            p.bias[b * p.bias_b + h * p.bias_h + bi * p.bias_r + bj] =
                __float2bfloat16_rn(rstd * (__uint_as_float(v[h]) - mean * s.wsum[c]) + s.bias[c]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.x_free);
    }
  } else {
    // thread = V channel c (head c / 32, d = c % 32); TMEM columns = the tile's pairs
    const int c = (warp & 3) * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint64_t wsv2 = f32x2(s.wsum[256 + c], s.wsum[256 + c]), bsv2 = f32x2(s.bias[256 + c], s.bias[256 + c]);
    // Each warp stages and stores its own 32 channels, one 64-pair half at a time (two
    // halves used in turn); the next 32-pair chunk's TMEM load is in flight while the
    // current one is converted.
    auto chunk = [&](int sb, int ch, const uint32_t (&v)[32]) {
      uint32_t packed[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {  // pairs (j, j + 1): rstd v - rstd mean wsum + bias
        const float4 st4 = s.stats[sb][(ch >> 1) + i];
        float a, bb;
        f32x2_split(fma_f32x2(f32x2(st4.x, st4.y), f32x2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1])),
                              fma_f32x2(f32x2(st4.z, st4.w), wsv2, bsv2)),
                    a, bb);
        packed[i] = pack_bf16(a, bb);
      }
      uint8_t* stage = s.vt[ch / 64];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        *reinterpret_cast<uint4*>(stage + sw128_offset(c, (ch % 64) + 8 * q)) =
            make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
    };
    int it = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++it) {
      const int sb = it & 1;
      const bool w1 = mbar_wait(&s.y_full, it & 1, p.err, kErrTimeoutMma);
      const bool w2 = mbar_wait(&s.st_full[sb], (it >> 1) & 1, p.err, kErrTimeoutLoad);
      // no barrier joins these warps, so each leaves on its own after a failed wait
      if (!__all_sync(0xFFFFFFFFu, w1 && w2)) break;
      tc_fence_after();
      const int c0 = (tile % tiles_per_row) * kTile;
      const int rr = tile / tiles_per_row;
      uint32_t va[32], vb[32];
      tmem_ld32(tmem0 + lane_off + kColY, va);
#pragma unroll 1
      for (int ch = 0; ch < kTile; ch += 64) {
        // this warp's store of this half two stores ago has finished reading it
        if (lane == 0) tma_store_wait_read1();
        __syncwarp();
        tmem_ld_wait();
        tmem_ld32(tmem0 + lane_off + kColY + ch + 32, vb);
        chunk(sb, ch, va);
        tmem_ld_wait();
        if (ch + 64 < kTile) tmem_ld32(tmem0 + lane_off + kColY + ch + 64, va);
        chunk(sb, ch + 32, vb);
        if (ch + 64 == kTile) {
          // the tile's accumulator and statistics have been read
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&s.y_free);
            mbar_arrive(&s.st_free[sb]);
          }
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          // V^T rows (b, r, head, d) = rr * 128 + c for this warp's 32 channels; pairs past
          // N are clipped by the map, a half wholly past N is not stored (empty group)
          if (c0 + ch < p.N) tma_store_2d(&map_vt, s.vt[ch / 64] + (warp & 3) * 32 * 128, c0 + ch, rr * kC + (warp & 3) * 32);
          tma_store_commit();
        }
      }
    }
    if (lane == 0) tma_store_wait_all0();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem0, 512);
  }
}

// ====================================================================== 2. attention
// Per CTA, a flat sequence of (unit, 64-key block) steps; a unit is 256 queries (two groups
// of 128) of one (batch, row, head).
//   warp 0      TMA: Q per unit (double-buffered), K, V^T and the two groups' bias tiles
//               per block through a 4-stage ring
//   warps 1, 10 MMA, one thread per group (on different SM sub-partitions): S = Q K^T of
//               step i + 2 (into the group's S/P buffer (i + 2) % 3) ahead of O += P V of
//               step i, with P read from TMEM (A operand) and O accumulated in TMEM across
//               the unit's blocks (one O buffer per group: the next unit's first P V waits
//               until the previous output has been read). Three S/P buffers let the tensor
//               pipe run two steps ahead of the softmax. With a head width of 32 the
//               products are small and each tcgen05 instruction costs its issuing thread
//               tens of cycles, so one thread issuing both groups' 12 products and their
//               commits per step would pace the kernel.
//   warps 2-9   softmax, thread = query row (TMEM lane): logits = S + bias (+ key mask),
//               P = 2^(x - m) written back over S as bf16. The running maximum m is raised
//               lazily: only when a block's maximum exceeds m + kRescale does the warp
//               rescale O (and the row sum) in TMEM, after the previous P V has landed, so
//               P <= 2^kRescale. V^T carries a row of ones (B operand row 32), so O column 32
//               is the row sum of P as the tensor core multiplied it. A unit's output is
//               read, normalised and stored while the next unit's first block runs.
constexpr int kKB = 64;        // keys per block
constexpr int kKVStages = 4;
constexpr int kAttnThreads = 352;  // warp 0 TMA, warps 1 / 10 MMA (group 0 / 1), warps 2..9 softmax
constexpr int kMmaWarp1 = 10;
constexpr int kMaxMaskWords = 2048;  // B * ceil(N / 64) * 2 words of key-mask bits
constexpr int kPolyEvery = 4;        // one key pair in four takes the FMA-pipe exponential
constexpr int kVtRows = 48;          // V^T (32 rows), a row of ones, 15 zero rows
constexpr int kOCols = 48;           // O (32 columns), the row sum, 15 unused
constexpr int kSBufs = 3;            // S/P buffers per group
constexpr int kGroupCols = 256;      // per group: S/P buffers at +0 / +64 / +128, O at +192
constexpr uint32_t kOCol = 192;
constexpr float kRescale = 8.0f;     // lazy-rescale threshold in log2 units

struct AttnSmem {
  alignas(1024) uint8_t q[2][kGroups][kTile * kD * 2];       // 8 KB each, SW64, by unit parity
  alignas(1024) uint8_t k[kKVStages][kKB * kD * 2];          // 4 KB, SW64
  alignas(1024) uint8_t vt[kKVStages][kVtRows * kKB * 2];    // 6 KB, SW128
  alignas(1024) uint8_t bias[kKVStages][kGroups][kTile * kKB * 2];  // 16 KB each, SW128
  uint32_t mask_words[kMaxMaskWords];
  uint64_t q_full[2], q_empty[2];
  uint64_t kv_full[kKVStages], kv_empty[kKVStages];
  uint64_t s_full[kGroups][kSBufs];
  uint64_t p_full[kGroups][kSBufs];
  uint64_t pv_done[kGroups][kSBufs];  // the group's P V of step i, on barrier i % kSBufs
  uint64_t o_full[kGroups], o_free[kGroups];
  uint64_t mma_done[kGroups];
  uint32_t tmem_base;
};

static_assert(sizeof(AttnSmem) + 1024 <= 232448, "attention shared memory exceeds the per-CTA limit");

struct AttnParams {
  const uint8_t* mask;   // [B, N]
  __nv_bfloat16* o;      // natural pair layout [B, R, N, 128]
  int B, N;
  int R, row0;           // problem rows held and the first one's global index
  int starting;
  int qpairs;            // ceil(ceil(N / 128) / 2)
  int words_per_batch;   // 2 * ceil(N / 64)
  int* err;
};

__device__ __forceinline__ void unit_coords(int unit, const AttnParams& p, int& b, int& r, int& h, int& qp) {
  qp = unit % p.qpairs;
  int rest = unit / p.qpairs;
  h = rest % kHeads;
  rest /= kHeads;
  r = rest % p.R;
  b = rest / p.R;
}

__global__ void __launch_bounds__(kAttnThreads, 1)
    triattn_attn_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                        const __grid_constant__ CUtensorMap map_vt, const __grid_constant__ CUtensorMap map_bias,
                        AttnParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  AttnSmem& s = *reinterpret_cast<AttnSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int units = p.B * p.R * kHeads * p.qpairs;
  const int nkb = (p.N + kKB - 1) / kKB;
  const int my_units = blockIdx.x < units ? (units - 1 - static_cast<int>(blockIdx.x)) / gridDim.x + 1 : 0;
  const int steps = my_units * nkb;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.q_full[i], 1);
      mbar_init(&s.q_empty[i], kGroups);  // one commit per MMA thread
    }
    for (int i = 0; i < kKVStages; ++i) {
      mbar_init(&s.kv_full[i], 1);
      mbar_init(&s.kv_empty[i], kGroups + 8);  // a commit per MMA thread + 8 softmax warps (bias read)
    }
    for (int g = 0; g < kGroups; ++g) {
      mbar_init(&s.o_full[g], 1);
      mbar_init(&s.o_free[g], 4);
      for (int i = 0; i < kSBufs; ++i) {
        mbar_init(&s.p_full[g][i], 4);
        mbar_init(&s.s_full[g][i], 1);
        mbar_init(&s.pv_done[g][i], 1);
      }
    }
    for (int g = 0; g < kGroups; ++g) mbar_init(&s.mma_done[g], 1);
    fence_mbar_init();
  }
  // key-mask bits, per batch padded to whole 64-key blocks (zero beyond N)
  for (int w = threadIdx.x; w < p.B * p.words_per_batch; w += kAttnThreads) {
    const int b = w / p.words_per_batch;
    const int k0 = (w % p.words_per_batch) * 32;
    uint32_t bits = 0;
    for (int i = 0; i < 32; ++i) {
      const int k = k0 + i;
      if (k < p.N && p.mask[b * p.N + k]) bits |= 1u << i;
    }
    s.mask_words[w] = bits;
  }
  // constant rows 32..47 of every V^T stage: bf16 ones, then zeros (TMA writes rows 0..31)
  for (int w = threadIdx.x; w < kKVStages * (kVtRows - kD) * 32; w += kAttnThreads) {
    const int st = w / ((kVtRows - kD) * 32);
    const int row = kD + (w / 32) % (kVtRows - kD);
    reinterpret_cast<uint32_t*>(s.vt[st] + row * 128)[w % 32] = row == kD ? 0x3F803F80u : 0u;
  }
  fence_async_smem();
  if (warp == 0) {
    tmem_alloc(&s.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem0 = s.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_map(&map_q);
      tma_prefetch_map(&map_k);
      tma_prefetch_map(&map_vt);
      tma_prefetch_map(&map_bias);
      int kv_it = 0, ul = 0;
      bool ok = true;
      for (int unit = blockIdx.x; unit < units && ok; unit += gridDim.x, ++ul) {
        int b, r, h, qp;
        unit_coords(unit, p, b, r, h, qp);
        const int qrow = (b * p.R + r) * kHeads + h;
        const int qb = ul & 1;
        if (!mbar_wait(&s.q_empty[qb], ((ul >> 1) & 1) ^ 1, p.err, kErrTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&s.q_full[qb], kGroups * kTile * kD * 2);
        for (int g = 0; g < kGroups; ++g) tma_load_3d(s.q[qb][g], &map_q, &s.q_full[qb], 0, (qp * 2 + g) * kTile, qrow);
        for (int j = 0; j < nkb; ++j, ++kv_it) {
          const int st = kv_it % kKVStages;
          if (!mbar_wait(&s.kv_empty[st], ((kv_it / kKVStages) & 1) ^ 1, p.err, kErrTimeoutEmpty)) { ok = false; break; }
          mbar_arrive_expect_tx(&s.kv_full[st], kKB * kD * 2 * 2 + kGroups * kTile * kKB * 2);
          tma_load_3d(s.k[st], &map_k, &s.kv_full[st], 0, j * kKB, qrow);
          tma_load_3d(s.vt[st], &map_vt, &s.kv_full[st], j * kKB, 0, qrow);
          for (int g = 0; g < kGroups; ++g)
            tma_load_3d(s.bias[st][g], &map_bias, &s.kv_full[st], j * kKB, (qp * 2 + g) * kTile, b * kHeads + h);
        }
        if (!ok) {
          ++ul;
          break;
        }
      }
      // every issued copy lands before the CTA may exit
      for (int k = 0; k < kKVStages && k < kv_it; ++k) {
        const int i = kv_it - 1 - k;
        mbar_wait(&s.kv_full[i % kKVStages], (i / kKVStages) & 1, p.err, kErrTimeoutLoad);
      }
      for (int k = 0; k < 2 && k < ul; ++k) {
        const int i = ul - 1 - k;
        mbar_wait(&s.q_full[i & 1], (i >> 1) & 1, p.err, kErrTimeoutLoad);
      }
    }
  } else if (warp == 1 || warp == kMmaWarp1) {
    // ------------------------------------------------------------ MMA issuers (one per group)
    if (lane == 0) {
      const int g = warp == 1 ? 0 : 1;
      const uint32_t idesc_s = idesc_bf16_f32(128, kKB);
      const uint32_t idesc_o = idesc_bf16_f32(128, kOCols);
      // The loop is kept short (no runtime division, descriptors advanced by constant
      // strides): this thread shares its sub-partition with softmax warps that are always
      // ready to issue. Descriptor start addresses are in 16-byte units (14 bits; shared
      // memory < 256 KB).
      constexpr uint32_t kQStep = kTile * kD * 2 / 16, kKStep = kKB * kD * 2 / 16, kVStep = kVtRows * kKB * 2 / 16;
      const uint64_t dq0 = desc_kmajor_sw64(smem_u32(s.q[0][g]));
      const uint64_t dk0 = desc_kmajor_sw64(smem_u32(s.k[0]));
      const uint64_t dv0 = desc_kmajor_sw128(smem_u32(s.vt[0]));
      const uint32_t gcols = tmem0 + g * kGroupCols;
      // S = Q K^T of step i (block j of unit ul) for this group into S/P buffer i % kSBufs
      auto issue_s = [&](int i, int j, int ul) -> bool {
        const int st = i % kKVStages, buf = i % kSBufs, qb = ul & 1;
        if (j == 0 && !mbar_wait(&s.q_full[qb], (ul >> 1) & 1, p.err, kErrTimeoutLoad)) return false;
        if (!mbar_wait(&s.kv_full[st], (i / kKVStages) & 1, p.err, kErrTimeoutLoad)) return false;
        tc_fence_after();
        const uint32_t d = gcols + buf * 64;
        const uint64_t da = dq0 + static_cast<uint64_t>(qb * kGroups * kQStep);
        const uint64_t db = dk0 + static_cast<uint64_t>(st * kKStep);
        mma_bf16(d, da, db, idesc_s, 0);
        mma_bf16(d, da + 2, db + 2, idesc_s, 1);
        mma_commit(&s.s_full[g][buf]);
        if (j == nkb - 1) mma_commit(&s.q_empty[qb]);  // the unit's Q may be refilled once these finish
        return true;
      };
      bool ok = true;
      int si = 0, sj = 0, sul = 0;  // the next S step and its (block, unit)
      for (; si < 2 && si < steps && ok; ++si) {
        ok = issue_s(si, sj, sul);
        if (++sj == nkb) sj = 0, ++sul;
      }
      int j = 0, ul = 0;
      for (int i = 0; i < steps && ok; ++i) {
        // S two steps ahead: its buffer's last P was read by the P V issued one step ago
        // (same thread, so the tensor pipe keeps the order)
        if (si < steps) {
          if (!issue_s(si, sj, sul)) break;
          ++si;
          if (++sj == nkb) sj = 0, ++sul;
        }
        const int st = i % kKVStages, buf = i % kSBufs;
        if (!mbar_wait(&s.p_full[g][buf], (i / kSBufs) & 1, p.err, kErrTimeoutMma)) break;
        // the single O buffer: the previous unit's output has been read
        if (j == 0 && !mbar_wait(&s.o_free[g], (ul & 1) ^ 1, p.err, kErrTimeoutEmpty)) break;
        tc_fence_after();
        const uint32_t d = gcols + kOCol;
        const uint32_t a = gcols + buf * 64;
        const uint64_t db = dv0 + static_cast<uint64_t>(st * kVStep);
        mma_bf16_tmem_a(d, a, db, idesc_o, j != 0);
        mma_bf16_tmem_a(d, a + 8, db + 2, idesc_o, 1);
        mma_bf16_tmem_a(d, a + 16, db + 4, idesc_o, 1);
        mma_bf16_tmem_a(d, a + 24, db + 6, idesc_o, 1);
        if (j == nkb - 1) mma_commit(&s.o_full[g]);
        // this group's P V of step i. One barrier per S/P buffer: when the softmax of step
        // i + 1 waits for it, S(i + 1) has landed, so every P V of the group up to step i - 2
        // has too, and the barrier's previous phase (step i - 3) is complete: the parity wait
        // is exact
        mma_commit(&s.pv_done[g][buf]);
        mma_commit(&s.kv_empty[st]);
        if (++j == nkb) j = 0, ++ul;
      }
      // every issued MMA completes before TMEM is released
      mma_commit(&s.mma_done[g]);
      mbar_wait(&s.mma_done[g], 0, p.err, kErrTimeoutMma);
    }
  } else {
    // ------------------------------------------------------------ softmax warpgroups
    const int g = (warp - 2) / 4;
    const int t = (warp & 3) * 32 + lane;  // TMEM lane == query row in the group's tile
    const uint32_t gbase = tmem0 + (static_cast<uint32_t>((warp & 3) * 32) << 16) + g * kGroupCols;
    const float kMasked = -1.0e9f * kLog2e;
    const float kNegInf = -__int_as_float(0x7f800000);
    bool ok = true;
    int i = 0;                                   // step index
    int prev_q = 0, prev_b = 0, prev_r = 0, prev_h = 0;  // the unit awaiting its output
    // read, normalise and store the output of unit `pu` (O buffer pu % 2)
    auto finalize = [&](int pu) -> bool {
      const bool w = mbar_wait(&s.o_full[g], pu & 1, p.err, kErrTimeoutMma);
      if (!__all_sync(0xFFFFFFFFu, w)) return false;
      tc_fence_after();
      uint32_t ov[32], os;
      tmem_ld32(gbase + kOCol, ov);
      tmem_ld1(gbase + kOCol + kD, os);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.o_free[g]);
      if (prev_q < p.N) {
        const float inv = 1.0f / __uint_as_float(os);
        // natural pair position: starting (i=r, j=q), ending (i=q, j=r)
        const int64_t pi = p.starting ? prev_r : prev_q;
        const int64_t pj = p.starting ? prev_q : prev_r;
        uint4* dst = reinterpret_cast<uint4*>(
            p.o + (((static_cast<int64_t>(prev_b) * p.R + pi) * p.N + pj) * kC + prev_h * kD));
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float* f = reinterpret_cast<const float*>(ov) + 8 * k;
          dst[k] = make_uint4(pack_bf16(f[0] * inv, f[1] * inv), pack_bf16(f[2] * inv, f[3] * inv),
                              pack_bf16(f[4] * inv, f[5] * inv), pack_bf16(f[6] * inv, f[7] * inv));
        }
      }
      return true;
    };
    int ul = 0;
    for (int unit = blockIdx.x; unit < units && ok; unit += gridDim.x, ++ul) {
      int b, r, h, qp;
      unit_coords(unit, p, b, r, h, qp);
      const int q = (qp * 2 + g) * kTile + t;
      const bool row_on = p.mask[b * p.N + p.row0 + r] != 0;
      const uint32_t* mw = s.mask_words + b * p.words_per_batch;
      float m = 0.f;
      for (int j = 0; j < nkb; ++j, ++i) {
        const int st = i % kKVStages;
        const int buf = i % kSBufs;
        const bool w1 = mbar_wait(&s.s_full[g][buf], (i / kSBufs) & 1, p.err, kErrTimeoutMma);
        const bool w2 = mbar_wait(&s.kv_full[st], (i / kKVStages) & 1, p.err, kErrTimeoutLoad);
        if (!__all_sync(0xFFFFFFFFu, w1 && w2)) { ok = false; break; }
        tc_fence_after();
        uint32_t sv[64];
        tmem_ld32(gbase + buf * 64, *reinterpret_cast<uint32_t(*)[32]>(sv));
        tmem_ld32(gbase + buf * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(sv + 32));
        tmem_ld_wait();
        // logits (base 2): s + bias, then the mask
        float x[64];
        const uint8_t* bt = s.bias[st][g];
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          const uint4 bv = *reinterpret_cast<const uint4*>(bt + sw128_offset(t, c8 * 8));
          const uint32_t w[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int c = c8 * 8 + 2 * e;
            f32x2_split(add_f32x2(f32x2(__uint_as_float(sv[c]), __uint_as_float(sv[c + 1])),
                                  f32x2(bf16_lo(w[e]), bf16_hi(w[e]))),
                        x[c], x[c + 1]);
          }
        }
        const int k0 = j * kKB;
        const uint64_t keep = row_on ? ((static_cast<uint64_t>(mw[2 * j + 1]) << 32) | mw[2 * j]) : 0ull;
        const int nvalid = p.N - k0 < kKB ? p.N - k0 : kKB;
        if (keep != ~0ull) {
#pragma unroll
          for (int c = 0; c < kKB; ++c) {
            if (!((keep >> c) & 1ull)) x[c] = c < nvalid ? kMasked : kNegInf;
          }
        }
        // block maximum: a three-input max tree (depth 4)
        float t1[22];
#pragma unroll
        for (int k = 0; k < 21; ++k) t1[k] = max3f(x[3 * k], x[3 * k + 1], x[3 * k + 2]);
        t1[21] = x[63];
        float t2[8];
#pragma unroll
        for (int k = 0; k < 7; ++k) t2[k] = max3f(t1[3 * k], t1[3 * k + 1], t1[3 * k + 2]);
        t2[7] = t1[21];
        const float bm = max3f(max3f(t2[0], t2[1], t2[2]), max3f(t2[3], t2[4], t2[5]), fmaxf(t2[6], t2[7]));
        if (j == 0) {
          m = bm;  // the unit's first block: nothing accumulated yet
        } else {
          const bool need = bm > m + kRescale;
          if (__any_sync(0xFFFFFFFFu, need)) {
            // raise m: O and the row sum (in TMEM) scale by 2^(m - m_new) once the previous
            // P V has landed
            const float m_new = need ? bm : m;
            const float alpha = ex2(m - m_new);
            const bool w3 = mbar_wait(&s.pv_done[g][(i - 1) % kSBufs], ((i - 1) / kSBufs) & 1, p.err, kErrTimeoutMma);
            if (!__all_sync(0xFFFFFFFFu, w3)) { ok = false; break; }
            tc_fence_after();
            uint32_t ov[32], os;
            tmem_ld32(gbase + kOCol, ov);
            tmem_ld1(gbase + kOCol + kD, os);
            tmem_ld_wait();
#pragma unroll
            for (int d = 0; d < kD; ++d) ov[d] = __float_as_uint(__uint_as_float(ov[d]) * alpha);
            os = __float_as_uint(__uint_as_float(os) * alpha);
            tmem_st32(gbase + kOCol, ov);
            tmem_st1(gbase + kOCol + kD, os);
            tmem_st_wait();
            m = m_new;
          }
        }
        // P = 2^(x - m) <= 2^kRescale: one key pair in kPolyEvery on the FMA pipe (cubic),
        // the rest on MUFU; packed to bf16 and written over S in TMEM
        const uint64_t neg_m = f32x2(-m, -m);
        uint32_t pw[32];
#pragma unroll
        for (int c = 0; c < kKB; c += 2) {
          const uint64_t d = add_f32x2(f32x2(x[c], x[c + 1]), neg_m);
          float e0, e1;
          if ((c / 2) % kPolyEvery == kPolyEvery - 1) {
            exp2_poly_x2(d, e0, e1);
          } else {
            float d0, d1;
            f32x2_split(d, d0, d1);
            e0 = ex2(d0);
            e1 = ex2(d1);
          }
          pw[c / 2] = pack_bf16(e0, e1);
        }
        tmem_st32(gbase + buf * 64, pw);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&s.p_full[g][buf]);
          mbar_arrive(&s.kv_empty[st]);
        }
        // the previous unit's output, while this unit's first P V runs
        if (j == 0 && ul > 0 && !finalize(ul - 1)) { ok = false; break; }
      }
      prev_q = q;
      prev_b = b;
      prev_r = r;
      prev_h = h;
    }
    if (ok && ul > 0) finalize(ul - 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem0, 512);
  }
}

// ====================================================================== 3. output
// Warp-specialised, persistent, 128-pair tiles (natural pair layout for both nodes); TMEM
// lane = pair, column = channel:
//   gate[p][c]  = z[p] . W_g'[c]                       (folded input LayerNorm)
//   G[p][c]     = sigmoid(gate[p][c]) * o[p][c]        written over the o tile in place: it
//                                                      is the K-major A operand of
//   delta[p][c] = G[p] . W_o[c];   z'[p][c] = z[p][c] + delta[p][c]  (in place, TMA store)
// A thread owns one pair: its o and z rows are read and written as 16-byte swizzled
// vectors, its LayerNorm coefficients stay in registers, and the paired fp32 pipe handles
// two channels per instruction.
//   warp 0      TMA: z and o tiles, 2-stage ring; it also stores each finished tile from its
//               slot (after the eight epilogue warps arrive) before reloading it
//   warp 1      MMA: gate product (tile t + 1) ahead of the output product (tile t)
//   warps 2-3   per-pair LayerNorm statistics of z and the keep mask
//   warps 4-11  lane = pair; warps 4-7 channels 0-63, warps 8-11 channels 64-127
constexpr int kOTile = 128;
constexpr int kOStages = 2;
constexpr int kOThreads = 384;

struct OutSmem {
  alignas(1024) uint8_t wg[kGateBytes];                // [c][k]: 2 K-blocks of [128 c x 128 B]
  alignas(1024) uint8_t wo[kOutBytes];
  alignas(1024) uint8_t z[kOStages][kOTile * kC * 2];  // [p][c]: 2 K-blocks of [128 p x 128 B]
  alignas(1024) uint8_t o[kOStages][kOTile * kC * 2];  // [p][c], same layout; G replaces o
  float4 cg[kC / 2];       // channel pair (2i, 2i+1): wsum_gate x2, bias_gate / 2 x2
  float2 pc[2][kOTile];    // per pair: rstd / 2, -rstd mean / 2
  float keep[2][kOTile];
  uint64_t wbar;
  uint64_t full[kOStages], out_ready[kOStages];  // tile landed; tile's output written over its z (8 warps)
  uint64_t g_full[2], gt_ready[2], d_full[2], acc_free[2], st_full[2], st_free[2];
  uint32_t tmem_base;
};

static_assert(sizeof(OutSmem) + 1024 <= 232448, "output shared memory exceeds the per-CTA limit");

struct OutParams {
  const uint8_t* packed;
  const uint8_t* mask;
  int B, N;
  int R, row0;  // pair rows held and the first one's global index
  int masked_zero;
  int* err;
};

__global__ void __launch_bounds__(kOThreads, 1)
    triattn_out_kernel(const __grid_constant__ CUtensorMap map_z, const __grid_constant__ CUtensorMap map_o,
                       const __grid_constant__ CUtensorMap map_out, OutParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  OutSmem& s = *reinterpret_cast<OutSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int tiles_per_row = (p.N + kOTile - 1) / kOTile;
  const int total = p.B * p.R * tiles_per_row;

  if (threadIdx.x == 0) {
    mbar_init(&s.wbar, 1);
    for (int i = 0; i < kOStages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.out_ready[i], 8);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.g_full[i], 1);
      mbar_init(&s.gt_ready[i], 8);
      mbar_init(&s.d_full[i], 1);
      mbar_init(&s.acc_free[i], 8);
      mbar_init(&s.st_full[i], 2);
      mbar_init(&s.st_free[i], 8);
    }
    fence_mbar_init();
  }
  {
    const float* v = reinterpret_cast<const float*>(p.packed + kProjBytes + kGateBytes + kOutBytes) + 2 * kProjRows;
    for (int i = threadIdx.x; i < kC / 2; i += kOThreads)
      s.cg[i] = make_float4(v[2 * i], v[2 * i + 1], 0.5f * v[128 + 2 * i], 0.5f * v[128 + 2 * i + 1]);
  }
  if (warp == 0) {
    tmem_alloc(&s.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem0 = s.tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_map(&map_z);
      tma_prefetch_map(&map_o);
      tma_prefetch_map(&map_out);
      mbar_arrive_expect_tx(&s.wbar, kGateBytes + kOutBytes);
      bulk_load(s.wg, p.packed + kProjBytes, kGateBytes, &s.wbar);
      bulk_load(s.wo, p.packed + kProjBytes + kGateBytes, kOutBytes, &s.wbar);
      // the slot's previous tile: written over its z by the epilogue (which ran after both
      // products had read the slot), stored from there; the slot is free once the store has
      // read it. This thread, not an epilogue warp, waits for that read.
      auto store_tile = [&](int t_it, int t_tile) -> bool {
        const int sst = t_it % kOStages;
        if (!mbar_wait(&s.out_ready[sst], (t_it / kOStages) & 1, p.err, kErrTimeoutEmpty)) return false;
        const int sc0 = (t_tile % tiles_per_row) * kOTile;
        const int srr = t_tile / tiles_per_row;
        tma_store_3d(&map_out, s.z[sst], 0, sc0, srr);
        tma_store_3d(&map_out, s.z[sst] + kOTile * 128, 64, sc0, srr);
        tma_store_commit();
        tma_store_wait_read0();
        return true;
      };
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++it) {
        const int st = it % kOStages;
        if (it >= kOStages && !store_tile(it - kOStages, tile - kOStages * static_cast<int>(gridDim.x))) {
          ok = false;
          break;
        }
        const int c0 = (tile % tiles_per_row) * kOTile;
        const int rr = tile / tiles_per_row;
        mbar_arrive_expect_tx(&s.full[st], 2 * kOTile * kC * 2);
        for (int kb = 0; kb < 2; ++kb) {
          tma_load_3d(s.z[st] + kb * (kOTile * 128), &map_z, &s.full[st], kb * 64, c0, rr);
          tma_load_3d(s.o[st] + kb * (kOTile * 128), &map_o, &s.full[st], kb * 64, c0, rr);
        }
      }
      // the last tiles' stores; every issued load has landed and every store has completed
      // before the CTA can exit
      for (int k = it - kOStages; ok && k < it; ++k)
        if (k >= 0) ok = store_tile(k, static_cast<int>(blockIdx.x) + k * static_cast<int>(gridDim.x));
      mbar_wait(&s.wbar, 0, p.err, kErrTimeoutLoad);
      if (it > 0) mbar_wait(&s.full[(it - 1) % kOStages], ((it - 1) / kOStages) & 1, p.err, kErrTimeoutLoad);
      tma_store_wait_all0();
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(kOTile, kC);
      bool ok = mbar_wait(&s.wbar, 0, p.err, kErrTimeoutLoad);
      const uint32_t wg = smem_u32(s.wg), wo = smem_u32(s.wo);
      auto gate_mma = [&](int it) -> bool {
        const int st = it % kOStages, buf = it & 1;
        if (!mbar_wait(&s.full[st], (it / kOStages) & 1, p.err, kErrTimeoutLoad)) return false;
        if (!mbar_wait(&s.acc_free[buf], ((it >> 1) & 1) ^ 1, p.err, kErrTimeoutEmpty)) return false;
        tc_fence_after();
        const uint32_t za = smem_u32(s.z[st]);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_bf16(tmem0 + buf * 256, desc_kmajor_sw128(za + kb * (kOTile * 128)) + 2 * kk,
                     desc_kmajor_sw128(wg + kb * 16384) + 2 * kk, idesc, (kb | kk) != 0);
        mma_commit(&s.g_full[buf]);
        return true;
      };
      const int mine = (blockIdx.x < total) ? (total - 1 - blockIdx.x) / gridDim.x + 1 : 0;
      if (ok && mine > 0) ok = gate_mma(0);
      for (int it = 0; it < mine && ok; ++it) {
        if (it + 1 < mine && !gate_mma(it + 1)) break;
        const int st = it % kOStages, buf = it & 1;
        if (!mbar_wait(&s.gt_ready[buf], (it >> 1) & 1, p.err, kErrTimeoutMma)) break;
        tc_fence_after();
        const uint32_t ga = smem_u32(s.o[st]);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_bf16(tmem0 + buf * 256 + kC, desc_kmajor_sw128(ga + kb * (kOTile * 128)) + 2 * kk,
                     desc_kmajor_sw128(wo + kb * 16384) + 2 * kk, idesc, (kb | kk) != 0);
        mma_commit(&s.d_full[buf]);
      }
    }
  } else if (warp < 4) {
    // statistics: thread t handles pairs t and t + 64 of the tile
    const int t = (warp - 2) * 32 + lane;
    int it = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++it) {
      const int st = it % kOStages, buf = it & 1;
      // the keep mask first (global loads independent of the staged tile, so their latency
      // overlaps the waits below)
      const int c0 = (tile % tiles_per_row) * kOTile;
      const int rr = tile / tiles_per_row;
      const int b = rr / p.R, r = rr - b * p.R;
      const bool row_keep = !p.masked_zero || p.mask[b * p.N + p.row0 + r];
      bool kp[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int j = c0 + t + 64 * k;
        kp[k] = j < p.N && row_keep && (!p.masked_zero || p.mask[b * p.N + j]);
      }
      const bool w1 = mbar_wait(&s.full[st], (it / kOStages) & 1, p.err, kErrTimeoutLoad);
      const bool w2 = mbar_wait(&s.st_free[buf], ((it >> 1) & 1) ^ 1, p.err, kErrTimeoutEmpty);
      if (!__all_sync(0xFFFFFFFFu, w1 && w2)) break;
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int pp = t + 64 * k;
        float mean, rstd;
        ln_stats_c128(s.z[st], kOTile * 128, pp, mean, rstd);
        s.pc[buf][pp] = make_float2(0.5f * rstd, -0.5f * rstd * mean);
        s.keep[buf][pp] = kp[k] ? 1.f : 0.f;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.st_full[buf]);
    }
  } else {
    // lane = pair pp; half = which 64 channels
    const int half = (warp - 4) / 4;
    const int pp = (warp & 3) * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    int it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++it) {
      const int st = it % kOStages, buf = it & 1;
      if (ok) {
        const bool w1 = mbar_wait(&s.g_full[buf], (it >> 1) & 1, p.err, kErrTimeoutMma);
        const bool w2 = mbar_wait(&s.st_full[buf], (it >> 1) & 1, p.err, kErrTimeoutLoad);
        ok = __all_sync(0xFFFFFFFFu, w1 && w2);
      }
      tc_fence_after();
      uint8_t* orow = s.o[st] + half * (kOTile * 128);
      uint8_t* zrow = s.z[st] + half * (kOTile * 128);
      const bool keep = s.keep[buf][pp] != 0.f;
      if (ok) {
        // G = o * sigmoid(g) = (o / 2) tanh(g / 2) + o / 2, g / 2 = (rstd/2) gate - (rstd mean/2) wsum + b/2
        const float2 pc = s.pc[buf][pp];
        const uint64_t ga = f32x2(pc.x, pc.x), gb = f32x2(pc.y, pc.y), h2 = f32x2(0.5f, 0.5f);
#pragma unroll 1
        for (int ch = 0; ch < 64; ch += 32) {
          uint32_t vg[32];
          tmem_ld32(tmem0 + lane_off + buf * 256 + half * 64 + ch, vg);
          tmem_ld_wait();
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4* op = reinterpret_cast<uint4*>(orow + sw128_offset(pp, ch + 8 * q));
            const uint4 ov = *op;
            const uint32_t ow[4] = {ov.x, ov.y, ov.z, ov.w};
            uint32_t res[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int i = 8 * q + 2 * e;
              const float4 cg = s.cg[(half * 64 + ch + i) / 2];
              const uint64_t g = fma_f32x2(ga, f32x2(__uint_as_float(vg[i]), __uint_as_float(vg[i + 1])),
                                           fma_f32x2(gb, f32x2(cg.x, cg.y), f32x2(cg.z, cg.w)));
              float g0, g1;
              f32x2_split(g, g0, g1);
              const uint64_t o2 = mul_f32x2(f32x2(bf16_lo(ow[e]), bf16_hi(ow[e])), h2);
              const uint64_t gv = fma_f32x2(o2, f32x2(tanh_fast(g0), tanh_fast(g1)), o2);
              float r0, r1;
              f32x2_split(gv, r0, r1);
              res[e] = pack_bf16(r0, r1);
            }
            *op = make_uint4(res[0], res[1], res[2], res[3]);
          }
        }
      }
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.gt_ready[buf]);
      if (ok) {
        const bool w3 = mbar_wait(&s.d_full[buf], (it >> 1) & 1, p.err, kErrTimeoutMma);
        ok = __all_sync(0xFFFFFFFFu, w3);
      }
      tc_fence_after();
      if (ok) {
#pragma unroll 1
        for (int ch = 0; ch < 64; ch += 32) {
          uint32_t vd[32];
          tmem_ld32(tmem0 + lane_off + buf * 256 + kC + half * 64 + ch, vd);
          tmem_ld_wait();
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4* zp = reinterpret_cast<uint4*>(zrow + sw128_offset(pp, ch + 8 * q));
            const uint4 zv = *zp;
            const uint32_t zw[4] = {zv.x, zv.y, zv.z, zv.w};
            uint32_t res[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int i = 8 * q + 2 * e;
              const uint64_t zz = add_f32x2(f32x2(bf16_lo(zw[e]), bf16_hi(zw[e])),
                                            f32x2(__uint_as_float(vd[i]), __uint_as_float(vd[i + 1])));
              float r0, r1;
              f32x2_split(zz, r0, r1);
              res[e] = pack_bf16(r0, r1);
            }
            if (keep) *zp = make_uint4(res[0], res[1], res[2], res[3]);
          }
        }
      }
      tc_fence_before();
      fence_async_smem();
      __syncwarp();
      if (!ok) break;
      // this warp's pairs x channels are written over the staged z: the TMA thread stores the
      // tile once all eight warps have arrived
      if (lane == 0) {
        mbar_arrive(&s.acc_free[buf]);
        mbar_arrive(&s.st_free[buf]);
        mbar_arrive(&s.out_ready[st]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem0, 512);
  }
}

struct Workspace {
  __nv_bfloat16 *q, *k, *vt, *bias, *o;
};

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

Workspace carve(void* ws, int B, int N) {
  const size_t np = (static_cast<size_t>(N) + 7) / 8 * 8;
  uint8_t* p = static_cast<uint8_t*>(ws);
  Workspace w;
  const size_t qk = align256(static_cast<size_t>(B) * N * kHeads * N * kD * 2);
  const size_t vt = align256(static_cast<size_t>(B) * N * kHeads * kD * np * 2);
  const size_t bias = align256(static_cast<size_t>(B) * kHeads * N * np * 2);
  w.q = reinterpret_cast<__nv_bfloat16*>(p);
  w.k = reinterpret_cast<__nv_bfloat16*>(p + qk);
  w.vt = reinterpret_cast<__nv_bfloat16*>(p + 2 * qk);
  w.bias = reinterpret_cast<__nv_bfloat16*>(p + 2 * qk + vt);
  w.o = reinterpret_cast<__nv_bfloat16*>(p + 2 * qk + vt + bias);
  return w;
}

}  // namespace

size_t triattn_packed_bytes() { return kPackedBytes; }

size_t triattn_workspace_bytes(int B, int N) {
  const size_t np = (static_cast<size_t>(N) + 7) / 8 * 8;
  const size_t qk = align256(static_cast<size_t>(B) * N * kHeads * N * kD * 2);
  const size_t vt = align256(static_cast<size_t>(B) * N * kHeads * kD * np * 2);
  const size_t bias = align256(static_cast<size_t>(B) * kHeads * N * np * 2);
  const size_t o = align256(static_cast<size_t>(B) * N * N * kC * 2);
  return 2 * qk + vt + bias + o;
}

int triattn_prepare(const TriAttnWeights& w, void* packed, cudaStream_t stream) {
  uint8_t* img = static_cast<uint8_t*>(packed);
  float* vec = reinterpret_cast<float*>(img + kProjBytes + kGateBytes + kOutBytes);
  int rc = static_cast<int>(cudaMemsetAsync(packed, 0, kPackedBytes, stream));
  const float qscale = kLog2e / sqrtf(static_cast<float>(kD));
  if (rc == 0)
    rc = launch_pack_weight(w.to_query, 128, kC, w.ln_w, w.ln_b, img, 0, kProjRows, vec, vec + kProjRows, stream,
                            qscale);
  if (rc == 0)
    rc = launch_pack_weight(w.to_key, 128, kC, w.ln_w, w.ln_b, img, 128, kProjRows, vec, vec + kProjRows, stream);
  if (rc == 0)
    rc = launch_pack_weight(w.to_value, 128, kC, w.ln_w, w.ln_b, img, 256, kProjRows, vec, vec + kProjRows, stream);
  if (rc == 0)
    rc = launch_pack_weight(w.to_bias, kHeads, kC, w.ln_w, w.ln_b, img, 384, kProjRows, vec, vec + kProjRows, stream,
                            kLog2e);
  if (rc == 0)
    rc = launch_pack_weight(w.to_gate, 128, kC, w.ln_w, w.ln_b, img + kProjBytes, 0, 128, vec + 2 * kProjRows,
                            vec + 2 * kProjRows + 128, stream);
  if (rc == 0)
    rc = launch_pack_weight(w.to_out, 128, kC, nullptr, nullptr, img + kProjBytes + kGateBytes, 0, 128, nullptr,
                            nullptr, stream);
  return rc;
}

namespace {

// z-shaped map ([B * R] rows of N pairs x 128 channels) with a box of `rows` pairs along a
// row (row tiles) or along a column (column tiles, R == N)
int pair_map(CUtensorMap* m, const void* base, int B, int R, int N, int rows, bool column_tiles) {
  const uint64_t dims[3] = {kC, static_cast<uint64_t>(N), static_cast<uint64_t>(B) * R};
  const uint64_t strides[2] = {kC * 2, static_cast<uint64_t>(N) * kC * 2};
  const uint32_t box_row[3] = {64, static_cast<uint32_t>(rows), 1};
  const uint32_t box_col[3] = {64, 1, static_cast<uint32_t>(rows)};
  return make_map(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, column_tiles ? box_col : box_row,
                  CU_TENSOR_MAP_SWIZZLE_128B);
}

int launch_proj(const void* z, const void* packed, __nv_bfloat16* q, __nv_bfloat16* k, __nv_bfloat16* vt,
                __nv_bfloat16* bias, int64_t bias_b, int64_t bias_h, int64_t bias_r, int B, int R, int N,
                int starting, const DeviceInfo& info, cudaStream_t stream) {
  const int np = (N + 7) / 8 * 8;
  CUtensorMap map_z, map_vt;
  int st = pair_map(&map_z, z, B, R, N, kTile, !starting);
  if (st) return st;
  {
    // V^T as rows (b, r, head, d) of N pairs (row stride Np), stored in [128 x 64] boxes
    const uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(B) * R * kC};
    const uint64_t strides[1] = {static_cast<uint64_t>(np) * 2};
    const uint32_t box[2] = {64, 32};  // one warp's 32 channels of a 64-pair half
    st = make_map(&map_vt, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, vt, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
  }
  ProjParams pp{static_cast<const uint8_t*>(packed), q, k, bias, B, N, np, R, 0, bias_b, bias_h, bias_r,
                starting, info.err};
  const int tiles = B * R * ((N + kTile - 1) / kTile);
  const int grid = tiles < info.num_sms ? tiles : info.num_sms;
  const size_t smem = sizeof(ProjSmem) + 1024;
  cudaFuncSetAttribute(triattn_proj_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  triattn_proj_kernel<<<grid, kProjThreads, smem, stream>>>(map_z, map_vt, pp);
  return cuda_status(static_cast<int>(cudaGetLastError()), "triattn_proj launch");
}

// bias: rows = queries, element strides of query row `bq` and of (batch * H + head) `bbh`
int launch_attn(const __nv_bfloat16* q, const __nv_bfloat16* k, const __nv_bfloat16* vt, const __nv_bfloat16* bias,
                int64_t bq, int64_t bbh, const uint8_t* mask, __nv_bfloat16* o, int B, int R, int N, int row0,
                int starting, const DeviceInfo& info, cudaStream_t stream) {
  const int np = (N + 7) / 8 * 8;
  CUtensorMap map_q, map_k, map_vt, map_bias;
  const uint64_t qdims[3] = {kD, static_cast<uint64_t>(N), static_cast<uint64_t>(B) * R * kHeads};
  const uint64_t qstrides[2] = {kD * 2, static_cast<uint64_t>(N) * kD * 2};
  const uint32_t qbox[3] = {kD, kTile, 1};
  const uint32_t kbox[3] = {kD, kKB, 1};
  int st = make_map(&map_q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, q, qdims, qstrides, qbox, CU_TENSOR_MAP_SWIZZLE_64B);
  if (st) return st;
  st = make_map(&map_k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, k, qdims, qstrides, kbox, CU_TENSOR_MAP_SWIZZLE_64B);
  if (st) return st;
  const uint64_t vdims[3] = {static_cast<uint64_t>(N), kD, static_cast<uint64_t>(B) * R * kHeads};
  const uint64_t vstrides[2] = {static_cast<uint64_t>(np) * 2, static_cast<uint64_t>(kD) * np * 2};
  const uint32_t vbox[3] = {kKB, kD, 1};
  st = make_map(&map_vt, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, vt, vdims, vstrides, vbox, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  const uint64_t bdims[3] = {static_cast<uint64_t>(N), static_cast<uint64_t>(N), static_cast<uint64_t>(B) * kHeads};
  const uint64_t bstrides[2] = {static_cast<uint64_t>(bq) * 2, static_cast<uint64_t>(bbh) * 2};
  const uint32_t bbox[3] = {kKB, kTile, 1};  // [q rows][64 keys], 128-byte rows
  st = make_map(&map_bias, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, bias, bdims, bstrides, bbox, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  AttnParams ap;
  ap.mask = mask;
  ap.o = o;
  ap.B = B;
  ap.N = N;
  ap.R = R;
  ap.row0 = row0;
  ap.starting = starting;
  ap.qpairs = ((N + kTile - 1) / kTile + 1) / 2;
  ap.words_per_batch = 2 * ((N + kKB - 1) / kKB);
  ap.err = info.err;
  if (B * ap.words_per_batch > kMaxMaskWords) return fail(2, "triattn: B * N too large for the key-mask cache");
  const int units = B * R * kHeads * ap.qpairs;
  const int grid = units < info.num_sms ? units : info.num_sms;
  const size_t smem = sizeof(AttnSmem) + 1024;
  cudaFuncSetAttribute(triattn_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  triattn_attn_kernel<<<grid, kAttnThreads, smem, stream>>>(map_q, map_k, map_vt, map_bias, ap);
  return cuda_status(static_cast<int>(cudaGetLastError()), "triattn_attn launch");
}

int launch_out(const void* z, const uint8_t* mask, const void* packed, const void* o, void* out, int B, int R, int N,
               int row0, int masked_zero, const DeviceInfo& info, cudaStream_t stream) {
  CUtensorMap map_z, map_o, map_out;
  int st = pair_map(&map_z, z, B, R, N, kOTile, false);
  if (st) return st;
  st = pair_map(&map_o, o, B, R, N, kOTile, false);
  if (st) return st;
  st = pair_map(&map_out, out, B, R, N, kOTile, false);
  if (st) return st;
  OutParams op{static_cast<const uint8_t*>(packed), mask, B, N, R, row0, masked_zero, info.err};
  const int tiles = B * R * ((N + kOTile - 1) / kOTile);
  const int grid = tiles < info.num_sms ? tiles : info.num_sms;
  const size_t smem = sizeof(OutSmem) + 1024;
  cudaFuncSetAttribute(triattn_out_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  triattn_out_kernel<<<grid, kOThreads, smem, stream>>>(map_z, map_o, map_out, op);
  return cuda_status(static_cast<int>(cudaGetLastError()), "triattn_out launch");
}

}  // namespace

int triattn_forward(const void* z, const uint8_t* mask, const void* packed, void* out, void* workspace, int B, int N,
                    int starting, int masked_zero, int stages, const DeviceInfo& info, cudaStream_t stream) {
  const int64_t np = (N + 7) / 8 * 8;
  Workspace ws = carve(workspace, B, N);
  // bias [B, H, N, Np] in the natural pair layout
  const int64_t bias_r = np, bias_h = static_cast<int64_t>(N) * np, bias_b = kHeads * bias_h;
  int st = 0;
  if (stages & 1) {
    st = launch_proj(z, packed, ws.q, ws.k, ws.vt, ws.bias, bias_b, bias_h, bias_r, B, N, N, starting, info, stream);
    if (st) return st;
  }
  if (stages & 2) {
    st = launch_attn(ws.q, ws.k, ws.vt, ws.bias, bias_r, bias_h, mask, ws.o, B, N, N, 0, starting, info, stream);
    if (st) return st;
  }
  if (stages & 4) st = launch_out(z, mask, packed, ws.o, out, B, N, N, 0, masked_zero, info, stream);
  return st;
}

// ---- row-sharded entry points (B = 1): the rank holds rows [row0, row0 + R) of the pair
// (for the ending node: of the transposed pair). Q, K [R, H, N, 32], V^T [R, H, 32, Np],
// o [R, N, 128]; the rank's bias rows [R][H][Np] concatenate under an all-gather into the
// [N][H][Np] bias (rows = queries) the attention reads.
int triattn_shard_proj(const void* z, const void* packed, void* q, void* k, void* vt, void* bias_rows, int R, int N,
                       const DeviceInfo& info, cudaStream_t stream) {
  const int64_t np = (N + 7) / 8 * 8;
  return launch_proj(z, packed, static_cast<__nv_bfloat16*>(q), static_cast<__nv_bfloat16*>(k),
                     static_cast<__nv_bfloat16*>(vt), static_cast<__nv_bfloat16*>(bias_rows), R * kHeads * np, np,
                     kHeads * np, 1, R, N, 1, info, stream);
}

int triattn_shard_attn(const void* q, const void* k, const void* vt, const void* bias_all, const uint8_t* mask, void* o,
                       int R, int N, int row0, const DeviceInfo& info, cudaStream_t stream) {
  const int64_t np = (N + 7) / 8 * 8;
  return launch_attn(static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
                     static_cast<const __nv_bfloat16*>(vt), static_cast<const __nv_bfloat16*>(bias_all), kHeads * np,
                     np, mask, static_cast<__nv_bfloat16*>(o), 1, R, N, row0, 1, info, stream);
}

int triattn_shard_out(const void* z, const uint8_t* mask, const void* packed, const void* o, void* out, int R, int N,
                      int row0, int masked_zero, const DeviceInfo& info, cudaStream_t stream) {
  return launch_out(z, mask, packed, o, out, 1, R, N, row0, masked_zero, info, stream);
}

}  // namespace ffb
