// Triangle multiplicative update (outgoing / incoming), bf16 activations, c_z = h = 128.
//
//   x = LN(z);  L = sigmoid(W_lg x) * (W_l x) * m_a m_k;  R = likewise;
//   u_ij = sum_k L_ik R_jk (outgoing) | sum_k L_ki R_kj (incoming);
//   z' = z + W_o LN_out(u) * sigmoid(W_g x)
// (legacy/reference/triangle.py:19-50, engine left/right per legacy/released.py:135-173).
//
// Three launches:
//  1. trimul_proj: 64-pair tiles of raw z (TMA, 128B swizzle) times the resident packed
//     projection [W_l; W_lg; W_r; W_rg] (tcgen05, fp32 in TMEM); the LayerNorm is folded
//     into the epilogue; L and R are written CHANNEL-MAJOR [c][a][k] so that step 2 is a
//     plain K-major GEMM per channel. The incoming direction reads COLUMN tiles of z
//     (pairs (k, a) for fixed a), which makes its contraction the same GEMM.
//  2. the per-channel contraction U_c = L_c R_c^T on the batched tcgen05 GEMM (gemm.cu).
//  3. trimul_out: per 128-pair tile, two tcgen05 GEMMs (gate from raw z, output
//     projection from raw u) with both LayerNorms folded into the epilogue through the
//     per-pair statistics (z's from step 1, u's taken from the staged u tile by the
//     statistics warps), sigmoid gate, mask and residual, written back through the z tile
//     and a TMA store.
//
// Kernels 1 and 3 are persistent (one CTA per SM) and warp-specialised: a TMA warp, an MMA
// warp, statistics warps and eight epilogue warps, with the resident weights, a ring of
// input tiles and double-buffered TMEM accumulators.
#include "abi_util.h"
#include "common.cuh"
#include "kernels.h"

namespace ffb {
namespace {

constexpr int kC = 128;       // pair channels
constexpr int kH = 128;       // hidden channels

// ---------------------------------------------------------------- packed weight image
// [0, 128K)            projection operand: rows 0..127 W_l', 128..255 W_lg', 256..383 W_r', 384..511 W_rg'
//                      (each scaled by 1/2: the epilogue's sigmoid is 1/2 + tanh(x / 2) / 2)
// [128K, 160K)         gate operand W_g' (rows = output channels)
// [160K, 192K)         output operand W_o' = W_o diag(gamma_out)
// [192K, +)            fp32: wsum_proj[512] bias_proj[512] wsum_gate[128] bias_gate[128] bias_out[128]
//                      wsum_out[128]
constexpr size_t kProjBytes = 512 * kC * 2;
constexpr size_t kGateBytes = kC * kC * 2;
constexpr size_t kOutBytes = kC * kH * 2;
constexpr size_t kVecFloats = 512 + 512 + 128 + 128 + 128 + 128;
constexpr size_t kPackedBytes = kProjBytes + kGateBytes + kOutBytes + kVecFloats * 4;

struct Vecs {
  float wsum_proj[512];
  float bias_proj[512];
  float wsum_gate[128];
  float bias_gate[128];
  float bias_out[128];
};

// ====================================================================== kernel 1
// Warp-specialised, persistent, 64-pair tiles. The projection is computed TRANSPOSED,
// D[channel][pair] = W'[channel][:] . z[pair][:], so a TMEM lane is an output channel and
// its columns are consecutive pairs: each epilogue thread owns one channel of L (or R),
// writes its 64 pairs into a 128-byte-swizzled [channel][pair] staging tile, and one thread
// per part stores the tile with a TMA store (pairs past N are clipped by the tensor map).
//   warp 0      TMA: z tiles into a 3-stage ring
//   warp 1      MMA: 4 x (M 128 channels, N 64 pairs, K 128) per tile -> 256 TMEM columns,
//               double-buffered (512 columns)
//   warps 2-3   LayerNorm statistics and pair mask of the tile's 64 pairs -> shared memory
//   warps 4-11  epilogue: warps 4-7 produce L, warps 8-11 produce R
constexpr int kPTile = 64;
constexpr int kPStages = 3;
constexpr int kPThreads = 384;

struct ProjSmem {
  alignas(1024) uint8_t w[kProjBytes];
  alignas(1024) uint8_t z[kPStages][kPTile * kC * 2];
  // L / R staging per part, two halves of 32 pairs used in turn: [128 channels][32 pairs], SW64
  alignas(1024) uint8_t out[2][2][kH * 32 * 2];
  float wsum[512];
  float bias[512];
  float4 coef[2][kPTile / 2];  // per pair couple (2i, 2i + 1): rstd, rstd; -rstd mean, -rstd mean
  float2 pm[2][kPTile / 2];    // per pair couple: the pair mask
  uint64_t wbar;
  uint64_t z_full[kPStages], z_empty[kPStages];
  uint64_t acc_full[2], acc_free[2];
  uint64_t st_full[2], st_free[2];
  uint32_t tmem_base;
};

struct ProjParams {
  const uint8_t* packed;
  const uint8_t* mask;  // [B, N]
  __nv_bfloat16* left;  // [B*h, N, Np]
  __nv_bfloat16* right;
  float2* zstats;       // [B, R, N] (mean, rstd) of the input LayerNorm, natural pair order
  int B, N, Np;
  int R, row0;          // problem rows held (N unless row-sharded) and the first one's global index
  int64_t ls_b, ls_c, ls_r;  // L / R element strides of batch, channel and row
  int outgoing;
  int* err;
};

static_assert(sizeof(ProjSmem) + 1024 <= 232448, "projection shared memory exceeds the per-CTA limit");

__global__ void __launch_bounds__(kPThreads, 1)
    trimul_proj_kernel(const __grid_constant__ CUtensorMap map_z, const __grid_constant__ CUtensorMap map_l,
                       const __grid_constant__ CUtensorMap map_r, ProjParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  ProjSmem& s = *reinterpret_cast<ProjSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int tiles_per_row = (p.N + kPTile - 1) / kPTile;
  const int total = p.B * p.R * tiles_per_row;

  if (threadIdx.x == 0) {
    mbar_init(&s.wbar, 1);
    for (int i = 0; i < kPStages; ++i) {
      mbar_init(&s.z_full[i], 1);
      mbar_init(&s.z_empty[i], 1 + 2);  // MMA commit + the two statistics warps
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.acc_full[i], 1);
      mbar_init(&s.acc_free[i], 8);
      mbar_init(&s.st_full[i], 2);
      mbar_init(&s.st_free[i], 8);
    }
    fence_mbar_init();
  }
  {
    const float* v = reinterpret_cast<const float*>(p.packed + kProjBytes + kGateBytes + kOutBytes);
    for (int i = threadIdx.x; i < 512; i += kPThreads) {
      s.wsum[i] = v[i];
      s.bias[i] = v[512 + i];
    }
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
      tma_prefetch_map(&map_l);
      tma_prefetch_map(&map_r);
      mbar_arrive_expect_tx(&s.wbar, kProjBytes);
      for (int off = 0; off < static_cast<int>(kProjBytes); off += 32768)
        bulk_load(s.w + off, p.packed + off, 32768, &s.wbar);
      int it = 0;
      for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++it) {
        const int st = it % kPStages;
        if (!mbar_wait(&s.z_empty[st], ((it / kPStages) & 1) ^ 1, p.err, kErrTimeoutEmpty)) break;
        const int c0 = (tile % tiles_per_row) * kPTile;
        const int rr = tile / tiles_per_row;
        const int b = rr / p.R, r = rr - b * p.R;
        mbar_arrive_expect_tx(&s.z_full[st], kPTile * kC * 2);
        for (int kb = 0; kb < 2; ++kb) {
          uint8_t* dst = s.z[st] + kb * (kPTile * 128);
          if (p.outgoing)
            tma_load_3d(dst, &map_z, &s.z_full[st], kb * 64, c0, rr);          // z[b, r, c0 + t]
          else
            tma_load_3d(dst, &map_z, &s.z_full[st], kb * 64, r, b * p.N + c0);  // z[b, c0 + t, r]
        }
      }
      mbar_wait(&s.wbar, 0, p.err, kErrTimeoutLoad);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(128, kPTile);
      bool ok = mbar_wait(&s.wbar, 0, p.err, kErrTimeoutLoad);
      int it = 0;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, ++it) {
        const int st = it % kPStages, buf = it & 1;
        if (!mbar_wait(&s.z_full[st], (it / kPStages) & 1, p.err, kErrTimeoutLoad)) break;
        if (!mbar_wait(&s.acc_free[buf], ((it >> 1) & 1) ^ 1, p.err, kErrTimeoutEmpty)) break;
        tc_fence_after();
        const uint32_t wa = smem_u32(s.w), za = smem_u32(s.z[st]);
#pragma unroll
        for (int m = 0; m < 4; ++m)
#pragma unroll
          for (int kb = 0; kb < 2; ++kb)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_bf16(tmem0 + buf * 256 + m * kPTile, desc_kmajor_sw128(wa + kb * 65536 + m * 16384) + 2 * kk,
                       desc_kmajor_sw128(za + kb * (kPTile * 128)) + 2 * kk, idesc, (kb | kk) != 0);
        mma_commit(&s.acc_full[buf]);
        mma_commit(&s.z_empty[st]);
      }
    }
  } else if (warp < 4) {
    // statistics: thread t = pair t of the tile
    const int t = (warp - 2) * 32 + lane;
    int it = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++it) {
      const int st = it % kPStages, buf = it & 1;
      bool w1 = mbar_wait(&s.z_full[st], (it / kPStages) & 1, p.err, kErrTimeoutLoad);
      bool w2 = mbar_wait(&s.st_free[buf], ((it >> 1) & 1) ^ 1, p.err, kErrTimeoutEmpty);
      if (!__all_sync(0xFFFFFFFFu, w1 && w2)) break;
      const uint8_t* zt = s.z[st];
      // one pass over the pair's 128 channels on the paired fp32 pipe: sums of x - x0 and
      // of its square (shifted by the first channel, so the variance does not cancel)
      uint4 v[16];
#pragma unroll
      for (int kb = 0; kb < 2; ++kb)
#pragma unroll
        for (int q = 0; q < 8; ++q)
          v[kb * 8 + q] = *reinterpret_cast<const uint4*>(zt + kb * (kPTile * 128) + sw128_offset(t, q * 8));
      const float x0 = bf16_lo(v[0].x);
      const uint64_t shift = f32x2(-x0, -x0);
      uint64_t s1 = 0, s2 = 0;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint64_t d = add_f32x2(f32x2(bf16_lo(w[j]), bf16_hi(w[j])), shift);
          s1 = add_f32x2(s1, d);
          s2 = fma_f32x2(d, d, s2);
        }
      }
      float a1, b1, a2, b2;
      f32x2_split(s1, a1, b1);
      f32x2_split(s2, a2, b2);
      const float dm = (a1 + b1) * (1.0f / kC);
      const float mean = x0 + dm;
      const float var = fmaxf((a2 + b2) * (1.0f / kC) - dm * dm, 0.f);
      const int c0 = (tile % tiles_per_row) * kPTile;
      const int rr = tile / tiles_per_row;
      const int b = rr / p.R, r = rr - b * p.R;
      const int k = c0 + t;
      const float rstd = rsqrtf(var + 1e-5f);
      reinterpret_cast<float*>(&s.coef[buf][t >> 1])[t & 1] = rstd;
      reinterpret_cast<float*>(&s.coef[buf][t >> 1])[2 + (t & 1)] = -rstd * mean;
      if (k < p.N) {
        // natural pair (i, j) of the rows held: outgoing row tile (r, k), incoming column
        // tile (k, r) (the incoming direction always holds all N rows)
        const int64_t pi = p.outgoing ? r : k, pj = p.outgoing ? k : r;
        p.zstats[(static_cast<int64_t>(b) * p.R + pi) * p.N + pj] = make_float2(mean, rstd);
      }
      reinterpret_cast<float*>(&s.pm[buf][t >> 1])[t & 1] =
          (k < p.N && p.mask[b * p.N + p.row0 + r] && p.mask[b * p.N + k]) ? 1.0f : 0.0f;
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&s.st_full[buf]);
        mbar_arrive(&s.z_empty[st]);
      }
    }
  } else {
    // epilogue: warp 4..7 -> L, 8..11 -> R; lane = output channel
    const int part = (warp - 4) / 4;
    const int c = (warp & 3) * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int rp = part * 256 + c, rg = part * 256 + 128 + c;
    // W_l / W_r and their gates carry 1/2 (packed that way), so with yp' = yp / 2 and
    // yg' = yg / 2: yp sigmoid(yg) = yp' (1 + tanh(yg'))
    const uint64_t wsp = f32x2(s.wsum[rp], s.wsum[rp]), bsp = f32x2(s.bias[rp], s.bias[rp]);
    const uint64_t wsg = f32x2(s.wsum[rg], s.wsum[rg]), bsg = f32x2(s.bias[rg], s.bias[rg]);
    const CUtensorMap* map_out = part == 0 ? &map_l : &map_r;
    // Software-pipelined over 32-pair chunks: a chunk's TMEM load is in flight while the
    // previous chunk is staged and stored (the next tile's first chunk included).
    uint32_t vp[32], vg[32], packed[16];
    auto compute = [&](int buf, int ch) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        // pairs (j, j + 1) of this channel on the paired pipe: y = rstd acc - rstd mean wsum + b
        const float4 cf = s.coef[buf][(ch >> 1) + i];
        const float2 pm2 = s.pm[buf][(ch >> 1) + i];
        const uint64_t rs = f32x2(cf.x, cf.y), nm = f32x2(cf.z, cf.w);
        const uint64_t yp = fma_f32x2(rs, f32x2(__uint_as_float(vp[2 * i]), __uint_as_float(vp[2 * i + 1])),
                                      fma_f32x2(nm, wsp, bsp));
        const uint64_t yg = fma_f32x2(rs, f32x2(__uint_as_float(vg[2 * i]), __uint_as_float(vg[2 * i + 1])),
                                      fma_f32x2(nm, wsg, bsg));
        float g0, g1;
        f32x2_split(yg, g0, g1);
        const uint64_t o = mul_f32x2(fma_f32x2(yp, f32x2(tanh_fast(g0), tanh_fast(g1)), yp), f32x2(pm2.x, pm2.y));
        float o0, o1;
        f32x2_split(o, o0, o1);
        packed[i] = pack_bf16(o0, o1);
      }
    };
    // each warp stages and stores its own 32 channels; half h's previous store from this
    // warp (two stores ago) has finished reading it. Pairs c0 + ch .. + 31 of row r, batch
    // b; a half wholly past N is not stored (its group stays empty, so groups alternate halves)
    auto stage_store = [&](int tile, int ch) {
      const int c0 = (tile % tiles_per_row) * kPTile;
      const int rr = tile / tiles_per_row;
      const int b = rr / p.R, r = rr - b * p.R;
      const int h = ch >> 5;
      if (lane == 0) tma_store_wait_read1();
      __syncwarp();
      uint8_t* stage = s.out[part][h];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        *reinterpret_cast<uint4*>(stage + sw64_offset(c, 8 * q)) =
            make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        if (c0 + ch < p.N) tma_store_4d(map_out, stage + (warp & 3) * 32 * 64, c0 + ch, (warp & 3) * 32, r, b);
        tma_store_commit();
      }
    };
    // wait for tile `it`'s accumulators and statistics, then start its first chunk's load
    // (no barrier joins the epilogue warps, so each leaves on its own after a failed wait)
    auto begin = [&](int it) -> bool {
      const int buf = it & 1;
      const bool w1 = mbar_wait(&s.acc_full[buf], (it >> 1) & 1, p.err, kErrTimeoutMma);
      const bool w2 = mbar_wait(&s.st_full[buf], (it >> 1) & 1, p.err, kErrTimeoutLoad);
      if (!__all_sync(0xFFFFFFFFu, w1 && w2)) return false;
      tc_fence_after();
      const uint32_t tb = tmem0 + lane_off + buf * 256 + (2 * part) * kPTile;
      tmem_ld32(tb, vp);
      tmem_ld32(tb + kPTile, vg);
      return true;
    };
    int it = 0;
    bool ok = blockIdx.x < total && begin(0);
    for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, ++it) {
      const int buf = it & 1;
      const uint32_t tb = tmem0 + lane_off + buf * 256 + (2 * part) * kPTile;
      tmem_ld_wait();
      compute(buf, 0);
      tmem_ld32(tb + 32, vp);
      tmem_ld32(tb + kPTile + 32, vg);
      stage_store(tile, 0);
      tmem_ld_wait();
      compute(buf, 32);
      // the tile's accumulators and statistics have been read
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&s.acc_free[buf]);
        mbar_arrive(&s.st_free[buf]);
      }
      if (tile + static_cast<int>(gridDim.x) < total) ok = begin(it + 1);
      stage_store(tile, 32);
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

// ====================================================================== kernel 3
// Warp-specialised, persistent, 128-pair tiles; TMEM lane = pair, column = channel:
//   gate[p][c] = z[p] . W_g'[c]          A = the z tile (K-major, as TMA lands it)
//   out[p][c]  = u[:, p] . W_o'[c]       A = the channel-major u tile read as an MN-major
//                                        operand (no transposition in shared memory)
// with both LayerNorms folded into the epilogue through per-pair statistics:
//   delta[p][c] = (ru_p (out - mu_p wsum_o[c]) + b_o[c]) * sigmoid(rz_p (gate - mz_p wsum_g[c]) + b_g[c])
// A thread owns one pair and adds delta into that pair's row of the z tile in place
// (16-byte swizzled vectors); the per-pair coefficients stay in registers and the paired
// fp32 pipe computes two channels per instruction.
//   warp 0      TMA: z and u tiles into a 2-stage ring; it also stores each finished tile
//               from its slot (after the eight epilogue warps arrive) before reloading it
//   warp 1      MMA: gate and out products -> 256 TMEM columns, double-buffered
//   warps 2-3   per-pair coefficients (z statistics from step 1, u statistics from the
//               staged u tile) and the keep mask
//   warps 4-11  epilogue: lane = pair, warps 4-7 channels 0-63, warps 8-11 channels 64-127
constexpr int kOTile = 128;
constexpr int kOStages = 2;
constexpr int kOThreads = 384;

struct OutSmem {
  alignas(1024) uint8_t wg[kGateBytes];                // [c][k]: 2 K-blocks of [128 c x 128 B]
  alignas(1024) uint8_t wo[kOutBytes];
  alignas(1024) uint8_t z[kOStages][kOTile * kC * 2];  // [p][c]: 2 K-blocks of [128 p x 128 B]
  alignas(1024) uint8_t u[kOStages][kH * kOTile * 2];  // [c][p]: 2 p-blocks of [128 c x 128 B]
  float4 cg[kC / 2];  // channel pair (2i, 2i+1): wsum_gate x2, bias_gate / 2 x2
  float4 co[kC / 2];  // channel pair: wsum_out x2, bias_out / 2 x2
  float4 pc[2][kOTile];  // per pair: rz / 2, -rz mz / 2, ru / 2, -ru mu / 2
  float keep[2][kOTile];
  uint64_t wbar;
  uint64_t full[kOStages], out_ready[kOStages];  // tile landed; tile's output written over its z (8 warps)
  uint64_t acc_full[2], acc_free[2], st_full[2], st_free[2];
  uint32_t tmem_base;
};

static_assert(sizeof(OutSmem) + 1024 <= 232448, "output shared memory exceeds the per-CTA limit");

struct OutParams {
  const uint8_t* packed;
  const uint8_t* mask;
  const float2* zstats;  // [B, R, N] (mean, rstd) of z (input LayerNorm)
  int B, N;
  int R, row0;           // rows held and the first one's global index
  int masked_zero;
  int* err;
};

__global__ void __launch_bounds__(kOThreads, 1)
    trimul_out_kernel(const __grid_constant__ CUtensorMap map_z, const __grid_constant__ CUtensorMap map_u,
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
      mbar_init(&s.acc_full[i], 1);
      mbar_init(&s.acc_free[i], 8);
      mbar_init(&s.st_full[i], 2);
      mbar_init(&s.st_free[i], 8);
    }
    fence_mbar_init();
  }
  {
    const float* v = reinterpret_cast<const float*>(p.packed + kProjBytes + kGateBytes + kOutBytes);
    for (int i = threadIdx.x; i < kC / 2; i += kOThreads) {
      s.cg[i] = make_float4(v[1024 + 2 * i], v[1024 + 2 * i + 1], 0.5f * v[1152 + 2 * i], 0.5f * v[1152 + 2 * i + 1]);
      s.co[i] = make_float4(v[1408 + 2 * i], v[1408 + 2 * i + 1], 0.5f * v[1280 + 2 * i], 0.5f * v[1280 + 2 * i + 1]);
    }
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
      tma_prefetch_map(&map_u);
      tma_prefetch_map(&map_out);
      mbar_arrive_expect_tx(&s.wbar, kGateBytes + kOutBytes);
      bulk_load(s.wg, p.packed + kProjBytes, kGateBytes, &s.wbar);
      bulk_load(s.wo, p.packed + kProjBytes + kGateBytes, kOutBytes, &s.wbar);
      // the slot's previous tile: written over its z by the epilogue (which ran after the MMA
      // and the statistics had read the slot), stored from there; the slot is free once the
      // store has read it. This thread, not an epilogue warp, waits for that read.
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
        const int b = rr / p.R, r = rr - b * p.R;
        mbar_arrive_expect_tx(&s.full[st], 2 * kOTile * kC * 2);
        for (int kb = 0; kb < 2; ++kb) {
          tma_load_3d(s.z[st] + kb * (kOTile * 128), &map_z, &s.full[st], kb * 64, c0, rr);
          tma_load_3d(s.u[st] + kb * (kH * 128), &map_u, &s.full[st], c0 + kb * 64, r, b * kH);
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
      const uint32_t idesc_g = idesc_bf16_f32(kOTile, kC);
      const uint32_t idesc_o = idesc_bf16_f32_amn(kOTile, kC);
      bool ok = mbar_wait(&s.wbar, 0, p.err, kErrTimeoutLoad);
      int it = 0;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, ++it) {
        const int st = it % kOStages, buf = it & 1;
        if (!mbar_wait(&s.full[st], (it / kOStages) & 1, p.err, kErrTimeoutLoad)) break;
        if (!mbar_wait(&s.acc_free[buf], ((it >> 1) & 1) ^ 1, p.err, kErrTimeoutEmpty)) break;
        tc_fence_after();
        const uint32_t wg = smem_u32(s.wg), wo = smem_u32(s.wo), za = smem_u32(s.z[st]), ua = smem_u32(s.u[st]);
        const uint32_t dg = tmem0 + buf * 256, dout = tmem0 + buf * 256 + kC;
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_bf16(dg, desc_kmajor_sw128(za + kb * (kOTile * 128)) + 2 * kk, desc_kmajor_sw128(wg + kb * 16384) + 2 * kk,
                     idesc_g, (kb | kk) != 0);
#pragma unroll
        for (int ks = 0; ks < kH / 16; ++ks)
          mma_bf16(dout, desc_mnmajor_sw128(ua + ks * 2048, kH * 128, 1024),
                   desc_kmajor_sw128(wo + (ks / 4) * 16384) + 2 * (ks % 4), idesc_o, ks != 0);
        mma_commit(&s.acc_full[buf]);
      }
    }
  } else if (warp < 4) {
    // per-pair coefficients and keep mask: z statistics precomputed by the projection, u
    // statistics over the 128 channel rows of the staged u tile (one pass, sums about the
    // pair's channel-0 value); thread t owns the pair couple (2t, 2t + 1), one 4-byte load
    // per channel
    const int t = (warp - 2) * 32 + lane;
    const int pp0 = 2 * t, pb = pp0 / 64, pcol = pp0 % 64;
    int it = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++it) {
      const int st = it % kOStages, buf = it & 1;
      // the pairs' global inputs first (the z statistics from the projection and the masks):
      // they do not depend on the staged tile, so their latency overlaps the waits below
      const int c0 = (tile % tiles_per_row) * kOTile;
      const int rr = tile / tiles_per_row;
      const int b = rr / p.R, r = rr - b * p.R;
      float2 zs[2];
      bool kp[2];
      const bool row_keep = !p.masked_zero || p.mask[b * p.N + p.row0 + r];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int j = c0 + pp0 + k;
        zs[k] = j < p.N ? p.zstats[(static_cast<int64_t>(b) * p.R + r) * p.N + j] : make_float2(0.f, 0.f);
        kp[k] = j < p.N && row_keep && (!p.masked_zero || p.mask[b * p.N + j]);
      }
      const bool w1 = mbar_wait(&s.full[st], (it / kOStages) & 1, p.err, kErrTimeoutLoad);
      const bool w2 = mbar_wait(&s.st_free[buf], ((it >> 1) & 1) ^ 1, p.err, kErrTimeoutEmpty);
      if (!__all_sync(0xFFFFFFFFu, w1 && w2)) break;
      const uint8_t* ut = s.u[st] + pb * (kH * 128);
      const uint32_t w0 = *reinterpret_cast<const uint32_t*>(ut + sw128_offset(0, pcol));
      const float sh0 = bf16_lo(w0), sh1 = bf16_hi(w0);
      const uint64_t nsh = f32x2(-sh0, -sh1);
      uint64_t a1 = f32x2(0.f, 0.f), a2 = f32x2(0.f, 0.f);
#pragma unroll 16
      for (int c = 0; c < kH; ++c) {
        const uint32_t w = *reinterpret_cast<const uint32_t*>(ut + sw128_offset(c, pcol));
        const uint64_t d = add_f32x2(f32x2(bf16_lo(w), bf16_hi(w)), nsh);
        a1 = add_f32x2(a1, d);
        a2 = fma_f32x2(d, d, a2);
      }
      float s1[2], s2[2];
      f32x2_split(a1, s1[0], s1[1]);
      f32x2_split(a2, s2[0], s2[1]);
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int pp = pp0 + k;
        const float m1 = s1[k] * (1.0f / kH);
        const float mu = (k ? sh1 : sh0) + m1;
        const float ru = rsqrtf(fmaxf(s2[k] * (1.0f / kH) - m1 * m1, 0.f) + 1e-5f);
        s.pc[buf][pp] = make_float4(0.5f * zs[k].y, -0.5f * zs[k].y * zs[k].x, 0.5f * ru, -0.5f * ru * mu);
        s.keep[buf][pp] = kp[k] ? 1.f : 0.f;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.st_full[buf]);
    }
  } else {
    // epilogue: lane = pair pp of the tile; half = which 64 channels. Per channel pair:
    //   g/2 = (rz/2) gate + (-rz mz/2) wsum_g + b_g/2,   o/2 likewise with ru, mu, W_o's vectors,
    //   z' = z + o * sigmoid(g) = z + (o/2) tanh(g/2) + o/2
    const int half = (warp - 4) / 4;
    const int pp = (warp & 3) * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    int it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++it) {
      const int st = it % kOStages, buf = it & 1;
      if (ok) {
        const bool w1 = mbar_wait(&s.acc_full[buf], (it >> 1) & 1, p.err, kErrTimeoutMma);
        const bool w2 = mbar_wait(&s.st_full[buf], (it >> 1) & 1, p.err, kErrTimeoutLoad);
        ok = __all_sync(0xFFFFFFFFu, w1 && w2);
      }
      tc_fence_after();
      uint8_t* zrow = s.z[st] + half * (kOTile * 128);
      if (ok) {
        const float4 pc = s.pc[buf][pp];
        const bool keep = s.keep[buf][pp] != 0.f;
        const uint64_t ga = f32x2(pc.x, pc.x), gb = f32x2(pc.y, pc.y), oa = f32x2(pc.z, pc.z), ob = f32x2(pc.w, pc.w);
#pragma unroll 1
        for (int ch = 0; ch < 64; ch += 32) {
          const int cb = half * 64 + ch;
          uint32_t vg[32], vo[32];
          tmem_ld32(tmem0 + lane_off + buf * 256 + cb, vg);
          tmem_ld32(tmem0 + lane_off + buf * 256 + kC + cb, vo);
          tmem_ld_wait();
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4* zp = reinterpret_cast<uint4*>(zrow + sw128_offset(pp, ch + 8 * q));
            const uint4 zv = *zp;
            const uint32_t zw[4] = {zv.x, zv.y, zv.z, zv.w};
            uint32_t res[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int i = 8 * q + 2 * e;  // channel pair (cb + i, cb + i + 1)
              const float4 cg = s.cg[(cb + i) / 2], co = s.co[(cb + i) / 2];
              const uint64_t g = fma_f32x2(ga, f32x2(__uint_as_float(vg[i]), __uint_as_float(vg[i + 1])),
                                           fma_f32x2(gb, f32x2(cg.x, cg.y), f32x2(cg.z, cg.w)));
              const uint64_t o = fma_f32x2(oa, f32x2(__uint_as_float(vo[i]), __uint_as_float(vo[i + 1])),
                                           fma_f32x2(ob, f32x2(co.x, co.y), f32x2(co.z, co.w)));
              float g0, g1;
              f32x2_split(g, g0, g1);
              const uint64_t d = fma_f32x2(o, f32x2(tanh_fast(g0), tanh_fast(g1)), o);
              const uint64_t zz = add_f32x2(d, f32x2(bf16_lo(zw[e]), bf16_hi(zw[e])));
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

}  // namespace

size_t trimul_packed_bytes() { return kPackedBytes; }

size_t trimul_workspace_bytes(int B, int N) {
  const size_t np = (static_cast<size_t>(N) + 7) / 8 * 8;
  const size_t one = static_cast<size_t>(B) * kH * N * np * 2;
  const size_t aligned = (one + 255) / 256 * 256;
  const size_t stats = (static_cast<size_t>(B) * N * N * 8 + 255) / 256 * 256;
  return 3 * aligned + stats;  // L, R, U, z statistics
}

int trimul_prepare(const TriMulWeights& w, void* packed, cudaStream_t stream) {
  uint8_t* img = static_cast<uint8_t*>(packed);
  float* vec = reinterpret_cast<float*>(img + kProjBytes + kGateBytes + kOutBytes);
  const float* mats[4] = {w.to_left, w.to_left_gate, w.to_right, w.to_right_gate};
  int rc = 0;
  for (int i = 0; i < 4 && rc == 0; ++i)
    rc = launch_pack_weight(mats[i], kH, kC, w.ln_w, w.ln_b, img, i * kH, 512, vec + 0, vec + 512, stream, 0.5f);
  if (rc == 0)
    rc = launch_pack_weight(w.to_gate, kC, kC, w.ln_w, w.ln_b, img + kProjBytes, 0, kC, vec + 1024, vec + 1152,
                            stream);
  if (rc == 0)
    rc = launch_pack_weight(w.to_out, kC, kH, w.ln_out_w, w.ln_out_b, img + kProjBytes + kGateBytes, 0, kC,
                            vec + 1408, vec + 1280, stream);
  return rc;
}

namespace {

// z tensor map over the rows held ([B * R] rows of N pairs x 128 channels), box of `rows`
// pairs of one row (row tiles) or, for the incoming direction, one pair of `rows` rows
// (column tiles, R == N).
int z_map(CUtensorMap* m, const void* z, int B, int R, int N, int rows, bool column_tiles) {
  const uint64_t dims[3] = {kC, static_cast<uint64_t>(N), static_cast<uint64_t>(B) * R};
  const uint64_t strides[2] = {kC * 2, static_cast<uint64_t>(N) * kC * 2};
  const uint32_t box_row[3] = {64, static_cast<uint32_t>(rows), 1};
  const uint32_t box_col[3] = {64, 1, static_cast<uint32_t>(rows)};
  return make_map(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, z, dims, strides, column_tiles ? box_col : box_row,
                  CU_TENSOR_MAP_SWIZZLE_128B);
}

int launch_proj(const void* z, const uint8_t* mask, const void* packed, void* left, void* right, float2* zstats,
                int B, int R, int N, int row0, int64_t ls_b, int64_t ls_c, int64_t ls_r, int outgoing,
                const DeviceInfo& info, cudaStream_t stream) {
  const int np = (N + 7) / 8 * 8;
  CUtensorMap map_z, map_l, map_r;
  int st = z_map(&map_z, z, B, R, N, kPTile, !outgoing);
  if (st) return st;
  {
    // L / R as [pair k (N, clipped)][channel][row][batch] with the caller's strides
    const uint64_t dims[4] = {static_cast<uint64_t>(N), kH, static_cast<uint64_t>(R), static_cast<uint64_t>(B)};
    const uint64_t strides[3] = {static_cast<uint64_t>(ls_c) * 2, static_cast<uint64_t>(ls_r) * 2,
                                 static_cast<uint64_t>(ls_b) * 2};
    const uint32_t box[4] = {32, 32, 1, 1};  // one warp's 32 channels of a staging half
    st = make_map(&map_l, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, left, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B);
    if (st) return st;
    st = make_map(&map_r, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, right, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B);
    if (st) return st;
  }
  ProjParams pp{static_cast<const uint8_t*>(packed), mask, static_cast<__nv_bfloat16*>(left),
                static_cast<__nv_bfloat16*>(right), zstats, B, N, np, R, row0, ls_b, ls_c, ls_r, outgoing, info.err};
  const int ptiles = B * R * ((N + kPTile - 1) / kPTile);
  const int pgrid = ptiles < info.num_sms ? ptiles : info.num_sms;
  const size_t proj_smem = sizeof(ProjSmem) + 1024;
  cudaFuncSetAttribute(trimul_proj_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(proj_smem));
  trimul_proj_kernel<<<pgrid, kPThreads, proj_smem, stream>>>(map_z, map_l, map_r, pp);
  return cuda_status(static_cast<int>(cudaGetLastError()), "trimul_proj launch");
}

// U[c] (R x N) = L[c] (R x N(k)) R[c]^T for `channels` channels of each of B batch entries;
// element strides of L / R: channel `l_c` / `r_c`, row `l_r` / `r_r` (batch entries follow
// their channels); U is [B * channels][R][Np].
int launch_contract(const void* left, const void* right, void* u, int B, int channels, int R, int N, int64_t l_c,
                    int64_t l_r, int64_t r_c, int64_t r_r, const DeviceInfo& info, cudaStream_t stream) {
  const int np = (N + 7) / 8 * 8;
  CUtensorMap map_l, map_r;
  const int bn = N > 128 ? 256 : 128;
  const uint64_t ldims[3] = {static_cast<uint64_t>(N), static_cast<uint64_t>(R), static_cast<uint64_t>(B) * channels};
  const uint64_t lstrides[2] = {static_cast<uint64_t>(l_r) * 2, static_cast<uint64_t>(l_c) * 2};
  const uint64_t rdims[3] = {static_cast<uint64_t>(N), static_cast<uint64_t>(N), static_cast<uint64_t>(B) * channels};
  const uint64_t rstrides[2] = {static_cast<uint64_t>(r_r) * 2, static_cast<uint64_t>(r_c) * 2};
  const uint32_t box_a[3] = {64, 128, 1};
  const uint32_t box_b[3] = {64, static_cast<uint32_t>(bn), 1};
  int st = make_map(&map_l, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, left, ldims, lstrides, box_a, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  st = make_map(&map_r, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, right, rdims, rstrides, box_b, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  GemmParams gp;
  gp.M = R;
  gp.N = N;
  gp.K = N;
  gp.batch = B * channels;
  gp.D = u;
  gp.ldd = np;
  gp.batch_stride_d = static_cast<int64_t>(R) * np;
  gp.d_is_f32 = 0;
  gp.epilogue = kEpiStore;
  gp.bias = nullptr;
  gp.residual = nullptr;
  gp.row_mask = nullptr;
  gp.err = info.err;
  return cuda_status(launch_gemm_nt(map_l, map_r, gp, bn, info.num_sms, stream), "trimul contraction launch");
}

int launch_out(const void* z, const uint8_t* mask, const void* packed, const void* u, const float2* zstats, void* out,
               int B, int R, int N, int row0, int masked_zero, const DeviceInfo& info, cudaStream_t stream) {
  const int np = (N + 7) / 8 * 8;
  CUtensorMap map_zo, map_out, map_u;
  int st = z_map(&map_zo, z, B, R, N, kOTile, false);
  if (st) return st;
  st = z_map(&map_out, out, B, R, N, kOTile, false);
  if (st) return st;
  const uint64_t udims[3] = {static_cast<uint64_t>(N), static_cast<uint64_t>(R), static_cast<uint64_t>(B) * kH};
  const uint64_t ustrides[2] = {static_cast<uint64_t>(np) * 2, static_cast<uint64_t>(R) * np * 2};
  const uint32_t ubox[3] = {64, 1, kH};  // [128 channels][64 pairs], 128-byte swizzled rows
  st = make_map(&map_u, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, u, udims, ustrides, ubox, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  OutParams op{static_cast<const uint8_t*>(packed), mask, zstats, B, N, R, row0, masked_zero, info.err};
  const size_t out_smem = sizeof(OutSmem) + 1024;
  const int otiles = B * R * ((N + kOTile - 1) / kOTile);
  const int ogrid = otiles < info.num_sms ? otiles : info.num_sms;
  cudaFuncSetAttribute(trimul_out_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(out_smem));
  trimul_out_kernel<<<ogrid, kOThreads, out_smem, stream>>>(map_zo, map_u, map_out, op);
  return cuda_status(static_cast<int>(cudaGetLastError()), "trimul_out launch");
}

}  // namespace

int trimul_forward(const void* z, const uint8_t* mask, const void* packed, void* out, void* workspace, int B, int N,
                   int outgoing, int masked_zero, int stages, const DeviceInfo& info, cudaStream_t stream) {
  const int np = (N + 7) / 8 * 8;
  const size_t one = static_cast<size_t>(B) * kH * N * np * 2;
  const size_t aligned = (one + 255) / 256 * 256;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* left = ws;
  void* right = ws + aligned;
  void* u = ws + 2 * aligned;
  float2* zstats = reinterpret_cast<float2*>(ws + 3 * aligned);
  // channel-major L, R, U: [B * 128][N][Np]
  const int64_t s_c = static_cast<int64_t>(N) * np, s_b = kH * s_c;
  int st = 0;
  if (stages & 1) {
    st = launch_proj(z, mask, packed, left, right, zstats, B, N, N, 0, s_b, s_c, np, outgoing, info, stream);
    if (st) return st;
  }
  if (stages & 2) {
    st = launch_contract(left, right, u, B, kH, N, N, s_c, np, s_c, np, info, stream);
    if (st) return st;
  }
  if (stages & 4) st = launch_out(z, mask, packed, u, zstats, out, B, N, N, 0, masked_zero, info, stream);
  return st;
}

// ---- row-sharded entry points (B = 1): the rank holds rows [row0, row0 + R) of the pair.
// L, R (and the gathered right operand): [rows][128][Np] so that an all-gather over rows
// concatenates whole tensors; U: [128][R][Np]; statistics [R][N].
int trimul_shard_proj(const void* z, const uint8_t* mask, const void* packed, void* left, void* right, void* zstats,
                      int R, int N, int row0, const DeviceInfo& info, cudaStream_t stream) {
  const int64_t np = (N + 7) / 8 * 8;
  return launch_proj(z, mask, packed, left, right, static_cast<float2*>(zstats), 1, R, N, row0, R * kH * np, np,
                     kH * np, 1, info, stream);
}

int trimul_shard_contract(const void* left, const void* right_all, void* u, int R, int N, const DeviceInfo& info,
                          cudaStream_t stream) {
  const int64_t np = (N + 7) / 8 * 8;
  return launch_contract(left, right_all, u, 1, kH, R, N, np, kH * np, np, kH * np, info, stream);
}

// Channel-sharded contraction: L, R [C][N][Np] (C of the 128 channels, all N rows) ->
// U [C][N][Np].
int trimul_channel_contract(const void* left, const void* right, void* u, int C, int N, const DeviceInfo& info,
                            cudaStream_t stream) {
  const int64_t np = (N + 7) / 8 * 8;
  return launch_contract(left, right, u, 1, C, N, N, static_cast<int64_t>(N) * np, np, static_cast<int64_t>(N) * np, np,
                         info, stream);
}

int trimul_shard_out(const void* z, const uint8_t* mask, const void* packed, const void* u, const void* zstats,
                     void* ustats, void* out, int R, int N, int row0, int masked_zero, const DeviceInfo& info,
                     cudaStream_t stream) {
  (void)ustats;  // the u statistics are taken inside the output kernel; the argument is kept for the ABI
  return launch_out(z, mask, packed, u, static_cast<const float2*>(zstats), out, 1, R, N, row0, masked_zero, info, stream);
}

}  // namespace ffb
