// Pair transition, fused: z' = z + W_sq (silu(W_a LN(z)) * W_b LN(z)), c_z = 128, n = 4
// (legacy/primitives.py:20-37, legacy/reference/transition.py:28-59; swiglu
// modules/dense/diffusion_transformer.py:36-44).
//
// One CTA owns 128 pair rows at a time (one TMEM lane block) and walks the 512 hidden
// units in 8 chunks of 64:
//   MMA1  A1[j % 2] = Z x [W_a'; W_b'](j)^T       (M 128, N 128 = 64 a | 64 b, K 128)
//   SwiGLU on A1 (+ bias W beta) -> H[j % 2] (bf16)
//   MMA2  ACC2 += H[j % 2] x W_sq(j)^T             (M 128, N 128, K 64)
// Both products take their A operand from TMEM (Z: the tile's rows normalised by the
// statistics warps, (z - mean) * rstd in bf16; H: written by the SwiGLU warps), so the
// first product already is W_a' LN(z) up to the bias W beta (gamma is folded into W' and
// 1/2 into the a rows, so the SwiGLU is  h = a/2 + b_a/2,  silu(a) b = (h + h tanh h) b).
// Shared memory only feeds the weight operands. The first product runs two chunks ahead of the
// second. z tiles (double-buffered) and weight chunks arrive by TMA / bulk copy, the
// chunks' first- and second-product parts through separate 3-stage rings, each stage
// released by the product that reads it (so loads run up to three chunks ahead); the residual (pair mask applied in "zero" mode) is written over the staged z tile
// and leaves through a TMA store. The next tile's statistics are taken before this tile's
// residual, so its first products overlap the residual.
//
// TMEM columns: Z 0..63 (bf16 pairs) | A1[0] 64..191 | A1[1] 192..319 | H[0] 320..351 |
// H[1] 352..383 | ACC2 384..511.
// Warps 0..15: Z staging, SwiGLU and residual, four warps per TMEM lane quarter (warp / 4 =
// which 16 of a chunk's hidden units, which 32 of the channels of Z and of the output; the
// row's LayerNorm sums, taken about its channel 0, are combined over the four through shared
// memory); warp 16: TMA; warp 17: first products; warp 18: second products (two issuing
// threads, so neither product's operand waits hold up the other's issue).
#include "../../include/foldforge_b200.h"
#include "abi_util.h"
#include "common.cuh"
#include "kernels.h"

namespace ffb {
namespace {

constexpr int kC = 128;
constexpr int kHidden = 512;
constexpr int kChunk = 64;
constexpr int kChunks = kHidden / kChunk;
constexpr int kRows = 128;
constexpr int kThreads = 608;  // 16 SwiGLU / residual warps, TMA warp 16, MMA warps 17 (first) and 18 (second)
constexpr int kWStages = 3;
constexpr size_t kW1Chunk = 128 * kC * 2;      // 32 KB: [64 a | 64 b] x 128, two SW128 K-blocks
constexpr size_t kW2Chunk = kC * kChunk * 2;   // 16 KB: 128 out x 64 hidden, SW128
constexpr size_t kW1Bytes = kW1Chunk * kChunks;
constexpr size_t kW2Bytes = kW2Chunk * kChunks;
constexpr size_t kPackedBytes = kW1Bytes + kW2Bytes + 2 * 2 * kHidden * 4;
constexpr uint32_t kColZ = 0, kColA1 = 64, kColH = 320, kColAcc2 = 384;

struct Smem {
  alignas(1024) uint8_t z[2][kRows * kC * 2];   // per tile parity: 2 K-blocks of [128 x 128 B]
  alignas(1024) uint8_t w1[kWStages][kW1Chunk];
  alignas(1024) uint8_t w2[kWStages][kW2Chunk];
  float bias[2 * kHidden];
  uint64_t z_full[2], z_empty[2];
  uint64_t w1_full[kWStages], w1_empty[kWStages];  // first-product weight chunks
  uint64_t w2_full[kWStages], w2_empty[kWStages];  // second-product weight chunks
  float2 zx[2][4][kRows];   // LayerNorm partial sums of a row's four channel quarters, by tile parity
  uint64_t zx_bar[2][4];    // a lane quarter's four partial sums written, by tile parity
  uint64_t zt_full, zt_free;
  uint64_t a1_full[2], h_full[2];
  uint64_t a1_free[2], h_free[2];  // A1[i] read out by the SwiGLU warps; H[i] read by its second product
  uint64_t acc2_full, acc2_free;
  uint32_t tmem_base;
};

static_assert(sizeof(Smem) + 1024 <= 232448, "transition shared memory exceeds the per-CTA limit");

struct Params {
  const uint8_t* packed;
  const uint8_t* mask;
  int64_t rows;  // B * R * N pair rows
  int N;
  int R, row0;   // problem rows held (N unless row-sharded) and the first one's global index
  int masked_zero;
  int* err;
};

__global__ void __launch_bounds__(kThreads, 1)
    transition_kernel(const __grid_constant__ CUtensorMap map_z, const __grid_constant__ CUtensorMap map_out,
                      Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int tiles = static_cast<int>((p.rows + kRows - 1) / kRows);
  const int my_tiles = static_cast<int>(blockIdx.x) < tiles ? (tiles - 1 - static_cast<int>(blockIdx.x)) / gridDim.x + 1 : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.z_full[i], 1);
      mbar_init(&s.z_empty[i], 1);
      mbar_init(&s.a1_full[i], 1);
      mbar_init(&s.h_full[i], 16);
      mbar_init(&s.a1_free[i], 16);
      mbar_init(&s.h_free[i], 1);
    }
    for (int i = 0; i < kWStages; ++i) {
      mbar_init(&s.w1_full[i], 1);
      mbar_init(&s.w1_empty[i], 1);
      mbar_init(&s.w2_full[i], 1);
      mbar_init(&s.w2_empty[i], 1);
    }
    mbar_init(&s.zt_full, 16);
    for (int i = 0; i < 8; ++i) mbar_init(&s.zx_bar[i / 4][i % 4], 4);
    mbar_init(&s.zt_free, 1);
    mbar_init(&s.acc2_full, 1);
    mbar_init(&s.acc2_free, 16);
    fence_mbar_init();
  }
  {
    const float* v = reinterpret_cast<const float*>(p.packed + kW1Bytes + kW2Bytes);
    for (int i = threadIdx.x; i < 2 * kHidden; i += kThreads) s.bias[i] = v[2 * kHidden + i];
  }
  if (warp == 0) {
    tmem_alloc(&s.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem0 = s.tmem_base;

  if (warp == 16) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_map(&map_z);
      tma_prefetch_map(&map_out);
      int zl = 0, n1 = 0, n2 = 0;  // z tiles, first- and second-product weight chunks issued
      bool ok = true;
      auto load_z = [&](int ti) -> bool {  // tile ti of this CTA into buffer ti % 2
        const int zb = ti & 1;
        if (!mbar_wait(&s.z_empty[zb], ((ti >> 1) & 1) ^ 1, p.err, kErrTimeoutEmpty)) return false;
        const int row0 = (static_cast<int>(blockIdx.x) + ti * static_cast<int>(gridDim.x)) * kRows;
        mbar_arrive_expect_tx(&s.z_full[zb], kRows * kC * 2);
        for (int kb = 0; kb < 2; ++kb) tma_load_2d(s.z[zb] + kb * 16384, &map_z, &s.z_full[zb], kb * 64, row0);
        ++zl;
        return true;
      };
      // global chunk wc = tile * kChunks + j; each ring stage is released by the product that
      // reads it, so the loads run up to kWStages chunks ahead of their product
      auto load_w1 = [&](int wc) -> bool {
        const int st = wc % kWStages;
        if (!mbar_wait(&s.w1_empty[st], ((wc / kWStages) & 1) ^ 1, p.err, kErrTimeoutEmpty)) return false;
        mbar_arrive_expect_tx(&s.w1_full[st], kW1Chunk);
        bulk_load(s.w1[st], p.packed + (wc % kChunks) * kW1Chunk, kW1Chunk, &s.w1_full[st]);
        ++n1;
        return true;
      };
      auto load_w2 = [&](int wc) -> bool {
        const int st = wc % kWStages;
        if (!mbar_wait(&s.w2_empty[st], ((wc / kWStages) & 1) ^ 1, p.err, kErrTimeoutEmpty)) return false;
        mbar_arrive_expect_tx(&s.w2_full[st], kW2Chunk);
        bulk_load(s.w2[st], p.packed + kW1Bytes + (wc % kChunks) * kW2Chunk, kW2Chunk, &s.w2_full[st]);
        ++n2;
        return true;
      };
      // the order the MMA thread consumes them: first products run two chunks ahead
      const int total = my_tiles * kChunks;
      if (my_tiles > 0) ok = load_z(0);
      for (int wc = 0; wc < 2 && wc < total && ok; ++wc) ok = load_w1(wc);
      for (int wc = 0; wc < total && ok; ++wc) {
        if (!load_w2(wc)) break;
        if (wc + 2 < total && !load_w1(wc + 2)) break;
        // the next tile's z follows the third chunk of this one
        const int ti = wc / kChunks;
        if (wc % kChunks == 2 && ti + 1 < my_tiles && !load_z(ti + 1)) break;
      }
      // every issued copy lands before the CTA may exit
      for (int k = 0; k < 2 && k < zl; ++k) {
        const int i = zl - 1 - k;
        mbar_wait(&s.z_full[i & 1], (i >> 1) & 1, p.err, kErrTimeoutLoad);
      }
      for (int k = 0; k < kWStages && k < n1; ++k) {
        const int i = n1 - 1 - k;
        mbar_wait(&s.w1_full[i % kWStages], (i / kWStages) & 1, p.err, kErrTimeoutLoad);
      }
      for (int k = 0; k < kWStages && k < n2; ++k) {
        const int i = n2 - 1 - k;
        mbar_wait(&s.w2_full[i % kWStages], (i / kWStages) & 1, p.err, kErrTimeoutLoad);
      }
    }
  } else if (warp == 17) {
    // ------------------------------------------------------------ first products
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(128, 128);
      bool ok = true;
      for (int ti = 0; ti < my_tiles && ok; ++ti) {
        if (!mbar_wait(&s.zt_full, ti & 1, p.err, kErrTimeoutLoad)) break;
        for (int j = 0; j < kChunks; ++j) {
          // chunk j into A1[j % 2] (use n of that buffer, once its use n - 1 is read out);
          // A = Z from TMEM
          const int wc = ti * kChunks + j;
          const int st = wc % kWStages;
          const int n = ti * (kChunks / 2) + j / 2;
          if (n > 0 && !mbar_wait(&s.a1_free[j & 1], (n - 1) & 1, p.err, kErrTimeoutEmpty)) { ok = false; break; }
          if (!mbar_wait(&s.w1_full[st], (wc / kWStages) & 1, p.err, kErrTimeoutLoad)) { ok = false; break; }
          tc_fence_after();
          const uint32_t b0 = smem_u32(s.w1[st]);
          const uint32_t d = tmem0 + kColA1 + (j & 1) * 128;
#pragma unroll
          for (int kb = 0; kb < 2; ++kb)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_bf16_tmem_a(d, tmem0 + kColZ + (kb * 4 + kk) * 8, desc_kmajor_sw128(b0 + kb * 16384) + 2 * kk, idesc,
                              (kb | kk) != 0);
          mma_commit(&s.a1_full[j & 1]);
          mma_commit(&s.w1_empty[st]);
          if (j == kChunks - 1) mma_commit(&s.zt_free);  // the tile's last first product is issued
        }
      }
    }
  } else if (warp == 18) {
    // ------------------------------------------------------------ second products
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(128, 128);
      bool ok = true;
      for (int ti = 0; ti < my_tiles && ok; ++ti) {
        for (int j = 0; j < kChunks; ++j) {
          const int wc = ti * kChunks + j;
          const int st = wc % kWStages;
          const int u = ti * (kChunks / 2) + j / 2;  // use count of H buffer j % 2
          if (!mbar_wait(&s.h_full[j & 1], u & 1, p.err, kErrTimeoutMma)) { ok = false; break; }
          if (j == 0 && !mbar_wait(&s.acc2_free, (ti & 1) ^ 1, p.err, kErrTimeoutEmpty)) { ok = false; break; }
          if (!mbar_wait(&s.w2_full[st], (wc / kWStages) & 1, p.err, kErrTimeoutLoad)) { ok = false; break; }
          tc_fence_after();
          const uint32_t b0 = smem_u32(s.w2[st]);
#pragma unroll
          for (int kk = 0; kk < kChunk / 16; ++kk)
            mma_bf16_tmem_a(tmem0 + kColAcc2, tmem0 + kColH + (j & 1) * 32 + kk * 8, desc_kmajor_sw128(b0) + 2 * kk,
                            idesc, (j | kk) != 0);
          mma_commit(&s.w2_empty[st]);
          mma_commit(&s.h_free[j & 1]);
        }
        if (!ok) break;
        mma_commit(&s.acc2_full);
      }
    }
  } else if (warp < 16) {
    // ------------------------------------------------------------ SwiGLU / residual warps
    // warp w: lane quarter w % 4 (TMEM lanes = the tile's rows); part w / 4 takes 16 of a
    // chunk's 64 hidden units and 32 of the 128 channels of Z and of the output
    const int part = warp / 4;
    const int t = (warp & 3) * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tl = tmem0 + lane_off;
    const int kb = part / 2, cb = (part % 2) * 32;  // this part's channels: z-tile K-block kb, columns cb..cb+31
    bool ok = true;
    // row t of tile ti, LayerNorm-normalised (no affine: gamma and beta are in the weights),
    // into Z; the row's sums, taken about its channel 0, are combined over the four parts
    // through shared memory
    auto stage_z = [&](int ti) {
      const int zb = ti & 1;
      bool w = mbar_wait(&s.z_full[zb], (ti >> 1) & 1, p.err, kErrTimeoutLoad);
      if (ti > 0) w = w && mbar_wait(&s.zt_free, (ti - 1) & 1, p.err, kErrTimeoutMma);
      const bool good = __all_sync(0xFFFFFFFFu, w);
      const uint8_t* zt = s.z[zb] + kb * 16384;
      uint32_t zw[16];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 v = *reinterpret_cast<const uint4*>(zt + sw128_offset(t, cb + q * 8));
        zw[4 * q] = v.x;
        zw[4 * q + 1] = v.y;
        zw[4 * q + 2] = v.z;
        zw[4 * q + 3] = v.w;
      }
      const float shift = bf16_lo(*reinterpret_cast<const uint32_t*>(s.z[zb] + sw128_offset(t, 0)));
      const uint64_t sh = f32x2(-shift, -shift);
      uint64_t a1 = f32x2(0.f, 0.f), a2 = f32x2(0.f, 0.f);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint64_t d = add_f32x2(f32x2(bf16_lo(zw[i]), bf16_hi(zw[i])), sh);
        a1 = add_f32x2(a1, d);
        a2 = fma_f32x2(d, d, a2);
      }
      float s1a, s1b, s2a, s2b;
      f32x2_split(a1, s1a, s1b);
      f32x2_split(a2, s2a, s2b);
      s.zx[zb][part][t] = make_float2(s1a + s1b, s2a + s2b);
      // the quarter's four warps (bounded wait: a warp that left on an error cannot hold the others)
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.zx_bar[zb][warp & 3]);
      const bool wx =
          __all_sync(0xFFFFFFFFu, mbar_wait(&s.zx_bar[zb][warp & 3], (ti >> 1) & 1, p.err, kErrTimeoutEmpty));
      float t1 = 0.f, t2 = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 v = s.zx[zb][k][t];
        t1 += v.x;
        t2 += v.y;
      }
      const float m1 = t1 * (1.0f / kC);
      const float var = fmaxf(t2 * (1.0f / kC) - m1 * m1, 0.f);
      const float rstd = rsqrtf(var + 1e-5f);
      const float nm = -(shift + m1) * rstd;
#pragma unroll
      for (int i = 0; i < 16; ++i) zw[i] = pack_bf16(fmaf(bf16_lo(zw[i]), rstd, nm), fmaf(bf16_hi(zw[i]), rstd, nm));
      if (!good || !wx) {
        ok = false;
        return;
      }
      tmem_st16(tl + kColZ + part * 16, zw);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.zt_full);
    };
    if (my_tiles > 0) stage_z(0);
    for (int ti = 0; ti < my_tiles; ++ti) {
      const int zb = ti & 1;
      const int64_t row = (static_cast<int64_t>(blockIdx.x) + static_cast<int64_t>(ti) * gridDim.x) * kRows + t;
      for (int j = 0; j < kChunks && ok; ++j) {
        const int u = ti * (kChunks / 2) + j / 2;
        if (!__all_sync(0xFFFFFFFFu, mbar_wait(&s.a1_full[j & 1], u & 1, p.err, kErrTimeoutMma))) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t va[16], vb[16];
        tmem_ld16(tl + kColA1 + (j & 1) * 128 + part * 16, va);
        tmem_ld16(tl + kColA1 + (j & 1) * 128 + 64 + part * 16, vb);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.a1_free[j & 1]);  // the chunk after next may overwrite A1[j % 2]
        const float4* bs4 = reinterpret_cast<const float4*>(s.bias + j * 128 + part * 16);
        uint32_t hw[8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 ba = bs4[q], bb = bs4[16 + q];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int c = 4 * q + 2 * e;
            // h = a / 2 (the a rows carry the 1/2), b; silu(a) b = (h + h tanh h) b
            const uint64_t hh = add_f32x2(f32x2(__uint_as_float(va[c]), __uint_as_float(va[c + 1])),
                                          e == 0 ? f32x2(ba.x, ba.y) : f32x2(ba.z, ba.w));
            const uint64_t b = add_f32x2(f32x2(__uint_as_float(vb[c]), __uint_as_float(vb[c + 1])),
                                         e == 0 ? f32x2(bb.x, bb.y) : f32x2(bb.z, bb.w));
            float h0, h1;
            f32x2_split(hh, h0, h1);
            const uint64_t sa = fma_f32x2(hh, f32x2(tanh_fast(h0), tanh_fast(h1)), hh);
            float o0, o1;
            f32x2_split(mul_f32x2(sa, b), o0, o1);
            hw[c / 2] = pack_bf16(o0, o1);
          }
        }
        // H[j % 2] was read by the second product of the chunk before last
        if (u > 0 && !__all_sync(0xFFFFFFFFu, mbar_wait(&s.h_free[j & 1], (u - 1) & 1, p.err, kErrTimeoutMma))) {
          ok = false;
          break;
        }
        tc_fence_after();
        tmem_st8(tl + kColH + (j & 1) * 32 + part * 8, hw);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.h_full[j & 1]);
      }
      // the next tile's statistics and Z, so its first products overlap this residual
      if (ok && ti + 1 < my_tiles) stage_z(ti + 1);
      // residual: z (staged tile) + ACC2 written over the tile, then one TMA store
      if (ok) ok = __all_sync(0xFFFFFFFFu, mbar_wait(&s.acc2_full, ti & 1, p.err, kErrTimeoutMma));
      if (ok) {
        tc_fence_after();
        bool keep = true;
        if (p.masked_zero && row < p.rows) {
          const int64_t jj = row % p.N;
          const int64_t bi = row / p.N;  // b * R + i
          const int64_t b = bi / p.R, i = bi - b * p.R;
          keep = p.mask[b * p.N + p.row0 + i] && p.mask[b * p.N + jj];
        }
        uint8_t* zt = s.z[zb] + kb * 16384;
        uint32_t vo[32];
        tmem_ld32(tl + kColAcc2 + part * 32, vo);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.acc2_free);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint8_t* addr = zt + sw128_offset(t, cb + q * 8);
          const uint4 zv = *reinterpret_cast<const uint4*>(addr);
          const uint32_t zw[4] = {zv.x, zv.y, zv.z, zv.w};
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float d0 = keep ? __uint_as_float(vo[q * 8 + 2 * e]) : 0.f;
            const float d1 = keep ? __uint_as_float(vo[q * 8 + 2 * e + 1]) : 0.f;
            o[e] = pack_bf16(bf16_lo(zw[e]) + d0, bf16_hi(zw[e]) + d1);
          }
          *reinterpret_cast<uint4*>(addr) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
      fence_async_smem();
      ok = !named_barrier_or(1, 512, !ok);  // uniform over the sixteen warps from here on
      if (threadIdx.x == 0) {
        if (ok) {
          const int r0 = static_cast<int>(row - t);
          tma_store_2d(&map_out, s.z[zb], 0, r0);
          tma_store_2d(&map_out, s.z[zb] + 16384, 64, r0);
          tma_store_commit();
          tma_store_wait_read0();
        }
        mbar_arrive(&s.z_empty[zb]);
      }
      if (!ok) break;
    }
    if (threadIdx.x == 0) tma_store_wait_all0();
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

size_t transition_packed_bytes() { return kPackedBytes; }

int transition_prepare(const TransitionWeights& w, void* packed, cudaStream_t stream) {
  uint8_t* img = static_cast<uint8_t*>(packed);
  float* vec = reinterpret_cast<float*>(img + kW1Bytes + kW2Bytes);
  int rc = 0;
  for (int j = 0; j < kChunks && rc == 0; ++j) {
    // first-product rows: 1/2 W_a rows [64 j, 64 j + 64) then W_b rows, gamma folded; the
    // bias entries (W beta) j * 128 + [0, 128) follow the same row order
    rc = launch_pack_weight(w.expand_a + static_cast<int64_t>(j) * kChunk * kC, kChunk, kC, w.ln_w, w.ln_b,
                            img + j * kW1Chunk, 0, 128, vec + j * 128, vec + 2 * kHidden + j * 128, stream, 0.5f);
    if (rc == 0)
      rc = launch_pack_weight(w.expand_b + static_cast<int64_t>(j) * kChunk * kC, kChunk, kC, w.ln_w, w.ln_b,
                              img + j * kW1Chunk, 64, 128, vec + j * 128, vec + 2 * kHidden + j * 128, stream);
  }
  // W_sq [128 x 512]: chunk j = 64-column block j of the K-major SW128 image (16 KB each)
  if (rc == 0)
    rc = launch_pack_weight(w.squeeze, kC, kHidden, nullptr, nullptr, img + kW1Bytes, 0, kC, nullptr, nullptr, stream);
  return rc;
}

namespace {

int launch_transition(const void* z, const uint8_t* mask, const void* packed, void* out, int B, int R, int N, int row0,
                      int masked_zero, const DeviceInfo& info, cudaStream_t stream) {
  const int64_t rows = static_cast<int64_t>(B) * R * N;
  if (rows >= (static_cast<int64_t>(1) << 31))
    return fail(FFB_ERR_UNSUPPORTED, "transition: %lld pair rows exceed the 2^31 TMA row range",
                static_cast<long long>(rows));
  CUtensorMap map_z, map_out;
  const uint64_t dims[2] = {kC, static_cast<uint64_t>(rows)};
  const uint64_t strides[1] = {kC * 2};
  const uint32_t box[2] = {64, kRows};
  int st = make_map(&map_z, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, z, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  st = make_map(&map_out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, out, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  Params pp{static_cast<const uint8_t*>(packed), mask, rows, N, R, row0, masked_zero, info.err};
  const int tiles = static_cast<int>((rows + kRows - 1) / kRows);
  const int grid = tiles < info.num_sms ? tiles : info.num_sms;
  const size_t smem = sizeof(Smem) + 1024;
  cudaFuncSetAttribute(transition_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  transition_kernel<<<grid, kThreads, smem, stream>>>(map_z, map_out, pp);
  return cuda_status(static_cast<int>(cudaGetLastError()), "transition launch");
}

}  // namespace

int transition_forward(const void* z, const uint8_t* mask, const void* packed, void* out, int B, int N,
                       int masked_zero, const DeviceInfo& info, cudaStream_t stream) {
  return launch_transition(z, mask, packed, out, B, N, N, 0, masked_zero, info, stream);
}

// row-sharded (B = 1): the rank holds pair rows [row0, row0 + R)
int transition_shard_forward(const void* z, const uint8_t* mask, const void* packed, void* out, int R, int N, int row0,
                             int masked_zero, const DeviceInfo& info, cudaStream_t stream) {
  return launch_transition(z, mask, packed, out, 1, R, N, row0, masked_zero, info, stream);
}

}  // namespace ffb
