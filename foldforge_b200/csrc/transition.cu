// Pair transition, fused: z' = z + W_sq (silu(W_a LN(z)) * W_b LN(z)), c_z = 128, n = 4
// (legacy/primitives.py:20-37, legacy/reference/transition.py:28-59; swiglu
// modules/dense/diffusion_transformer.py:36-44).
//
// One CTA owns 256 pair rows (two halves of 128, one TMEM lane block each) and walks the
// 512 hidden units in 8 chunks of 64:
//   MMA1  acc1[h] = z[h] x [W_a'; W_b'](chunk)^T    (M 128, N 128 = 64 a | 64 b, K 128)
//   SwiGLU on acc1 with the folded input LayerNorm -> H[h] (bf16, K-major, smem)
//   MMA2  acc2[h] += H[h] x W_sq(chunk)^T           (M 128, N 128, K 64)
// then z + acc2 (pair mask applied in "zero" mode) goes back through the z tile and a TMA
// store. The hidden activation never leaves the SM. Weight chunks stream through a
// 2-deep TMA ring; the two halves alternate so one half's SwiGLU overlaps the other's MMAs.
//
// Warps 0..7: epilogue (half = warp / 4); warp 8: TMA; warp 9: MMA issue.
#include "abi_util.h"
#include "common.cuh"
#include "kernels.h"

namespace ffb {
namespace {

constexpr int kC = 128;
constexpr int kHidden = 512;
constexpr int kChunk = 64;
constexpr int kChunks = kHidden / kChunk;
constexpr int kRows = 256;
constexpr int kThreads = 320;
constexpr size_t kW1Chunk = 128 * kC * 2;      // 32 KB: [64 a | 64 b] x 128
constexpr size_t kW2Chunk = kC * kChunk * 2;   // 16 KB: 128 out x 64
constexpr size_t kW1Bytes = kW1Chunk * kChunks;
constexpr size_t kW2Bytes = kW2Chunk * kChunks;
constexpr size_t kPackedBytes = kW1Bytes + kW2Bytes + 2 * 2 * kHidden * 4;

struct Smem {
  alignas(1024) uint8_t z[2][kC * 128 * 2];       // per half: 2 K-blocks of [128 x 128 B]
  alignas(1024) uint8_t w1[2][kW1Chunk];
  alignas(1024) uint8_t w2[2][kW2Chunk];
  alignas(1024) uint8_t hbuf[2][128 * kChunk * 2];  // per half: [128 x 64] bf16
  float wsum[2 * kHidden];
  float bias[2 * kHidden];
  uint64_t z_full, z_empty;
  uint64_t w_full[2], w_empty[2];
  uint64_t acc1_full[2], h_full[2], acc2_full[2], acc2_free[2];
  uint32_t tmem_base;
};

struct Params {
  const uint8_t* packed;
  const uint8_t* mask;
  int64_t rows;  // B * N * N
  int N;
  int masked_zero;
  int* err;
};

__device__ __forceinline__ float silu_(float a) {
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(0.5f * a));
  return 0.5f * a * (1.0f + t);
}

__global__ void __launch_bounds__(kThreads, 1)
    transition_kernel(const __grid_constant__ CUtensorMap map_z, const __grid_constant__ CUtensorMap map_out,
                      Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int tiles = static_cast<int>((p.rows + kRows - 1) / kRows);

  if (threadIdx.x == 0) {
    mbar_init(&s.z_full, 1);
    mbar_init(&s.z_empty, 2);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.w_full[i], 1);
      mbar_init(&s.w_empty[i], 1);
      mbar_init(&s.acc1_full[i], 1);
      mbar_init(&s.h_full[i], 4);
      mbar_init(&s.acc2_full[i], 1);
      mbar_init(&s.acc2_free[i], 4);
    }
    fence_mbar_init();
  }
  {
    const float* v = reinterpret_cast<const float*>(p.packed + kW1Bytes + kW2Bytes);
    for (int i = threadIdx.x; i < 2 * kHidden; i += kThreads) {
      s.wsum[i] = v[i];
      s.bias[i] = v[2 * kHidden + i];
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

  if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_map(&map_z);
      tma_prefetch_map(&map_out);
      int t_it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++t_it) {
        const int row0 = tile * kRows;
        if (!mbar_wait(&s.z_empty, (t_it & 1) ^ 1, p.err, kErrTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&s.z_full, 2 * kC * 128 * 2);
        for (int h = 0; h < 2; ++h)
          for (int kb = 0; kb < 2; ++kb) tma_load_2d(s.z[h] + kb * 16384, &map_z, &s.z_full, kb * 64, row0 + h * 128);
        for (int j = 0; j < kChunks; ++j) {
          const int w_it = t_it * kChunks + j;
          const int buf = w_it & 1;
          if (!mbar_wait(&s.w_empty[buf], ((w_it >> 1) & 1) ^ 1, p.err, kErrTimeoutEmpty)) { ok = false; break; }
          mbar_arrive_expect_tx(&s.w_full[buf], kW1Chunk + kW2Chunk);
          bulk_load(s.w1[buf], p.packed + j * kW1Chunk, kW1Chunk, &s.w_full[buf]);
          bulk_load(s.w2[buf], p.packed + kW1Bytes + j * kW2Chunk, kW2Chunk, &s.w_full[buf]);
        }
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc1 = idesc_bf16_f32(128, 128);
      const uint32_t idesc2 = idesc_bf16_f32(128, 128);
      int t_it = 0;
      bool ok = true;
      auto mma1 = [&](int h, int buf) {
        const uint32_t a0 = smem_u32(s.z[h]);
        const uint32_t b0 = smem_u32(s.w1[buf]);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_bf16(tmem0 + h * 128, desc_kmajor_sw128(a0 + kb * 16384) + 2 * kk,
                     desc_kmajor_sw128(b0 + kb * 16384) + 2 * kk, idesc1, (kb | kk) != 0);
        mma_commit(&s.acc1_full[h]);
      };
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++t_it) {
        if (!mbar_wait(&s.z_full, t_it & 1, p.err, kErrTimeoutLoad)) break;
        const int w0 = t_it * kChunks;
        if (!mbar_wait(&s.w_full[w0 & 1], (w0 >> 1) & 1, p.err, kErrTimeoutLoad)) break;
        tc_fence_after();
        mma1(0, w0 & 1);
        mma1(1, w0 & 1);
        for (int j = 0; j < kChunks && ok; ++j) {
          const int w_it = w0 + j;
          const int buf = w_it & 1;
          for (int h = 0; h < 2; ++h) {
            if (!mbar_wait(&s.h_full[h], j & 1, p.err, kErrTimeoutMma)) { ok = false; break; }
            if (j == 0 && !mbar_wait(&s.acc2_free[h], (t_it & 1) ^ 1, p.err, kErrTimeoutEmpty)) { ok = false; break; }
            tc_fence_after();
            const uint32_t a0 = smem_u32(s.hbuf[h]);
            const uint32_t b0 = smem_u32(s.w2[buf]);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_bf16(tmem0 + 256 + h * 128, desc_kmajor_sw128(a0) + 2 * kk, desc_kmajor_sw128(b0) + 2 * kk, idesc2,
                       (j | kk) != 0);
            if (j + 1 < kChunks) {
              const int nb = (w_it + 1) & 1;
              if (h == 0 && !mbar_wait(&s.w_full[nb], ((w_it + 1) >> 1) & 1, p.err, kErrTimeoutLoad)) {
                ok = false;
                break;
              }
              tc_fence_after();
              mma1(h, nb);
            }
          }
          if (!ok) break;
          mma_commit(&s.w_empty[buf]);
        }
        if (!ok) break;
        mma_commit(&s.acc2_full[0]);
        mma_commit(&s.acc2_full[1]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue warps
    const int h = warp / 4;
    const int t = (warp & 3) * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    uint8_t* zt = s.z[h];
    uint8_t* hb = s.hbuf[h];
    int t_it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++t_it) {
      const int64_t row = static_cast<int64_t>(tile) * kRows + h * 128 + t;
      bool w = mbar_wait(&s.z_full, t_it & 1, p.err, kErrTimeoutLoad);
      ok = __all_sync(0xFFFFFFFFu, w) && ok;
      float mean = 0.f, rstd = 0.f;
      if (ok) {
        float sum = 0.f;
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const uint4 v = *reinterpret_cast<const uint4*>(zt + kb * 16384 + sw128_offset(t, q * 8));
            const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) sum += bf16_lo(u[e]) + bf16_hi(u[e]);
          }
        mean = sum * (1.0f / kC);
        float q2 = 0.f;
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const uint4 v = *reinterpret_cast<const uint4*>(zt + kb * 16384 + sw128_offset(t, q * 8));
            const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float a = bf16_lo(u[e]) - mean, b = bf16_hi(u[e]) - mean;
              q2 += a * a + b * b;
            }
          }
        rstd = rsqrtf(q2 * (1.0f / kC) + 1e-5f);
      }
      for (int j = 0; j < kChunks; ++j) {
        bool w1 = ok && mbar_wait(&s.acc1_full[h], j & 1, p.err, kErrTimeoutMma);
        ok = __all_sync(0xFFFFFFFFu, w1);
        tc_fence_after();
        if (ok) {
          const float* ws = s.wsum + j * 128;
          const float* bs = s.bias + j * 128;
#pragma unroll 1
          for (int half32 = 0; half32 < 2; ++half32) {
            uint32_t va[32], vb[32];
            tmem_ld32(tmem0 + lane_off + h * 128 + half32 * 32, va);
            tmem_ld32(tmem0 + lane_off + h * 128 + 64 + half32 * 32, vb);
            tmem_ld_wait();
            uint32_t packed[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              float hv[2];
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const int c = half32 * 32 + 2 * i + e;
                const float a = rstd * (__uint_as_float(va[2 * i + e]) - mean * ws[c]) + bs[c];
                const float b = rstd * (__uint_as_float(vb[2 * i + e]) - mean * ws[64 + c]) + bs[64 + c];
                hv[e] = silu_(a) * b;
              }
              packed[i] = pack_bf16(hv[0], hv[1]);
            }
#pragma unroll
            for (int q = 0; q < 4; ++q)
              *reinterpret_cast<uint4*>(hb + sw128_offset(t, half32 * 32 + q * 8)) =
                  make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
          }
        }
        fence_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.h_full[h]);
      }
      bool w2 = ok && mbar_wait(&s.acc2_full[h], t_it & 1, p.err, kErrTimeoutMma);
      ok = __all_sync(0xFFFFFFFFu, w2);
      tc_fence_after();
      if (ok) {
        bool keep = true;
        if (p.masked_zero && row < p.rows) {
          const int64_t j = row % p.N;
          const int64_t bi = row / p.N;  // b * N + i
          const int64_t b = bi / p.N;
          keep = p.mask[bi] && p.mask[b * p.N + j];
        }
#pragma unroll 1
        for (int cc = 0; cc < kC; cc += 32) {
          uint32_t vo[32];
          tmem_ld32(tmem0 + lane_off + 256 + h * 128 + cc, vo);
          tmem_ld_wait();
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int ch = cc + q * 8;
            uint8_t* addr = zt + (ch / 64) * 16384 + sw128_offset(t, ch % 64);
            const uint4 zv = *reinterpret_cast<const uint4*>(addr);
            const uint32_t u[4] = {zv.x, zv.y, zv.z, zv.w};
            uint32_t o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float d0 = keep ? __uint_as_float(vo[q * 8 + 2 * e]) : 0.f;
              const float d1 = keep ? __uint_as_float(vo[q * 8 + 2 * e + 1]) : 0.f;
              o[e] = pack_bf16(bf16_lo(u[e]) + d0, bf16_hi(u[e]) + d1);
            }
            *reinterpret_cast<uint4*>(addr) = make_uint4(o[0], o[1], o[2], o[3]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.acc2_free[h]);
      fence_async_smem();
      ok = !named_barrier_or(1 + h, 128, !ok);  // half-uniform from here on
      if (t == 0) {
        if (ok) {
          const int r0 = static_cast<int>(static_cast<int64_t>(tile) * kRows + h * 128);
          tma_store_2d(&map_out, zt, 0, r0);
          tma_store_2d(&map_out, zt + 16384, 64, r0);
          tma_store_commit();
          tma_store_wait_read0();
        }
        mbar_arrive(&s.z_empty);
      }
      if (!ok) break;
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

size_t transition_packed_bytes() { return kPackedBytes; }

int transition_prepare(const TransitionWeights& w, void* packed, cudaStream_t stream) {
  uint8_t* img = static_cast<uint8_t*>(packed);
  float* vec = reinterpret_cast<float*>(img + kW1Bytes + kW2Bytes);
  int rc = 0;
  for (int j = 0; j < kChunks && rc == 0; ++j) {
    rc = launch_pack_weight(w.expand_a + static_cast<int64_t>(j) * kChunk * kC, kChunk, kC, w.ln_w, w.ln_b,
                            img + j * kW1Chunk, 0, 128, vec + j * 128, vec + 2 * kHidden + j * 128, stream);
    if (rc == 0)
      rc = launch_pack_weight(w.expand_b + static_cast<int64_t>(j) * kChunk * kC, kChunk, kC, w.ln_w, w.ln_b,
                              img + j * kW1Chunk, 64, 128, vec + j * 128, vec + 2 * kHidden + j * 128, stream);
  }
  if (rc == 0)
    rc = launch_pack_weight(w.squeeze, kC, kHidden, nullptr, nullptr, img + kW1Bytes, 0, kC, nullptr, nullptr, stream);
  return rc;
}

int transition_forward(const void* z, const uint8_t* mask, const void* packed, void* out, int B, int N,
                       int masked_zero, const DeviceInfo& info, cudaStream_t stream) {
  const int64_t rows = static_cast<int64_t>(B) * N * N;
  CUtensorMap map_z, map_out;
  const uint64_t dims[2] = {kC, static_cast<uint64_t>(rows)};
  const uint64_t strides[1] = {kC * 2};
  const uint32_t box[2] = {64, 128};
  int st = make_map(&map_z, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, z, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  st = make_map(&map_out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, out, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  Params pp{static_cast<const uint8_t*>(packed), mask, rows, N, masked_zero, info.err};
  const int tiles = static_cast<int>((rows + kRows - 1) / kRows);
  const int grid = tiles < info.num_sms ? tiles : info.num_sms;
  const size_t smem = sizeof(Smem) + 1024;
  cudaFuncSetAttribute(transition_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  transition_kernel<<<grid, kThreads, smem, stream>>>(map_z, map_out, pp);
  return cuda_status(static_cast<int>(cudaGetLastError()), "transition launch");
}

}  // namespace ffb
