// Batched bf16 GEMM on tcgen05: D[b] = epilogue(A[b] * B[b]^T), A [M, K], B [N, K], both
// K-major (row-major with K innermost), fp32 accumulation in TMEM.
//
// Persistent, warp-specialised: warp 0 issues TMA loads into a STAGES-deep ring of
// shared-memory stages, warp 1 (one elected lane) issues tcgen05.mma and commits, warps
// 2..5 drain the accumulator (TMEM -> registers) and run the epilogue. Two TMEM
// accumulators of BN columns let the MMA of tile t+1 overlap the epilogue of tile t.
// The plain bf16 store (the contraction's epilogue) leaves through 64-column chunks staged
// 128-byte-swizzled in shared memory (two buffers, alternated) and written by TMA stores,
// so the tile's rows reach memory as whole lines; the other epilogues store per thread.
//
// Used for the triangle-multiplication contraction (one GEMM per hidden channel, batch =
// B * hidden) and for the single-track projections.
#include "abi_util.h"
#include "common.cuh"
#include "kernels.h"

namespace ffb {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;  // one 128-byte swizzle row of bf16
constexpr int kStages = 4;

template <int BN>
struct GemmSmem {
  alignas(1024) uint8_t a[kStages][kBM * kBK * 2];
  alignas(1024) uint8_t b[kStages][BN * kBK * 2];
  uint64_t full[kStages];
  uint64_t empty[kStages];
  alignas(1024) uint8_t out[2][kBM * 64 * 2];  // bf16 store staging: [128 rows][64 columns], SW128
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint32_t tmem_base;
};

static_assert(sizeof(GemmSmem<256>) + 1024 <= 232448, "GEMM shared memory exceeds the per-CTA limit");

__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int& b, int& tm, int& tn) {
  const int per_batch = tiles_m * tiles_n;
  b = tile / per_batch;
  const int r = tile - b * per_batch;
  tm = r / tiles_n;
  tn = r - tm * tiles_n;
}

// element offset of batch b's output
__device__ __forceinline__ int64_t batch_offset(const GemmParams& p, int b) {
  if (p.batch_inner > 0)
    return static_cast<int64_t>(b % p.batch_inner) * p.batch_stride_d + static_cast<int64_t>(b / p.batch_inner) * p.batch_stride_d2;
  return static_cast<int64_t>(b) * p.batch_stride_d;
}

template <int BN>
__device__ __forceinline__ void epilogue_chunk(const GemmParams& p, int b, int m, int n0, const uint32_t (&v)[32]) {
  if (m >= p.M) return;
  const int out_cols = (p.epilogue == kEpiSwiGLU) ? (p.N / 2) : p.N;
  if (p.epilogue == kEpiSwiGLU) {
    // the packed weight interleaves a and b in blocks of 16 rows, so accumulator columns
    // [n0, n0 + 32) hold a[h0 : h0 + 16] then b[h0 : h0 + 16], h0 = n0 / 2
    const int h0 = n0 / 2;
    float out[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float a = __uint_as_float(v[i]);
      const float bb = __uint_as_float(v[16 + i]);
      out[i] = a / (1.0f + __expf(-a)) * bb;
    }
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.D) + batch_offset(p, b) +
                         static_cast<int64_t>(m) * p.ldd + h0;
    if (h0 + 16 <= out_cols && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
      uint4 w0 = make_uint4(pack_bf16(out[0], out[1]), pack_bf16(out[2], out[3]), pack_bf16(out[4], out[5]),
                            pack_bf16(out[6], out[7]));
      uint4 w1 = make_uint4(pack_bf16(out[8], out[9]), pack_bf16(out[10], out[11]), pack_bf16(out[12], out[13]),
                            pack_bf16(out[14], out[15]));
      reinterpret_cast<uint4*>(dst)[0] = w0;
      reinterpret_cast<uint4*>(dst)[1] = w1;
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (h0 + i < out_cols) dst[i] = __float2bfloat16_rn(out[i]);
    }
    return;
  }
  const bool full = (n0 + 32 <= p.N);
  float acc[32];
  if (p.bias != nullptr && full && (reinterpret_cast<uintptr_t>(p.bias + n0) & 15u) == 0) {
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      const float4 bb = *reinterpret_cast<const float4*>(p.bias + n0 + i);
      acc[i] = __uint_as_float(v[i]) + bb.x;
      acc[i + 1] = __uint_as_float(v[i + 1]) + bb.y;
      acc[i + 2] = __uint_as_float(v[i + 2]) + bb.z;
      acc[i + 3] = __uint_as_float(v[i + 3]) + bb.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      float x = __uint_as_float(v[i]);
      if (p.bias != nullptr && n0 + i < p.N) x += p.bias[n0 + i];
      acc[i] = x;
    }
  }
  if (p.col_gate != nullptr) {
    const float* gr = p.col_gate + static_cast<int64_t>(m % p.gate_rows) * p.N + n0;
    if (full && (reinterpret_cast<uintptr_t>(gr) & 15u) == 0) {
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        const float4 gv = *reinterpret_cast<const float4*>(gr + i);
        acc[i] *= 1.0f / (1.0f + __expf(-gv.x));
        acc[i + 1] *= 1.0f / (1.0f + __expf(-gv.y));
        acc[i + 2] *= 1.0f / (1.0f + __expf(-gv.z));
        acc[i + 3] *= 1.0f / (1.0f + __expf(-gv.w));
      }
    } else {
      for (int i = 0; i < 32; ++i)
        if (n0 + i < p.N) acc[i] *= 1.0f / (1.0f + __expf(-gr[i]));
    }
  }
  float rowscale = 1.0f;
  if (p.row_mask != nullptr) rowscale = p.row_mask[static_cast<int64_t>(b) * p.M + m] ? 1.0f : 0.0f;
  if (p.row_scale != nullptr) {
    rowscale *= p.row_scale[static_cast<int64_t>(b) * p.M + m];
    if (p.epilogue != kEpiResidual) {
#pragma unroll
      for (int i = 0; i < 32; ++i) acc[i] *= rowscale;
    }
  }
  const int64_t off = batch_offset(p, b) + static_cast<int64_t>(m) * p.ldd + n0;
  if (p.epilogue == kEpiResidual) {
    // D = R + acc * rowscale, R and D share the layout and dtype. All of the chunk's residual
    // values are read before the first store (R may alias D), 16 bytes at a time when the
    // chunk is whole and aligned.
    if (p.d_is_f32) {
      const float* r = reinterpret_cast<const float*>(p.residual) + off;
      float* d = reinterpret_cast<float*>(p.D) + off;
      if (full && ((reinterpret_cast<uintptr_t>(r) | reinterpret_cast<uintptr_t>(d)) & 15u) == 0) {
        float4 rv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) rv[i] = reinterpret_cast<const float4*>(r)[i];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          reinterpret_cast<float4*>(d)[i] =
              make_float4(fmaf(acc[4 * i], rowscale, rv[i].x), fmaf(acc[4 * i + 1], rowscale, rv[i].y),
                          fmaf(acc[4 * i + 2], rowscale, rv[i].z), fmaf(acc[4 * i + 3], rowscale, rv[i].w));
      } else {
        float rv[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) rv[i] = (n0 + i < p.N) ? r[i] : 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (n0 + i < p.N) d[i] = fmaf(acc[i], rowscale, rv[i]);
      }
    } else {
      const __nv_bfloat16* r = reinterpret_cast<const __nv_bfloat16*>(p.residual) + off;
      __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(p.D) + off;
      if (full && ((reinterpret_cast<uintptr_t>(r) | reinterpret_cast<uintptr_t>(d)) & 15u) == 0) {
        uint4 rv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) rv[i] = reinterpret_cast<const uint4*>(r)[i];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t w[4] = {rv[i].x, rv[i].y, rv[i].z, rv[i].w};
          uint32_t o[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int e = 8 * i + 2 * k;
            o[k] = pack_bf16(fmaf(acc[e], rowscale, bf16_lo(w[k])), fmaf(acc[e + 1], rowscale, bf16_hi(w[k])));
          }
          reinterpret_cast<uint4*>(d)[i] = make_uint4(o[0], o[1], o[2], o[3]);
        }
      } else {
        float rv[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) rv[i] = (n0 + i < p.N) ? __bfloat162float(r[i]) : 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (n0 + i < p.N) d[i] = __float2bfloat16_rn(fmaf(acc[i], rowscale, rv[i]));
      }
    }
    return;
  }
  if (p.d_is_f32) {
    float* d = reinterpret_cast<float*>(p.D) + off;
    if (full && (reinterpret_cast<uintptr_t>(d) & 15u) == 0) {
#pragma unroll
      for (int i = 0; i < 32; i += 4) *reinterpret_cast<float4*>(d + i) = make_float4(acc[i], acc[i + 1], acc[i + 2], acc[i + 3]);
    } else {
      for (int i = 0; i < 32; ++i)
        if (n0 + i < p.N) d[i] = acc[i];
    }
  } else {
    __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(p.D) + off;
    if (full && (reinterpret_cast<uintptr_t>(d) & 15u) == 0) {
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
        uint4 w = make_uint4(pack_bf16(acc[i], acc[i + 1]), pack_bf16(acc[i + 2], acc[i + 3]),
                             pack_bf16(acc[i + 4], acc[i + 5]), pack_bf16(acc[i + 6], acc[i + 7]));
        *reinterpret_cast<uint4*>(d + i) = w;
      }
    } else {
      for (int i = 0; i < 32; ++i)
        if (n0 + i < p.N) d[i] = __float2bfloat16_rn(acc[i]);
    }
  }
}

template <int BN>
__global__ void __launch_bounds__(192, 1)
    gemm_nt_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                   const __grid_constant__ CUtensorMap map_d, GemmParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  GemmSmem<BN>& s = *reinterpret_cast<GemmSmem<BN>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int tiles_m = (p.M + kBM - 1) / kBM;
  const int tiles_n = (p.N + BN - 1) / BN;
  const int total = p.batch * tiles_m * tiles_n;
  const int kblocks = (p.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.acc_full[i], 1);
      mbar_init(&s.acc_empty[i], 4);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&s.tmem_base, 2 * BN);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&map_a);
    tma_prefetch_map(&map_b);
    if (p.tma_store) tma_prefetch_map(&map_d);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        int b, tm, tn;
        tile_coords(tile, tiles_m, tiles_n, b, tm, tn);
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int st = it % kStages;
          const uint32_t ph = (it / kStages) & 1;
          if (!mbar_wait(&s.empty[st], ph ^ 1, p.err, kErrTimeoutEmpty)) { ok = false; break; }
          mbar_arrive_expect_tx(&s.full[st], (kBM + BN) * kBK * 2);
          if (p.batch_inner > 0) {
            const int bi = b % p.batch_inner, bo = b / p.batch_inner;
            tma_load_4d(s.a[st], &map_a, &s.full[st], kb * kBK, tm * kBM, bi, bo);
            tma_load_4d(s.b[st], &map_b, &s.full[st], kb * kBK, tn * BN, bi, bo);
          } else {
            tma_load_3d(s.a[st], &map_a, &s.full[st], kb * kBK, tm * kBM, b);
            tma_load_3d(s.b[st], &map_b, &s.full[st], kb * kBK, tn * BN, b);
          }
        }
      }
      // drain: every issued stage must land before the CTA may exit
      for (int k = 0; k < kStages && k < it; ++k) {
        const int j = it - 1 - k;
        mbar_wait(&s.full[j % kStages], (j / kStages) & 1, p.err, kErrTimeoutLoad);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(kBM, BN);
      int it = 0, local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        if (!mbar_wait(&s.acc_empty[acc], ((local >> 1) & 1) ^ 1, p.err, kErrTimeoutEmpty)) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * BN;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int st = it % kStages;
          if (!mbar_wait(&s.full[st], (it / kStages) & 1, p.err, kErrTimeoutLoad)) { ok = false; break; }
          tc_fence_after();
          const uint64_t da = desc_kmajor_sw128(smem_u32(s.a[st]));
          const uint64_t db = desc_kmajor_sw128(smem_u32(s.b[st]));
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            mma_bf16(d, da + 2 * kk, db + 2 * kk, idesc, (kb | kk) != 0);
          mma_commit(&s.empty[st]);
        }
        mma_commit(&s.acc_full[acc]);
      }
    }
  } else {
    // epilogue warps 2..5: TMEM lane quarter = warp % 4
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const bool issuer = warp == 2 && lane == 0;
    int local = 0, chunk = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++local) {
      int b, tm, tn;
      tile_coords(tile, tiles_m, tiles_n, b, tm, tn);
      const int acc = local & 1;
      const bool ok = mbar_wait(&s.acc_full[acc], (local >> 1) & 1, p.err, kErrTimeoutMma);
      // uniform over the four warps: the staged store below synchronises them per chunk
      if (named_barrier_or(1, 128, !ok)) break;
      tc_fence_after();
      const uint32_t base = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
      const int m = tm * kBM + row;
      if (p.tma_store) {
        for (int c = 0; c < BN; c += 64, ++chunk) {
          // nothing of this chunk (or the later ones) lies inside the output: stop, so that
          // every staged chunk is a committed store and the two-buffer wait below pairs each
          // buffer with the store that last read it
          if (tn * BN + c >= p.N) break;
          uint8_t* stage = s.out[chunk & 1];
          // the store issued two chunks ago has finished reading this staging buffer
          if (issuer) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
          named_barrier(1, 128);
          uint32_t v[32], w[32];
          tmem_ld32(base + c, v);
          tmem_ld32(base + c + 32, w);
          tmem_ld_wait();
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            *reinterpret_cast<uint4*>(stage + sw128_offset(row, 8 * q)) =
                make_uint4(pack_bf16(__uint_as_float(v[8 * q]), __uint_as_float(v[8 * q + 1])),
                           pack_bf16(__uint_as_float(v[8 * q + 2]), __uint_as_float(v[8 * q + 3])),
                           pack_bf16(__uint_as_float(v[8 * q + 4]), __uint_as_float(v[8 * q + 5])),
                           pack_bf16(__uint_as_float(v[8 * q + 6]), __uint_as_float(v[8 * q + 7])));
            *reinterpret_cast<uint4*>(stage + sw128_offset(row, 32 + 8 * q)) =
                make_uint4(pack_bf16(__uint_as_float(w[8 * q]), __uint_as_float(w[8 * q + 1])),
                           pack_bf16(__uint_as_float(w[8 * q + 2]), __uint_as_float(w[8 * q + 3])),
                           pack_bf16(__uint_as_float(w[8 * q + 4]), __uint_as_float(w[8 * q + 5])),
                           pack_bf16(__uint_as_float(w[8 * q + 6]), __uint_as_float(w[8 * q + 7])));
          }
          fence_async_smem();
          named_barrier(1, 128);
          // rows past M and columns past N are clipped by the tensor map
          if (issuer) {
            tma_store_3d(&map_d, stage, tn * BN + c, tm * kBM, b);
            tma_store_commit();
          }
        }
      } else {
        for (int c = 0; c < BN; c += 32) {
          uint32_t v[32];
          tmem_ld32(base + c, v);
          tmem_ld_wait();
          if (tn * BN + c < p.N) epilogue_chunk<BN>(p, b, m, tn * BN + c, v);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.acc_empty[acc]);
    }
    if (issuer) tma_store_wait_all0();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 2 * BN);
  }
}

}  // namespace

size_t gemm_smem_bytes(int bn) {
  return (bn == 256 ? sizeof(GemmSmem<256>) : sizeof(GemmSmem<128>)) + 1024;
}

int launch_gemm_nt(const CUtensorMap& map_a, const CUtensorMap& map_b, const GemmParams& p_in, int bn, int num_sms,
                   cudaStream_t stream) {
  GemmParams p = p_in;
  const int tiles = p.batch * ((p.M + kBM - 1) / kBM) * ((p.N + bn - 1) / bn);
  if (tiles <= 0) return 0;
  // the plain bf16 store goes through a TMA store map when the output's strides allow it
  CUtensorMap map_d;
  memset(&map_d, 0, sizeof(map_d));
  p.tma_store = 0;
  if (p.epilogue == kEpiStore && !p.d_is_f32 && p.bias == nullptr && p.row_scale == nullptr && p.batch_inner == 0 &&
      (reinterpret_cast<uintptr_t>(p.D) & 15u) == 0 &&
      (p.ldd * 2) % 16 == 0 &&
      (p.batch_stride_d * 2) % 16 == 0) {
    const uint64_t dims[3] = {static_cast<uint64_t>(p.N), static_cast<uint64_t>(p.M), static_cast<uint64_t>(p.batch)};
    const uint64_t strides[2] = {static_cast<uint64_t>(p.ldd) * 2, static_cast<uint64_t>(p.batch_stride_d) * 2};
    const uint32_t box[3] = {64, kBM, 1};
    if (make_map(&map_d, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, p.D, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B) == 0)
      p.tma_store = 1;
  }
  const int grid = tiles < num_sms ? tiles : num_sms;
  const size_t smem = gemm_smem_bytes(bn);
  if (bn == 256) {
    cudaFuncSetAttribute(gemm_nt_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    gemm_nt_kernel<256><<<grid, 192, smem, stream>>>(map_a, map_b, map_d, p);
  } else {
    cudaFuncSetAttribute(gemm_nt_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    gemm_nt_kernel<128><<<grid, 192, smem, stream>>>(map_a, map_b, map_d, p);
  }
  return static_cast<int>(cudaGetLastError());
}

}  // namespace ffb
