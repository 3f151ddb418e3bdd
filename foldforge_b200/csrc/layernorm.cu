// Standalone LayerNorm over the channel axis (the engine `layernorm` op).
//
// The pair tensor's rows are c_z = 128 bf16 = 256 bytes: 16 lanes each load one 16-byte
// vector, so a warp covers two rows per load instruction and every load is a full
// 128-bit access; mean and variance are two-pass in fp32 from registers with half-warp
// shuffle reductions. Each warp keeps several rows in flight to cover HBM latency. The
// single track's bf16 rows (c_s = 384) are held in registers by one warp each; other widths
// and fp32 use a one-warp-per-row kernel that reads the row three times.
#include "common.cuh"
#include "kernels.h"

namespace ffb {
namespace {

constexpr int kRowsInFlight = 8;  // per half-warp

__device__ __forceinline__ float half_warp_sum(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

__global__ void __launch_bounds__(256) ln128_bf16_kernel(const uint4* __restrict__ x, uint4* __restrict__ y,
                                                          const float* __restrict__ gamma,
                                                          const float* __restrict__ beta, int64_t rows, float eps) {
  const int lane = threadIdx.x & 31;
  const int sub = lane >> 4;   // which row of the pair this half-warp owns
  const int part = lane & 15;  // 16-byte vector index inside the row
  float g[8], bt[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    g[i] = gamma ? gamma[part * 8 + i] : 1.0f;
    bt[i] = beta ? beta[part * 8 + i] : 0.0f;
  }
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  const int64_t warp_id = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
  const int64_t step = warps * 2 * kRowsInFlight;
  for (int64_t base = warp_id * 2 * kRowsInFlight; base < rows; base += step) {
    uint4 v[kRowsInFlight];
#pragma unroll
    for (int u = 0; u < kRowsInFlight; ++u) {
      const int64_t r = base + u * 2 + sub;
      v[u] = r < rows ? __ldcs(x + r * 16 + part) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kRowsInFlight; ++u) {
      const int64_t r = base + u * 2 + sub;
      const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
      float f[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        f[2 * i] = bf16_lo(w[i]);
        f[2 * i + 1] = bf16_hi(w[i]);
      }
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) s += f[i];
      const float mean = half_warp_sum(s) * (1.0f / 128.0f);
      float q = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float d = f[i] - mean;
        q += d * d;
      }
      const float rstd = rsqrtf(half_warp_sum(q) * (1.0f / 128.0f) + eps);
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        o[i] = pack_bf16((f[2 * i] - mean) * rstd * g[2 * i] + bt[2 * i],
                         (f[2 * i + 1] - mean) * rstd * g[2 * i + 1] + bt[2 * i + 1]);
      if (r < rows) __stcs(y + r * 16 + part, make_uint4(o[0], o[1], o[2], o[3]));
    }
  }
}

// bf16 rows of c = 384 (the single track): one warp per row, the row held in registers (each
// lane loads three 8-byte words: channels 4 lane + 128 k), one read and one write per element.
__global__ void __launch_bounds__(256) ln384_bf16_kernel(const uint2* __restrict__ x, uint2* __restrict__ y,
                                                          const float* __restrict__ gamma,
                                                          const float* __restrict__ beta, int64_t rows, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32; r < rows; r += warps) {
    uint2 v[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) v[k] = x[r * 96 + k * 32 + lane];
    float f[12];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      f[4 * k] = bf16_lo(v[k].x);
      f[4 * k + 1] = bf16_hi(v[k].x);
      f[4 * k + 2] = bf16_lo(v[k].y);
      f[4 * k + 3] = bf16_hi(v[k].y);
    }
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < 12; ++i) sum += f[i];
    const float mean = warp_sum(sum) / 384.0f;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < 12; ++i) {
      const float d = f[i] - mean;
      q += d * d;
    }
    const float rstd = rsqrtf(warp_sum(q) / 384.0f + eps);
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      float o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int c = k * 128 + 4 * lane + e;
        float t = (f[4 * k + e] - mean) * rstd;
        if (gamma) t *= gamma[c];
        if (beta) t += beta[c];
        o[e] = t;
      }
      y[r * 96 + k * 32 + lane] = make_uint2(pack_bf16(o[0], o[1]), pack_bf16(o[2], o[3]));
    }
  }
}

template <typename T>
__device__ __forceinline__ float load_f(const T* p);
template <>
__device__ __forceinline__ float load_f<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float load_f<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }

template <typename T>
__device__ __forceinline__ void store_f(T* p, float v);
template <>
__device__ __forceinline__ void store_f<float>(float* p, float v) { *p = v; }
template <>
__device__ __forceinline__ void store_f<__nv_bfloat16>(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

template <typename T>
__global__ void __launch_bounds__(256) ln_rowwarp_kernel(const T* __restrict__ x, T* __restrict__ y,
                                                          const float* __restrict__ gamma,
                                                          const float* __restrict__ beta, int64_t rows, int c,
                                                          float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32; r < rows; r += warps) {
    const T* xr = x + r * c;
    float s = 0.f;
    for (int i = lane; i < c; i += 32) s += load_f(xr + i);
    const float mean = warp_sum(s) / c;
    float q = 0.f;
    for (int i = lane; i < c; i += 32) {
      const float d = load_f(xr + i) - mean;
      q += d * d;
    }
    const float rstd = rsqrtf(warp_sum(q) / c + eps);
    for (int i = lane; i < c; i += 32) {
      float v = (load_f(xr + i) - mean) * rstd;
      if (gamma) v *= gamma[i];
      if (beta) v += beta[i];
      store_f(y + r * c + i, v);
    }
  }
}

}  // namespace

int launch_layernorm(const void* x, void* y, const float* gamma, const float* beta, int64_t rows, int c, float eps,
                     int is_f32, int num_sms, cudaStream_t stream) {
  if (rows <= 0) return 0;
  if (!is_f32 && c == 128) {
    const int64_t need = (rows + 2 * kRowsInFlight - 1) / (2 * kRowsInFlight);  // warps
    int64_t blocks = (need + 7) / 8;
    const int64_t cap = static_cast<int64_t>(num_sms) * 8;
    if (blocks > cap) blocks = cap;
    ln128_bf16_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(
        reinterpret_cast<const uint4*>(x), reinterpret_cast<uint4*>(y), gamma, beta, rows, eps);
  } else if (!is_f32 && c == 384 && (reinterpret_cast<uintptr_t>(x) & 7u) == 0 &&
             (reinterpret_cast<uintptr_t>(y) & 7u) == 0) {
    int64_t blocks = (rows + 7) / 8;
    const int64_t cap = static_cast<int64_t>(num_sms) * 16;
    if (blocks > cap) blocks = cap;
    ln384_bf16_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(
        reinterpret_cast<const uint2*>(x), reinterpret_cast<uint2*>(y), gamma, beta, rows, eps);
  } else {
    int64_t blocks = (rows + 7) / 8;
    const int64_t cap = static_cast<int64_t>(num_sms) * 16;
    if (blocks > cap) blocks = cap;
    if (is_f32)
      ln_rowwarp_kernel<float><<<static_cast<int>(blocks), 256, 0, stream>>>(
          reinterpret_cast<const float*>(x), reinterpret_cast<float*>(y), gamma, beta, rows, c, eps);
    else
      ln_rowwarp_kernel<__nv_bfloat16><<<static_cast<int>(blocks), 256, 0, stream>>>(
          reinterpret_cast<const __nv_bfloat16*>(x), reinterpret_cast<__nv_bfloat16*>(y), gamma, beta, rows, c,
          eps);
  }
  return static_cast<int>(cudaGetLastError());
}

}  // namespace ffb
