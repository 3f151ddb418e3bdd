// Row-shard exchanges over NVLink peer memory: the pair transpose (the all-to-all between the
// row-wise and the column-wise ops) and the all-gather over rows, written by one kernel
// straight into the peers' buffers in their final layout, plus a bounded wait for the peers'
// writes. No counterpart in the reference (FoldForge has no multi-GPU Pairformer).
//
// Buffers are plain cudaMalloc allocations shared through CUDA IPC handles (no multicast
// object is created or bound); each rank maps its peers' buffers with
// cudaIpcOpenMemHandle and passes the peer base addresses to the kernels as a device array.
//
// Signalling: every exchange kernel ends with its last CTA (an arrival counter in the
// rank's `sync` words) fencing at system scope and storing a new epoch, with release
// semantics, into slot [rank] of every peer's flag array (its own included). The epoch is
// counted on the device (sync[1]), so a CUDA graph replaying the exchange signals new
// epochs. ffb_shard_wait_p2p then waits, with acquire loads and a spin bounded by a
// caller-given wall-clock limit (2 s by default), until every slot of this rank's flags has
// reached the epoch: the peers' writes into this rank's buffers are then visible. A wait
// that runs out records kErrTimeoutPeer in the device error word and returns; it never
// traps.
//
// The kernels assume one rank per GPU (they wait on other ranks' kernels, which need not
// run concurrently on a shared GPU): the host uses this path only then.
#include "../../include/foldforge_b200.h"
#include "abi_util.h"
#include "common.cuh"

namespace ffb {
namespace {

constexpr int kMaxRanks = 8;
constexpr int kXThreads = 256;
constexpr int64_t kDefaultPeerWaitNs = 2000000000ll;  // 2 s

// The last CTA of the grid publishes a new epoch to every peer's flag slot [rank].
__device__ __forceinline__ void signal_peers(const uint64_t* flag_ptrs, uint32_t* sync, int rank, int P) {
  asm volatile("fence.acq_rel.sys;" ::: "memory");  // this thread's peer stores before the arrival
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t done;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(done) : "l"(sync) : "memory");
    if (done + 1 == gridDim.x) {
      sync[0] = 0;  // arrival counter ready for the next launch
      const uint32_t e = sync[1] + 1;
      sync[1] = e;
      asm volatile("fence.acq_rel.sys;" ::: "memory");
      for (int q = 0; q < P; ++q) {
        uint32_t* slot = reinterpret_cast<uint32_t*>(flag_ptrs[q]) + rank;
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(slot), "r"(e) : "memory");
      }
    }
  }
}

// x: this rank's pair rows [R][N][128] bf16 (global rows row0 + i). Pair (i, c), c = q R + a,
// goes to rank q's receive buffer at [a][row0 + i]: the rows of z^T that rank q holds.
// One warp per (source column c, chunk of kTRows rows): column c of this rank's rows goes to
// rank q = c / R, row a = c % R of its buffer, at columns row0 + i, so the chunk's pairs land
// as ONE contiguous run there (kTRows x 256 bytes over NVLink) while the source pairs are read
// with a stride of N pairs (each a coalesced 256-byte piece). Lanes 0-15 move one pair's 16
// words, lanes 16-31 the next pair's; the index arithmetic is 32-bit and once per chunk.
// Items are (a, chunk, destination) with the destination fastest; N = P R, so each
// (column, chunk) is one item.
constexpr int kTRows = 64;

__global__ void __launch_bounds__(kXThreads) pair_transpose_scatter_kernel(const uint4* __restrict__ x,
                                                                           const uint64_t* __restrict__ dst,
                                                                           const uint64_t* __restrict__ flag_ptrs,
                                                                           uint32_t* sync, int R, int N, int row0,
                                                                           int rank, int P) {
  __shared__ uint64_t sdst[kMaxRanks];
  if (threadIdx.x < P) sdst[threadIdx.x] = dst[threadIdx.x];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int part = lane & 15, half = lane >> 4;
  const int chunks = (R + kTRows - 1) / kTRows;
  const int items = N * chunks;
  const int warps = static_cast<int>(gridDim.x) * (kXThreads / 32);
  for (int item = static_cast<int>(blockIdx.x) * (kXThreads / 32) + static_cast<int>(threadIdx.x >> 5); item < items;
       item += warps) {
    // destination rank fastest (staggered by rank): the warps in flight write to every peer
    // at once, so no rank's incoming links take all the ranks' traffic at one time
    const int qq = item % P, rest = item / P;
    const int a = rest / chunks, i0 = (rest - a * chunks) * kTRows;
    const int q = qq + rank + 1 < P ? qq + rank + 1 : qq + rank + 1 - P;
    const int c = q * R + a;
    const int rows = R - i0 < kTRows ? R - i0 : kTRows;
    const uint4* src = x + (static_cast<int64_t>(i0) * N + c) * 16 + part;
    uint4* d = reinterpret_cast<uint4*>(sdst[q]) + (static_cast<int64_t>(a) * N + row0 + i0) * 16 + part;
    const int64_t sstep = static_cast<int64_t>(N) * 16;
    constexpr int kUnroll = 4;  // pairs per half-warp in flight
    for (int i = half; i < rows; i += 2 * kUnroll) {
      uint4 v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u)
        if (i + 2 * u < rows) v[u] = src[(i + 2 * u) * sstep];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u)
        if (i + 2 * u < rows) d[(i + 2 * u) * 16] = v[u];
    }
  }
  signal_peers(flag_ptrs, sync, rank, P);
}

// src: this rank's chunk of `bytes` (a multiple of 16); copied to offset rank * bytes of every
// rank's gather buffer (dst[q]), so the buffers end up as the rank-ordered concatenation.
__global__ void __launch_bounds__(kXThreads) row_gather_kernel(const uint4* __restrict__ src,
                                                               const uint64_t* __restrict__ dst,
                                                               const uint64_t* __restrict__ flag_ptrs, uint32_t* sync,
                                                               int64_t words, int rank, int P) {
  __shared__ uint64_t sdst[kMaxRanks];
  if (threadIdx.x < P) sdst[threadIdx.x] = dst[threadIdx.x];
  __syncthreads();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kXThreads;
  for (int64_t w = static_cast<int64_t>(blockIdx.x) * kXThreads + threadIdx.x; w < words; w += stride) {
    const uint4 v = src[w];
    for (int q = 0; q < P; ++q) reinterpret_cast<uint4*>(sdst[q])[static_cast<int64_t>(rank) * words + w] = v;
  }
  signal_peers(flag_ptrs, sync, rank, P);
}

// Row scatters of the channel-sharded TriMul contraction (rows of Np bf16, `row_words`
// 16-byte words each; cpp = 128 / P channels per rank):
//   mode 0 (L / R to the channel owners): src [R][128][Np] (this rank's rows i); row (i, c)
//          goes to rank q = c / cpp at [c % cpp][row0 + i] of its [cpp][N][Np] buffer;
//   mode 1 (U back to the row owners): src [cpp][N][Np] (this rank's channels c'); row
//          (c', g) goes to rank q = g / R at [rank cpp + c'][g % R] of its [128][R][Np] buffer.
__global__ void __launch_bounds__(kXThreads) row_scatter_kernel(const uint4* __restrict__ src,
                                                                const uint64_t* __restrict__ dst,
                                                                const uint64_t* __restrict__ flag_ptrs, uint32_t* sync,
                                                                int mode, int R, int N, int cpp, int row_words,
                                                                int rank, int P) {
  __shared__ uint64_t sdst[kMaxRanks];
  if (threadIdx.x < P) sdst[threadIdx.x] = dst[threadIdx.x];
  __syncthreads();
  // one warp per row (its destination worked out once), lanes striding over its words
  const int lane = threadIdx.x & 31;
  const int rows = mode == 0 ? R * 128 : cpp * N;
  const int warps = static_cast<int>(gridDim.x) * (kXThreads / 32);
  for (int r = static_cast<int>(blockIdx.x) * (kXThreads / 32) + static_cast<int>(threadIdx.x >> 5); r < rows;
       r += warps) {
    int q;
    int64_t drow;
    if (mode == 0) {
      const int i = r >> 7, c = r & 127;
      q = c / cpp;
      drow = static_cast<int64_t>(c - q * cpp) * N + rank * R + i;
    } else {
      const int cl = r / N, g = r - cl * N;
      q = g / R;
      drow = static_cast<int64_t>(rank * cpp + cl) * R + (g - q * R);
    }
    const uint4* s = src + static_cast<int64_t>(r) * row_words;
    uint4* d = reinterpret_cast<uint4*>(sdst[q]) + drow * row_words;
    constexpr int kUnroll = 4;
    for (int k = lane; k < row_words; k += 32 * kUnroll) {
      uint4 v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u)
        if (k + 32 * u < row_words) v[u] = s[k + 32 * u];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u)
        if (k + 32 * u < row_words) d[k + 32 * u] = v[u];
    }
  }
  signal_peers(flag_ptrs, sync, rank, P);
}

// One thread per rank q: wait until flags[q] has reached this rank's current epoch, for at
// most `limit_ns` nanoseconds of the GPU's global timer; then record kErrTimeoutPeer and
// return (the stream continues; the host reads the error word).
__global__ void shard_wait_kernel(const uint32_t* flags, const uint32_t* sync, int P, int64_t limit_ns, int* err) {
  const int q = threadIdx.x;
  if (q >= P) return;
  const uint32_t e = sync[1];
  uint64_t start;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(start));
  while (true) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + q) : "memory");
    if (static_cast<int32_t>(v - e) >= 0) break;
    uint64_t now;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
    if (static_cast<int64_t>(now - start) > limit_ns || error_raised(err)) {
      set_error(err, kErrTimeoutPeer);
      break;
    }
    __nanosleep(200);
  }
}

int exchange_grid(const DeviceInfo& info) { return info.num_sms * 4; }

}  // namespace
}  // namespace ffb

using namespace ffb;

extern "C" {

int ffb_p2p_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return fail(FFB_ERR_ARG, "p2p_alloc: null pointer or zero size");
  void* p = nullptr;
  int st = cuda_status(static_cast<int>(cudaMalloc(&p, bytes)), "p2p_alloc: cudaMalloc");
  if (st) return st;
  st = cuda_status(static_cast<int>(cudaMemset(p, 0, bytes)), "p2p_alloc: cudaMemset");
  if (st) {
    cudaFree(p);
    return st;
  }
  cudaIpcMemHandle_t h;
  st = cuda_status(static_cast<int>(cudaIpcGetMemHandle(&h, p)), "p2p_alloc: cudaIpcGetMemHandle");
  if (st) {
    cudaFree(p);
    return st;
  }
  memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return FFB_OK;
}

int ffb_p2p_handle_bytes(void) { return static_cast<int>(sizeof(cudaIpcMemHandle_t)); }

int ffb_p2p_open(const void* handle, void** ptr) {
  if (!ptr || !handle) return fail(FFB_ERR_ARG, "p2p_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cuda_status(static_cast<int>(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess)),
                     "p2p_open: cudaIpcOpenMemHandle");
}

int ffb_p2p_close(void* ptr) {
  if (!ptr) return FFB_OK;
  return cuda_status(static_cast<int>(cudaIpcCloseMemHandle(ptr)), "p2p_close: cudaIpcCloseMemHandle");
}

int ffb_p2p_free(void* ptr) {
  if (!ptr) return FFB_OK;
  return cuda_status(static_cast<int>(cudaFree(ptr)), "p2p_free: cudaFree");
}

int ffb_shard_transpose_p2p(const void* x, const void* dst_ptrs, const void* flag_ptrs, void* sync, int R, int N,
                            int row0, int rank, int P, void* stream) {
  if (!x || !dst_ptrs || !flag_ptrs || !sync) return fail(FFB_ERR_ARG, "shard_transpose_p2p: null pointer");
  if (P < 1 || P > kMaxRanks || rank < 0 || rank >= P || R <= 0 || N != R * P || row0 != rank * R)
    return fail(FFB_ERR_ARG, "shard_transpose_p2p: R=%d N=%d row0=%d rank=%d P=%d", R, N, row0, rank, P);
  if ((reinterpret_cast<uintptr_t>(x) & 15u) != 0) return fail(FFB_ERR_ARG, "shard_transpose_p2p: misaligned x");
  DeviceInfo info;
  int st = device_info(&info);
  if (st != FFB_OK) return st;
  pair_transpose_scatter_kernel<<<exchange_grid(info), kXThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(x), static_cast<const uint64_t*>(dst_ptrs), static_cast<const uint64_t*>(flag_ptrs),
      static_cast<uint32_t*>(sync), R, N, row0, rank, P);
  return cuda_status(static_cast<int>(cudaGetLastError()), "shard_transpose_p2p launch");
}

int ffb_shard_gather_p2p(const void* src, size_t bytes, const void* dst_ptrs, const void* flag_ptrs, void* sync,
                         int rank, int P, void* stream) {
  if (!src || !dst_ptrs || !flag_ptrs || !sync) return fail(FFB_ERR_ARG, "shard_gather_p2p: null pointer");
  if (P < 1 || P > kMaxRanks || rank < 0 || rank >= P || bytes == 0 || bytes % 16 != 0)
    return fail(FFB_ERR_ARG, "shard_gather_p2p: bytes=%zu rank=%d P=%d", bytes, rank, P);
  if ((reinterpret_cast<uintptr_t>(src) & 15u) != 0) return fail(FFB_ERR_ARG, "shard_gather_p2p: misaligned src");
  DeviceInfo info;
  int st = device_info(&info);
  if (st != FFB_OK) return st;
  row_gather_kernel<<<exchange_grid(info), kXThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), static_cast<const uint64_t*>(dst_ptrs), static_cast<const uint64_t*>(flag_ptrs),
      static_cast<uint32_t*>(sync), static_cast<int64_t>(bytes / 16), rank, P);
  return cuda_status(static_cast<int>(cudaGetLastError()), "shard_gather_p2p launch");
}

int ffb_shard_rows_p2p(const void* src, int mode, int R, int N, const void* dst_ptrs, const void* flag_ptrs,
                       void* sync, int rank, int P, void* stream) {
  if (!src || !dst_ptrs || !flag_ptrs || !sync) return fail(FFB_ERR_ARG, "shard_rows_p2p: null pointer");
  if (P < 1 || P > kMaxRanks || 128 % P != 0 || rank < 0 || rank >= P || R <= 0 || N != R * P || (mode != 0 && mode != 1))
    return fail(FFB_ERR_ARG, "shard_rows_p2p: mode=%d R=%d N=%d rank=%d P=%d", mode, R, N, rank, P);
  if ((reinterpret_cast<uintptr_t>(src) & 15u) != 0) return fail(FFB_ERR_ARG, "shard_rows_p2p: misaligned src");
  DeviceInfo info;
  int st = device_info(&info);
  if (st != FFB_OK) return st;
  const int np = (N + 7) / 8 * 8;
  row_scatter_kernel<<<exchange_grid(info), kXThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), static_cast<const uint64_t*>(dst_ptrs), static_cast<const uint64_t*>(flag_ptrs),
      static_cast<uint32_t*>(sync), mode, R, N, 128 / P, np / 8, rank, P);
  return cuda_status(static_cast<int>(cudaGetLastError()), "shard_rows_p2p launch");
}

int ffb_shard_wait_p2p(const void* flags, const void* sync, int P, int64_t limit_us, void* stream) {
  if (!flags || !sync) return fail(FFB_ERR_ARG, "shard_wait_p2p: null pointer");
  if (P < 1 || P > kMaxRanks) return fail(FFB_ERR_ARG, "shard_wait_p2p: P=%d", P);
  if (limit_us > 3600ll * 1000000ll) return fail(FFB_ERR_ARG, "shard_wait_p2p: limit_us=%lld", static_cast<long long>(limit_us));
  DeviceInfo info;
  int st = device_info(&info);
  if (st != FFB_OK) return st;
  const int64_t limit_ns = limit_us > 0 ? limit_us * 1000 : kDefaultPeerWaitNs;
  shard_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint32_t*>(flags), static_cast<const uint32_t*>(sync), P, limit_ns, info.err);
  return cuda_status(static_cast<int>(cudaGetLastError()), "shard_wait_p2p launch");
}

}  // extern "C"
