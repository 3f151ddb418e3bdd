// The single transition without a caller-provided workspace.
//
// Some callers cannot allocate device memory at the point where they run the op: a host
// framework whose device memory is owned by its own pool or arena (and forbids the
// library from calling cudaMalloc behind it), or a real-time or embedded pipeline that
// performs all its allocations at start-up. For them this file keeps the single
// transition's scratch (the LayerNorm output and the SwiGLU hidden activation) in a fixed
// file-scope device array instead of a workspace argument. Inputs, outputs and the packed
// weights are still the caller's.
//
// * The array holds at most kMaxTokens = 1024 tokens (B * N), 3,932,160 bytes. Every GPU
//   that loads this library reserves it for the life of the process.
// * Its device address is looked up once per device, on that device's first call (with
//   the device current). Make that first call before any stream capture.
// * All calls share the one array and leave the last call's values in it. Nothing in it
//   has to start at zero: each call writes every byte it later reads. Two calls whose GPU
//   work overlaps (on different streams, or from several host threads) race on the array
//   and may corrupt each other's results; serialise them.
// * No cudaMalloc, cudaFree or other allocating routine is called.
#include <mutex>

#include "../../include/foldforge_b200.h"
#include "abi_util.h"
#include "common.cuh"
#include "kernels.h"

namespace ffb {
namespace {

constexpr int kCs = 384;
constexpr int kMaxTokens = 1024;
constexpr size_t kScratchBytes = static_cast<size_t>(kMaxTokens) * (kCs * 2 + 4 * kCs * 2);  // y + hidden

static __device__ __align__(256) uint8_t g_single_transition_scratch[kScratchBytes];

std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxDevices];

// Device address of the scratch array on the current device (looked up once per device).
int scratch_address(int device, void** out) {
  if (device < 0 || device >= kMaxDevices)
    return fail(FFB_ERR_ARG, "single_transition_fwd_noalloc: device index %d out of range", device);
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[device] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_single_transition_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(FFB_ERR_CUDA, "single_transition_fwd_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_scratch_ptr[device] = p;
  }
  *out = g_scratch_ptr[device];
  return FFB_OK;
}

}  // namespace
}  // namespace ffb

using namespace ffb;

extern "C" int ffb_single_transition_fwd_noalloc(const void* s, const uint8_t* mask, const void* packed, void* out,
                                                 int B, int N, int masked, void* stream) {
  if (B <= 0 || N <= 0) return fail(FFB_ERR_ARG, "single_transition_fwd_noalloc: empty problem B=%d N=%d", B, N);
  if (static_cast<int64_t>(B) * N > kMaxTokens)
    return fail(FFB_ERR_UNSUPPORTED,
                "single_transition_fwd_noalloc: B*N = %lld tokens exceeds the built-in scratch limit of %d tokens "
                "(use ffb_single_transition_fwd with a workspace)",
                static_cast<long long>(B) * N, kMaxTokens);
  if (!s || !packed || !out) return fail(FFB_ERR_ARG, "single_transition_fwd_noalloc: null pointer");
  if (masked == FFB_MASKED_ZERO && !mask)
    return fail(FFB_ERR_ARG, "single_transition_fwd_noalloc: masked zero needs the mask");
  if (masked != FFB_MASKED_COMPUTE && masked != FFB_MASKED_ZERO)
    return fail(FFB_ERR_ARG, "single_transition_fwd_noalloc: masked=%d", masked);
  if (s == out) return fail(FFB_ERR_ARG, "single_transition_fwd_noalloc: out must not alias s");
  if (((reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(out)) & 15u) ||
      (reinterpret_cast<uintptr_t>(packed) & 255u))
    return fail(FFB_ERR_ARG, "single_transition_fwd_noalloc: misaligned pointer");
  DeviceInfo info;
  int st = device_info(&info);
  if (st != FFB_OK) return st;
  void* scratch = nullptr;
  st = scratch_address(info.device, &scratch);
  if (st != FFB_OK) return st;
  if (single_transition_workspace_bytes(B, N) > kScratchBytes)
    return fail(FFB_ERR_UNSUPPORTED, "single_transition_fwd_noalloc: scratch too small for B=%d N=%d", B, N);
  return single_transition_forward(s, mask, packed, out, scratch, B, N, masked == FFB_MASKED_ZERO, info,
                                   static_cast<cudaStream_t>(stream));
}
