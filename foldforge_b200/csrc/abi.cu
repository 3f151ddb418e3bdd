// The C ABI (include/foldforge_b200.h): argument checks, tensor-map encoding, per-device
// caches and status reporting around the kernel launchers.
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/foldforge_b200.h"
#include "abi_util.h"
#include "common.cuh"
#include "kernels.h"

namespace ffb {

__device__ int g_error_word;

namespace {
thread_local std::string t_last_error;
std::mutex g_mutex;
int g_num_sms[kMaxDevices];
int* g_err_ptr[kMaxDevices];
PFN_encodeTiled g_encode = nullptr;
}  // namespace

int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return status;
}

int cuda_status(int rc, const char* what) {
  if (rc == 0) return FFB_OK;
  return fail(FFB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(static_cast<cudaError_t>(rc)));
}

int device_info(DeviceInfo* info) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(FFB_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(FFB_ERR_ARG, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_num_sms[dev] == 0) {
    int sms = 0, major = 0, minor = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (major != 10 || minor != 0)
      return fail(FFB_ERR_UNSUPPORTED, "device %d is sm_%d%d; these kernels are built for sm_100a only", dev, major,
                  minor);
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_error_word);
    if (e != cudaSuccess) return fail(FFB_ERR_CUDA, "cudaGetSymbolAddress(error word): %s", cudaGetErrorString(e));
    g_err_ptr[dev] = static_cast<int*>(p);
    g_num_sms[dev] = sms;
  }
  if (g_encode == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || fn == nullptr || q != cudaDriverEntryPointSuccess)
      return fail(FFB_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    g_encode = reinterpret_cast<PFN_encodeTiled>(fn);
  }
  info->device = dev;
  info->num_sms = g_num_sms[dev];
  info->err = g_err_ptr[dev];
  return FFB_OK;
}

int make_map(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
             const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return fail(FFB_ERR_ARG, "tensor base %p is not 16-byte aligned", base);
  for (int i = 0; i + 1 < rank; ++i)
    if (strides_bytes[i] % 16 != 0)
      return fail(FFB_ERR_ARG, "tensor stride %llu bytes is not a multiple of 16", (unsigned long long)strides_bytes[i]);
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t bdim[5];
  cuuint32_t estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) gstride[i] = strides_bytes[i];
  CUresult r = g_encode(map, dtype, rank, const_cast<void*>(base), gdim, gstride, bdim, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FFB_ERR_ARG, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return FFB_OK;
}

}  // namespace ffb

using namespace ffb;

extern "C" {

int ffb_version(void) { return 100; }

const char* ffb_last_error(void) { return t_last_error.c_str(); }

int ffb_device_error(int* code, void* stream) {
  DeviceInfo info;
  int st = device_info(&info);
  if (st != FFB_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return fail(FFB_ERR_CUDA, "cudaStreamSynchronize: %s", cudaGetErrorString(e));
  int value = 0;
  e = cudaMemcpy(&value, info.err, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fail(FFB_ERR_CUDA, "reading the error word: %s", cudaGetErrorString(e));
  if (value != 0) {
    const int zero = 0;
    cudaMemcpy(info.err, &zero, sizeof(int), cudaMemcpyHostToDevice);
  }
  if (code) *code = value;
  return value == 0 ? FFB_OK : fail(FFB_ERR_DEVICE, "device error word %d", value);
}

int ffb_layernorm_fwd(const void* x, void* y, const float* gamma, const float* beta, int64_t rows, int c, float eps,
                      int dtype, void* stream) {
  if (rows < 0 || c <= 0) return fail(FFB_ERR_ARG, "layernorm: rows=%lld c=%d", (long long)rows, c);
  if (rows > 0 && (x == nullptr || y == nullptr)) return fail(FFB_ERR_ARG, "layernorm: null tensor");
  if (dtype != FFB_BF16 && dtype != FFB_F32) return fail(FFB_ERR_UNSUPPORTED, "layernorm: dtype %d", dtype);
  if (dtype == FFB_BF16 && c == 128 &&
      ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15u) != 0)
    return fail(FFB_ERR_ARG, "layernorm: bf16 rows of 128 need 16-byte aligned tensors");
  DeviceInfo info;
  int st = device_info(&info);
  if (st != FFB_OK) return st;
  return cuda_status(launch_layernorm(x, y, gamma, beta, rows, c, eps, dtype == FFB_F32, info.num_sms,
                                      static_cast<cudaStream_t>(stream)),
                     "layernorm launch");
}

int ffb_gemm_bf16_nt(const void* a, const void* b, void* d, int batch, int m, int n, int k, int64_t lda,
                     int64_t ldb, int64_t ldd, int64_t sa, int64_t sb, int64_t sd, int d_dtype, const float* bias,
                     int epilogue, const void* residual, const uint8_t* row_mask, void* stream) {
  if (batch <= 0 || m <= 0 || n <= 0 || k <= 0) return fail(FFB_ERR_ARG, "gemm: empty problem");
  if (k % 8 != 0 || lda % 8 != 0 || ldb % 8 != 0) return fail(FFB_ERR_ARG, "gemm: k, lda, ldb must be multiples of 8");
  if (epilogue < 0 || epilogue > 2) return fail(FFB_ERR_ARG, "gemm: epilogue %d", epilogue);
  if (epilogue == kEpiResidual && residual == nullptr) return fail(FFB_ERR_ARG, "gemm: residual epilogue needs R");
  if (epilogue == kEpiSwiGLU && (n % 32 != 0 || d_dtype != FFB_BF16))
    return fail(FFB_ERR_ARG, "gemm: SwiGLU needs n % 32 == 0 and a bf16 output");
  if (batch > 1 && (sa % 8 != 0 || sb % 8 != 0)) return fail(FFB_ERR_ARG, "gemm: batch strides must be multiples of 8");
  DeviceInfo info;
  int st = device_info(&info);
  if (st != FFB_OK) return st;
  const int bn = n >= 256 ? 256 : 128;
  CUtensorMap ma, mb;
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(k), static_cast<uint64_t>(m), static_cast<uint64_t>(batch)};
    const uint64_t strides[2] = {static_cast<uint64_t>(lda) * 2, static_cast<uint64_t>(batch > 1 ? sa : lda * m) * 2};
    const uint32_t box[3] = {64, 128, 1};
    st = make_map(&ma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != FFB_OK) return st;
  }
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(k), static_cast<uint64_t>(n), static_cast<uint64_t>(batch)};
    const uint64_t strides[2] = {static_cast<uint64_t>(ldb) * 2, static_cast<uint64_t>(batch > 1 ? sb : ldb * n) * 2};
    const uint32_t box[3] = {64, static_cast<uint32_t>(bn), 1};
    st = make_map(&mb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, b, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != FFB_OK) return st;
  }
  GemmParams p;
  p.M = m;
  p.N = n;
  p.K = k;
  p.batch = batch;
  p.D = d;
  p.ldd = ldd;
  p.batch_stride_d = sd;
  p.d_is_f32 = d_dtype == FFB_F32;
  p.epilogue = epilogue;
  p.bias = bias;
  p.residual = residual;
  p.row_mask = row_mask;
  p.err = info.err;
  return cuda_status(launch_gemm_nt(ma, mb, p, bn, info.num_sms, static_cast<cudaStream_t>(stream)), "gemm launch");
}

size_t ffb_trimul_packed_bytes(void) { return trimul_packed_bytes(); }

size_t ffb_trimul_workspace_bytes(int B, int N) { return (B <= 0 || N <= 0) ? 0 : trimul_workspace_bytes(B, N); }

int ffb_trimul_prepare(const float* ln_w, const float* ln_b, const float* ln_out_w, const float* ln_out_b,
                       const float* to_left, const float* to_right, const float* to_left_gate,
                       const float* to_right_gate, const float* to_out, const float* to_gate, void* packed,
                       void* stream) {
  if (!ln_w || !ln_b || !ln_out_w || !ln_out_b || !to_left || !to_right || !to_left_gate || !to_right_gate ||
      !to_out || !to_gate || !packed)
    return fail(FFB_ERR_ARG, "trimul_prepare: null pointer");
  if ((reinterpret_cast<uintptr_t>(packed) & 15u) != 0) return fail(FFB_ERR_ARG, "trimul_prepare: packed not 16-byte aligned");
  DeviceInfo info;
  int st = device_info(&info);
  if (st != FFB_OK) return st;
  TriMulWeights w{ln_w, ln_b, ln_out_w, ln_out_b, to_left, to_right, to_left_gate, to_right_gate, to_out, to_gate};
  return cuda_status(trimul_prepare(w, packed, static_cast<cudaStream_t>(stream)), "trimul_prepare");
}

int ffb_trimul_fwd(const void* z, const uint8_t* mask, const void* packed, void* out, void* workspace,
                   size_t workspace_bytes, int B, int N, int outgoing, int masked, void* stream) {
  return ffb_trimul_fwd_stages(z, mask, packed, out, workspace, workspace_bytes, B, N, outgoing, masked, 7, stream);
}

int ffb_trimul_fwd_stages(const void* z, const uint8_t* mask, const void* packed, void* out, void* workspace,
                          size_t workspace_bytes, int B, int N, int outgoing, int masked, int stages, void* stream) {
  if (stages <= 0 || stages > 7) return fail(FFB_ERR_ARG, "trimul_fwd: stages=%d", stages);
  if (B <= 0 || N <= 0) return fail(FFB_ERR_ARG, "trimul_fwd: empty problem B=%d N=%d", B, N);
  if (!z || !mask || !packed || !out || !workspace) return fail(FFB_ERR_ARG, "trimul_fwd: null pointer");
  if (z == out) return fail(FFB_ERR_ARG, "trimul_fwd: out must not alias z");
  if (masked != FFB_MASKED_COMPUTE && masked != FFB_MASKED_ZERO) return fail(FFB_ERR_ARG, "trimul_fwd: masked=%d", masked);
  if (workspace_bytes < trimul_workspace_bytes(B, N))
    return fail(FFB_ERR_ARG, "trimul_fwd: workspace %zu < %zu bytes", workspace_bytes, trimul_workspace_bytes(B, N));
  if (((reinterpret_cast<uintptr_t>(z) | reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(packed)) & 15u) ||
      (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return fail(FFB_ERR_ARG, "trimul_fwd: misaligned pointer");
  if (static_cast<int64_t>(B) * N > (1 << 30) / 128) return fail(FFB_ERR_UNSUPPORTED, "trimul_fwd: B*N too large");
  DeviceInfo info;
  int st = device_info(&info);
  if (st != FFB_OK) return st;
  return trimul_forward(z, mask, packed, out, workspace, B, N, outgoing != 0, masked == FFB_MASKED_ZERO, stages, info,
                        static_cast<cudaStream_t>(stream));
}

size_t ffb_triattn_packed_bytes(void) { return triattn_packed_bytes(); }

size_t ffb_triattn_workspace_bytes(int B, int N) { return (B <= 0 || N <= 0) ? 0 : triattn_workspace_bytes(B, N); }

int ffb_triattn_prepare(const float* ln_w, const float* ln_b, const float* to_bias, const float* to_query,
                        const float* to_key, const float* to_value, const float* to_gate, const float* to_out,
                        void* packed, void* stream) {
  if (!ln_w || !ln_b || !to_bias || !to_query || !to_key || !to_value || !to_gate || !to_out || !packed)
    return fail(FFB_ERR_ARG, "triattn_prepare: null pointer");
  if ((reinterpret_cast<uintptr_t>(packed) & 15u) != 0) return fail(FFB_ERR_ARG, "triattn_prepare: packed not 16-byte aligned");
  DeviceInfo info;
  int st = device_info(&info);
  if (st != FFB_OK) return st;
  TriAttnWeights w{ln_w, ln_b, to_bias, to_query, to_key, to_value, to_gate, to_out};
  return cuda_status(triattn_prepare(w, packed, static_cast<cudaStream_t>(stream)), "triattn_prepare");
}

int ffb_triattn_fwd(const void* z, const uint8_t* mask, const void* packed, void* out, void* workspace,
                    size_t workspace_bytes, int B, int N, int starting, int masked, void* stream) {
  return ffb_triattn_fwd_stages(z, mask, packed, out, workspace, workspace_bytes, B, N, starting, masked, 7, stream);
}

int ffb_triattn_fwd_stages(const void* z, const uint8_t* mask, const void* packed, void* out, void* workspace,
                           size_t workspace_bytes, int B, int N, int starting, int masked, int stages, void* stream) {
  if (stages <= 0 || stages > 7) return fail(FFB_ERR_ARG, "triattn_fwd: stages=%d", stages);
  if (B <= 0 || N <= 0) return fail(FFB_ERR_ARG, "triattn_fwd: empty problem B=%d N=%d", B, N);
  if (!z || !mask || !packed || !out || !workspace) return fail(FFB_ERR_ARG, "triattn_fwd: null pointer");
  if (z == out) return fail(FFB_ERR_ARG, "triattn_fwd: out must not alias z");
  if (masked != FFB_MASKED_COMPUTE && masked != FFB_MASKED_ZERO) return fail(FFB_ERR_ARG, "triattn_fwd: masked=%d", masked);
  if (workspace_bytes < triattn_workspace_bytes(B, N))
    return fail(FFB_ERR_ARG, "triattn_fwd: workspace %zu < %zu bytes", workspace_bytes, triattn_workspace_bytes(B, N));
  if (((reinterpret_cast<uintptr_t>(z) | reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(packed)) & 15u) ||
      (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return fail(FFB_ERR_ARG, "triattn_fwd: misaligned pointer");
  if (static_cast<int64_t>(B) * N * 4 > (1 << 30) / 128) return fail(FFB_ERR_UNSUPPORTED, "triattn_fwd: B*N too large");
  DeviceInfo info;
  int st = device_info(&info);
  if (st != FFB_OK) return st;
  return triattn_forward(z, mask, packed, out, workspace, B, N, starting != 0, masked == FFB_MASKED_ZERO, stages,
                         info, static_cast<cudaStream_t>(stream));
}

size_t ffb_transition_packed_bytes(void) { return transition_packed_bytes(); }

int ffb_transition_prepare(const float* ln_w, const float* ln_b, const float* expand_a, const float* expand_b,
                           const float* squeeze, void* packed, void* stream) {
  if (!ln_w || !ln_b || !expand_a || !expand_b || !squeeze || !packed)
    return fail(FFB_ERR_ARG, "transition_prepare: null pointer");
  if ((reinterpret_cast<uintptr_t>(packed) & 15u) != 0) return fail(FFB_ERR_ARG, "transition_prepare: packed not 16-byte aligned");
  DeviceInfo info;
  int st = device_info(&info);
  if (st != FFB_OK) return st;
  TransitionWeights w{ln_w, ln_b, expand_a, expand_b, squeeze};
  return cuda_status(transition_prepare(w, packed, static_cast<cudaStream_t>(stream)), "transition_prepare");
}

int ffb_transition_fwd(const void* z, const uint8_t* mask, const void* packed, void* out, int B, int N, int masked,
                       void* stream) {
  if (B <= 0 || N <= 0) return fail(FFB_ERR_ARG, "transition_fwd: empty problem B=%d N=%d", B, N);
  if (!z || !packed || !out) return fail(FFB_ERR_ARG, "transition_fwd: null pointer");
  if (masked == FFB_MASKED_ZERO && !mask) return fail(FFB_ERR_ARG, "transition_fwd: masked zero needs the mask");
  if (masked != FFB_MASKED_COMPUTE && masked != FFB_MASKED_ZERO) return fail(FFB_ERR_ARG, "transition_fwd: masked=%d", masked);
  if (z == out) return fail(FFB_ERR_ARG, "transition_fwd: out must not alias z");
  if ((reinterpret_cast<uintptr_t>(z) | reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(packed)) & 15u)
    return fail(FFB_ERR_ARG, "transition_fwd: misaligned pointer");
  if (static_cast<int64_t>(B) * N * N >= (int64_t(1) << 31) - 256) return fail(FFB_ERR_UNSUPPORTED, "transition_fwd: too many rows");
  DeviceInfo info;
  int st = device_info(&info);
  if (st != FFB_OK) return st;
  return transition_forward(z, mask, packed, out, B, N, masked == FFB_MASKED_ZERO, info,
                            static_cast<cudaStream_t>(stream));
}

size_t ffb_apb_packed_bytes(void) { return apb_packed_bytes(); }

size_t ffb_apb_workspace_bytes(int B, int N) { return (B <= 0 || N <= 0) ? 0 : apb_workspace_bytes(B, N); }

int ffb_apb_prepare(const float* ln_single_w, const float* ln_single_b, const float* to_query,
                    const float* query_bias, const float* to_key, const float* to_value, const float* to_gate,
                    const float* to_out, const float* ln_pair_w, const float* to_bias, void* packed, void* stream) {
  if (!ln_single_w || !ln_single_b || !to_query || !query_bias || !to_key || !to_value || !to_gate || !to_out ||
      !ln_pair_w || !to_bias || !packed)
    return fail(FFB_ERR_ARG, "apb_prepare: null pointer");
  if ((reinterpret_cast<uintptr_t>(packed) & 255u) != 0) return fail(FFB_ERR_ARG, "apb_prepare: packed not 256-byte aligned");
  DeviceInfo info;
  int st = device_info(&info);
  if (st != FFB_OK) return st;
  ApbWeights w{ln_single_w, ln_single_b, to_query, query_bias, to_key, to_value, to_gate, to_out, ln_pair_w, to_bias};
  return cuda_status(apb_prepare(w, packed, static_cast<cudaStream_t>(stream)), "apb_prepare");
}

int ffb_apb_fwd(const void* s, const void* z, const uint8_t* mask, const void* packed, const void* extra_pair_bias,
                int extra_dtype, float gate_bias, void* out, void* workspace, size_t workspace_bytes, int B, int N,
                int masked, void* stream) {
  if (B <= 0 || N <= 0) return fail(FFB_ERR_ARG, "apb_fwd: empty problem B=%d N=%d", B, N);
  if (!s || !z || !mask || !packed || !out || !workspace) return fail(FFB_ERR_ARG, "apb_fwd: null pointer");
  if (s == out) return fail(FFB_ERR_ARG, "apb_fwd: out must not alias s");
  if (masked != FFB_MASKED_COMPUTE && masked != FFB_MASKED_ZERO) return fail(FFB_ERR_ARG, "apb_fwd: masked=%d", masked);
  if (extra_pair_bias && extra_dtype != FFB_BF16 && extra_dtype != FFB_F32) return fail(FFB_ERR_ARG, "apb_fwd: extra dtype");
  if (workspace_bytes < apb_workspace_bytes(B, N))
    return fail(FFB_ERR_ARG, "apb_fwd: workspace %zu < %zu bytes", workspace_bytes, apb_workspace_bytes(B, N));
  if (((reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(z) | reinterpret_cast<uintptr_t>(out)) & 15u) ||
      ((reinterpret_cast<uintptr_t>(packed) | reinterpret_cast<uintptr_t>(workspace)) & 255u))
    return fail(FFB_ERR_ARG, "apb_fwd: misaligned pointer");
  if (static_cast<int64_t>(B) * N * N >= (int64_t(1) << 31) - 256) return fail(FFB_ERR_UNSUPPORTED, "apb_fwd: too many pairs");
  DeviceInfo info;
  int st = device_info(&info);
  if (st != FFB_OK) return st;
  return apb_forward(s, z, mask, packed, extra_pair_bias, extra_dtype == FFB_F32, gate_bias, out, workspace, B, N,
                     masked == FFB_MASKED_ZERO, info, static_cast<cudaStream_t>(stream));
}

size_t ffb_single_transition_packed_bytes(void) { return single_transition_packed_bytes(); }

size_t ffb_single_transition_workspace_bytes(int B, int N) {
  return (B <= 0 || N <= 0) ? 0 : single_transition_workspace_bytes(B, N);
}

int ffb_single_transition_prepare(const float* ln_w, const float* ln_b, const float* expand_a,
                                  const float* expand_b, const float* squeeze, void* packed, void* stream) {
  if (!ln_w || !ln_b || !expand_a || !expand_b || !squeeze || !packed)
    return fail(FFB_ERR_ARG, "single_transition_prepare: null pointer");
  if ((reinterpret_cast<uintptr_t>(packed) & 255u) != 0)
    return fail(FFB_ERR_ARG, "single_transition_prepare: packed not 256-byte aligned");
  DeviceInfo info;
  int st = device_info(&info);
  if (st != FFB_OK) return st;
  TransitionWeights w{ln_w, ln_b, expand_a, expand_b, squeeze};
  return cuda_status(single_transition_prepare(w, packed, static_cast<cudaStream_t>(stream)),
                     "single_transition_prepare");
}

int ffb_single_transition_fwd(const void* s, const uint8_t* mask, const void* packed, void* out, void* workspace,
                              size_t workspace_bytes, int B, int N, int masked, void* stream) {
  if (B <= 0 || N <= 0) return fail(FFB_ERR_ARG, "single_transition_fwd: empty problem B=%d N=%d", B, N);
  if (!s || !packed || !out || !workspace) return fail(FFB_ERR_ARG, "single_transition_fwd: null pointer");
  if (masked == FFB_MASKED_ZERO && !mask) return fail(FFB_ERR_ARG, "single_transition_fwd: masked zero needs the mask");
  if (masked != FFB_MASKED_COMPUTE && masked != FFB_MASKED_ZERO)
    return fail(FFB_ERR_ARG, "single_transition_fwd: masked=%d", masked);
  if (s == out) return fail(FFB_ERR_ARG, "single_transition_fwd: out must not alias s");
  if (workspace_bytes < single_transition_workspace_bytes(B, N))
    return fail(FFB_ERR_ARG, "single_transition_fwd: workspace too small");
  if (((reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(out)) & 15u) ||
      ((reinterpret_cast<uintptr_t>(packed) | reinterpret_cast<uintptr_t>(workspace)) & 255u))
    return fail(FFB_ERR_ARG, "single_transition_fwd: misaligned pointer");
  DeviceInfo info;
  int st = device_info(&info);
  if (st != FFB_OK) return st;
  return single_transition_forward(s, mask, packed, out, workspace, B, N, masked == FFB_MASKED_ZERO, info,
                                   static_cast<cudaStream_t>(stream));
}

}  // extern "C"

// ---- row-sharded pieces (axial parallelism; B = 1; the rank holds pair rows
// [row0, row0 + R) of an N x N pair, or of its transpose for the column-wise ops)
namespace {
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
int shard_args(const char* what, int R, int N, int row0) {
  if (R <= 0 || N <= 0 || row0 < 0 || row0 + R > N)
    return fail(FFB_ERR_ARG, "%s: rows [%d, %d) of N=%d", what, row0, row0 + R, N);
  if (static_cast<int64_t>(R) * N >= (int64_t(1) << 31) - 256) return fail(FFB_ERR_UNSUPPORTED, "%s: too many pairs", what);
  return FFB_OK;
}
}  // namespace

extern "C" {

int ffb_trimul_shard_proj(const void* z, const uint8_t* mask, const void* packed, void* left, void* right,
                          void* zstats, int R, int N, int row0, void* stream) {
  int st = shard_args("trimul_shard_proj", R, N, row0);
  if (st) return st;
  if (!z || !mask || !packed || !left || !right || !zstats) return fail(FFB_ERR_ARG, "trimul_shard_proj: null pointer");
  if (!aligned16(z) || !aligned16(packed) || !aligned16(left) || !aligned16(right) || !aligned16(zstats))
    return fail(FFB_ERR_ARG, "trimul_shard_proj: misaligned pointer");
  DeviceInfo info;
  st = device_info(&info);
  if (st != FFB_OK) return st;
  return trimul_shard_proj(z, mask, packed, left, right, zstats, R, N, row0, info, static_cast<cudaStream_t>(stream));
}

int ffb_trimul_shard_contract(const void* left, const void* right_all, void* u, int R, int N, void* stream) {
  int st = shard_args("trimul_shard_contract", R, N, 0);
  if (st) return st;
  if (!left || !right_all || !u) return fail(FFB_ERR_ARG, "trimul_shard_contract: null pointer");
  if (!aligned16(left) || !aligned16(right_all) || !aligned16(u))
    return fail(FFB_ERR_ARG, "trimul_shard_contract: misaligned pointer");
  DeviceInfo info;
  st = device_info(&info);
  if (st != FFB_OK) return st;
  return trimul_shard_contract(left, right_all, u, R, N, info, static_cast<cudaStream_t>(stream));
}

int ffb_trimul_channel_contract(const void* left, const void* right, void* u, int C, int N, void* stream) {
  if (C <= 0 || C > 128 || N <= 0 || static_cast<int64_t>(C) * N >= (int64_t(1) << 31) - 256)
    return fail(FFB_ERR_ARG, "trimul_channel_contract: C=%d N=%d", C, N);
  if (!left || !right || !u) return fail(FFB_ERR_ARG, "trimul_channel_contract: null pointer");
  if (!aligned16(left) || !aligned16(right) || !aligned16(u))
    return fail(FFB_ERR_ARG, "trimul_channel_contract: misaligned pointer");
  DeviceInfo info;
  int st = device_info(&info);
  if (st != FFB_OK) return st;
  return trimul_channel_contract(left, right, u, C, N, info, static_cast<cudaStream_t>(stream));
}

int ffb_trimul_shard_out(const void* z, const uint8_t* mask, const void* packed, const void* u, const void* zstats,
                         void* ustats, void* out, int R, int N, int row0, int masked, void* stream) {
  int st = shard_args("trimul_shard_out", R, N, row0);
  if (st) return st;
  if (!z || !mask || !packed || !u || !zstats || !out) return fail(FFB_ERR_ARG, "trimul_shard_out: null pointer");
  if (z == out) return fail(FFB_ERR_ARG, "trimul_shard_out: out must not alias z");
  if (masked != FFB_MASKED_COMPUTE && masked != FFB_MASKED_ZERO) return fail(FFB_ERR_ARG, "trimul_shard_out: masked=%d", masked);
  if (!aligned16(z) || !aligned16(packed) || !aligned16(u) || !aligned16(zstats) || !aligned16(out))
    return fail(FFB_ERR_ARG, "trimul_shard_out: misaligned pointer");
  DeviceInfo info;
  st = device_info(&info);
  if (st != FFB_OK) return st;
  return trimul_shard_out(z, mask, packed, u, zstats, ustats, out, R, N, row0, masked == FFB_MASKED_ZERO, info,
                          static_cast<cudaStream_t>(stream));
}

int ffb_triattn_shard_proj(const void* z, const void* packed, void* q, void* k, void* vt, void* bias_rows, int R, int N,
                           void* stream) {
  int st = shard_args("triattn_shard_proj", R, N, 0);
  if (st) return st;
  if (!z || !packed || !q || !k || !vt || !bias_rows) return fail(FFB_ERR_ARG, "triattn_shard_proj: null pointer");
  if (!aligned16(z) || !aligned16(packed) || !aligned16(q) || !aligned16(k) || !aligned16(vt) || !aligned16(bias_rows))
    return fail(FFB_ERR_ARG, "triattn_shard_proj: misaligned pointer");
  DeviceInfo info;
  st = device_info(&info);
  if (st != FFB_OK) return st;
  return triattn_shard_proj(z, packed, q, k, vt, bias_rows, R, N, info, static_cast<cudaStream_t>(stream));
}

int ffb_triattn_shard_attn(const void* q, const void* k, const void* vt, const void* bias_all, const uint8_t* mask,
                           void* o, int R, int N, int row0, void* stream) {
  int st = shard_args("triattn_shard_attn", R, N, row0);
  if (st) return st;
  if (!q || !k || !vt || !bias_all || !mask || !o) return fail(FFB_ERR_ARG, "triattn_shard_attn: null pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(vt) || !aligned16(bias_all) || !aligned16(o))
    return fail(FFB_ERR_ARG, "triattn_shard_attn: misaligned pointer");
  DeviceInfo info;
  st = device_info(&info);
  if (st != FFB_OK) return st;
  return triattn_shard_attn(q, k, vt, bias_all, mask, o, R, N, row0, info, static_cast<cudaStream_t>(stream));
}

int ffb_triattn_shard_out(const void* z, const uint8_t* mask, const void* packed, const void* o, void* out, int R, int N,
                          int row0, int masked, void* stream) {
  int st = shard_args("triattn_shard_out", R, N, row0);
  if (st) return st;
  if (!z || !mask || !packed || !o || !out) return fail(FFB_ERR_ARG, "triattn_shard_out: null pointer");
  if (z == out) return fail(FFB_ERR_ARG, "triattn_shard_out: out must not alias z");
  if (masked != FFB_MASKED_COMPUTE && masked != FFB_MASKED_ZERO) return fail(FFB_ERR_ARG, "triattn_shard_out: masked=%d", masked);
  if (!aligned16(z) || !aligned16(packed) || !aligned16(o) || !aligned16(out))
    return fail(FFB_ERR_ARG, "triattn_shard_out: misaligned pointer");
  DeviceInfo info;
  st = device_info(&info);
  if (st != FFB_OK) return st;
  return triattn_shard_out(z, mask, packed, o, out, R, N, row0, masked == FFB_MASKED_ZERO, info,
                           static_cast<cudaStream_t>(stream));
}

int ffb_transition_shard_fwd(const void* z, const uint8_t* mask, const void* packed, void* out, int R, int N, int row0,
                             int masked, void* stream) {
  int st = shard_args("transition_shard_fwd", R, N, row0);
  if (st) return st;
  if (!z || !packed || !out) return fail(FFB_ERR_ARG, "transition_shard_fwd: null pointer");
  if (masked == FFB_MASKED_ZERO && !mask) return fail(FFB_ERR_ARG, "transition_shard_fwd: masked zero needs the mask");
  if (masked != FFB_MASKED_COMPUTE && masked != FFB_MASKED_ZERO) return fail(FFB_ERR_ARG, "transition_shard_fwd: masked=%d", masked);
  if (z == out) return fail(FFB_ERR_ARG, "transition_shard_fwd: out must not alias z");
  if (!aligned16(z) || !aligned16(out) || !aligned16(packed)) return fail(FFB_ERR_ARG, "transition_shard_fwd: misaligned pointer");
  DeviceInfo info;
  st = device_info(&info);
  if (st != FFB_OK) return st;
  return transition_shard_forward(z, mask, packed, out, R, N, row0, masked == FFB_MASKED_ZERO, info,
                                  static_cast<cudaStream_t>(stream));
}

int ffb_apb_shard_pair_bias(const void* z, const void* packed, void* pb_rows, int R, int N, void* stream) {
  int st = shard_args("apb_shard_pair_bias", R, N, 0);
  if (st) return st;
  if (!z || !packed || !pb_rows) return fail(FFB_ERR_ARG, "apb_shard_pair_bias: null pointer");
  if (!aligned16(z) || (reinterpret_cast<uintptr_t>(packed) & 255u) || !aligned16(pb_rows))
    return fail(FFB_ERR_ARG, "apb_shard_pair_bias: misaligned pointer");
  DeviceInfo info;
  st = device_info(&info);
  if (st != FFB_OK) return st;
  return apb_shard_pair_bias(z, packed, pb_rows, R, N, info, static_cast<cudaStream_t>(stream));
}

size_t ffb_apb_single_workspace_bytes(int N) { return N <= 0 ? 0 : apb_single_workspace_bytes(N); }

int ffb_apb_shard_single(const void* s, const uint8_t* mask, const void* packed, const void* pb_all,
                         const void* extra_pair_bias, int extra_dtype, float gate_bias, void* out, void* workspace,
                         size_t workspace_bytes, int N, int masked, void* stream) {
  if (N <= 0) return fail(FFB_ERR_ARG, "apb_shard_single: N=%d", N);
  if (!s || !mask || !packed || !pb_all || !out || !workspace) return fail(FFB_ERR_ARG, "apb_shard_single: null pointer");
  if (s == out) return fail(FFB_ERR_ARG, "apb_shard_single: out must not alias s");
  if (masked != FFB_MASKED_COMPUTE && masked != FFB_MASKED_ZERO) return fail(FFB_ERR_ARG, "apb_shard_single: masked=%d", masked);
  if (extra_pair_bias && extra_dtype != FFB_BF16 && extra_dtype != FFB_F32)
    return fail(FFB_ERR_ARG, "apb_shard_single: extra dtype");
  if (workspace_bytes < apb_single_workspace_bytes(N))
    return fail(FFB_ERR_ARG, "apb_shard_single: workspace %zu < %zu bytes", workspace_bytes, apb_single_workspace_bytes(N));
  if (!aligned16(s) || !aligned16(out) || !aligned16(pb_all) ||
      ((reinterpret_cast<uintptr_t>(packed) | reinterpret_cast<uintptr_t>(workspace)) & 255u))
    return fail(FFB_ERR_ARG, "apb_shard_single: misaligned pointer");
  DeviceInfo info;
  int st = device_info(&info);
  if (st != FFB_OK) return st;
  return apb_shard_single(s, mask, packed, pb_all, extra_pair_bias, extra_dtype == FFB_F32, gate_bias, out, workspace,
                          N, masked == FFB_MASKED_ZERO, info, static_cast<cudaStream_t>(stream));
}

// The rank's rows of the single track's attention with pair bias from its own pair-bias rows.
int ffb_apb_shard_single_rows(const void* s, const uint8_t* mask, const void* packed, const void* pb_rows,
                              float gate_bias, void* out_rows, void* workspace, size_t workspace_bytes, int N,
                              int row0, int R, int masked, void* stream) {
  if (N <= 0 || R <= 0 || row0 < 0 || row0 + R > N)
    return fail(FFB_ERR_ARG, "apb_shard_single_rows: N=%d row0=%d R=%d", N, row0, R);
  if (!s || !mask || !packed || !pb_rows || !out_rows || !workspace)
    return fail(FFB_ERR_ARG, "apb_shard_single_rows: null pointer");
  if (masked != FFB_MASKED_COMPUTE && masked != FFB_MASKED_ZERO)
    return fail(FFB_ERR_ARG, "apb_shard_single_rows: masked=%d", masked);
  if (workspace_bytes < apb_single_workspace_bytes(N))
    return fail(FFB_ERR_ARG, "apb_shard_single_rows: workspace %zu < %zu bytes", workspace_bytes,
                apb_single_workspace_bytes(N));
  const uint8_t* s_rows = static_cast<const uint8_t*>(s) + static_cast<size_t>(row0) * 384 * 2;
  if (!aligned16(s) || !aligned16(out_rows) || !aligned16(pb_rows) ||
      ((reinterpret_cast<uintptr_t>(packed) | reinterpret_cast<uintptr_t>(workspace)) & 255u))
    return fail(FFB_ERR_ARG, "apb_shard_single_rows: misaligned pointer");
  const uint8_t* o = static_cast<const uint8_t*>(out_rows);
  if (o < s_rows + static_cast<size_t>(R) * 384 * 2 && s_rows < o + static_cast<size_t>(R) * 384 * 2)
    return fail(FFB_ERR_ARG, "apb_shard_single_rows: out_rows must not overlap s");
  DeviceInfo info;
  int st = device_info(&info);
  if (st != FFB_OK) return st;
  return apb_shard_single_rows(s, mask, packed, pb_rows, gate_bias, out_rows, workspace, N, row0, R,
                               masked == FFB_MASKED_ZERO, info, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
