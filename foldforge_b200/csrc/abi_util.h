// Helpers shared by the C-ABI translation units: status reporting, per-device info and
// tensor-map encoding through the driver entry point (no link-time libcuda dependency).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>

namespace ffb {

typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// Devices a process may use with this library (per-device caches are arrays of this size).
constexpr int kMaxDevices = 64;

struct DeviceInfo {
  int device;
  int num_sms;
  int* err;  // device address of this device's error word
};

// Records a formatted message for ffb_last_error() and returns `status`.
int fail(int status, const char* fmt, ...);
// FFB_OK for cudaSuccess, else FFB_ERR_CUDA with the runtime's message.
int cuda_status(int rc, const char* what);
// Current device's cached info; checks the device is sm_100.
int device_info(DeviceInfo* info);
// Encodes a tiled tensor map; dims innermost first, strides (rank - 1 of them) in bytes.
int make_map(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
             const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle);

}  // namespace ffb
