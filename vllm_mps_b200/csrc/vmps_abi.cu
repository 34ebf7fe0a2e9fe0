// Shared pieces of the C ABI: error reporting, the device error word, the
// per-device SM count, and access to the driver's tensor-map encoder.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "vmps_abi_internal.h"

namespace vmps {

__device__ int g_error_word = 0;

static thread_local char t_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return code;
}

void clear_error() { t_last_error[0] = '\0'; }

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return fail(VMPS_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  }
  return VMPS_OK;
}

int device_sm_count(int* out) {
  static int cached[64];
  static std::once_flag flags[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    return fail(VMPS_ERR_CUDA, "cudaGetDevice failed");
  }
  std::call_once(flags[dev], [&] {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) n = 0;
    cached[dev] = n;
  });
  if (cached[dev] <= 0) return fail(VMPS_ERR_CUDA, "could not read the SM count");
  *out = cached[dev];
  return VMPS_OK;
}

int device_error_word(int** out) {
  static int* cached[64];
  static std::once_flag flags[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    return fail(VMPS_ERR_CUDA, "cudaGetDevice failed");
  }
  std::call_once(flags[dev], [&] {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_error_word) != cudaSuccess) p = nullptr;
    cached[dev] = static_cast<int*>(p);
  });
  if (!cached[dev]) return fail(VMPS_ERR_CUDA, "could not resolve the device error word");
  *out = cached[dev];
  return VMPS_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int encode_tiled(CUtensorMap* map, CUtensorMapDataType dt, int rank, void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swizzle) {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  });
  if (!fn) return fail(VMPS_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(map, dt, (cuuint32_t)rank, base, (const cuuint64_t*)dims,
                  (const cuuint64_t*)strides_bytes, (const cuuint32_t*)box, elem_strides,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(VMPS_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return VMPS_OK;
}

}  // namespace vmps

extern "C" {

const char* vmps_version(void) { return "vmps 0.1.0 sm_100a"; }

const char* vmps_last_error(void) { return vmps::t_last_error; }

int vmps_debug_error_word(void* stream, int* word_out) {
  if (!word_out) return vmps::fail(VMPS_ERR_INVALID_ARG, "word_out is NULL");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int zero = 0;
  int host = 0;
  if (cudaMemcpyFromSymbolAsync(&host, vmps::g_error_word, sizeof(int), 0,
                                cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess ||
      cudaMemcpyToSymbolAsync(vmps::g_error_word, &zero, sizeof(int), 0,
                              cudaMemcpyHostToDevice, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess) {
    return vmps::fail(VMPS_ERR_CUDA, "reading the error word failed: %s",
                      cudaGetErrorString(cudaGetLastError()));
  }
  *word_out = host;
  vmps::clear_error();
  return VMPS_OK;
}

}  // extern "C"
