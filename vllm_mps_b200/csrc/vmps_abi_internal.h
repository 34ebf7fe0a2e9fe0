// Host-side helpers shared by the .cu files of libvmps_kernels.so.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/vmps.h"

namespace vmps {

// Records a printf-style message for vmps_last_error() and returns `code`.
int fail(int code, const char* fmt, ...);
void clear_error();
// Turns a pending launch error into VMPS_ERR_CUDA.
int check_launch(const char* what);
// Device address of the error word of the current device (cached per device).
int device_error_word(int** out);
// Number of SMs of the current device (cached per device).
int device_sm_count(int* out);
// cuTensorMapEncodeTiled through the runtime's driver entry point, so the
// library does not link libcuda directly.
int encode_tiled(CUtensorMap* map, CUtensorMapDataType dt, int rank, void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swizzle);

// Bytes at the start of a decode workspace that hold the split-K merge
// counters one call of this shape uses (n_kv * num_seqs ints), or 0 when the
// shape is outside what the decode kernel accepts.
size_t decode_counter_bytes(int num_seqs, int n_kv);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace vmps
