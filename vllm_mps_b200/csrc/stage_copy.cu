// Stage copy: moves a step's inputs from pinned host memory into device
// memory with the GPU's own loads and stores, as one link of a chain of
// kernels launched with programmatic dependent launch (PDL).
//
// A copy-engine memcpy placed between two PDL-chained kernels (in a stream
// or as a CUDA-graph node feeding the second kernel) makes that kernel wait
// for the first one to finish entirely before it may even launch, which
// costs the decode step its launch overlap (measured on a B200: ~17 us per
// config-1 step as a pure PDL chain, ~27 us with an event-ordered copy node
// feeding every step).  This kernel instead starts while the previous
// kernel in the stream still runs (it triggers its dependents at once),
// reads the host buffer over the host link and writes the destination
// without waiting for anything, and only then waits for the previous kernel
// to finish -- so the kernel after it still finds every earlier kernel
// complete.  Its CTAs need no shared memory and few registers, so they fit
// beside a running decode step's CTAs.
#include "vmps_abi_internal.h"
#include "vmps_common.cuh"

namespace vmps {
namespace {

constexpr int kCopyThreads = 256;
constexpr int kCopyUnroll = 4;

__global__ void __launch_bounds__(kCopyThreads)
    stage_copy_kernel(uint4* __restrict__ dst, const uint4* __restrict__ src, size_t n16) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const size_t stride = static_cast<size_t>(gridDim.x) * kCopyThreads;
  size_t i = static_cast<size_t>(blockIdx.x) * kCopyThreads + threadIdx.x;
  // kCopyUnroll independent 16-byte loads in flight per thread: the host
  // link's latency is paid once per round, not once per load.
  for (; i + (kCopyUnroll - 1) * stride < n16; i += kCopyUnroll * stride) {
    uint4 v[kCopyUnroll];
#pragma unroll
    for (int u = 0; u < kCopyUnroll; ++u) v[u] = src[i + u * stride];
#pragma unroll
    for (int u = 0; u < kCopyUnroll; ++u) dst[i + u * stride] = v[u];
  }
  for (; i < n16; i += stride) dst[i] = src[i];
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

}  // namespace
}  // namespace vmps

extern "C" int vmps_stage_copy(void* dst, const void* src, size_t bytes, void* stream) {
  using namespace vmps;
  clear_error();
  if (bytes == 0) return VMPS_OK;
  if (!dst || !src) return fail(VMPS_ERR_INVALID_ARG, "stage_copy: NULL pointer");
  if (!aligned16(dst) || !aligned16(src) || (bytes & 15)) {
    return fail(VMPS_ERR_ALIGNMENT,
                "stage_copy: both pointers must be 16-byte aligned and bytes a multiple of 16");
  }
  int sms = 0;
  if (int rc = device_sm_count(&sms)) return rc;
  const size_t n16 = bytes / 16;
  const size_t per_cta = static_cast<size_t>(kCopyThreads) * kCopyUnroll;
  size_t grid = (n16 + per_cta - 1) / per_cta;
  if (grid > static_cast<size_t>(sms)) grid = static_cast<size_t>(sms);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kCopyThreads);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, stage_copy_kernel, static_cast<uint4*>(dst),
                                           static_cast<const uint4*>(src), n16);
  if (e != cudaSuccess) {
    return fail(VMPS_ERR_CUDA, "stage_copy: launch failed: %s", cudaGetErrorString(e));
  }
  return VMPS_OK;
}
