// Allocation-free variant of vmps_paged_decode_attention.
//
// Who needs it: callers that must not allocate device memory once they are
// running -- e.g. a host binding (Go/Java/C through the C ABI) that has no
// caching allocator and a fixed device-memory budget decided at start-up,
// or a serving process that reserves all free HBM for its KV pool up front,
// so a later cudaMalloc would fail or fragment the pool.  Such callers
// cannot provide the split-K workspace that vmps_paged_decode_attention
// asks for, so this entry point uses a fixed scratch array that lives in
// the library itself.
//
// Limits and sharing rules:
//   * The scratch is one file-scope device array of kNoAllocScratchBytes
//     (8 MiB).  Every GPU on which the library's kernels are loaded holds
//     it until the process exits.
//   * A call whose workspace would exceed it (see
//     vmps_paged_decode_workspace_bytes) is rejected with
//     VMPS_ERR_WORKSPACE before anything is launched.  On a 148-SM B200 this
//     admits every supported shape with up to 8 query heads per kv head
//     (~6 MB: 1 MiB of merge counters plus the split-K partials of the
//     grid) and rejects 16 query heads per kv head (~10.8 MB).
//   * All calls on a device share the array and it keeps the last call's
//     contents.  The kernel's split-K merge counters must be zero when it
//     starts.  A call that completes leaves them at zero, but one whose
//     kernel gave up a bounded wait (error bit 8) can leave some behind, and
//     the caller has no handle on the array to reset it.  So every call
//     first clears the counters it will use -- n_kv * num_seqs ints at the
//     start of the array -- with cudaMemsetAsync on its own stream (a memset,
//     not an allocation); the partial results are always written before
//     they are read.  Calls whose kernels may overlap on the GPU (different
//     streams without ordering) race on the array and must not be issued.
//   * The first call on a device resolves the array's device address with
//     cudaGetSymbolAddress (with that device current) and caches it; make
//     that first call before any stream capture on the device.
//   * Nothing here calls cudaMalloc, cudaFree or any allocating routine.
#include <mutex>

#include "vmps_abi_internal.h"

namespace vmps {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;

static __device__ __align__(256) uint8_t g_decode_scratch[kNoAllocScratchBytes];

// Device address of g_decode_scratch on the current device.  The name is a
// host-side stand-in in host code; only this address may be given to a
// kernel.
static int noalloc_scratch(void** out) {
  static void* cached[64];
  static int status[64];
  static std::once_flag flags[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    return fail(VMPS_ERR_CUDA, "paged_decode_attention_noalloc: cudaGetDevice failed");
  }
  std::call_once(flags[dev], [&] {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
    status[dev] = static_cast<int>(e);
    cached[dev] = (e == cudaSuccess) ? p : nullptr;
  });
  if (!cached[dev]) {
    return fail(VMPS_ERR_CUDA,
                "paged_decode_attention_noalloc: resolving the scratch array failed: %s",
                cudaGetErrorString(static_cast<cudaError_t>(status[dev])));
  }
  *out = cached[dev];
  return VMPS_OK;
}

}  // namespace vmps

extern "C" int vmps_paged_decode_attention_noalloc(void* out, const void* q, const void* pool,
                                                   const int32_t* block_tables,
                                                   int max_blocks_per_seq,
                                                   const int32_t* seq_lens, int num_seqs,
                                                   int n_q, int n_kv, int head_dim,
                                                   int block_size, int num_blocks, float scale,
                                                   int dtype, void* stream) {
  using namespace vmps;
  clear_error();
  if (num_seqs < 0) {
    return fail(VMPS_ERR_INVALID_ARG, "paged_decode_attention_noalloc: num_seqs %d", num_seqs);
  }
  if (num_seqs == 0) return VMPS_OK;
  const size_t need =
      vmps_paged_decode_workspace_bytes(num_seqs, n_q, n_kv, head_dim, dtype);
  if (need == 0) {
    return fail(VMPS_ERR_UNSUPPORTED,
                "paged_decode_attention_noalloc: n_q=%d n_kv=%d head_dim=%d dtype=%d not "
                "supported",
                n_q, n_kv, head_dim, dtype);
  }
  if (need > kNoAllocScratchBytes) {
    return fail(VMPS_ERR_WORKSPACE,
                "paged_decode_attention_noalloc: this call needs %zu bytes of scratch, more "
                "than the library's fixed %zu-byte array (use "
                "vmps_paged_decode_attention with a caller-provided workspace)",
                need, kNoAllocScratchBytes);
  }
  const size_t counter_bytes = decode_counter_bytes(num_seqs, n_kv);
  if (counter_bytes == 0) {
    return fail(VMPS_ERR_UNSUPPORTED,
                "paged_decode_attention_noalloc: num_seqs=%d n_kv=%d outside the kernel's limits",
                num_seqs, n_kv);
  }
  void* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  // Counters left behind by an earlier call that gave up a wait would make
  // this call skip merges; clear the ones it uses.
  const cudaError_t e = cudaMemsetAsync(scratch, 0, counter_bytes, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    return fail(VMPS_ERR_CUDA, "paged_decode_attention_noalloc: clearing the merge counters failed: %s",
                cudaGetErrorString(e));
  }
  return vmps_paged_decode_attention(out, q, pool, block_tables, max_blocks_per_seq, seq_lens,
                                     num_seqs, n_q, n_kv, head_dim, block_size, num_blocks, scale,
                                     scratch, kNoAllocScratchBytes, dtype, stream);
}
