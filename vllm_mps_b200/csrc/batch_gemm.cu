// Kernel 5: the projections of a decode step at batch sizes 16..256 on the
// sm_100a tensor cores (tcgen05 MMA, TMEM accumulator, TMA-fed ring).
//
// out[M, N] = x[M, K] . w[N, K]^T, 16-bit inputs, fp32 accumulation, one
// rounding to the 16-bit type (the nn.Linear the reference's HF decoder
// layers run, models/llama_adapter.py:137-207, at the engine's batch).
//
// At M = 256 these GEMMs sit at the B200's ridge point (2 M FLOP per 2-byte
// weight ~ 256 FLOP/B against ~251 for the measured peaks), and the narrow
// ones (QKV, O, down of Llama-3-8B: 32-48 tiles of 128 output features) give
// too few tiles for 148 SMs unless K is split.  The design:
//
//  * Swap AB: the MMA's M (128) runs over output features (weight rows, K-
//    major), its N over the batch (x rows, K-major, N = M rounded up to 16),
//    so one CTA's tile is 128 features x the whole batch and the weights --
//    the HBM traffic -- are read exactly once.
//  * Warp 0 streams 64-wide K chunks of W (16 KB) and x (Mp x 128 B) into a
//    3-4 stage ring with 3-D TMA loads (128-byte swizzle, rows of x past M
//    read as zeros); the first stages' weight loads are issued before the
//    programmatic-dependent-launch wait (weights never depend on the kernel
//    before), the x loads after it.  Warp 1 (one lane) issues four
//    tcgen05.mma (K = 16 each) per chunk into one TMEM accumulator of Mp
//    fp32 columns and frees each stage with tcgen05.commit.
//  * Split-K over a thread-block cluster of S CTAs (same tile, K split in S
//    ranges), reduced through distributed shared memory: when every CTA's
//    MMAs are done (cluster barrier), each CTA owns 1/S of the batch columns
//    and the others write their fp32 partials of those columns straight
//    into its freed ring (st.shared::cluster); after a second cluster
//    barrier each CTA adds them to its own accumulator in rank order and
//    stores the rounded result.  No partial tile touches HBM.
//  * Warps 2-5 are the epilogue: one thread per output feature (TMEM lane),
//    16 batch columns per tcgen05.ld.
//
// Every mbarrier wait is bounded (kDevErrTimeout and an abort flag on expiry);
// an aborting CTA still takes both cluster barriers, waits (bounded) for its
// own TMA loads in flight and frees its TMEM.  No TMA multicast.
#include <type_traits>
#include <mutex>

#include "vmps_abi_internal.h"
#include "vmps_common.cuh"

namespace vmps {
namespace {

constexpr int kBgThreads = 192;  // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int kBgRows = 128;     // output features per CTA (MMA M)
constexpr int kBgWBytes = kBgRows * 128;  // one 64-wide K chunk of W
constexpr int kBgMaxStages = 4;
constexpr int kBgSmemLimit = 227 * 1024;
constexpr int kBgBarBytes = 256;
constexpr int kBgMaxSplit = 8;   // portable cluster size
constexpr int kBgMaxM = 256;     // MMA N limit

struct BgParams {
  void* out;
  int64_t out_stride;
  int M, Mp, N, K;
  int kc;      // K / 64 chunks
  int split;   // CTAs per tile (cluster size along x)
  int stages;
  int groups;  // Mp / 16 column groups
  int recv_row_floats;  // row stride of a received partial slot
  uint32_t tmem_cols;
  int* err;
};

__device__ __forceinline__ void bg_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void bg_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void bg_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void bg_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n"
      "}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void bg_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// 128-byte-swizzled K-major operand: 8-row atoms 1024 bytes apart.
__device__ __forceinline__ uint64_t bg_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(16 >> 4) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}
// kind::f16, fp32 accumulation, A and B K-major, M = 128, N = n.
template <typename T>
__device__ __forceinline__ uint32_t bg_idesc(int n) {
  const uint32_t fmt = std::is_same<T, __half>::value ? 0u : 1u;
  return (1u << 4) | (fmt << 7) | (fmt << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(kBgRows >> 4) << 24);
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b),
               "f"(c), "f"(d)
               : "memory");
}

}  // namespace
}  // namespace vmps

namespace vmps {
namespace {

template <typename T>
__global__ void __launch_bounds__(kBgThreads, 1)
    batch_gemm_kernel(const __grid_constant__ CUtensorMap wmap,
                      const __grid_constant__ CUtensorMap xmap, const BgParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.split;
  const uint32_t rank = S > 1 ? cluster_rank() : 0u;
  const int n0 = static_cast<int>(blockIdx.y) * kBgRows;
  const int c_begin = static_cast<int>((static_cast<long long>(rank) * p.kc) / S);
  const int c_end = static_cast<int>((static_cast<long long>(rank + 1) * p.kc) / S);
  const int nch = c_end - c_begin;
  const uint32_t xbytes = static_cast<uint32_t>(p.Mp) * 128u;
  const uint32_t stage_bytes = kBgWBytes + xbytes;
  // The swizzled tiles need 1024-byte alignment: the window carries 1 KB of
  // slack (the same offset in every CTA, so ring addresses map across the
  // cluster).
  uint8_t* ring = smem + ((1024u - (smem_u32(smem) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + p.stages * stage_bytes);
  uint64_t* empty = full + kBgMaxStages;
  uint64_t* mma_done = empty + kBgMaxStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kBgMaxStages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(p.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  bg_fence_before();
  __syncthreads();
  bg_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ── TMA producer ────────────────────────────────────────────────────────
    if (lane == 0) {
      int issued = 0;
      if (!*abort_flag) {
        prefetch_tmap(&wmap);
        prefetch_tmap(&xmap);
        const int pre = nch < p.stages ? nch : p.stages;
        for (int i = 0; i < pre; ++i) {
          mbar_arrive_expect_tx(full + i, stage_bytes);
          tma_load_3d(ring + i * stage_bytes, &wmap, full + i, 0, n0, c_begin + i);
        }
        // x may be the output of the kernel before this one.
        asm volatile("griddepcontrol.wait;" ::: "memory");
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
        for (int i = 0; i < pre; ++i) {
          tma_load_3d(ring + i * stage_bytes + kBgWBytes, &xmap, full + i, 0, 0, c_begin + i);
        }
        issued = pre;
        for (int i = pre; i < nch; ++i) {
          const int s = i % p.stages;
          if (!mbar_wait(empty + s, static_cast<uint32_t>((i / p.stages) - 1) & 1u, p.err)) {
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(full + s, stage_bytes);
          tma_load_3d(ring + s * stage_bytes, &wmap, full + s, 0, n0, c_begin + i);
          tma_load_3d(ring + s * stage_bytes + kBgWBytes, &xmap, full + s, 0, 0, c_begin + i);
          issued = i + 1;
        }
      }
      // Never leave with a load in flight: wait (bounded) for the last load
      // issued into each stage.
      for (int i = issued - p.stages > 0 ? issued - p.stages : 0; i < issued; ++i) {
        mbar_wait(full + (i % p.stages), static_cast<uint32_t>(i / p.stages) & 1u, p.err);
      }
    }
  } else if (warp == 1) {
    // ── MMA issue (one lane) ────────────────────────────────────────────────
    if (lane == 0) {
      const uint32_t idesc = bg_idesc<T>(p.Mp);
      for (int i = 0; i < nch && !*abort_flag; ++i) {
        const int s = i % p.stages;
        if (!mbar_wait(full + s, static_cast<uint32_t>(i / p.stages) & 1u, p.err)) {
          *abort_flag = 1;
          break;
        }
        bg_fence_after();
        const uint32_t w_addr = smem_u32(ring + s * stage_bytes);
        const uint32_t x_addr = w_addr + kBgWBytes;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          bg_mma(tmem_base, bg_desc(w_addr + k * 32), bg_desc(x_addr + k * 32), idesc,
                 (i > 0 || k > 0) ? 1u : 0u);
        }
        bg_commit(empty + s);  // the stage is free once these MMAs have read it
      }
      bg_commit(mma_done);  // arrives when every MMA issued above is complete
    }
  } else {
    // Epilogue threads: wait for the accumulator (the output may still be
    // read by the kernel before this one until the dependency wait returns).
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (!mbar_wait(mma_done, 0, p.err)) *abort_flag = 1;
    bg_fence_after();
  }
  __syncwarp();

  // ── epilogue (warps 2-5) and the split-K reduction ───────────────────────
  const bool epi = warp >= 2;
  const int quarter = warp & 3;  // the TMEM lane quarter this warp may access
  const int row = quarter * 32 + lane;
  const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
  const int G = p.groups;
  T* outp = static_cast<T*>(p.out) + static_cast<size_t>(n0 + row);
  auto store16 = [&](int g, const float (&v)[16]) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int b = g * 16 + j;
      if (b < p.M) outp[static_cast<size_t>(b) * p.out_stride] = Elt<T>::from_f(v[j]);
    }
  };
  if (S == 1) {
    if (epi) {
      for (int g = 0; g < G; ++g) {
        float v[16];
        bg_ld16(t_row + g * 16, v);
        store16(g, v);
      }
    }
  } else {
    // Every CTA of the cluster is past its MMAs and its loads: all rings free.
    cluster_sync_all();
    if (epi) {
      // Send this CTA's partial of every other CTA's columns into that CTA's
      // ring: slot q (senders in rank order, the receiver skipped), row, 16
      // floats per column group.
      for (int d = 0; d < S; ++d) {
        if (d == static_cast<int>(rank)) continue;
        const int gb = d * G / S, ge = (d + 1) * G / S;
        const int q = static_cast<int>(rank) < d ? static_cast<int>(rank) : static_cast<int>(rank) - 1;
        const uint32_t base = map_to_rank(smem_u32(ring), static_cast<uint32_t>(d)) +
                              static_cast<uint32_t>((q * kBgRows + row) * p.recv_row_floats) * 4u;
        for (int g = gb; g < ge; ++g) {
          float v[16];
          bg_ld16(t_row + g * 16, v);
          const uint32_t a = base + static_cast<uint32_t>(g - gb) * 64u;
#pragma unroll
          for (int j = 0; j < 16; j += 4) st_cluster_v4(a + j * 4, v[j], v[j + 1], v[j + 2], v[j + 3]);
        }
      }
    }
    // Every partial of this CTA's columns has arrived.
    cluster_sync_all();
    if (epi) {
      const int gb = static_cast<int>(rank) * G / S, ge = (static_cast<int>(rank) + 1) * G / S;
      for (int g = gb; g < ge; ++g) {
        float own[16], acc[16];
        bg_ld16(t_row + g * 16, own);
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[j] = 0.f;
        // Sum in rank order, so the result does not depend on arrival order.
        for (int src = 0; src < S; ++src) {
          if (src == static_cast<int>(rank)) {
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[j] += own[j];
          } else {
            const int q = src < static_cast<int>(rank) ? src : src - 1;
            const float4* slot = reinterpret_cast<const float4*>(
                ring + static_cast<size_t>((q * kBgRows + row) * p.recv_row_floats + (g - gb) * 16) * 4);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float4 f = slot[j];
              acc[4 * j] += f.x;
              acc[4 * j + 1] += f.y;
              acc[4 * j + 2] += f.z;
              acc[4 * j + 3] += f.w;
            }
          }
        }
        store16(g, acc);
      }
    }
  }

  // Free the accumulator once every TMEM read is done.
  bg_fence_before();
  __syncthreads();
  if (warp == 1) {
    bg_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(p.tmem_cols)
                 : "memory");
  }
}

}  // namespace
}  // namespace vmps

// ── host side ────────────────────────────────────────────────────────────────

namespace vmps {
namespace {

struct BgPlan {
  int Mp, groups, split, stages, recv_row_floats;
  uint32_t tmem_cols;
  size_t smem;
};

// Split: enough CTAs for one wave over the SMs (at most 8 per cluster, at
// least two K chunks each); stages: as many 48 KB-or-smaller stages as fit,
// up to 4; the ring must also hold the partials a CTA receives.
bool bg_plan(int M, int N, int K, int sms, BgPlan* pl) {
  if (M < 1 || M > kBgMaxM || N < kBgRows || N % kBgRows || K < 64 || K % 64) return false;
  const int Mp = (M + 15) / 16 * 16;
  const int tiles = N / kBgRows, kc = K / 64;
  const size_t stage_bytes = kBgWBytes + static_cast<size_t>(Mp) * 128;
  const size_t avail = kBgSmemLimit - 1024 - kBgBarBytes;
  int stages = static_cast<int>(avail / stage_bytes);
  if (stages > kBgMaxStages) stages = kBgMaxStages;
  if (stages < 2) return false;
  int split = sms / tiles;
  if (split > kBgMaxSplit) split = kBgMaxSplit;
  if (split > kc / 2) split = kc / 2;
  if (split < 1) split = 1;
  const int groups = Mp / 16;
  int rf = 0;
  for (; split > 1; --split) {
    rf = ((groups + split - 1) / split) * 16 + 4;
    const size_t recv = static_cast<size_t>(split - 1) * kBgRows * rf * 4;
    if (recv <= static_cast<size_t>(stages) * stage_bytes) break;
  }
  uint32_t cols = 32;
  while (cols < static_cast<uint32_t>(Mp)) cols <<= 1;
  pl->Mp = Mp;
  pl->groups = groups;
  pl->split = split;
  pl->stages = stages;
  pl->recv_row_floats = split > 1 ? rf : 0;
  pl->tmem_cols = cols;
  pl->smem = 1024 + static_cast<size_t>(stages) * stage_bytes + kBgBarBytes;
  return true;
}

template <typename T>
cudaError_t bg_launch(const CUtensorMap& wmap, const CUtensorMap& xmap, const BgParams& p,
                      dim3 grid, size_t smem, cudaStream_t s) {
  static std::once_flag flags[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64) {
    std::call_once(flags[dev], [] {
      cudaFuncSetAttribute(batch_gemm_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kBgSmemLimit);
    });
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kBgThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int n = 0;
  attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[n].val.programmaticStreamSerializationAllowed = 1;
  ++n;
  if (p.split > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = static_cast<unsigned>(p.split);
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, batch_gemm_kernel<T>, wmap, xmap, p);
}

}  // namespace
}  // namespace vmps

using namespace vmps;

extern "C" int vmps_batch_gemm_split(int M, int N, int K) {
  int sms = 0;
  if (device_sm_count(&sms)) return 0;
  BgPlan pl;
  return bg_plan(M, N, K, sms, &pl) ? pl.split : 0;
}

extern "C" int vmps_batch_gemm(void* out, int64_t out_row_stride, const void* x,
                               int64_t x_row_stride, const void* w, int M, int N, int K, int dtype,
                               void* stream) {
  clear_error();
  int sms = 0;
  if (int rc = device_sm_count(&sms)) return rc;
  BgPlan pl;
  if (!bg_plan(M, N, K, sms, &pl)) {
    return fail(VMPS_ERR_UNSUPPORTED,
                "batch_gemm: M=%d N=%d K=%d (1 <= M <= %d, N %% 128 == 0, K %% 64 == 0)", M, N, K,
                kBgMaxM);
  }
  if (!out || !x || !w) return fail(VMPS_ERR_INVALID_ARG, "batch_gemm: NULL pointer");
  if (dtype != VMPS_DTYPE_F16 && dtype != VMPS_DTYPE_BF16) {
    return fail(VMPS_ERR_INVALID_ARG, "batch_gemm: dtype %d", dtype);
  }
  if (!aligned16(x) || !aligned16(w) || (x_row_stride % 8) || x_row_stride < K ||
      (reinterpret_cast<uintptr_t>(out) & 1) || out_row_stride < N) {
    return fail(VMPS_ERR_ALIGNMENT,
                "batch_gemm: x and w 16-byte aligned, x rows a multiple of 8 elements apart, "
                "out rows at least N apart");
  }
  const CUtensorMapDataType tdt =
      dtype == VMPS_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const int kc = K / 64;
  // W as {64 elements, row, 64-column chunk}: a box is 128 rows of one chunk.
  CUtensorMap wmap, xmap;
  {
    const uint64_t dims[3] = {64, (uint64_t)N, (uint64_t)kc};
    const uint64_t strides[2] = {(uint64_t)K * 2, 128};
    const uint32_t box[3] = {64, (uint32_t)kBgRows, 1};
    if (int rc = encode_tiled(&wmap, tdt, 3, const_cast<void*>(w), dims, strides, box,
                              CU_TENSOR_MAP_SWIZZLE_128B)) {
      return rc;
    }
  }
  // x the same way; a box is Mp rows (rows past M read as zeros).
  {
    const uint64_t dims[3] = {64, (uint64_t)M, (uint64_t)kc};
    const uint64_t strides[2] = {(uint64_t)x_row_stride * 2, 128};
    const uint32_t box[3] = {64, (uint32_t)pl.Mp, 1};
    if (int rc = encode_tiled(&xmap, tdt, 3, const_cast<void*>(x), dims, strides, box,
                              CU_TENSOR_MAP_SWIZZLE_128B)) {
      return rc;
    }
  }
  int* err = nullptr;
  if (int rc = device_error_word(&err)) return rc;
  BgParams p;
  p.out = out;
  p.out_stride = out_row_stride;
  p.M = M;
  p.Mp = pl.Mp;
  p.N = N;
  p.K = K;
  p.kc = kc;
  p.split = pl.split;
  p.stages = pl.stages;
  p.groups = pl.groups;
  p.recv_row_floats = pl.recv_row_floats;
  p.tmem_cols = pl.tmem_cols;
  p.err = err;
  const dim3 grid(pl.split, N / kBgRows);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const cudaError_t e = dtype == VMPS_DTYPE_F16
                            ? bg_launch<__half>(wmap, xmap, p, grid, pl.smem, s)
                            : bg_launch<__nv_bfloat16>(wmap, xmap, p, grid, pl.smem, s);
  if (e != cudaSuccess) {
    return fail(VMPS_ERR_CUDA, "batch_gemm: launch failed: %s", cudaGetErrorString(e));
  }
  return VMPS_OK;
}
