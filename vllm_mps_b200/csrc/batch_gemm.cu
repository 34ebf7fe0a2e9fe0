// Kernel 5: the projections of a decode step at batch sizes 1..256 on the
// sm_100a tensor cores (tcgen05 MMA, TMEM accumulator, TMA-fed rings).
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
//  * Two rings fed by two producer warps with 3-D TMA loads (128-byte
//    swizzle, no multicast): 64-wide K chunks of W (16 KB) in a deep ring
//    (up to 8 stages: the weights come from HBM and need many bytes in
//    flight per SM), chunks of x (Mp x 128 B, rows past M read as zeros) in
//    a shallow one (they come from L2).  The first weight chunks are loaded
//    before the programmatic-dependent-launch wait (weights never depend on
//    the kernel before), x only after it.  Warp 1 (one lane) issues four
//    tcgen05.mma (K = 16 each) per chunk into one TMEM accumulator of Mp
//    fp32 columns and frees both stages with tcgen05.commit.
//  * Split-K over a thread-block cluster of S <= 4 CTAs (same tile, K split
//    in S ranges), S chosen so the whole grid is resident at once
//    (cudaOccupancyMaxActiveClusters).  Each CTA owns 1/S of the batch
//    columns; the others store their fp32 partials of those columns to the
//    caller's workspace, which stays in L2 (coalesced 16-byte stores), one cluster
//    barrier orders them, and the owner adds them to its own accumulator in
//    rank order (deterministic) before rounding.
//  * Warps 3-6 are the epilogue, one thread per output feature (TMEM lane):
//    the rounded results go through shared memory (transposed to batch-row
//    major) and out with TMA tensor stores of 16 x 128 tiles (rows past M
//    are clipped by the TMA).
//
// Every mbarrier wait is bounded (kDevErrTimeout and an abort flag on expiry);
// an aborting CTA still takes the cluster barrier, waits (bounded) for its
// own TMA loads in flight and frees its TMEM.  Calls that may overlap on the
// GPU need different workspaces; a stream's calls never overlap.
#include <type_traits>
#include <mutex>

#include "vmps_abi_internal.h"
#include "vmps_common.cuh"

namespace vmps {
namespace {

constexpr int kBgThreads = 224;  // warp 0 W loads, 1 MMA, 2 x loads, 3-6 epilogue
constexpr int kBgRows = 128;     // output features per CTA (MMA M)
constexpr int kBgWBytes = kBgRows * 128;  // one 64-wide K chunk of W
constexpr int kBgMaxWStages = 8;
constexpr int kBgMaxXStages = 4;
constexpr int kBgSmemLimit = 227 * 1024;
constexpr int kBgBarBytes = 256;
constexpr int kBgMaxSplit = 4;
constexpr int kBgMaxM = 256;     // MMA N limit
constexpr int kBgOutTile = 16 * kBgRows * 2;  // one 16-row output tile (16-bit)
// Split-K workspace: [tile][owner][sender][group][row][16] fp32.  The split
// is chosen so that it needs at most this much.
constexpr size_t kBgScratchFloats = (16u << 20) / 4;

struct BgParams {
  void* out;
  int M, Mp, N, K;
  int kc;      // K / 64 chunks
  int split;   // CTAs per tile (cluster size along x)
  int wstages, xstages;
  int groups;  // Mp / 16 column groups
  int maxg;    // most groups one CTA owns
  uint32_t tmem_cols;
  float* scratch;  // the caller's workspace (split > 1)
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
// 2-D TMA tensor store of one shared-memory tile (bulk-group completion).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0,
                                             int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(c0), "r"(c1)
      : "memory");
}

}  // namespace
}  // namespace vmps

namespace vmps {
namespace {

template <typename T>
__global__ void __launch_bounds__(kBgThreads, 1)
    batch_gemm_kernel(const __grid_constant__ CUtensorMap wmap,
                      const __grid_constant__ CUtensorMap xmap,
                      const __grid_constant__ CUtensorMap omap, const BgParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.split;
  const int rank = S > 1 ? static_cast<int>(cluster_rank()) : 0;
  const int tile = static_cast<int>(blockIdx.y);
  const int n0 = tile * kBgRows;
  const int c_begin = rank * p.kc / S;
  const int nch = (rank + 1) * p.kc / S - c_begin;
  const uint32_t xbytes = static_cast<uint32_t>(p.Mp) * 128u;
  // The swizzled tiles need 1024-byte alignment: the window carries 1 KB of
  // slack.
  uint8_t* wring = smem + ((1024u - (smem_u32(smem) & 1023u)) & 1023u);
  uint8_t* xring = wring + p.wstages * kBgWBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(xring + p.xstages * xbytes);
  uint64_t* w_full = bars;
  uint64_t* w_empty = bars + kBgMaxWStages;
  uint64_t* x_full = bars + 2 * kBgMaxWStages;
  uint64_t* x_empty = x_full + kBgMaxXStages;
  uint64_t* mma_done = x_empty + kBgMaxXStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kBgMaxWStages; ++s) {
      mbar_init(w_full + s, 1);
      mbar_init(w_empty + s, 1);
    }
    for (int s = 0; s < kBgMaxXStages; ++s) {
      mbar_init(x_full + s, 1);
      mbar_init(x_empty + s, 1);
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

  if (warp == 0 || warp == 2) {
    // ── producers: warp 0 the weights (before and after the PDL wait), warp 2
    // the activations (after it) ─────────────────────────────────────────────
    if (lane == 0) {
      const bool is_w = warp == 0;
      const int stages = is_w ? p.wstages : p.xstages;
      const uint32_t bytes = is_w ? static_cast<uint32_t>(kBgWBytes) : xbytes;
      uint64_t* full = is_w ? w_full : x_full;
      uint64_t* empty = is_w ? w_empty : x_empty;
      uint8_t* ring = is_w ? wring : xring;
      const CUtensorMap* map = is_w ? &wmap : &xmap;
      prefetch_tmap(map);
      if (!is_w) {
        // x may be the output of the kernel before this one.
        asm volatile("griddepcontrol.wait;" ::: "memory");
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
      }
      int issued = 0;
      for (int i = 0; i < nch; ++i) {
        const int s = i % stages;
        if (i >= stages &&
            !mbar_wait(empty + s, static_cast<uint32_t>((i / stages) - 1) & 1u, p.err)) {
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        mbar_arrive_expect_tx(full + s, bytes);
        tma_load_3d(ring + static_cast<size_t>(s) * bytes, map, full + s, 0, is_w ? n0 : 0,
                    c_begin + i);
        issued = i + 1;
      }
      // Never leave with a load in flight: wait (bounded) for the last load
      // issued into each stage.
      for (int i = issued - stages > 0 ? issued - stages : 0; i < issued; ++i) {
        mbar_wait(full + (i % stages), static_cast<uint32_t>(i / stages) & 1u, p.err);
      }
    }
  } else if (warp == 1) {
    // ── MMA issue (one lane) ────────────────────────────────────────────────
    if (lane == 0) {
      const uint32_t idesc = bg_idesc<T>(p.Mp);
      for (int i = 0; i < nch && !*abort_flag; ++i) {
        const int sw = i % p.wstages, sx = i % p.xstages;
        if (!mbar_wait(w_full + sw, static_cast<uint32_t>(i / p.wstages) & 1u, p.err) ||
            !mbar_wait(x_full + sx, static_cast<uint32_t>(i / p.xstages) & 1u, p.err)) {
          *abort_flag = 1;
          break;
        }
        bg_fence_after();
        const uint32_t w_addr = smem_u32(wring + static_cast<size_t>(sw) * kBgWBytes);
        const uint32_t x_addr = smem_u32(xring + static_cast<size_t>(sx) * xbytes);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          bg_mma(tmem_base, bg_desc(w_addr + k * 32), bg_desc(x_addr + k * 32), idesc,
                 (i > 0 || k > 0) ? 1u : 0u);
        }
        bg_commit(w_empty + sw);  // the stages are free once these MMAs have read them
        bg_commit(x_empty + sx);
      }
      bg_commit(mma_done);  // arrives when every MMA issued above is complete
    }
  } else {
    // Epilogue warps: the output may still be read by the kernel before this
    // one until the dependency wait returns.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (!mbar_wait(mma_done, 0, p.err)) *abort_flag = 1;
    bg_fence_after();
  }
  __syncwarp();

  // ── epilogue (warps 3-6) and the split-K reduction ───────────────────────
  const bool epi = warp >= 3;
  const int quarter = warp & 3;  // the TMEM lane quarter this warp may access
  const int row = quarter * 32 + lane;
  const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
  const int G = p.groups;
  // Scratch slot of (owner d, sender slot q, owner-local group gi): 128 rows x 16.
  auto slot = [&](int d, int q, int gi) {
    return p.scratch +
           ((((static_cast<size_t>(tile) * S + d) * (S - 1) + q) * p.maxg + gi) * kBgRows + row) * 16;
  };
  if (S > 1) {
    if (epi) {
      for (int d = 0; d < S; ++d) {
        if (d == rank) continue;
        const int gb = d * G / S, ge = (d + 1) * G / S;
        const int q = rank < d ? rank : rank - 1;
        for (int g = gb; g < ge; ++g) {
          float v[16];
          bg_ld16(t_row + g * 16, v);
          float4* o = reinterpret_cast<float4*>(slot(d, q, g - gb));
#pragma unroll
          for (int j = 0; j < 4; ++j) __stcg(o + j, make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]));
        }
      }
    }
    // Every partial of every CTA in the cluster is in the scratch area.
    cluster_sync_all();
  }
  if (epi) {
    const int gb = rank * G / S, ge = (rank + 1) * G / S;
    // The weight ring is free (every MMA has completed): stage the rounded
    // 16 x 128 output tiles there, batch-row major.
    for (int g = gb; g < ge; ++g) {
      float own[16], acc[16];
      bg_ld16(t_row + g * 16, own);
#pragma unroll
      for (int j = 0; j < 16; ++j) acc[j] = 0.f;
      // Sum in rank order, so the result does not depend on arrival order.
      for (int src = 0; src < S; ++src) {
        if (src == rank) {
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[j] += own[j];
        } else {
          const float4* sp =
              reinterpret_cast<const float4*>(slot(rank, src < rank ? src : src - 1, g - gb));
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float4 f = __ldcg(sp + j);
            acc[4 * j] += f.x;
            acc[4 * j + 1] += f.y;
            acc[4 * j + 2] += f.z;
            acc[4 * j + 3] += f.w;
          }
        }
      }
      T* tp = reinterpret_cast<T*>(wring + static_cast<size_t>(g - gb) * kBgOutTile);
#pragma unroll
      for (int j = 0; j < 16; ++j) tp[j * kBgRows + row] = Elt<T>::from_f(acc[j]);
    }
    // Make the generic-proxy stores visible to the TMA, then one thread
    // stores every tile of this CTA (rows past M are clipped).
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    named_barrier_sync(1, 128);
    if (warp == 3 && lane == 0) {
      for (int g = gb; g < ge && g * 16 < p.M; ++g) {
        tma_store_2d(&omap, wring + static_cast<size_t>(g - gb) * kBgOutTile, n0, g * 16);
      }
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
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
  int Mp, groups, split, wstages, xstages, maxg;
  uint32_t tmem_cols;
  size_t smem;
  size_t scratch_bytes;  // split-K partials: the workspace a call needs
};

size_t bg_smem_bytes(int wstages, int xstages, int Mp) {
  return 1024 + static_cast<size_t>(wstages) * kBgWBytes +
         static_cast<size_t>(xstages) * Mp * 128 + kBgBarBytes;
}

template <typename T>
void bg_set_smem_attr() {
  static std::once_flag flags[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return;
  std::call_once(flags[dev], [] {
    cudaFuncSetAttribute(batch_gemm_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kBgSmemLimit);
  });
}

// Clusters of `split` CTAs of this configuration that fit on the device at
// once (cached per device, dtype, batch group count and split).
template <typename T>
int bg_max_clusters(int split, int Mp, size_t smem) {
  static int cache[64][2][17][kBgMaxSplit + 1];
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 0;
  const int ti = std::is_same<T, __half>::value ? 0 : 1;
  std::lock_guard<std::mutex> lock(mu);
  int& c = cache[dev][ti][Mp / 16][split];
  if (c == 0) {
    bg_set_smem_attr<T>();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(split, 1);
    cfg.blockDim = dim3(kBgThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute a[1];
    a[0].id = cudaLaunchAttributeClusterDimension;
    a[0].val.clusterDim.x = static_cast<unsigned>(split);
    a[0].val.clusterDim.y = 1;
    a[0].val.clusterDim.z = 1;
    cfg.attrs = a;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, batch_gemm_kernel<T>, &cfg) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    c = n > 0 ? n : -1;
  }
  return c > 0 ? c : 0;
}

// Rings: x in 2-4 stages of Mp x 128 B, W in as many 16 KB stages as fit (up
// to 8).  Split: the largest S <= 4 (each CTA keeping at least four K chunks)
// whose grid of clusters fits on the device at once and whose partials fit
// in kBgScratchFloats; otherwise none.
template <typename T>
bool bg_plan(int M, int N, int K, BgPlan* pl) {
  if (M < 1 || M > kBgMaxM || N < kBgRows || N % kBgRows || K < 64 || K % 64) return false;
  const int Mp = (M + 15) / 16 * 16;
  const int tiles = N / kBgRows, kc = K / 64, groups = Mp / 16;
  // x chunks are Mp / 128 times a weight chunk: at large batches they need
  // as many stages in flight as the weights.
  const int xstages = Mp > 128 ? 4 : (Mp > 64 ? 3 : 4);
  const size_t avail = kBgSmemLimit - bg_smem_bytes(0, xstages, Mp);
  int wstages = static_cast<int>(avail / kBgWBytes);
  if (wstages > kBgMaxWStages) wstages = kBgMaxWStages;
  // The ring must hold the staged output tiles (at most 16 x 4 KB).
  if (wstages < 4) return false;
  const size_t smem = bg_smem_bytes(wstages, xstages, Mp);
  int split = 1;
  for (int s = (kc / 4 < kBgMaxSplit ? kc / 4 : kBgMaxSplit); s > 1; --s) {
    const int maxg = (groups + s - 1) / s;
    const size_t scratch = static_cast<size_t>(tiles) * s * (s - 1) * maxg * kBgRows * 16;
    if (scratch > kBgScratchFloats) continue;
    if (bg_max_clusters<T>(s, Mp, smem) >= tiles) {
      split = s;
      break;
    }
  }
  uint32_t cols = 32;
  while (cols < static_cast<uint32_t>(Mp)) cols <<= 1;
  pl->Mp = Mp;
  pl->groups = groups;
  pl->split = split;
  pl->wstages = wstages;
  pl->xstages = xstages;
  pl->maxg = (groups + split - 1) / split;
  pl->tmem_cols = cols;
  pl->smem = smem;
  pl->scratch_bytes = split > 1 ? static_cast<size_t>(tiles) * split * (split - 1) * pl->maxg *
                                      kBgRows * 16 * sizeof(float)
                                : 0;
  return true;
}

template <typename T>
cudaError_t bg_launch(const CUtensorMap& wmap, const CUtensorMap& xmap, const CUtensorMap& omap,
                      const BgParams& p, dim3 grid, size_t smem, cudaStream_t s) {
  bg_set_smem_attr<T>();
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
  return cudaLaunchKernelEx(&cfg, batch_gemm_kernel<T>, wmap, xmap, omap, p);
}

}  // namespace
}  // namespace vmps

using namespace vmps;

extern "C" int vmps_batch_gemm_split(int M, int N, int K) {
  BgPlan pl;
  return bg_plan<__nv_bfloat16>(M, N, K, &pl) ? pl.split : 0;
}

extern "C" size_t vmps_batch_gemm_workspace_bytes(int M, int N, int K, int dtype) {
  BgPlan pl;
  if (dtype == VMPS_DTYPE_F16) return bg_plan<__half>(M, N, K, &pl) ? pl.scratch_bytes : 0;
  if (dtype == VMPS_DTYPE_BF16) return bg_plan<__nv_bfloat16>(M, N, K, &pl) ? pl.scratch_bytes : 0;
  return 0;
}

extern "C" int vmps_batch_gemm(void* out, int64_t out_row_stride, const void* x,
                               int64_t x_row_stride, const void* w, int M, int N, int K,
                               void* workspace, size_t workspace_bytes, int dtype, void* stream) {
  clear_error();
  if (dtype != VMPS_DTYPE_F16 && dtype != VMPS_DTYPE_BF16) {
    return fail(VMPS_ERR_INVALID_ARG, "batch_gemm: dtype %d", dtype);
  }
  BgPlan pl;
  const bool ok = dtype == VMPS_DTYPE_F16 ? bg_plan<__half>(M, N, K, &pl)
                                          : bg_plan<__nv_bfloat16>(M, N, K, &pl);
  if (!ok) {
    return fail(VMPS_ERR_UNSUPPORTED,
                "batch_gemm: M=%d N=%d K=%d (1 <= M <= %d, N %% 128 == 0, K %% 64 == 0)", M, N, K,
                kBgMaxM);
  }
  if (pl.scratch_bytes > 0 && (!workspace || workspace_bytes < pl.scratch_bytes ||
                               !aligned16(workspace))) {
    return fail(VMPS_ERR_WORKSPACE,
                "batch_gemm: this shape splits K over %d CTAs and needs a 16-byte aligned "
                "workspace of %zu bytes (got %zu; see vmps_batch_gemm_workspace_bytes)",
                pl.split, pl.scratch_bytes, workspace ? workspace_bytes : size_t(0));
  }
  if (!out || !x || !w) return fail(VMPS_ERR_INVALID_ARG, "batch_gemm: NULL pointer");
  if (!aligned16(x) || !aligned16(w) || !aligned16(out) || (x_row_stride % 8) || x_row_stride < K ||
      (out_row_stride % 8) || out_row_stride < N) {
    return fail(VMPS_ERR_ALIGNMENT,
                "batch_gemm: x, w and out 16-byte aligned, x and out rows a multiple of 8 "
                "elements apart (x rows at least K, out rows at least N)");
  }
  const CUtensorMapDataType tdt =
      dtype == VMPS_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const int kc = K / 64;
  CUtensorMap wmap, xmap, omap;
  // W as {64 elements, row, 64-column chunk}: a box is 128 rows of one chunk.
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
  // out as {feature, batch row}: a box is one 16-row x 128-feature tile.
  {
    const uint64_t dims[2] = {(uint64_t)N, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)out_row_stride * 2};
    const uint32_t box[2] = {(uint32_t)kBgRows, 16};
    if (int rc = encode_tiled(&omap, tdt, 2, out, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE)) {
      return rc;
    }
  }
  int* err = nullptr;
  if (int rc = device_error_word(&err)) return rc;
  BgParams p;
  p.out = out;
  p.M = M;
  p.Mp = pl.Mp;
  p.N = N;
  p.K = K;
  p.kc = kc;
  p.split = pl.split;
  p.wstages = pl.wstages;
  p.xstages = pl.xstages;
  p.groups = pl.groups;
  p.maxg = pl.maxg;
  p.tmem_cols = pl.tmem_cols;
  p.scratch = static_cast<float*>(workspace);
  p.err = err;
  const dim3 grid(pl.split, N / kBgRows);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const cudaError_t e = dtype == VMPS_DTYPE_F16
                            ? bg_launch<__half>(wmap, xmap, omap, p, grid, pl.smem, s)
                            : bg_launch<__nv_bfloat16>(wmap, xmap, omap, p, grid, pl.smem, s);
  if (e != cudaSuccess) {
    return fail(VMPS_ERR_CUDA, "batch_gemm: launch failed: %s", cudaGetErrorString(e));
  }
  return VMPS_OK;
}
