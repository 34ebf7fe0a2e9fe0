// Decode GEMM: Y[M, N] = X[M, K] . W[N, K]^T for the small batches of a
// decode step (M <= 8), optionally with the gated-MLP epilogue
// Y[M, I] = silu(X . Wg^T) * (X . Wu^T) on a fused [gate; up] weight.
//
// These are the projections of the Llama decoder layer around the paged
// attention step (transformers LlamaAttention q/k/v/o_proj, LlamaMLP
// gate/up/down_proj; the reference runs them as nn.Linear through
// models/llama_adapter.py:137-207).  At decode batch sizes a projection
// reads every weight once and does 2*M FLOPs per weight: it is bound by the
// weight stream from HBM, and cuBLAS's small-M kernels reach only 1.2-1.6 TB/s
// on these shapes (TinyLlama QKV, O and down projections on a B200).
//
// Design (B200):
//  * Work unit = a row block of 16 output features (with the gated epilogue,
//    16 gate rows and the matching 16 up rows) over the whole K: no split-K, so
//    no partial sums and no merge round trips.  Row blocks are dealt out in
//    contiguous, equal shares to one persistent CTA per SM.
//  * A producer warp streams the weight rows with the tiled TMA
//    (cp.async.bulk.tensor, no multicast): one 32 KiB box = 16 rows x 1024 K
//    as 128-byte swizzled chunks, into a ring of 2-6 stages.  The row pieces
//    of a box must be long: boxes of 8 rows x 1 KiB streamed at 3.9 TB/s
//    (without the math), 8 x 4 KiB at 6.2 and 16 x 2 KiB at 6.3.
//  * The weights never depend on the previous kernel, so the producer starts
//    streaming them before the programmatic-dependent-launch wait: under PDL
//    the ring fills while the previous kernel finishes.  Only the consumers
//    wait, then stage X (M x K, at most 8 rows) in shared memory once.
//  * Eight consumer warps split each stage by 64-column chunks (two
//    accumulator chains each; two warps per scheduler, so MMA and
//    shared-memory latencies overlap).  mma.m16n8k16 with 16 weight rows as
//    the A side and the batch (up to 8) as the n8 B side: D[feature][batch],
//    no padded rows.  Each warp hands its partial sums of a row block to
//    a dedicated epilogue warp through two mbarrier-guarded shared-memory
//    slots, so no consumer waits for the adds and stores.
//  * The epilogue keeps the modules' rounding points: each projection's
//    result is rounded to the 16-bit type; the gated form computes
//    round(round(silu(g)) * u) from the rounded g and u (LlamaMLP:
//    act_fn(gate_proj(x)) * up_proj(x)).
#include <mutex>

#include "vmps_abi_internal.h"
#include "vmps_common.cuh"

namespace vmps {
namespace {

constexpr int kGemmRows = 16;         // output features per row block (the mma's 16-row A side)
#ifndef VMPS_GEMM_KTILE
#define VMPS_GEMM_KTILE 1024
#endif
constexpr int kGemmKTile = VMPS_GEMM_KTILE;  // K per stage, in chunks of 64 elements
constexpr int kGemmStageBytes = kGemmRows * kGemmKTile * 2;
constexpr int kGemmConsumers = 8;
constexpr int kGemmChunksPerWarp = kGemmKTile / 64 / kGemmConsumers;
static_assert(kGemmChunksPerWarp >= 1 && kGemmKTile % (64 * kGemmConsumers) == 0, "stage tiling");
constexpr int kGemmEpilogueWarp = 1 + kGemmConsumers;
constexpr int kGemmThreads = 32 * (2 + kGemmConsumers);  // producer, consumers, epilogue
constexpr int kGemmRedSlots = 2;
constexpr int kGemmMaxStages = 16;
constexpr int kGemmMaxM = 8;
constexpr int kGemmMaxK = 8192;
constexpr int kGemmSmemLimit = 227 * 1024;

struct GemmParams {
  void* out;
  int64_t out_stride;  // elements between output rows
  const void* x;
  int64_t x_stride;    // elements between X rows
  int M, N, K;         // N = output features (the inter size with the gated epilogue)
  int silu;            // 1: gated epilogue on a [gate; up] weight of 2N rows
  int kt;              // K tiles of kGemmKTile
  int stages;          // ring depth
  int row_blocks;
  int* err;
};

__device__ __forceinline__ void gemm_pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void gemm_pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void cp_async16_g(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src)
               : "memory");
}

template <typename T>
__global__ void __launch_bounds__(kGemmThreads, 1)
decode_gemm_kernel(const __grid_constant__ CUtensorMap wmap, const GemmParams p) {
  __shared__ uint64_t full_bar[kGemmMaxStages];
  __shared__ uint64_t empty_bar[kGemmMaxStages];
  __shared__ volatile int s_abort;
  __shared__ float4 red[kGemmRedSlots][kGemmConsumers][2][32];  // [gate|plain, up] partial sums
  __shared__ uint64_t red_full[kGemmRedSlots];
  __shared__ uint64_t red_empty[kGemmRedSlots];
  extern __shared__ uint8_t dyn_smem[];

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int S = p.stages;
  // Dynamic shared memory: [ring, 1024-aligned][X rows, K + 8 elements each].
  const uint32_t dyn_base = smem_u32(dyn_smem);
  const uint32_t ring_off = ((dyn_base + 1023u) & ~1023u) - dyn_base;
  uint8_t* ring = dyn_smem + ring_off;
  T* xs = reinterpret_cast<T*>(ring + S * kGemmStageBytes);
  const int xrow = p.K + 8;  // padded row: conflict-free ldmatrix

  if (tid == 0) {
    s_abort = 0;
    for (int i = 0; i < S; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], kGemmConsumers);
    }
    for (int i = 0; i < kGemmRedSlots; ++i) {
      mbar_init(&red_full[i], kGemmConsumers);
      mbar_init(&red_empty[i], 1);
    }
    fence_mbar_init();
  }
  __syncthreads();

  const int G = gridDim.x;
  const int rb0 = static_cast<int>(static_cast<long long>(blockIdx.x) * p.row_blocks / G);
  const int rb1 = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * p.row_blocks / G);
  const int nst = p.silu ? 2 * p.kt : p.kt;  // stages per row block

  if (warp == 0) {
    // ── producer: weights only, so no PDL wait ───────────────────────────────
    if (lane == 0) {
      prefetch_tmap(&wmap);
      int it = 0;
      for (int rb = rb0; rb < rb1 && !s_abort; ++rb) {
        for (int s = 0; s < nst; ++s, ++it) {
          const int stage = it % S;
          const uint32_t round = static_cast<uint32_t>(it / S);
          if (!mbar_wait(&empty_bar[stage], (round & 1u) ^ 1u, p.err)) {
            s_abort = 1;
            break;
          }
          const int half = s >= p.kt;  // gated form: the up rows follow the gate rows
          const int row = rb * kGemmRows + (half ? p.N : 0);
          const int kt = half ? s - p.kt : s;
          mbar_arrive_expect_tx(&full_bar[stage], kGemmStageBytes);
          // Box {64 elements, kGemmRows rows, kGemmKTile / 64 chunks}: chunks past K read
          // as zeros.
          tma_load_3d(ring + stage * kGemmStageBytes, &wmap, &full_bar[stage], 0, row,
                      kt * (kGemmKTile / 64));
        }
      }
      // Drain: every load still in flight lands before the CTA exits.
      const int first = it > S ? it - S : 0;
      for (int j = first; j < it; ++j) {
        mbar_wait(&full_bar[j % S], static_cast<uint32_t>(j / S) & 1u, p.err);
      }
    }
    return;
  }

  if (warp == kGemmEpilogueWarp) {
    // ── epilogue: adds the consumers' partial sums of each row block ─────────
    gemm_pdl_wait();  // out may still be read by the previous kernel
    const int g = lane >> 2, c = lane & 3;
    T* out = static_cast<T*>(p.out);
    for (int rb = rb0; rb < rb1; ++rb) {
      const int slot = (rb - rb0) % kGemmRedSlots;
      const uint32_t round = static_cast<uint32_t>((rb - rb0) / kGemmRedSlots);
      if (!s_abort && !mbar_wait(&red_full[slot], round & 1u, p.err)) s_abort = 1;
      float4 vg = make_float4(0.f, 0.f, 0.f, 0.f), vu = vg;
#pragma unroll
      for (int q = 0; q < kGemmConsumers; ++q) {
        const float4 a = red[slot][q][0][lane];
        vg.x += a.x;
        vg.y += a.y;
        vg.z += a.z;
        vg.w += a.w;
        if (p.silu) {
          const float4 b = red[slot][q][1][lane];
          vu.x += b.x;
          vu.y += b.y;
          vu.z += b.z;
          vu.w += b.w;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&red_empty[slot]);
      // D fragment: (feature g, batch 2c), (g, 2c + 1), (g + 8, 2c), (g + 8, 2c + 1).
      const float gv[4] = {vg.x, vg.y, vg.z, vg.w};
      const float uv[4] = {vu.x, vu.y, vu.z, vu.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int f = rb * kGemmRows + g + (e >> 1) * 8;
        const int b = 2 * c + (e & 1);
        if (b >= p.M || f >= p.N) continue;
        float o = gv[e];
        if (p.silu) {
          const float g0 = Elt<T>::to_f(Elt<T>::from_f(gv[e]));
          const float u0 = Elt<T>::to_f(Elt<T>::from_f(uv[e]));
          o = Elt<T>::to_f(Elt<T>::from_f(g0 / (1.f + expf(-g0)))) * u0;
        }
        out[static_cast<int64_t>(b) * p.out_stride + f] = Elt<T>::from_f(o);
      }
    }
    return;
  }

  // ── consumers: warp w owns 64-column chunk w of every stage ───────────────
  const int w = warp - 1;
  const int ctid = tid - 32;
  gemm_pdl_wait();  // X is the previous kernel's output
  {
    const int n16 = p.K / 8;  // 16-byte pieces per row
    for (int e = ctid; e < p.M * n16; e += 32 * kGemmConsumers) {
      const int r = e / n16, c = e - r * n16;
      cp_async16_g(xs + r * xrow + c * 8,
                   static_cast<const T*>(p.x) + static_cast<int64_t>(r) * p.x_stride + c * 8);
    }
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
  }
  named_barrier_sync(1, 32 * kGemmConsumers);
  gemm_pdl_trigger();

  const int mi = lane >> 3, r8 = lane & 7;
  // Warp w owns chunks w, w + 8, ... of every stage.  ldmatrix addresses of
  // this lane: weight row (mi & 1) * 8 + r8 of a chunk (128-byte swizzled line
  // chunk*16 + row, 16-byte unit 2*ks + (mi >> 1) for k-step ks), and X row r8
  // (the batch; rows >= M are unused columns of the B side) at k = mi * 8.
  const int wrow = (mi & 1) * 8 + r8;
  uint32_t a_off[4];
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    a_off[ks] = static_cast<uint32_t>((w * kGemmRows + wrow) * 128 + (((2 * ks + (mi >> 1)) ^ r8) << 4));
  }
  const uint32_t ring_u32 = smem_u32(ring);
  const uint32_t x_lane = smem_u32(xs) + static_cast<uint32_t>((r8 * xrow + w * 64 + mi * 8) * 2);
  int it = 0;
  for (int rb = rb0; rb < rb1; ++rb) {
    // Two independent accumulator chains (even and odd k-steps) per projection.
    float ga[4] = {0.f, 0.f, 0.f, 0.f}, gb[4] = {0.f, 0.f, 0.f, 0.f};
    float ua[4] = {0.f, 0.f, 0.f, 0.f}, ub[4] = {0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < nst; ++s, ++it) {
      const int stage = it % S;
      if (!s_abort && !mbar_wait(&full_bar[stage], static_cast<uint32_t>(it / S) & 1u, p.err)) {
        s_abort = 1;
      }
      const bool up = s >= p.kt;
      const int kt = up ? s - p.kt : s;
#pragma unroll
      for (int i = 0; i < kGemmChunksPerWarp; ++i) {
        const int kc = kt * kGemmKTile + (w + i * kGemmConsumers) * 64;  // first k of the chunk
        if (s_abort || kc >= p.K) break;
        const uint32_t sb = ring_u32 + stage * kGemmStageBytes + i * kGemmConsumers * kGemmRows * 128;
        const uint32_t xb = x_lane + static_cast<uint32_t>((kc - w * 64) * 2);
#ifndef VMPS_GEMM_NOMATH
        uint32_t a0[4], a1[4], a2[4], a3[4], x01[4], x23[4];
        ldmatrix_x4(a0, sb + a_off[0]);  // W rows 0-15, k-step 0
        ldmatrix_x4(a1, sb + a_off[1]);
        ldmatrix_x4(a2, sb + a_off[2]);
        ldmatrix_x4(a3, sb + a_off[3]);
        ldmatrix_x4(x01, xb);            // b0, b1 of k-steps 0 and 1
        ldmatrix_x4(x23, xb + 64);       // of k-steps 2 and 3
        if (up) {
          Mma<T>::run(ua, a0, x01[0], x01[1]);
          Mma<T>::run(ub, a1, x01[2], x01[3]);
          Mma<T>::run(ua, a2, x23[0], x23[1]);
          Mma<T>::run(ub, a3, x23[2], x23[3]);
        } else {
          Mma<T>::run(ga, a0, x01[0], x01[1]);
          Mma<T>::run(gb, a1, x01[2], x01[3]);
          Mma<T>::run(ga, a2, x23[0], x23[1]);
          Mma<T>::run(gb, a3, x23[2], x23[3]);
        }
#endif
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[stage]);
    }
    // Hand this warp's partial sums of the row block to the epilogue warp
    // (two slots, so consumers run ahead while it stores the previous one).
    const int slot = (rb - rb0) % kGemmRedSlots;
    const uint32_t round = static_cast<uint32_t>((rb - rb0) / kGemmRedSlots);
    if (!s_abort && !mbar_wait(&red_empty[slot], (round & 1u) ^ 1u, p.err)) s_abort = 1;
    red[slot][w][0][lane] = make_float4(ga[0] + gb[0], ga[1] + gb[1], ga[2] + gb[2], ga[3] + gb[3]);
    if (p.silu) {
      red[slot][w][1][lane] = make_float4(ua[0] + ub[0], ua[1] + ub[1], ua[2] + ub[2], ua[3] + ub[3]);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&red_full[slot]);
  }
}


// X region: kGemmMaxM rows of K + 8 elements, plus 64 bytes that the last
// k-step pair's ldmatrix may touch past the last row.
size_t gemm_x_bytes(int K) { return static_cast<size_t>(kGemmMaxM) * (K + 8) * 2 + 64; }

int gemm_stages(int K) {
  const size_t x_bytes = gemm_x_bytes(K);
  const size_t fixed = 1024 + 20 * 1024;  // alignment slack + static shared memory
  if (x_bytes + fixed + 2 * static_cast<size_t>(kGemmStageBytes) > kGemmSmemLimit) return 0;
  size_t s = (kGemmSmemLimit - fixed - x_bytes) / kGemmStageBytes;
  return static_cast<int>(s > kGemmMaxStages ? kGemmMaxStages : s);
}

}  // namespace
}  // namespace vmps

using namespace vmps;

extern "C" int vmps_decode_gemm_supported(int M, int N, int K, int silu) {
  // K % 64 == 0: the weight rows are whole 128-byte chunks, so no box reads
  // past the end of the last row.
  if (M < 0 || M > kGemmMaxM || N <= 0 || N % 8 || K <= 0 || K % 64 || K > kGemmMaxK) return 0;
  (void)silu;
  return gemm_stages(K) > 0 ? 1 : 0;
}

extern "C" int vmps_decode_gemm(void* out, int64_t out_row_stride, const void* x,
                                int64_t x_row_stride, const void* w, int M, int N, int K,
                                int silu_mul, int dtype, void* stream) {
  clear_error();
  if (!vmps_decode_gemm_supported(M, N, K, silu_mul)) {
    return fail(VMPS_ERR_UNSUPPORTED,
                "decode_gemm: M=%d N=%d K=%d (M <= %d, N %% 8 == 0, K %% 64 == 0, K <= %d)", M, N,
                K, kGemmMaxM, kGemmMaxK);
  }
  if (M == 0) return VMPS_OK;
  if (!out || !x || !w) return fail(VMPS_ERR_INVALID_ARG, "decode_gemm: NULL pointer");
  if (dtype != VMPS_DTYPE_F16 && dtype != VMPS_DTYPE_BF16) {
    return fail(VMPS_ERR_INVALID_ARG, "decode_gemm: dtype %d", dtype);
  }
  if (!aligned16(x) || !aligned16(w) || (x_row_stride % 8) || x_row_stride < K ||
      (reinterpret_cast<uintptr_t>(out) & 3) || (out_row_stride % 2) || out_row_stride < N) {
    return fail(VMPS_ERR_ALIGNMENT,
                "decode_gemm: x and w must be 16-byte aligned with x rows a multiple of 8 "
                "elements apart; out 4-byte aligned with an even row stride");
  }
  const int wrows = silu_mul ? 2 * N : N;
  CUtensorMap wmap;
  // W as {64 elements, rows, K / 64 chunks}: one box is kGemmRows rows x kGemmKTile K.
  const uint64_t dims[3] = {64, (uint64_t)wrows, (uint64_t)((K + 63) / 64)};
  const uint64_t strides[2] = {(uint64_t)K * 2, 128};
  const uint32_t box[3] = {64, (uint32_t)kGemmRows, (uint32_t)(kGemmKTile / 64)};
  if (int rc = encode_tiled(&wmap,
                            dtype == VMPS_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                    : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                            3, const_cast<void*>(w), dims, strides, box,
                            CU_TENSOR_MAP_SWIZZLE_128B)) {
    return rc;
  }
  int sms = 0;
  if (int rc = device_sm_count(&sms)) return rc;
  int* err = nullptr;
  if (int rc = device_error_word(&err)) return rc;
  GemmParams p;
  p.out = out;
  p.out_stride = out_row_stride;
  p.x = x;
  p.x_stride = x_row_stride;
  p.M = M;
  p.N = N;
  p.K = K;
  p.silu = silu_mul ? 1 : 0;
  p.kt = (K + kGemmKTile - 1) / kGemmKTile;
  p.stages = gemm_stages(K);
  p.row_blocks = (N + kGemmRows - 1) / kGemmRows;
  p.err = err;
  const int grid = p.row_blocks < sms ? p.row_blocks : sms;
  const size_t smem = 1024 + static_cast<size_t>(p.stages) * kGemmStageBytes + gemm_x_bytes(K);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  static std::once_flag flags[2][64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return fail(VMPS_ERR_CUDA, "device index %d", dev);
  cudaError_t e;
  if (dtype == VMPS_DTYPE_F16) {
    std::call_once(flags[0][dev], [] {
      cudaFuncSetAttribute(decode_gemm_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kGemmSmemLimit - 20 * 1024);
    });
    e = cudaLaunchKernelEx(&cfg, decode_gemm_kernel<__half>, wmap, p);
  } else {
    std::call_once(flags[1][dev], [] {
      cudaFuncSetAttribute(decode_gemm_kernel<__nv_bfloat16>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmemLimit - 20 * 1024);
    });
    e = cudaLaunchKernelEx(&cfg, decode_gemm_kernel<__nv_bfloat16>, wmap, p);
  }
  if (e != cudaSuccess) {
    return fail(VMPS_ERR_CUDA, "decode_gemm: launch failed: %s", cudaGetErrorString(e));
  }
  return VMPS_OK;
}
