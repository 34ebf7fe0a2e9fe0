// Kernel 3: causal paged prefill attention on the sm_100a tensor cores
// (tcgen05 MMA with TMEM accumulators).
//
// Replaces the reference's prompt handling, which feeds a prompt through the
// single-token path one token at a time (layers/paged_attention_layer.py:175-241;
// benchmarks/batch_size_benchmark.py:49-60): token t of a sequence attends to
// the sequence's slots 0..position(t).  Here kernel 1 first writes every
// prompt row's rotated K and V into its slot, then this kernel computes all
// rows at once as a dense causal contraction.
//
// Work split.  A CTA owns one 128-row tile of one kv head of one sequence.
// The rows are (query token, query head) pairs: 128/G consecutive tokens x
// the G query heads that share the kv head, so every K/V tile loaded serves
// all G heads (GQA is never materialised).  Key tiles are 64 keys (4 pages).
//
// Data movement.  Warp 4 loads the Q tile with a 3-D TMA and the K pages,
// warp 5 the V pages, with 4-D TMAs (no multicast), all with the 128-byte
// swizzle, into a K ring and a V ring of two tiles each, so K(j+2) loads as
// soon as QK(j) is done and V(j+2) as soon as PV(j) is, neither waiting on
// the other.  Block ids are fetched 32 pages at a time, a batch ahead.  Pages past the sequence's
// table are fetched at an out-of-range coordinate (the TMA fills zeros).
//
// Math.  Warp 6 (one lane) issues tcgen05.mma (kind::f16, M=128, fp32
// accumulate).  S(j) = Q K(j)^T goes to one of two 64-column TMEM buffers,
// so QK(j+1) runs while the softmax works on S(j).  The softmax warps write
// P(j) as 16-bit pairs over the first 32 columns of S(j)'s own buffer and
// PV(j) reads it from there as a TMEM A operand (V as an MN-major shared-
// memory operand, no transpose), accumulating O in 128 more columns.  Warps
// 0-3 own one row each (TMEM lane = row): mask by position, running max and
// sum in fp32 with exp2; O is rescaled in TMEM only when a row's max grows by
// more than 2^8 (then after PV(j-1) has landed), so most tiles never wait on
// the previous PV.  Two CTAs share each SM (~96 KB of shared memory, 256
// TMEM columns each).
//
// Safety.  Every mbarrier wait is bounded; a wait that gives up sets
// kDevErrTimeout and a CTA-wide abort flag, all roles leave their loops,
// the MMA lane waits (bounded) for its own MMAs, the producer for its own
// loads, and the TMEM columns are always freed before the CTA exits.
#include <type_traits>
#include <mutex>

#include "vmps_abi_internal.h"
#include "vmps_common.cuh"

namespace vmps {
namespace {

constexpr int kPfRows = 128;       // MMA M: rows per tile
constexpr int kPfKeys = 64;        // keys per key tile (4 pages)
constexpr int kPfPages = kPfKeys / 16;
constexpr int kPfStages = 2;       // K ring and V ring depth
constexpr int kPfThreads = 224;    // warps 0-3 softmax, 4 K loads, 5 V loads, 6 MMA
constexpr int kKWarp = 4;
constexpr int kVWarp = 5;
constexpr int kMmaWarp = 6;
constexpr int kRegion = 128 * 128; // 128 rows x 64 16-bit columns (one swizzle span)
constexpr int kKRegion = kPfKeys * 128;  // one 64-column chunk of a key tile

template <int D>
struct PrefillShape {
  static constexpr int kChunks = D / 64;
  static constexpr int kQBytes = kChunks * kRegion;
  static constexpr int kTileBytes = kChunks * kKRegion;  // K (or V) of one key tile
  static constexpr int kBarBytes = 256;
  static constexpr int kSmemBytes = kQBytes + 2 * kPfStages * kTileBytes + kBarBytes;
  // TMEM: S double buffer in columns [0, 2 KEYS) (P(j) overwrites the first
  // KEYS/2 columns of S(j)), O in [2 KEYS, 2 KEYS + D).
  static constexpr uint32_t kTmemCols = 256;
};

struct PrefillParams {
  void* out;
  const int32_t* block_tables;
  const int32_t* q_start;
  const int32_t* q_lens;
  const int32_t* cu_q;
  int max_blocks;
  int num_seqs, total_q, max_q_len;
  int n_q, n_kv, G, g_shift, num_blocks;
  int tokens_per_tile;  // 128 / G
  float scale_log2;
  int* err;
};

// ── tcgen05 wrappers (PTX ISA 8.7, sm_100a) ──────────────────────────────────

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
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

// Same with A read from TMEM (K-major: row = lane, 16-bit pairs along K per
// 32-bit column, 8 columns per K-step of 16).
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n"
      "}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 16 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// Ties registers written by tcgen05.ld to the wait that follows it: the
// compiler sees each value pass through an asm placed after the wait, so no
// use can be scheduled before the load has landed.
__device__ __forceinline__ void tmem_ld_fence_regs(uint32_t (&r)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i) asm volatile("" : "+r"(r[i]));
}

// Shared-memory matrix descriptor for a 128-byte-swizzled operand
// (sm_100 format: start, leading and stride byte offsets in 16-byte units,
// descriptor version 1 at bit 46, layout type 2 = SWIZZLE_128B at bit 61).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo_bytes,
                                               uint32_t sbo_bytes) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) |
         (static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32) | (1ull << 46) |
         (2ull << 61);
}

// Instruction descriptor of kind::f16 with fp32 accumulation: A and B both
// fp16 or both bf16, A K-major, B K-major or MN-major, M = 128.
template <typename T>
__device__ __forceinline__ uint32_t f16_idesc(int n, bool b_mn_major) {
  const uint32_t fmt = std::is_same<T, __half>::value ? 0u : 1u;
  return (1u << 4) | (fmt << 7) | (fmt << 10) | (static_cast<uint32_t>(b_mn_major) << 16) |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(kPfRows >> 4) << 24);
}

__device__ __forceinline__ bool aborted(volatile int* flag) { return *flag != 0; }

// ── packed fp32 pairs (f32x2 arithmetic of sm_100) for the softmax ───────────
// Each op computes two independent fp32 results, rounded exactly as the
// scalar op would, in one instruction.

__device__ __forceinline__ uint64_t f2_make(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_split(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

template <typename T, int D>
__global__ void __launch_bounds__(kPfThreads, 2)
    paged_prefill_kernel(const __grid_constant__ CUtensorMap kv_map,
                         const __grid_constant__ CUtensorMap q_map, const PrefillParams p) {
  using Shape = PrefillShape<D>;
  constexpr int KEYS = kPfKeys;
  // The swizzled tiles need 1024-byte alignment; the dynamic window is
  // declared so, and a launch that did not get it reports it and does nothing.
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023u) {
    if (threadIdx.x == 0) set_error(p.err, kDevErrTimeout);
    return;
  }
  uint8_t* sQ = smem_raw;
  uint8_t* sK = sQ + Shape::kQBytes;                 // K ring: kPfStages tiles
  uint8_t* sV = sK + kPfStages * Shape::kTileBytes;  // V ring: kPfStages tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kPfStages * Shape::kTileBytes);
  uint64_t* q_full = bars + 0;
  uint64_t* o_ready = bars + 1;  // MMA -> softmax: PV(j) complete
  uint64_t* o_done = bars + 2;   // all MMAs complete
  uint64_t* s_full = bars + 3;   // [2]: S(j) in TMEM buffer j % 2
  // [2]: softmax -> MMA, P(j) in TMEM buffer j % 2 and O rescaled.  One per
  // buffer: a softmax warp may finish tile j + 1 (S(j + 1) is computed ahead)
  // before another warp finishes tile j, and its arrival must not count
  // toward tile j.
  uint64_t* p_full = bars + 5;
  uint64_t* k_full = bars + 7;   // [kPfStages]
  uint64_t* k_empty = k_full + kPfStages;
  uint64_t* v_full = k_empty + kPfStages;
  uint64_t* v_empty = v_full + kPfStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(v_empty + kPfStages);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int seq = blockIdx.z;
  const int kvh = blockIdx.y;
  const int tile = gridDim.x - 1 - blockIdx.x;  // the longest (last) tiles start first
  const int q_len = p.q_lens[seq];
  const int tok0 = tile * p.tokens_per_tile;
  if (tok0 >= q_len) return;  // uniform across the CTA, before any barrier
  const int q_start = p.q_start[seq];
  const int row0 = p.cu_q[seq];
  if (q_start < 0 || row0 < 0 || static_cast<long long>(row0) + q_len > p.total_q) {
    if (threadIdx.x == 0) set_error(p.err, kDevErrQueryRange);
    return;
  }
  if (threadIdx.x == 0 && tile == 0 && kvh == 0 && q_len > p.max_q_len) {
    set_error(p.err, kDevErrQueryRange);
  }
  const int tok_end = min(q_len, tok0 + p.tokens_per_tile);
  const int n_keys = q_start + tok_end;  // keys 0 .. last position of the tile
  const int n_key_tiles = (n_keys + KEYS - 1) / KEYS;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(p_full + 0, 4);
    mbar_init(p_full + 1, 4);
    mbar_init(o_ready, 1);
    mbar_init(o_done, 1);
    mbar_init(s_full + 0, 1);
    mbar_init(s_full + 1, 1);
    for (int s = 0; s < kPfStages; ++s) {
      mbar_init(k_full + s, 1);
      mbar_init(k_empty + s, 1);
      mbar_init(v_full + s, 1);
      mbar_init(v_empty + s, 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(Shape::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == kKWarp || warp == kVWarp) {
    // ── loads: one warp streams K tiles, another V tiles, so a K load never
    // queues behind a V slot that PV has not released yet.  The block ids
    // come 32 pages at a time (one coalesced load by the warp, the next batch
    // fetched one batch ahead), handed to lane 0 with shuffles.
    const bool is_v = warp == kVWarp;
    if (!is_v && lane == 0) {
      prefetch_tmap(&q_map);
      mbar_arrive_expect_tx(q_full, Shape::kQBytes);
#pragma unroll
      for (int c = 0; c < Shape::kChunks; ++c) {
        tma_load_3d(sQ + c * kRegion, &q_map, q_full, c * 64, kvh * p.G, row0 + tok0);
      }
    }
    if (lane == 0) prefetch_tmap(&kv_map);
    const int32_t* table = p.block_tables + static_cast<size_t>(seq) * p.max_blocks;
    const int n_pages = (n_keys + 15) >> 4;
    const int oob = 2 * p.num_blocks;  // past the pool: the TMA fills zeros
    auto fetch = [&](int page) -> int {  // block id of `page`, or -1
      if (page >= n_pages) return -1;
      if (page >= p.max_blocks) {
        set_error(p.err, kDevErrSeqLen);
        return -1;
      }
      const int b = table[page];
      if (b < 0 || b >= p.num_blocks) {
        set_error(p.err, kDevErrBlockRange);
        return -1;
      }
      return b;
    };
    int ids = fetch(lane), nxt = fetch(32 + lane), batch = 0;
    uint64_t* full = is_v ? v_full : k_full;
    uint64_t* empty = is_v ? v_empty : k_empty;
    uint8_t* ring = is_v ? sV : sK;
    int issued = 0;
    for (int j = 0; j < n_key_tiles; ++j) {
      const int page0 = j * kPfPages;
      if ((page0 >> 5) != batch) {
        batch = page0 >> 5;
        ids = nxt;
        nxt = fetch((batch + 1) * 32 + lane);
      }
      int blk[kPfPages];
#pragma unroll
      for (int pg = 0; pg < kPfPages; ++pg) blk[pg] = __shfl_sync(0xffffffffu, ids, (page0 + pg) & 31);
      bool go = true;
      if (lane == 0) {
        const int st = j % kPfStages;
        // Slot free once QK (K) or PV (V) of tile j - stages is done with it.
        if (j >= kPfStages &&
            (!mbar_wait(empty + st, ((j / kPfStages) - 1) & 1, p.err) || aborted(abort_flag))) {
          *abort_flag = 1;
          go = false;
        } else {
          mbar_arrive_expect_tx(full + st, Shape::kTileBytes);
#pragma unroll
          for (int pg = 0; pg < kPfPages; ++pg) {
            const int coord = blk[pg] < 0 ? oob : 2 * blk[pg] + (is_v ? 1 : 0);
#pragma unroll
            for (int c = 0; c < Shape::kChunks; ++c) {
              tma_load_4d(ring + st * Shape::kTileBytes + c * kKRegion + pg * 2048, &kv_map,
                          full + st, c * 64, 0, kvh, coord);
            }
          }
          issued = j + 1;
        }
      }
      if (!__shfl_sync(0xffffffffu, go ? 1 : 0, 0)) break;
    }
    if (lane == 0 && aborted(abort_flag)) {
      // Let this warp's own loads land before the shared memory is released.
      if (!is_v) mbar_wait(q_full, 0, p.err);
      for (int j = max(0, issued - kPfStages); j < issued; ++j) {
        mbar_wait(full + (j % kPfStages), (j / kPfStages) & 1, p.err);
      }
    }
  } else if (warp == kMmaWarp) {
    // ── MMA issue ─────────────────────────────────────────────────────────────
    // Order: QK(0), QK(1), then per tile j: PV(j) [after the softmax of j],
    // QK(j + 2) into the S buffer PV(j) just read P from (MMAs of one thread
    // execute in issue order).
    if (lane == 0) {
      const uint32_t t_o = tmem_base + 2 * KEYS;
      const uint32_t idesc_qk = f16_idesc<T>(KEYS, false);
      const uint32_t idesc_pv = f16_idesc<T>(D, true);
      const uint32_t q_addr = smem_u32(sQ);
      bool ok = mbar_wait(q_full, 0, p.err) && !aborted(abort_flag);
      auto issue_qk = [&](int j) -> bool {
        const int st = j % kPfStages;
        if (!mbar_wait(k_full + st, (j / kPfStages) & 1, p.err) || aborted(abort_flag)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + st * Shape::kTileBytes);
        const uint32_t t_s = tmem_base + (j & 1) * KEYS;
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint64_t a = sw128_desc(q_addr + (k >> 2) * kRegion + (k & 3) * 32, 16, 1024);
          const uint64_t b = sw128_desc(k_addr + (k >> 2) * kKRegion + (k & 3) * 32, 16, 1024);
          tc_mma(t_s, a, b, idesc_qk, k > 0 ? 1u : 0u);
        }
        tc_commit(k_empty + st);
        tc_commit(s_full + (j & 1));
        return true;
      };
      if (ok) ok = issue_qk(0);
      if (ok && n_key_tiles > 1) ok = issue_qk(1);
      for (int j = 0; ok && j < n_key_tiles; ++j) {
        // O += P(j) V(j), P(j) read from TMEM where S(j) was.
        if (!mbar_wait(p_full + (j & 1), (j >> 1) & 1, p.err) || aborted(abort_flag)) {
          ok = false;
          break;
        }
        const int st = j % kPfStages;
        if (!mbar_wait(v_full + st, (j / kPfStages) & 1, p.err) || aborted(abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + st * Shape::kTileBytes);
        const uint32_t t_p = tmem_base + (j & 1) * KEYS;
#pragma unroll
        for (int k = 0; k < KEYS / 16; ++k) {
          const uint64_t b = sw128_desc(v_addr + k * 2048, kKRegion, 1024);
          tc_mma_ts(t_o, t_p + k * 8, b, idesc_pv, (j > 0 || k > 0) ? 1u : 0u);
        }
        tc_commit(v_empty + st);
        tc_commit(o_ready);
        if (j + 2 < n_key_tiles) ok = issue_qk(j + 2);
      }
      if (!ok) *abort_flag = 1;
      // Whatever happened, every MMA this lane issued completes before the
      // TMEM is freed: o_done fires after all of them.
      tc_commit(o_done);
      mbar_wait(o_done, 0, p.err);
    }
  } else {
    // ── softmax and epilogue: one row per thread ─────────────────────────────
    const int m = threadIdx.x;  // row = TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    const uint32_t t_o = tmem_base + lane_base + 2 * KEYS;
    const int t = m >> p.g_shift;
    const int row_pos = q_start + tok0 + t;
    float m_run = -INFINITY;
    float l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n_key_tiles; ++j) {
      ok = mbar_wait(s_full + (j & 1), (j >> 1) & 1, p.err);
      ok = __all_sync(0xffffffffu, ok) && !aborted(abort_flag);
      if (!ok) break;
      tc_fence_after();
      const uint32_t t_s = tmem_base + lane_base + (j & 1) * KEYS;
      uint32_t s[KEYS / 16][16];
#pragma unroll
      for (int c = 0; c < KEYS / 16; ++c) tmem_ld16(t_s + c * 16, s[c]);
      tmem_ld_wait();
#pragma unroll
      for (int c = 0; c < KEYS / 16; ++c) tmem_ld_fence_regs(s[c]);
      const int key0 = j * KEYS;
      // The max is taken on raw scores (the scale is positive) and the scale
      // is folded into the exp2 argument: p = exp2(s * scale - m).  Masked
      // keys (position > row) become -inf; the warp takes the masked path
      // together whenever any of its rows needs it.
      const bool needs_mask = __any_sync(0xffffffffu, key0 + KEYS - 1 > row_pos);
      // Four independent partial maxima (short dependency chains), two
      // scores per three-input max.
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      if (needs_mask) {
#pragma unroll
        for (int c = 0; c < KEYS / 16; ++c) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            if (key0 + c * 16 + i > row_pos) s[c][i] = __float_as_uint(-INFINITY);
          }
        }
      }
#pragma unroll
      for (int c = 0; c < KEYS / 16; ++c) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          mx4[i & 3] = fmax3(mx4[i & 3], __uint_as_float(s[c][2 * i]),
                             __uint_as_float(s[c][2 * i + 1]));
        }
      }
      float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      mx *= p.scale_log2;
      const float m_new = fmaxf(m_run, mx);
      if (j == 0) {
        m_run = m_new;
      } else if (__any_sync(0xffffffffu, m_new > m_run + 8.f)) {
        // Rescale this warp's O rows once PV(j - 1) has landed; rows whose
        // max did not grow use 1.  (Only PV(j - 1) can have completed since
        // the last wait on o_ready, so its parity is unambiguous.)
        ok = mbar_wait(o_ready, (j - 1) & 1, p.err);
        ok = __all_sync(0xffffffffu, ok) && !aborted(abort_flag);
        if (!ok) break;
        tc_fence_after();
        const float alpha = fast_exp2(m_run - m_new);
#pragma unroll
        for (int c = 0; c < D / 16; ++c) {
          uint32_t o[16];
          tmem_ld16(t_o + c * 16, o);
          tmem_ld_wait();
          tmem_ld_fence_regs(o);
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st16(t_o + c * 16, o);
        }
        l_run *= alpha;
        m_run = m_new;
      }
      // P = exp2(s - m_run) as 16-bit pairs over the first KEYS/2 columns of
      // this S buffer (A operand of PV(j) in TMEM: row = lane, key pairs per
      // 32-bit column).
      // The scale-and-subtract and the row sum run as packed pairs.
      uint32_t pk[KEYS / 32][16];
      uint64_t acc2[2] = {0ull, 0ull};  // two independent packed partial sums
      const uint64_t scale2 = f2_make(p.scale_log2, p.scale_log2);
      const uint64_t neg_m2 = f2_make(-m_run, -m_run);
#pragma unroll
      for (int c = 0; c < KEYS / 16; ++c) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float a, b;
          f2_split(f2_fma(f2_make(__uint_as_float(s[c][2 * i]), __uint_as_float(s[c][2 * i + 1])),
                          scale2, neg_m2),
                   a, b);
          a = fast_exp2(a);
          b = fast_exp2(b);
          acc2[i & 1] = f2_add(acc2[i & 1], f2_make(a, b));
          pk[c >> 1][(c & 1) * 8 + i] = Elt<T>::pack(a, b);
        }
      }
      float s0, s1, s2, s3;
      f2_split(acc2[0], s0, s1);
      f2_split(acc2[1], s2, s3);
      const float sum = (s0 + s1) + (s2 + s3);
#pragma unroll
      for (int c = 0; c < KEYS / 32; ++c) tmem_st16(t_s + c * 16, pk[c]);
      tmem_st_wait();
      l_run += sum;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full + (j & 1));
    }
    // Epilogue: O / l for rows of this sequence.
    bool done = ok && mbar_wait(o_done, 0, p.err);
    done = __all_sync(0xffffffffu, done) && !aborted(abort_flag);
    if (done) {
      tc_fence_after();
      const float inv_l = 1.f / l_run;
      const bool valid = tok0 + t < q_len;
      T* orow = static_cast<T*>(p.out) +
                (static_cast<size_t>(row0 + tok0 + t) * p.n_q + kvh * p.G + (m & (p.G - 1))) * D;
#pragma unroll
      for (int c = 0; c < D / 16; ++c) {
        uint32_t o[16];
        tmem_ld16(t_o + c * 16, o);
        tmem_ld_wait();
        tmem_ld_fence_regs(o);
        uint32_t packed[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          packed[i] = Elt<T>::pack(__uint_as_float(o[2 * i]) * inv_l,
                                   __uint_as_float(o[2 * i + 1]) * inv_l);
        }
        if (valid) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 16);
          dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
          dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
        }
      }
    } else {
      *abort_flag = 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(Shape::kTmemCols)
                 : "memory");
  }
}

template <typename T, int D>
int launch_prefill(const CUtensorMap& kv_map, const CUtensorMap& q_map, const PrefillParams& p,
                   dim3 grid, cudaStream_t s) {
  using Shape = PrefillShape<D>;
  static std::once_flag flags[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return fail(VMPS_ERR_CUDA, "device index %d", dev);
  std::call_once(flags[dev], [] {
    cudaFuncSetAttribute(paged_prefill_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         Shape::kSmemBytes);
  });
  paged_prefill_kernel<T, D><<<grid, kPfThreads, Shape::kSmemBytes, s>>>(kv_map, q_map, p);
  return check_launch("paged_prefill_attention");
}

}  // namespace
}  // namespace vmps

using namespace vmps;

extern "C" int vmps_paged_prefill_attention(
    void* out, const void* q, int64_t q_row_stride, const void* pool,
    const int32_t* block_tables, int max_blocks_per_seq, const int32_t* q_start_pos,
    const int32_t* q_lens, const int32_t* cu_q, int num_seqs, int total_q, int max_q_len,
    int n_q, int n_kv, int head_dim, int block_size, int num_blocks, float scale, int dtype,
    void* stream) {
  const char* what = "paged_prefill_attention";
  clear_error();
  if (num_seqs < 0 || total_q < 0 || max_q_len < 0 || num_blocks <= 0 ||
      max_blocks_per_seq <= 0) {
    return fail(VMPS_ERR_INVALID_ARG,
                "%s: bad sizes (num_seqs=%d total_q=%d max_q_len=%d num_blocks=%d "
                "max_blocks=%d)",
                what, num_seqs, total_q, max_q_len, num_blocks, max_blocks_per_seq);
  }
  if (num_seqs == 0 || total_q == 0 || max_q_len == 0) return VMPS_OK;
  if (num_seqs > 65535) return fail(VMPS_ERR_UNSUPPORTED, "%s: num_seqs %d > 65535", what, num_seqs);
  if (dtype != VMPS_DTYPE_F16 && dtype != VMPS_DTYPE_BF16) {
    return fail(VMPS_ERR_INVALID_ARG, "%s: dtype %d", what, dtype);
  }
  if (block_size != 16) {
    return fail(VMPS_ERR_UNSUPPORTED, "%s: block_size %d (only 16 is built)", what, block_size);
  }
  if ((head_dim != 64 && head_dim != 128) || n_kv <= 0 || n_kv > 65535 || n_q <= 0 ||
      n_q % n_kv) {
    return fail(VMPS_ERR_UNSUPPORTED, "%s: n_q=%d n_kv=%d head_dim=%d not supported", what, n_q,
                n_kv, head_dim);
  }
  const int G = n_q / n_kv;
  if (G != 1 && G != 2 && G != 4 && G != 8 && G != 16) {
    return fail(VMPS_ERR_UNSUPPORTED, "%s: n_q/n_kv=%d (1, 2, 4, 8 or 16 are built)", what, G);
  }
  if (!out || !q || !pool || !block_tables || !q_start_pos || !q_lens || !cu_q) {
    return fail(VMPS_ERR_INVALID_ARG, "%s: NULL pointer", what);
  }
  if (!aligned16(pool) || !aligned16(q) || !aligned16(out) || (q_row_stride % 8)) {
    return fail(VMPS_ERR_ALIGNMENT,
                "%s: pool/q/out must be 16-byte aligned and the q row stride a multiple of 8 "
                "elements",
                what);
  }
  if (q_row_stride < static_cast<int64_t>(n_q) * head_dim) {
    return fail(VMPS_ERR_INVALID_ARG, "%s: q row stride smaller than a row", what);
  }
  if (!(scale > 0.f) || !(scale < 1e30f)) {
    return fail(VMPS_ERR_INVALID_ARG, "%s: scale %g", what, (double)scale);
  }
  int* err = nullptr;
  if (int rc = device_error_word(&err)) return rc;

  const CUtensorMapDataType tdt =
      dtype == VMPS_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint64_t e = 2;
  // Pool as {d, token, kv head, (block, K|V)}: a box [64][16][1][1] is one
  // page of one head, 16 rows of 128 bytes.
  CUtensorMap kv_map;
  {
    const uint64_t dims[4] = {(uint64_t)head_dim, 16, (uint64_t)n_kv, (uint64_t)2 * num_blocks};
    const uint64_t strides[3] = {(uint64_t)n_kv * head_dim * e, (uint64_t)head_dim * e,
                                 (uint64_t)16 * n_kv * head_dim * e};
    const uint32_t box[4] = {64, 16, 1, 1};
    if (int rc = encode_tiled(&kv_map, tdt, 4, const_cast<void*>(pool), dims, strides, box,
                              CU_TENSOR_MAP_SWIZZLE_128B)) {
      return rc;
    }
  }
  // Queries as {d, head, row}: a box [64][G][128/G] is the 128 tile rows
  // (token-major, head-minor) of one 64-column chunk.
  const int tpt = 128 / G;
  CUtensorMap q_map;
  {
    const uint64_t dims[3] = {(uint64_t)head_dim, (uint64_t)n_q, (uint64_t)total_q};
    const uint64_t strides[2] = {(uint64_t)head_dim * e, (uint64_t)q_row_stride * e};
    const uint32_t box[3] = {64, (uint32_t)G, (uint32_t)tpt};
    if (int rc = encode_tiled(&q_map, tdt, 3, const_cast<void*>(q), dims, strides, box,
                              CU_TENSOR_MAP_SWIZZLE_128B)) {
      return rc;
    }
  }
  PrefillParams p;
  p.out = out;
  p.block_tables = block_tables;
  p.q_start = q_start_pos;
  p.q_lens = q_lens;
  p.cu_q = cu_q;
  p.max_blocks = max_blocks_per_seq;
  p.num_seqs = num_seqs;
  p.total_q = total_q;
  p.max_q_len = max_q_len;
  p.n_q = n_q;
  p.n_kv = n_kv;
  p.G = G;
  p.g_shift = __builtin_ctz(static_cast<unsigned>(G));
  p.num_blocks = num_blocks;
  p.tokens_per_tile = tpt;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.err = err;
  const dim3 grid((max_q_len + tpt - 1) / tpt, n_kv, num_seqs);
  if (grid.x > 0x7fffffffu) return fail(VMPS_ERR_UNSUPPORTED, "%s: grid too large", what);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == VMPS_DTYPE_F16) {
    return head_dim == 64 ? launch_prefill<__half, 64>(kv_map, q_map, p, grid, s)
                          : launch_prefill<__half, 128>(kv_map, q_map, p, grid, s);
  }
  return head_dim == 64 ? launch_prefill<__nv_bfloat16, 64>(kv_map, q_map, p, grid, s)
                        : launch_prefill<__nv_bfloat16, 128>(kv_map, q_map, p, grid, s);
}
