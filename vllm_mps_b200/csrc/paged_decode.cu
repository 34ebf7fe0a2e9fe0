// Kernel 2: paged decode attention (one query token per sequence), sm_100a,
// optionally fused with kernel 1's RoPE and K/V write (the whole decode step
// of one layer in one launch).
//
// Replaces the gather/pad loop, the GQA repeat and the masked softmax
// attention of PagedAttentionLayer._forward_batch
// (layers/paged_attention_layer.py:326-359) and the Metal fused_attention
// shader (kernels/__init__.py:99-242); in fused mode also the RoPE loop and
// the write_kv loop (:275-286, :317-324).
//
// Design (B200):
//  * Work unit = one 16-token page of one head group (HPC kv heads, 16 KiB of
//    K+V) of one sequence.  The units of all sequences are laid end to end and
//    every CTA of a persistent grid takes one contiguous, equal share, so
//    ragged batches and single long sequences both keep every SM streaming
//    (flash-decoding with balanced splits).
//  * A producer warp streams pages with the tiled TMA (cp.async.bulk.tensor,
//    no multicast) into a shared-memory ring guarded by mbarriers.  The box
//    is [64 d][16 tokens][HPC heads][K,V] with the 128-byte swizzle, so K and
//    V of HPC kv heads arrive in one instruction per 64 columns.
//  * One consumer warp per kv head.  The G query heads of a kv head are the
//    N=8 side of the tensor-core MMA, so K and V are read once for the whole
//    group and GQA is never materialised:
//        S^T[16 tok x 8 heads] = K[16 x D] . Q^T[D x 8]        (mma.m16n8k16)
//        online softmax over tokens per head (warp shuffles, fp32, exp2)
//        O^T[D x 8]          += V^T[D x 16] . P^T[16 x 8]     (P via movmatrix)
//  * Fused mode: each warp rotates its Q fragments in registers, and the
//    warp that owns a sequence's last page rotates the new K, writes K and V
//    to the pool slot and patches them into its shared-memory copy of the
//    page (no other CTA reads that page in this launch).  RoPE uses the
//    reference's 16-bit rounding points, so the written K is bit-identical
//    to kernel 1's.
//  * A sequence cut between CTAs: every piece stores its fp32 state (running
//    max, sum, unnormalised output in MMA-fragment order) and arrives on an
//    atomic counter per kv head and sequence (one acq_rel add, issued a
//    couple of pages later so it never stalls the page pipeline).
//    The last piece to arrive stages all pieces into the freed shared-memory
//    ring with cp.async (one round trip) and merges them.  Nobody waits on
//    anybody.
//  * The per-segment inputs of a CTA's first segments (query rows, new K/V,
//    lengths, slots, RoPE tables) are staged in shared memory at the start,
//    so a segment switch never waits on a global load queued behind the page
//    stream.
//  * Launched with programmatic dependent launch: in the fused step the
//    prologue (page prefix sums, the first block-table entries, the loads of
//    the first segments' lengths, slots and RoPE inputs) runs while the
//    previous kernel in the stream finishes.  The producer's first page load
//    waits for nothing but its block-table entries; the consumers' prologue
//    overlaps it, with every global load issued before the first use, so a
//    CTA placed just as the previous kernel ends starts streaming at once.
#include <mutex>
#include <utility>

#include "vmps_abi_internal.h"
#include "vmps_common.cuh"

#ifndef VMPS_DECODE_STAGES
#define VMPS_DECODE_STAGES 4
#endif
#ifndef VMPS_DECODE_CTAS_PER_SM
#define VMPS_DECODE_CTAS_PER_SM 2
#endif
// CTAs the kernel is compiled to fit on one SM at once (registers and shared
// memory).  Above VMPS_DECODE_CTAS_PER_SM, CTAs of the next PDL-chained
// launch can be resident beside this launch's and start their L2 prefetch
// while it still runs.
#ifndef VMPS_DECODE_RESIDENT
#define VMPS_DECODE_RESIDENT VMPS_DECODE_CTAS_PER_SM
#endif

namespace vmps {

constexpr int kStages = VMPS_DECODE_STAGES;
constexpr int kCtasPerSm = VMPS_DECODE_CTAS_PER_SM;
constexpr int kMinPagesPerCta = 4;
// Work is split in a weighted page space: a page weighs kPageWeight and every
// non-empty sequence adds kSegmentWeight before its first page: the extra
// cost a CTA pays to start a sequence (query rows, RoPE tables, its own
// accumulators, the partial store of a split piece; ~2 us per extra sequence
// measured in a CTA; a sweep of the weight on C1 was best at 9 pages).
// CTA b owns the pages whose weighted position lies in
// [b*wchunk, (b+1)*wchunk), so CTAs whose chunk spans several sequences get
// fewer pages and all CTAs finish together.
#ifndef VMPS_DECODE_SEG_WEIGHT
#define VMPS_DECODE_SEG_WEIGHT 36
#endif
constexpr int kPageWeight = 4;
constexpr int kSegmentWeight = VMPS_DECODE_SEG_WEIGHT;
constexpr int kMaxSeqs = 4096;
constexpr int kMaxKvHeads = 64;
#ifndef VMPS_DECODE_SEG_TABLES
#define VMPS_DECODE_SEG_TABLES 4
#endif
// Segments per CTA whose inputs (RoPE table, query rows, new K/V) are staged
// in shared memory up front; later segments read them from global memory.
constexpr int kSegTables = VMPS_DECODE_SEG_TABLES;
constexpr int kPageTokens = 16;
// Bytes of its first pages that a CTA pulls into L2 before the PDL wait in
// the fused step.  296 CTAs x 256 KiB = 74 MiB stays well inside the 126 MB
// L2 whatever the workload; a C1-sized chunk (~14 pages of 16 KiB) is
// prefetched whole.
#ifndef VMPS_DECODE_PREFETCH_BYTES
#define VMPS_DECODE_PREFETCH_BYTES (256 * 1024)
#endif
constexpr int kPrefetchBytes = VMPS_DECODE_PREFETCH_BYTES;
// 1: a CTA lets the next launch in the stream start before its own PDL wait
// (the next launch's CTAs then wait for this one to finish, as always).
#ifndef VMPS_DECODE_EARLY_TRIGGER
#define VMPS_DECODE_EARLY_TRIGGER 0
#endif
constexpr bool kEarlyTrigger = VMPS_DECODE_EARLY_TRIGGER != 0;

struct DecodeParams {
  void* out;
  const void* q;
  int64_t q_stride;  // elements between sequences
  const void* k;
  int64_t k_stride;
  const void* v;
  int64_t v_stride;
  const int32_t* positions;
  const int32_t* slot_mapping;
  const float* inv_freq;  // fused mode: RoPE table; else nullptr
  void* pool;
  const int32_t* block_tables;
  const int32_t* seq_lens;
  int max_blocks;
  int num_seqs;
  int n_q;
  int n_kv;
  int G;
  int num_blocks;
  int num_hg;  // head groups = n_kv / HPC
  int n_cta;
  float scale_log2;    // scale * log2(e)
  int fused;           // 1: RoPE + K/V write inside the kernel
  int early_prologue;  // 1: seq_lens may be read before the PDL wait
  int* counters;       // [n_kv * num_seqs], zero between calls
  float* part_ml;      // [n_cta * 2 * HPC][NT][4 lanes][4]
  float* part_o;       // [n_cta * 2 * HPC][NT * D/16][32 lanes][4]
  int* err;
};

// Releases this piece and acquires the ones that arrived before it, in one
// acq_rel atomic (measured 0.5 us shorter per C1 step than a separate
// fence.acq_rel before and after a relaxed add): returns the counter value
// before the increment.
__device__ __forceinline__ int arrive_piece(int* counter) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(counter) : "memory");
  return old;
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src)
               : "memory");
}

__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Named barrier 1 over the consumer warps only (the producer warp never
// joins it; barrier 0 is __syncthreads).
__device__ __forceinline__ void consumer_sync(int threads) {
  asm volatile("bar.sync 1, %0;" ::"r"(threads) : "memory");
}
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <int D, int HPC>
struct DecodeShape {
  static constexpr int kDHalves = D / 64;
  static constexpr int kRowBytes = 128;  // 64 elements of 16 bits
  static constexpr int kTileBytes = 2 * kPageTokens * HPC * kRowBytes;  // [K,V][h][tok][64]
  static constexpr int kStageBytes = kTileBytes * kDHalves;
  static constexpr int kThreads = 32 * (1 + HPC);
};

__device__ __forceinline__ int upper_bound_pref(const int* pref, int n, int f) {
  // Largest s in [0, n) with pref[s] <= f (pref non-decreasing, pref[0] = 0).
  int lo = 0, hi = n;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (pref[mid] <= f) lo = mid; else hi = mid;
  }
  return lo;
}

// RoPE of one element pair with the reference's rounding points
// (layers/rotary_embedding.py:20-24): x*cos, rotate_half(x)*sin and their sum
// each rounded to T.  `lo` is element j, `hi` element j + D/2.
template <typename T>
__device__ __forceinline__ void rope_pair(float lo, float hi, float cs, float sn, float& out_lo,
                                          float& out_hi) {
  const float a_lo = Elt<T>::to_f(Elt<T>::from_f(lo * cs));
  const float b_lo = Elt<T>::to_f(Elt<T>::from_f(-hi * sn));
  const float a_hi = Elt<T>::to_f(Elt<T>::from_f(hi * cs));
  const float b_hi = Elt<T>::to_f(Elt<T>::from_f(lo * sn));
  out_lo = Elt<T>::to_f(Elt<T>::from_f(a_lo + b_lo));
  out_hi = Elt<T>::to_f(Elt<T>::from_f(a_hi + b_hi));
}

// Normalises the O^T fragments by l and stores the G query heads of kv head
// kvh of sequence s (fragment: d = mt*16 + g (+8), heads 2c, 2c+1 of n-tile nt).
template <typename T, int D, int NT>
__device__ __forceinline__ void store_output(T* obase, int s, int kvh, int n_q, int G, int g,
                                             int c, const float (&l)[NT][2],
                                             const float (&o)[NT][D / 16][4]) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const float inv0 = 1.f / l[nt][0], inv1 = 1.f / l[nt][1];
    const int n0 = nt * 8 + 2 * c;
#pragma unroll
    for (int mt = 0; mt < D / 16; ++mt) {
      const int d = mt * 16 + g;
      if (n0 < G) {
        T* row = obase + (static_cast<size_t>(s) * n_q + kvh * G + n0) * D;
        row[d] = Elt<T>::from_f(o[nt][mt][0] * inv0);
        row[d + 8] = Elt<T>::from_f(o[nt][mt][2] * inv0);
      }
      if (n0 + 1 < G) {
        T* row = obase + (static_cast<size_t>(s) * n_q + kvh * G + n0 + 1) * D;
        row[d] = Elt<T>::from_f(o[nt][mt][1] * inv1);
        row[d + 8] = Elt<T>::from_f(o[nt][mt][3] * inv1);
      }
    }
  }
}

// cos/sin of sequence s's position at frequency jj, rounded to T
// (rotary_embedding.py:47-53, 71-72): the fp32 angle pos * inv_freq[jj]
// (one product, as torch.outer computes it), evaluated in double precision.
template <typename T>
__device__ __forceinline__ void rope_value(int pos, float inv_freq, float* cs, float* sn) {
  const float ang = static_cast<float>(pos) * inv_freq;
  double sd, cd;
  sincos(static_cast<double>(ang), &sd, &cd);
  *cs = Elt<T>::to_f(Elt<T>::from_f(static_cast<float>(cd)));
  *sn = Elt<T>::to_f(Elt<T>::from_f(static_cast<float>(sd)));
}

template <typename T, typename Params>
__device__ __forceinline__ void rope_entry(const Params& p, int s, int jj, float* cs, float* sn) {
  const int pos = p.positions[s];
  if (pos < 0) set_error(p.err, kDevErrPositionRange);
  rope_value<T>(pos, p.inv_freq[jj], &cs[jj], &sn[jj]);
}

template <typename T>
__device__ __forceinline__ void unpack2(uint32_t w, float& a, float& b) {
  const T* e = reinterpret_cast<const T*>(&w);
  a = Elt<T>::to_f(e[0]);
  b = Elt<T>::to_f(e[1]);
}

template <typename T, int D, int HPC, int NT>
__global__ void __launch_bounds__(DecodeShape<D, HPC>::kThreads, VMPS_DECODE_RESIDENT)
paged_decode_kernel(const __grid_constant__ CUtensorMap tmap, const DecodeParams p) {
  using Shape = DecodeShape<D, HPC>;
  constexpr int KS = D / 16;  // k-steps over head_dim, and m-tiles of O^T
  constexpr int HALF = D / 2;

  __shared__ uint64_t full_bar[kStages];
  __shared__ uint64_t empty_bar[kStages];
  __shared__ int stage_blk[kStages];
  __shared__ volatile int s_abort;
  __shared__ float rope_cs[HPC][HALF];  // per-warp table beyond kSegTables segments
  __shared__ float rope_sn[HPC][HALF];
  __shared__ float seg_cs[kSegTables][HALF];  // tables of this CTA's first segments
  __shared__ float seg_sn[kSegTables][HALF];
  __shared__ int seg_seq[kSegTables];
  __shared__ int seg_hg[kSegTables];
  __shared__ int seg_ctx[kSegTables];
  __shared__ int seg_slot[kSegTables];
  __shared__ int n_seg_tables;
  // Per-segment inputs staged with cp.async right after the PDL wait, so a
  // segment switch never waits on a global load behind the page stream:
  // the query rows of each kv head, and (fused) the new token's K and V rows.
  __shared__ __align__(16) T seg_q[kSegTables][HPC][8 * NT][D];
  __shared__ __align__(16) T seg_kv[kSegTables][HPC][2][D];
  __shared__ uint64_t loop_done_bar;  // all consumer warps finished with the ring
  extern __shared__ uint8_t dyn_smem[];

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int num_seqs = p.num_seqs;

  // Dynamic shared memory: [stage ring, 1024-aligned][page prefix sums].
  const uint32_t dyn_base = smem_u32(dyn_smem);
  const uint32_t ring_off = ((dyn_base + 1023u) & ~1023u) - dyn_base;
  uint8_t* ring = dyn_smem + ring_off;
  int* pref = reinterpret_cast<int*>(ring + kStages * Shape::kStageBytes);
  int* wpref = pref + (num_seqs + 1);  // weighted prefix sums

  if (tid == 0) {
    s_abort = 0;
    n_seg_tables = 0;
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], HPC);
    }
    mbar_init(&loop_done_bar, HPC);
    fence_mbar_init();
  }
  // seq_lens are read before the PDL wait only when the caller knows the
  // kernel ahead of this one does not write them.
  if (!p.early_prologue) pdl_wait();

  // ── per-sequence page counts and their prefix sums ─────────────────────────
  for (int s = tid; s < num_seqs; s += blockDim.x) {
    const int L = p.seq_lens[s];
    int pages = L > 0 ? (L + kPageTokens - 1) / kPageTokens : 0;
    if (pages > p.max_blocks) {
      if (blockIdx.x == 0) set_error(p.err, kDevErrSeqLen);
      pages = p.max_blocks;
    }
    pref[s + 1] = pages;
    wpref[s + 1] = pages > 0 ? pages * kPageWeight + kSegmentWeight : 0;
  }
  if (tid == 0) {
    pref[0] = 0;
    wpref[0] = 0;
  }
  __syncthreads();
  if (warp == 0) {
    int carry = 0, wcarry = 0;
    for (int base = 0; base < num_seqs; base += 32) {
      const int s = base + lane;
      int v = s < num_seqs ? pref[s + 1] : 0;
      int w = s < num_seqs ? wpref[s + 1] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, v, o);
        const int z = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) {
          v += y;
          w += z;
        }
      }
      if (s < num_seqs) {
        pref[s + 1] = v + carry;
        wpref[s + 1] = w + wcarry;
      }
      carry += __shfl_sync(0xffffffffu, v, 31);
      wcarry += __shfl_sync(0xffffffffu, w, 31);
    }
  }
  __syncthreads();

  const int TP = pref[num_seqs];
  const int WTP = wpref[num_seqs];
  const long long U = static_cast<long long>(p.num_hg) * TP;
  const long long WU = static_cast<long long>(p.num_hg) * WTP;
  long long wchunk = (WU + p.n_cta - 1) / p.n_cta;
  // A chunk holds at least kMinPagesPerCta pages.  When sequences average
  // at most 2 * kMinPagesPerCta pages it also holds one sequence start, so
  // short sequences are not cut: a CTA loads a whole one in one or two
  // rounds of the ring, less than a split piece's merge costs (C0-sized
  // batches: 7.7 -> 5.9 us per layer).  Longer sequences still split finely,
  // which is what keeps a small batch of long contexts streaming on every SM.
  const long long nonempty = (WTP - static_cast<long long>(kPageWeight) * TP) / kSegmentWeight;
  const bool short_seqs = static_cast<long long>(TP) <= 2LL * kMinPagesPerCta * nonempty;
  const long long kMinChunk = kMinPagesPerCta * kPageWeight + (short_seqs ? kSegmentWeight : 0);
  if (wchunk < kMinChunk) wchunk = kMinChunk;
  // First page unit whose weighted position is >= w.
  auto unit_at = [&](long long w) -> long long {
    if (w >= WU) return U;
    const int hg = static_cast<int>(w / WTP);
    const int wf = static_cast<int>(w - static_cast<long long>(hg) * WTP);
    const int s = upper_bound_pref(wpref, num_seqs, wf);
    const int pages = pref[s + 1] - pref[s];
    int pg = (wf - wpref[s] - kSegmentWeight + kPageWeight - 1) / kPageWeight;
    if (wf - wpref[s] <= kSegmentWeight) pg = 0;
    if (pg > pages) pg = pages;
    return static_cast<long long>(hg) * TP + pref[s] + pg;
  };
  // The CTA that owns page `pg` of sequence s in head group hg.
  auto owner_cta = [&](int hg, int s, int pg) -> int {
    const long long w = static_cast<long long>(hg) * WTP + wpref[s] + kSegmentWeight +
                        static_cast<long long>(pg) * kPageWeight;
    return static_cast<int>(w / wchunk);
  };
  const long long u_begin = unit_at(static_cast<long long>(blockIdx.x) * wchunk);
  const long long u_end = unit_at(static_cast<long long>(blockIdx.x + 1) * wchunk);

  // Work decode for a unit: its head group and physical block (producer) or
  // its sequence (consumers).
  // (The block id is range-checked where it is used, so the load is not
  // waited for here.)
  auto unit_block = [&](long long u, int& hg, int& phys) {
    hg = static_cast<int>(u / TP);
    const int f = static_cast<int>(u - static_cast<long long>(hg) * TP);
    const int s = upper_bound_pref(pref, num_seqs, f);
    phys = p.block_tables[static_cast<size_t>(s) * p.max_blocks + (f - pref[s])];
  };
  if (warp == 0) {
    // ── producer: one TMA per 64 columns per page ────────────────────────────
    // Its prologue is only the first batch of block-table entries (host-written
    // inputs, fetched before the PDL wait in the fused step), so a CTA that is
    // placed on its SM just as the previous kernel ends issues its first page
    // load one table round trip after it starts; the consumers' prologue runs
    // while those pages are in flight.
    // Block-table entries are fetched one batch of 32 ahead, so their load
    // latency (long while the page stream keeps HBM queues full) is hidden.
    int cur_phys = 0, cur_hg = 0;
    if (u_begin + lane < u_end) unit_block(u_begin + lane, cur_hg, cur_phys);
    if (kEarlyTrigger) pdl_trigger();
    if (p.early_prologue) {
      // The pool may still be being written by the previous kernel, so pages
      // go to shared memory only after the PDL wait -- but they can be pulled
      // into L2 now (L2 is coherent with those writes): the first
      // kPrefetchUnits pages of this CTA's chunk stream from HBM while the
      // previous launch drains, and the loads after the wait hit L2.
      constexpr int kPrefetchUnits =
          (kPrefetchBytes / Shape::kStageBytes) < 32 ? (kPrefetchBytes / Shape::kStageBytes) : 32;
      if (lane < kPrefetchUnits && u_begin + lane < u_end && cur_phys >= 0 &&
          cur_phys < p.num_blocks) {
#pragma unroll
        for (int dh = 0; dh < Shape::kDHalves; ++dh) {
          tma_prefetch_l2_4d(&tmap, dh * 64, 0, cur_hg * HPC, 2 * cur_phys);
        }
      }
      pdl_wait();
    }
    if (!kEarlyTrigger) pdl_trigger();
    if (u_begin >= u_end) return;
    if (lane == 0) prefetch_tmap(&tmap);
    int it = 0;
    for (long long base = u_begin; base < u_end; base += 32) {
      int nxt_phys = 0, nxt_hg = 0;
      if (base + 32 + lane < u_end) unit_block(base + 32 + lane, nxt_hg, nxt_phys);
      const int phys = cur_phys, hg = cur_hg;
      if (base + lane < u_end && (phys < 0 || phys >= p.num_blocks)) {
        set_error(p.err, kDevErrBlockRange);
      }
      cur_phys = nxt_phys;
      cur_hg = nxt_hg;
      const int n = static_cast<int>(u_end - base < 32 ? u_end - base : 32);
      for (int k = 0; k < n; ++k, ++it) {
        const int ph = __shfl_sync(0xffffffffu, phys, k);
        const int hk = __shfl_sync(0xffffffffu, hg, k);
        if (lane == 0 && !s_abort) {
          const int stage = it % kStages;
          const uint32_t round = static_cast<uint32_t>(it / kStages);
          if (!mbar_wait(&empty_bar[stage], (round & 1u) ^ 1u, p.err)) {
            s_abort = 1;
          } else {
            stage_blk[stage] = ph;
            mbar_arrive_expect_tx(&full_bar[stage], Shape::kStageBytes);
            uint8_t* dst = ring + stage * Shape::kStageBytes;
#pragma unroll
            for (int dh = 0; dh < Shape::kDHalves; ++dh) {
              // Out-of-range block ids read as zeros (TMA bounds fill).
              tma_load_4d(dst + dh * Shape::kTileBytes, &tmap, &full_bar[stage], dh * 64, 0,
                          hk * HPC, 2 * ph);
            }
          }
        }
        __syncwarp();
      }
    }
    return;
  }

  // ── consumer prologue (overlaps the producer's first page loads) ──────────
  // Every global load of the prologue is issued before the first use of any
  // of them: under a full page stream one round trip costs ~2 us, and a CTA
  // placed on its SM just as the previous kernel ends pays each serial one.
  constexpr int kConsumerThreads = 32 * HPC;
  constexpr int kRopePer = (kSegTables * HALF + kConsumerThreads - 1) / kConsumerThreads;
  const int ctid = tid - 32;
  if (warp == 1 && lane == 0) {
    // This CTA's first segments (one sequence each), walked in the prefix sums.
    long long uu = u_begin;
    int k = 0;
    for (; k < kSegTables && uu < u_end; ++k) {
      const int hg = static_cast<int>(uu / TP);
      const int f = static_cast<int>(uu - static_cast<long long>(hg) * TP);
      const int sq = upper_bound_pref(pref, num_seqs, f);
      seg_seq[k] = sq;
      seg_hg[k] = hg;
      uu += pref[sq + 1] - f;
    }
    n_seg_tables = k;
  }
  consumer_sync(kConsumerThreads);
  const int n_seg = n_seg_tables;
  // Host-written inputs of those segments (lengths, new-token slots,
  // positions, RoPE frequencies): loaded before the PDL wait, used after it.
  int r_pos[kRopePer];
  float r_inv[kRopePer];
  if (p.fused) {
#pragma unroll
    for (int i = 0; i < kRopePer; ++i) {
      const int e = ctid + i * kConsumerThreads;
      r_pos[i] = 0;
      r_inv[i] = 0.f;
      if (e < n_seg * HALF) {
        r_pos[i] = p.positions[seg_seq[e / HALF]];
        r_inv[i] = p.inv_freq[e % HALF];
      }
    }
  }
  int l_ctx = 0, l_slot = -1;
  if (warp == 1 && lane < n_seg) {
    const int sq = seg_seq[lane];
    l_ctx = p.seq_lens[sq];
    l_slot = p.fused ? p.slot_mapping[sq] : -1;
  }

  if (p.early_prologue) {
    // The first segments' q rows and new K/V rows into L2 before the wait
    // (the previous kernel may still be writing them; L2 stays coherent),
    // so the cp.async staging after the wait hits L2.
    const int h = warp - 1;
    const int qbytes = p.G * D * static_cast<int>(sizeof(T));
    for (int k = 0; k < n_seg; ++k) {
      const int sq = seg_seq[k];
      const int kvh = seg_hg[k] * HPC + h;
      const char* qrow = reinterpret_cast<const char*>(
          static_cast<const T*>(p.q) + static_cast<size_t>(sq) * p.q_stride +
          static_cast<size_t>(kvh) * p.G * D);
      for (int off = lane * 128; off < qbytes; off += 32 * 128) {
        asm volatile("prefetch.global.L2 [%0];" ::"l"(qrow + off));
      }
      if (lane == 31 || lane == 30) {
        const T* src = lane == 31 ? static_cast<const T*>(p.k) + static_cast<size_t>(sq) * p.k_stride
                                  : static_cast<const T*>(p.v) + static_cast<size_t>(sq) * p.v_stride;
        asm volatile("prefetch.global.L2 [%0];" ::"l"(src + static_cast<size_t>(kvh) * D));
      }
    }
  }
  // q/k/v and the output may still be in use by the previous kernel.
  if (kEarlyTrigger) pdl_trigger();
  if (p.early_prologue) pdl_wait();
  if (!kEarlyTrigger) pdl_trigger();
  {
    // Stage this warp's kv-head rows of the first segments: the G query rows
    // and, in fused mode, the new token's K and V.
    const int h = warp - 1;
    for (int k = 0; k < n_seg; ++k) {
      const int sq = seg_seq[k];
      const int kvh = seg_hg[k] * HPC + h;
      const T* qsrc = static_cast<const T*>(p.q) + static_cast<size_t>(sq) * p.q_stride +
                      static_cast<size_t>(kvh) * p.G * D;
      T* qdst = &seg_q[k][h][0][0];
      for (int ci = lane; ci < p.G * (D / 8); ci += 32) cp_async16(qdst + ci * 8, qsrc + ci * 8);
      if (p.fused) {
        const T* ksrc = static_cast<const T*>(p.k) + static_cast<size_t>(sq) * p.k_stride +
                        static_cast<size_t>(kvh) * D;
        const T* vsrc = static_cast<const T*>(p.v) + static_cast<size_t>(sq) * p.v_stride +
                        static_cast<size_t>(kvh) * D;
        for (int ci = lane; ci < 2 * (D / 8); ci += 32) {
          const bool is_v = ci >= D / 8;
          const int cc = is_v ? ci - D / 8 : ci;
          cp_async16(&seg_kv[k][h][is_v ? 1 : 0][cc * 8], (is_v ? vsrc : ksrc) + cc * 8);
        }
      }
    }
    cp_async_commit();
  }
  // While those copies fly: the segment tables from the loaded values.
  if (warp == 1 && lane < n_seg) {
    seg_ctx[lane] = l_ctx;
    seg_slot[lane] = l_slot;
  }
  if (p.fused) {
#pragma unroll
    for (int i = 0; i < kRopePer; ++i) {
      const int e = ctid + i * kConsumerThreads;
      if (e < n_seg * HALF) {
        if (r_pos[i] < 0) set_error(p.err, kDevErrPositionRange);
        rope_value<T>(r_pos[i], r_inv[i], &seg_cs[e / HALF][e % HALF], &seg_sn[e / HALF][e % HALF]);
      }
    }
  }
  // Zero rows for empty sequences (they own no work unit, so in fused mode
  // their new K/V is not written either: flagged).  The rows are spread over
  // all CTAs, each written by the consumer warps with coalesced stores -- a
  // padded batch can hold hundreds of them.
  for (int s = blockIdx.x; s < num_seqs; s += gridDim.x) {
    if (pref[s + 1] != pref[s]) continue;
    if (ctid == 0 && p.fused && p.slot_mapping[s] >= 0) set_error(p.err, kDevErrSlotNotLast);
    T* o = static_cast<T*>(p.out) + static_cast<size_t>(s) * p.n_q * D;
    if ((reinterpret_cast<uintptr_t>(o) & 15) == 0) {
      uint4* o4 = reinterpret_cast<uint4*>(o);
      const int n16 = p.n_q * D * static_cast<int>(sizeof(T)) / 16;
      for (int e = ctid; e < n16; e += kConsumerThreads) o4[e] = make_uint4(0u, 0u, 0u, 0u);
    } else {
      for (int e = ctid; e < p.n_q * D; e += kConsumerThreads) o[e] = Elt<T>::from_f(0.f);
    }
  }
  consumer_sync(kConsumerThreads);  // segment and RoPE tables complete
  if (u_begin >= u_end) return;

  // ── consumers: warp h = kv head (hg * HPC + h) ──────────────────────────────
  const int h = warp - 1;
  const int g = lane >> 2;  // MMA row group
  const int c = lane & 3;   // MMA column pair
  const int mi = lane >> 3, r = lane & 7;
  uint32_t k_off[4], v_off[4];
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    const int tk = r + ((mi & 1) << 3);
    const int ck = ks * 2 + (mi >> 1);
    k_off[ks] = (uint32_t)(((0 * HPC + h) * kPageTokens + tk) * Shape::kRowBytes + ((ck ^ r) << 4));
    const int tv = r + ((mi >> 1) << 3);
    const int cv = ks * 2 + (mi & 1);
    v_off[ks] = (uint32_t)(((1 * HPC + h) * kPageTokens + tv) * Shape::kRowBytes + ((cv ^ r) << 4));
  }
  const uint32_t ring_u32 = smem_u32(ring);
  const T* qbase = static_cast<const T*>(p.q);
  T* obase = static_cast<T*>(p.out);
  int kseg = 0;

  {
    // Pull the Q rows of this CTA's first few segments into L2 now, so the
    // loads at later segment switches do not queue behind the page stream.
    long long uu = u_begin;
    for (int k = 0; k < 4 && uu < u_end; ++k) {
      const int hg = static_cast<int>(uu / TP);
      const int f = static_cast<int>(uu - static_cast<long long>(hg) * TP);
      const int s = upper_bound_pref(pref, num_seqs, f);
      const char* qrow = reinterpret_cast<const char*>(
          qbase + static_cast<size_t>(s) * p.q_stride + static_cast<size_t>((hg * HPC + h) * p.G) * D);
      const int bytes = p.G * D * static_cast<int>(sizeof(T));
      for (int off = lane * 128; off < bytes; off += 32 * 128) {
        asm volatile("prefetch.global.L2 [%0];" ::"l"(qrow + off));
      }
      uu += pref[s + 1] - pref[s] - (f - pref[s]);
    }
  }
  int pend_s[2], pend_kvh[2], pend_c0[2], pend_c1[2];
  int pend_old[2] = {-1, -1};  // counter value before our arrival (lane 0)
  int n_pend = 0, n_arrived = 0;
  int arrive_at = -1;  // page count after which the oldest piece arrives
  int it = 0;
  long long u = u_begin;
  while (u < u_end) {
    const int hg = static_cast<int>(u / TP);
    const int f = static_cast<int>(u - static_cast<long long>(hg) * TP);
    const int s = upper_bound_pref(pref, num_seqs, f);
    const int j0 = f - pref[s];
    const int seg_pages = pref[s + 1] - pref[s];
    const long long left = u_end - u;
    const int j1 = (seg_pages - j0) < left ? seg_pages : j0 + static_cast<int>(left);
    const int kvh = hg * HPC + h;
    const bool staged = kseg < n_seg_tables;
    if (kseg == 0) {
      asm volatile("cp.async.wait_all;" ::: "memory");
      __syncwarp();
    }
    const int ctx = staged ? seg_ctx[kseg] : p.seq_lens[s];
    const T* q_rows = staged ? &seg_q[kseg][h][0][0]
                             : qbase + static_cast<size_t>(s) * p.q_stride +
                                   static_cast<size_t>(kvh) * p.G * D;
    const T* new_k = staged ? &seg_kv[kseg][h][0][0]
                            : static_cast<const T*>(p.k) + static_cast<size_t>(s) * p.k_stride +
                                  static_cast<size_t>(kvh) * D;
    const T* new_v = staged ? &seg_kv[kseg][h][1][0]
                            : static_cast<const T*>(p.v) + static_cast<size_t>(s) * p.v_stride +
                                  static_cast<size_t>(kvh) * D;
    const int new_slot = staged ? seg_slot[kseg] : (p.fused ? p.slot_mapping[s] : -1);

    const float* cs_tab = rope_cs[h];
    const float* sn_tab = rope_sn[h];
    if (p.fused) {
      if (staged) {
        cs_tab = seg_cs[kseg];
        sn_tab = seg_sn[kseg];
      } else {
        for (int jj = lane; jj < HALF; jj += 32) rope_entry<T>(p, s, jj, rope_cs[h], rope_sn[h]);
        __syncwarp();
      }
    }
    ++kseg;

    // Q^T as the B operand: b0 = Q[n][ks*16 + 2c..], b1 = Q[n][ks*16 + 8 + 2c..].
    uint32_t qf[NT][KS][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int n = nt * 8 + g;
      const bool valid = n < p.G;
      const T* qrow = q_rows + static_cast<size_t>(valid ? n : 0) * D;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        qf[nt][ks][0] = valid ? *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 2 * c) : 0u;
        qf[nt][ks][1] = valid ? *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 8 + 2 * c) : 0u;
      }
      if (p.fused) {
        // Rotate in registers: element d pairs with d + D/2, which this lane
        // holds in k-step ks + KS/2 at the same offsets.
#pragma unroll
        for (int ks = 0; ks < KS / 2; ++ks) {
#pragma unroll
          for (int w = 0; w < 2; ++w) {
            const int j = ks * 16 + w * 8 + 2 * c;
            float l0, l1, h0, h1, o0, o1, p0, p1;
            unpack2<T>(qf[nt][ks][w], l0, l1);
            unpack2<T>(qf[nt][ks + KS / 2][w], h0, h1);
            rope_pair<T>(l0, h0, cs_tab[j], sn_tab[j], o0, p0);
            rope_pair<T>(l1, h1, cs_tab[j + 1], sn_tab[j + 1], o1, p1);
            qf[nt][ks][w] = Elt<T>::pack(o0, o1);
            qf[nt][ks + KS / 2][w] = Elt<T>::pack(p0, p1);
          }
        }
      }
    }
    float m_run[NT][2], l_run[NT][2], o[NT][KS][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      m_run[nt][0] = m_run[nt][1] = -INFINITY;
      l_run[nt][0] = l_run[nt][1] = 0.f;
#pragma unroll
      for (int mt = 0; mt < KS; ++mt) o[nt][mt][0] = o[nt][mt][1] = o[nt][mt][2] = o[nt][mt][3] = 0.f;
    }

    for (int j = j0; j < j1; ++j, ++it) {
      const int stage = it % kStages;
      if (!mbar_wait(&full_bar[stage], static_cast<uint32_t>(it / kStages) & 1u, p.err)) {
        s_abort = 1;
        break;
      }
      const uint32_t sbase = ring_u32 + stage * Shape::kStageBytes;

      if (p.fused && j == seg_pages - 1) {
        // This warp owns the new token of (s, kvh): rotate K, write K and V to
        // the pool slot and into this page's shared-memory copy.
        const int slot = new_slot;
        const int tok = slot & (kPageTokens - 1);
        const int blk = slot >> 4;
        const bool in_pool = slot >= 0 && blk < p.num_blocks;
        if (!in_pool && lane == 0 && slot >= 0) set_error(p.err, kDevErrSlotRange);
        const bool here = in_pool && blk == stage_blk[stage];
        // The new token must sit in the sequence's last page, which only this
        // CTA reads in this launch; anywhere else the write could race a read.
        if (in_pool && !here && lane == 0) set_error(p.err, kDevErrSlotNotLast);
        constexpr int kChunks = D / 8;  // 16-byte chunks per row
        if (lane < 2 * kChunks && in_pool) {
          const bool is_v = lane >= kChunks;
          const int ci = is_v ? lane - kChunks : lane;
          uint4 val;
          if (is_v) {
            val = *reinterpret_cast<const uint4*>(new_v + ci * 8);
          } else {
            const T* krow = new_k;
            const int base_e = ci * 8;
            const int partner = base_e < HALF ? base_e + HALF : base_e - HALF;
            const uint4 mine = *reinterpret_cast<const uint4*>(krow + base_e);
            const uint4 other = *reinterpret_cast<const uint4*>(krow + partner);
            const T* me = reinterpret_cast<const T*>(&mine);
            const T* ot = reinterpret_cast<const T*>(&other);
            T res[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int jj = (base_e + e) & (HALF - 1);
              float lo, hi, out_lo, out_hi;
              if (base_e < HALF) {
                lo = Elt<T>::to_f(me[e]);
                hi = Elt<T>::to_f(ot[e]);
              } else {
                lo = Elt<T>::to_f(ot[e]);
                hi = Elt<T>::to_f(me[e]);
              }
              rope_pair<T>(lo, hi, cs_tab[jj], sn_tab[jj], out_lo, out_hi);
              res[e] = Elt<T>::from_f(base_e < HALF ? out_lo : out_hi);
            }
            val = *reinterpret_cast<const uint4*>(res);
          }
          T* dst = static_cast<T*>(p.pool) +
                   ((static_cast<size_t>(blk) * 2 + (is_v ? 1 : 0)) * kPageTokens + tok) *
                       static_cast<size_t>(p.n_kv) * D +
                   static_cast<size_t>(kvh) * D + ci * 8;
          *reinterpret_cast<uint4*>(dst) = val;
          if (here) {
            const int dh = ci >> 3, cc = ci & 7;
            uint8_t* row = ring + stage * Shape::kStageBytes + dh * Shape::kTileBytes +
                           (((is_v ? 1 : 0) * HPC + h) * kPageTokens + tok) * Shape::kRowBytes;
            *reinterpret_cast<uint4*>(row + ((cc ^ (tok & 7)) << 4)) = val;
          }
        }
        __syncwarp();
      }

      // S^T = K . Q^T, the K steps in two independent accumulator chains
      // (even and odd steps) so the MMAs of one page do not wait on each other.
      float sc[NT][4], sc_odd[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
        sc_odd[nt][0] = sc_odd[nt][1] = sc_odd[nt][2] = sc_odd[nt][3] = 0.f;
      }
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        uint32_t a[4];
        ldmatrix_x4(a, sbase + (ks >> 2) * Shape::kTileBytes + k_off[ks & 3]);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          Mma<T>::run((ks & 1) ? sc_odd[nt] : sc[nt], a, qf[nt][ks][0], qf[nt][ks][1]);
        }
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[nt][e] += sc_odd[nt][e];
      }

      // Mask, scale into log2 units, online softmax per head.
      const int t0 = j * kPageTokens + g;
      const bool v0 = t0 < ctx, v1 = t0 + 8 < ctx;
      uint32_t pb[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const float x0 = v0 ? sc[nt][0] * p.scale_log2 : -INFINITY;
        const float x1 = v0 ? sc[nt][1] * p.scale_log2 : -INFINITY;
        const float x2 = v1 ? sc[nt][2] * p.scale_log2 : -INFINITY;
        const float x3 = v1 ? sc[nt][3] * p.scale_log2 : -INFINITY;
        float mx0 = fmaxf(x0, x2), mx1 = fmaxf(x1, x3);
        // The running max only has to bound the scores: it is raised (a
        // reduction over the row groups, and O and l rescaled) only when a
        // score of this page exceeds it by more than 2^8, so P <= 256 (exact
        // scaling in the 16-bit P and cancelled by l).  Most pages skip the
        // shuffles, the exponentials of alpha and the rescale.
        if (__any_sync(0xffffffffu, mx0 > m_run[nt][0] + 8.f || mx1 > m_run[nt][1] + 8.f)) {
#pragma unroll
          for (int sh = 4; sh < 32; sh <<= 1) {
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, sh));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, sh));
          }
          const float mn0 = fmaxf(m_run[nt][0], mx0), mn1 = fmaxf(m_run[nt][1], mx1);
          const float al0 = fast_exp2(m_run[nt][0] - mn0), al1 = fast_exp2(m_run[nt][1] - mn1);
          m_run[nt][0] = mn0;
          m_run[nt][1] = mn1;
          l_run[nt][0] *= al0;
          l_run[nt][1] *= al1;
#pragma unroll
          for (int mt = 0; mt < KS; ++mt) {
            o[nt][mt][0] *= al0;
            o[nt][mt][1] *= al1;
            o[nt][mt][2] *= al0;
            o[nt][mt][3] *= al1;
          }
        }
        const float p0 = fast_exp2(x0 - m_run[nt][0]), p1 = fast_exp2(x1 - m_run[nt][1]);
        const float p2 = fast_exp2(x2 - m_run[nt][0]), p3 = fast_exp2(x3 - m_run[nt][1]);
        l_run[nt][0] += p0 + p2;
        l_run[nt][1] += p1 + p3;
        // C fragment (row = token, col = head) -> B fragment (k = token, n = head).
        pb[nt][0] = movmatrix_trans(Elt<T>::pack(p0, p1));
        pb[nt][1] = movmatrix_trans(Elt<T>::pack(p2, p3));
      }

      // O^T += V^T . P^T
#pragma unroll
      for (int mt = 0; mt < KS; ++mt) {
        uint32_t a[4];
        ldmatrix_x4_trans(a, sbase + (mt >> 2) * Shape::kTileBytes + v_off[mt & 3]);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) Mma<T>::run(o[nt][mt], a, pb[nt][0], pb[nt][1]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[stage]);
      if (n_arrived < n_pend && it >= arrive_at) {
        // Arrive for a piece published a couple of pages ago: its stores are
        // done by now, so the release fence is cheap, and the counter's
        // answer is only needed after the last page.
        if (lane == 0) {
          pend_old[n_arrived] = arrive_piece(&p.counters[static_cast<size_t>(pend_kvh[n_arrived]) * num_seqs + pend_s[n_arrived]]);
        }
        ++n_arrived;
      }
    }
    if (s_abort) break;

    // Sum each head's l over the 8 row groups (m is already uniform).
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int sh = 4; sh < 32; sh <<= 1) {
        l_run[nt][0] += __shfl_xor_sync(0xffffffffu, l_run[nt][0], sh);
        l_run[nt][1] += __shfl_xor_sync(0xffffffffu, l_run[nt][1], sh);
      }
    }

    if (j0 == 0 && j1 == seg_pages) {
      // The whole sequence was in this CTA: normalise and store.
      store_output<T, D, NT>(obase, s, kvh, p.n_q, p.G, g, c, l_run, o);
    } else {
      // Split sequence: publish this piece now; the arrival (and the merge,
      // for the last piece) waits until this CTA's pages are all streamed,
      // so a round trip to the counter never stalls the page pipeline.
      const int c0 = owner_cta(hg, s, 0);
      const int c1 = owner_cta(hg, s, seg_pages - 1);
      const int slot = (static_cast<int>(blockIdx.x) == c0) ? 1 : 0;
      const size_t rec = (static_cast<size_t>(blockIdx.x) * 2 + slot) * HPC + h;
      float4* po = reinterpret_cast<float4*>(p.part_o) + rec * NT * KS * 32;
      float4* pml = reinterpret_cast<float4*>(p.part_ml) + rec * NT * 4;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
          __stcg(po + (nt * KS + mt) * 32 + lane,
                 make_float4(o[nt][mt][0], o[nt][mt][1], o[nt][mt][2], o[nt][mt][3]));
        }
        if (g == 0) {
          __stcg(pml + nt * 4 + c,
                 make_float4(m_run[nt][0], l_run[nt][0], m_run[nt][1], l_run[nt][1]));
        }
      }
      // Only a CTA's first and last segments can be split: at most two.
      if (n_pend == 2) {
        set_error(p.err, kDevErrSeqLen);
        break;
      }
      pend_s[n_pend] = s;
      pend_kvh[n_pend] = kvh;
      pend_c0[n_pend] = c0;
      pend_c1[n_pend] = c1;
      ++n_pend;
      arrive_at = it + 2;
    }
    u += (j1 - j0);
  }
  if (s_abort) return;

  // Remaining arrivals (the last segment's piece, just published).
  // __syncwarp orders every lane's partial stores before lane 0's release.
  __syncwarp();
  int last_mask = 0;
  if (lane == 0) {
    for (int i = n_arrived; i < n_pend; ++i) {
      pend_old[i] = arrive_piece(&p.counters[static_cast<size_t>(pend_kvh[i]) * num_seqs + pend_s[i]]);
    }
    for (int i = 0; i < n_pend; ++i) {
      if (pend_old[i] == pend_c1[i] - pend_c0[i]) last_mask |= 1 << i;
    }
  }
  last_mask = __shfl_sync(0xffffffffu, last_mask, 0);
  __syncwarp();  // every lane's loads below come after lane 0's acquire
  // The shared-memory ring is reused to stage the pieces to merge, once every
  // consumer warp is done reading pages from it.
  if (lane == 0) mbar_arrive(&loop_done_bar);
  if (!last_mask) return;
  if (!mbar_wait(&loop_done_bar, 0, p.err)) return;

  // Stage every piece of every segment this warp merges into its slice of
  // the ring with 16-byte cp.async (one round trip), then merge in registers.
  constexpr int kPartO = NT * KS * 32;  // float4 per piece (fragment order)
  constexpr int kPartML = NT * 4;
  constexpr int kPartBytes = (kPartO + kPartML) * 16;
  constexpr int kRegion = (kStages * Shape::kStageBytes / HPC) & ~15;
  constexpr int kCap = kRegion / kPartBytes;
  static_assert(kCap >= 2, "merge staging region too small");
  float4* region = reinterpret_cast<float4*>(ring + h * kRegion);
  for (int i = 0; i < n_pend; ++i) {
    if (!(last_mask & (1 << i))) continue;
    const int s = pend_s[i], kvh = pend_kvh[i], c0 = pend_c0[i], c1 = pend_c1[i];
    float m_run[NT][2], l_run[NT][2], o[NT][KS][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      m_run[nt][0] = m_run[nt][1] = -INFINITY;
      l_run[nt][0] = l_run[nt][1] = 0.f;
#pragma unroll
      for (int mt = 0; mt < KS; ++mt) o[nt][mt][0] = o[nt][mt][1] = o[nt][mt][2] = o[nt][mt][3] = 0.f;
    }
    for (int b0 = c0; b0 <= c1; b0 += kCap) {
      const int nb = (c1 - b0 + 1) < kCap ? (c1 - b0 + 1) : kCap;
      for (int b = 0; b < nb; ++b) {
        const int pc = b0 + b;
        const size_t rr = (static_cast<size_t>(pc) * 2 + (pc == c0 ? 1 : 0)) * HPC + h;
        const float4* qo = reinterpret_cast<const float4*>(p.part_o) + rr * kPartO;
        const float4* qml = reinterpret_cast<const float4*>(p.part_ml) + rr * kPartML;
        float4* so = region + b * (kPartO + kPartML);
#pragma unroll
        for (int v = 0; v < NT * KS; ++v) cp_async16(so + v * 32 + lane, qo + v * 32 + lane);
        if (lane < kPartML) cp_async16(so + kPartO + lane, qml + lane);
      }
      cp_async_wait_all();
      __syncwarp();
      for (int b = 0; b < nb; ++b) {
        const float4* so = region + b * (kPartO + kPartML);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const float4 m4 = so[kPartO + nt * 4 + c];
          const float n0 = fmaxf(m_run[nt][0], m4.x), n1 = fmaxf(m_run[nt][1], m4.z);
          const float a0 = fast_exp2(m_run[nt][0] - n0), a1 = fast_exp2(m_run[nt][1] - n1);
          const float e0 = fast_exp2(m4.x - n0), e1 = fast_exp2(m4.z - n1);
          m_run[nt][0] = n0;
          m_run[nt][1] = n1;
          l_run[nt][0] = l_run[nt][0] * a0 + m4.y * e0;
          l_run[nt][1] = l_run[nt][1] * a1 + m4.w * e1;
#pragma unroll
          for (int mt = 0; mt < KS; ++mt) {
            const float4 v4 = so[(nt * KS + mt) * 32 + lane];
            o[nt][mt][0] = o[nt][mt][0] * a0 + v4.x * e0;
            o[nt][mt][1] = o[nt][mt][1] * a1 + v4.y * e1;
            o[nt][mt][2] = o[nt][mt][2] * a0 + v4.z * e0;
            o[nt][mt][3] = o[nt][mt][3] * a1 + v4.w * e1;
          }
        }
      }
      __syncwarp();  // the slots are reused by the next batch
    }
    if (lane == 0) p.counters[static_cast<size_t>(kvh) * num_seqs + s] = 0;
    store_output<T, D, NT>(obase, s, kvh, p.n_q, p.G, g, c, l_run, o);
  }
}

// ── host side ────────────────────────────────────────────────────────────────

struct DecodeConfig {
  int hpc;  // kv heads per CTA
  int nt;   // 8-wide n-tiles of query heads per kv head
};

static bool pick_config(int n_q, int n_kv, int D, DecodeConfig* cfg) {
  if (D != 64 && D != 128) return false;
  if (n_kv <= 0 || n_kv > kMaxKvHeads || n_q <= 0 || n_q % n_kv) return false;
  const int G = n_q / n_kv;
  if (G != 1 && G != 2 && G != 4 && G != 8 && G != 16) return false;
  const int want = 256 / D;  // heads per CTA for a 16 KiB page tile
  int hpc = 1;
  for (int x = want; x >= 1; x >>= 1) {
    if (n_kv % x == 0) { hpc = x; break; }
  }
  cfg->hpc = hpc;
  cfg->nt = G > 8 ? 2 : 1;
  return true;
}

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Workspace layout: [counters][part_ml][part_o], each 256-byte aligned.  The
// counter region has a fixed size (kMaxSeqs * kMaxKvHeads ints) whatever the
// call's shape, so a workspace reused for another shape still finds zeros
// there: it must be zero before the first call, and every call leaves the
// counters it used at zero.
struct WorkspaceLayout {
  size_t counters, ml, o, total;
};

static WorkspaceLayout workspace_layout(int num_seqs, int n_kv, int D, const DecodeConfig& cfg,
                                        int n_cta) {
  WorkspaceLayout w;
  const size_t recs = static_cast<size_t>(n_cta) * 2 * cfg.hpc;
  (void)num_seqs;
  (void)n_kv;
  w.counters = 0;
  w.ml = align256(static_cast<size_t>(kMaxKvHeads) * kMaxSeqs * sizeof(int));
  w.o = w.ml + align256(recs * cfg.nt * 4 * 4 * sizeof(float));
  w.total = w.o + align256(recs * cfg.nt * (D / 16) * 32 * 4 * sizeof(float));
  return w;
}

size_t decode_counter_bytes(int num_seqs, int n_kv) {
  if (num_seqs <= 0 || num_seqs > kMaxSeqs || n_kv <= 0 || n_kv > kMaxKvHeads) return 0;
  return static_cast<size_t>(num_seqs) * n_kv * sizeof(int);
}

// Launches `kernel` with programmatic dependent launch enabled, so it may
// start while the previous kernel in the stream finishes; the kernel itself
// calls griddepcontrol.wait before touching that kernel's outputs.
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <typename T, int D, int HPC, int NT>
static int launch_decode(const CUtensorMap& tmap, const DecodeParams& p, cudaStream_t s) {
  using Shape = DecodeShape<D, HPC>;
  const size_t smem = 1024 + kStages * Shape::kStageBytes + 2 * (p.num_seqs + 1) * sizeof(int);
  static std::once_flag flags[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return fail(VMPS_ERR_CUDA, "device index %d", dev);
  std::call_once(flags[dev], [] {
    cudaFuncSetAttribute(paged_decode_kernel<T, D, HPC, NT>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                         1024 + kStages * Shape::kStageBytes + 2 * (kMaxSeqs + 1) * sizeof(int));
  });
  const cudaError_t e = launch_pdl(paged_decode_kernel<T, D, HPC, NT>, dim3(p.n_cta),
                                   dim3(Shape::kThreads), smem, s, tmap, p);
  if (e != cudaSuccess) {
    return fail(VMPS_ERR_CUDA, "paged_decode_attention: launch failed: %s", cudaGetErrorString(e));
  }
  return VMPS_OK;
}

template <typename T>
static int dispatch_decode(const DecodeConfig& cfg, int D, const CUtensorMap& tmap,
                           const DecodeParams& p, cudaStream_t s) {
#define VMPS_DECODE_CASE(DD, HH, NN)                                      \
  if (D == DD && cfg.hpc == HH && cfg.nt == NN) return launch_decode<T, DD, HH, NN>(tmap, p, s);
  VMPS_DECODE_CASE(64, 4, 1)
  VMPS_DECODE_CASE(64, 4, 2)
  VMPS_DECODE_CASE(64, 2, 1)
  VMPS_DECODE_CASE(64, 2, 2)
  VMPS_DECODE_CASE(64, 1, 1)
  VMPS_DECODE_CASE(64, 1, 2)
  VMPS_DECODE_CASE(128, 2, 1)
  VMPS_DECODE_CASE(128, 2, 2)
  VMPS_DECODE_CASE(128, 1, 1)
  VMPS_DECODE_CASE(128, 1, 2)
#undef VMPS_DECODE_CASE
  return fail(VMPS_ERR_UNSUPPORTED, "paged_decode_attention: no kernel for D=%d hpc=%d nt=%d", D,
              cfg.hpc, cfg.nt);
}

// Shared by both entry points.  `fused` adds RoPE + the K/V write.
static int decode_enqueue(void* out, const void* q, int64_t q_stride, const void* k,
                          int64_t k_stride, const void* v, int64_t v_stride,
                          const int32_t* positions, const int32_t* slot_mapping,
                          const float* inv_freq, void* pool, const int32_t* block_tables,
                          int max_blocks_per_seq, const int32_t* seq_lens, int num_seqs, int n_q,
                          int n_kv, int head_dim, int block_size, int num_blocks, float scale,
                          void* workspace, size_t workspace_bytes_given, int dtype, void* stream,
                          int fused, const char* what) {
  if (num_seqs < 0 || num_blocks <= 0 || max_blocks_per_seq <= 0) {
    return fail(VMPS_ERR_INVALID_ARG, "%s: bad sizes (num_seqs=%d num_blocks=%d max_blocks=%d)",
                what, num_seqs, num_blocks, max_blocks_per_seq);
  }
  if (num_seqs == 0) return VMPS_OK;
  if (num_seqs > kMaxSeqs) {
    return fail(VMPS_ERR_UNSUPPORTED, "%s: num_seqs %d > %d", what, num_seqs, kMaxSeqs);
  }
  if (dtype != VMPS_DTYPE_F16 && dtype != VMPS_DTYPE_BF16) {
    return fail(VMPS_ERR_INVALID_ARG, "%s: dtype %d", what, dtype);
  }
  if (block_size != kPageTokens) {
    return fail(VMPS_ERR_UNSUPPORTED, "%s: block_size %d (only 16 is built)", what, block_size);
  }
  DecodeConfig cfg;
  if (!pick_config(n_q, n_kv, head_dim, &cfg)) {
    return fail(VMPS_ERR_UNSUPPORTED,
                "%s: n_q=%d n_kv=%d head_dim=%d not supported (head_dim 64/128, n_kv <= 64, "
                "n_q/n_kv in 1,2,4,8,16)",
                what, n_q, n_kv, head_dim);
  }
  if (!out || !q || !pool || !block_tables || !seq_lens) {
    return fail(VMPS_ERR_INVALID_ARG, "%s: NULL pointer", what);
  }
  if (fused && (!k || !v || !positions || !slot_mapping || !inv_freq)) {
    return fail(VMPS_ERR_INVALID_ARG, "%s: NULL k/v/positions/slot_mapping/inv_freq", what);
  }
  if (!aligned16(pool) || !aligned16(q) || (q_stride % 8) ||
      (fused && (!aligned16(k) || !aligned16(v) || (k_stride % 8) || (v_stride % 8)))) {
    return fail(VMPS_ERR_ALIGNMENT,
                "%s: pool/q/k/v must be 16-byte aligned and q/k/v row strides multiples of 8 "
                "elements",
                what);
  }
  if (reinterpret_cast<uintptr_t>(out) & 1) {  // 16-bit element stores
    return fail(VMPS_ERR_ALIGNMENT, "%s: out must be 2-byte aligned", what);
  }
  if (q_stride < static_cast<int64_t>(n_q) * head_dim ||
      (fused && (k_stride < static_cast<int64_t>(n_kv) * head_dim ||
                 v_stride < static_cast<int64_t>(n_kv) * head_dim))) {
    return fail(VMPS_ERR_INVALID_ARG, "%s: row stride smaller than a row", what);
  }
  if (!(scale > 0.f) || !(scale < 1e30f)) {
    return fail(VMPS_ERR_INVALID_ARG, "%s: scale %g", what, (double)scale);
  }
  int sms = 0;
  if (int rc = device_sm_count(&sms)) return rc;
  const int n_cta = sms * kCtasPerSm;
  const WorkspaceLayout wl = workspace_layout(num_seqs, n_kv, head_dim, cfg, n_cta);
  if (!workspace || workspace_bytes_given < wl.total) {
    return fail(VMPS_ERR_WORKSPACE, "%s: workspace %zu bytes < %zu needed", what,
                workspace_bytes_given, wl.total);
  }
  if (reinterpret_cast<uintptr_t>(workspace) & 255) {
    return fail(VMPS_ERR_ALIGNMENT, "%s: workspace must be 256-byte aligned", what);
  }
  int* err = nullptr;
  if (int rc = device_error_word(&err)) return rc;

  // Pool as a 4-D tensor {d, token, kv head, (block, K|V)} so that the box
  // [64][16][hpc][2] lands as [K|V][head][token][64] rows of 128 bytes.
  const size_t e = 2;
  CUtensorMap tmap;
  const uint64_t dims[4] = {(uint64_t)head_dim, (uint64_t)block_size, (uint64_t)n_kv,
                            (uint64_t)2 * num_blocks};
  const uint64_t strides[3] = {(uint64_t)n_kv * head_dim * e, (uint64_t)head_dim * e,
                               (uint64_t)block_size * n_kv * head_dim * e};
  const uint32_t box[4] = {64, (uint32_t)block_size, (uint32_t)cfg.hpc, 2};
  if (int rc = encode_tiled(&tmap,
                            dtype == VMPS_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                    : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                            4, pool, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) {
    return rc;
  }

  DecodeParams p;
  p.out = out;
  p.q = q;
  p.q_stride = q_stride;
  p.k = k;
  p.k_stride = k_stride;
  p.v = v;
  p.v_stride = v_stride;
  p.positions = positions;
  p.slot_mapping = slot_mapping;
  p.inv_freq = inv_freq;
  p.pool = pool;
  p.block_tables = block_tables;
  p.seq_lens = seq_lens;
  p.max_blocks = max_blocks_per_seq;
  p.num_seqs = num_seqs;
  p.n_q = n_q;
  p.n_kv = n_kv;
  p.G = n_q / n_kv;
  p.num_blocks = num_blocks;
  p.num_hg = n_kv / cfg.hpc;
  p.n_cta = n_cta;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.fused = fused;
  p.early_prologue = fused;  // the fused step's seq_lens never come from the kernel before it
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.counters = reinterpret_cast<int*>(ws + wl.counters);
  p.part_ml = reinterpret_cast<float*>(ws + wl.ml);
  p.part_o = reinterpret_cast<float*>(ws + wl.o);
  p.err = err;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return dtype == VMPS_DTYPE_F16 ? dispatch_decode<__half>(cfg, head_dim, tmap, p, s)
                                 : dispatch_decode<__nv_bfloat16>(cfg, head_dim, tmap, p, s);
}

}  // namespace vmps

extern "C" size_t vmps_paged_decode_workspace_bytes(int num_seqs, int n_q, int n_kv, int head_dim,
                                                    int dtype) {
  using namespace vmps;
  DecodeConfig cfg;
  if (num_seqs < 0 || (dtype != VMPS_DTYPE_F16 && dtype != VMPS_DTYPE_BF16) ||
      !pick_config(n_q, n_kv, head_dim, &cfg)) {
    return 0;
  }
  int sms = 0;
  if (device_sm_count(&sms)) return 0;
  return workspace_layout(num_seqs > 0 ? num_seqs : 1, n_kv, head_dim, cfg, sms * kCtasPerSm)
      .total;
}

extern "C" int vmps_paged_decode_workspace_init(void* workspace, size_t workspace_bytes,
                                                void* stream) {
  using namespace vmps;
  clear_error();
  if (!workspace && workspace_bytes) return fail(VMPS_ERR_INVALID_ARG, "workspace is NULL");
  if (cudaMemsetAsync(workspace, 0, workspace_bytes, static_cast<cudaStream_t>(stream)) !=
      cudaSuccess) {
    return fail(VMPS_ERR_CUDA, "workspace memset failed: %s",
                cudaGetErrorString(cudaGetLastError()));
  }
  return VMPS_OK;
}

extern "C" int vmps_paged_decode_attention(void* out, const void* q, const void* pool,
                                           const int32_t* block_tables, int max_blocks_per_seq,
                                           const int32_t* seq_lens, int num_seqs, int n_q,
                                           int n_kv, int head_dim, int block_size,
                                           int num_blocks, float scale, void* workspace,
                                           size_t workspace_bytes, int dtype, void* stream) {
  vmps::clear_error();
  return vmps::decode_enqueue(out, q, static_cast<int64_t>(n_q) * head_dim, nullptr, 0, nullptr,
                              0, nullptr, nullptr, nullptr, const_cast<void*>(pool), block_tables,
                              max_blocks_per_seq, seq_lens, num_seqs, n_q, n_kv, head_dim,
                              block_size, num_blocks, scale, workspace, workspace_bytes, dtype,
                              stream, /*fused=*/0, "paged_decode_attention");
}

extern "C" int vmps_paged_decode_step(void* out, void* q, int64_t q_row_stride, const void* k,
                                      int64_t k_row_stride, const void* v, int64_t v_row_stride,
                                      const int32_t* positions, const int32_t* slot_mapping,
                                      const float* inv_freq, void* pool,
                                      const int32_t* block_tables, int max_blocks_per_seq,
                                      const int32_t* seq_lens, int num_seqs, int n_q, int n_kv,
                                      int head_dim, int block_size, int num_blocks, float scale,
                                      void* workspace, size_t workspace_bytes, int dtype,
                                      void* stream) {
  vmps::clear_error();
  return vmps::decode_enqueue(out, q, q_row_stride, k, k_row_stride, v, v_row_stride, positions,
                              slot_mapping, inv_freq, pool, block_tables, max_blocks_per_seq,
                              seq_lens, num_seqs, n_q, n_kv, head_dim, block_size, num_blocks,
                              scale, workspace, workspace_bytes, dtype, stream, /*fused=*/1,
                              "paged_decode_step");
}
