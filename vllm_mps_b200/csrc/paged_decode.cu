// Kernel 2: paged decode attention (one query token per sequence), sm_100a.
//
// Replaces the gather/pad loop, the GQA repeat and the masked softmax
// attention of PagedAttentionLayer._forward_batch
// (layers/paged_attention_layer.py:326-359) and Phases 2-4 of the Metal
// fused_attention shader (kernels/__init__.py:166-241).
//
// Design (B200):
//  * Work unit = one 16-token page of one head group of one sequence.  The
//    units of all sequences are laid end to end and every CTA of a persistent
//    grid (num_SMs x kCtasPerSm) takes one contiguous, equal share, so
//    ragged context lengths still keep all SMs busy (flash-decoding with
//    balanced splits).  A sequence cut between CTAs leaves fp32 partial
//    results (running max, sum, unnormalised output) in the workspace and a
//    small combine kernel merges them.  Both kernels are launched with
//    programmatic dependent launch, so each one's prologue (page prefix sums,
//    barrier set-up) overlaps the tail of the kernel before it.
//  * A producer warp streams pages with the tiled TMA (cp.async.bulk.tensor,
//    no multicast) into a 4-stage shared-memory ring guarded by mbarriers.
//    The box is [64 d][16 tokens][HPC heads][K,V] with the 128-byte swizzle,
//    so K and V of HPC kv heads arrive in one instruction per 64 columns.
//  * One consumer warp per kv head.  The G query heads of a kv head are the
//    N=8 side of the tensor-core MMA, so K and V are read once for the whole
//    group and GQA is never materialised:
//        S^T[16 tok x 8 heads] = K[16 x D] . Q^T[D x 8]        (mma.m16n8k16)
//        online softmax over tokens per head (warp shuffles, fp32, exp2)
//        O^T[D x 8]          += V^T[D x 16] . P^T[16 x 8]     (P via movmatrix)
//  * Scores, softmax state and accumulators are fp32; the output is rounded
//    once to the model dtype.
#include <mutex>
#include <utility>

#include "vmps_abi_internal.h"
#include "vmps_common.cuh"

namespace vmps {

constexpr int kStages = 4;
constexpr int kCtasPerSm = 3;
constexpr int kMinPagesPerCta = 4;
constexpr int kMaxSeqs = 4096;
constexpr int kPageTokens = 16;

struct DecodeParams {
  void* out;
  const void* q;
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
  float scale_log2;  // scale * log2(e)
  int early_prologue;  // 1: seq_lens/block tables may be read before the PDL wait
  int* meta;         // [0] = pages per CTA, [1] = total pages, [2..] = page prefix sums
  float* part_ml;    // [n_cta][2][HPC * GP][2]   (running max in log2 units, sum)
  float* part_o;     // [n_cta][2][HPC * GP][D]   (unnormalised output)
  int* err;
};

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <int D, int HPC, typename T>
struct DecodeShape {
  static constexpr int kDHalves = D / 64;
  static constexpr int kRowBytes = 128;  // 64 elements of 16 bits
  static constexpr int kTileBytes = 2 * kPageTokens * HPC * kRowBytes;  // [K,V][h][tok][64]
  static constexpr int kStageBytes = kTileBytes * kDHalves;
  static constexpr int kThreads = 32 * (1 + HPC);
};

__device__ __forceinline__ int upper_bound_pref(const int* pref, int n, int f) {
  // Largest s in [0, n) with pref[s] <= f (pref is non-decreasing, pref[0] = 0).
  int lo = 0, hi = n;  // invariant: pref[lo] <= f, answer in [lo, hi)
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (pref[mid] <= f) lo = mid; else hi = mid;
  }
  return lo;
}

template <typename T, int D, int HPC, int NT>
__global__ void __launch_bounds__(DecodeShape<D, HPC, T>::kThreads, kCtasPerSm)
paged_decode_kernel(const __grid_constant__ CUtensorMap tmap, const DecodeParams p) {
  using Shape = DecodeShape<D, HPC, T>;
  constexpr int GP = 8 * NT;
  constexpr int KS = D / 16;  // k-steps over head_dim, and m-tiles of O^T

  __shared__ uint64_t full_bar[kStages];
  __shared__ uint64_t empty_bar[kStages];
  __shared__ volatile int s_abort;
  extern __shared__ uint8_t dyn_smem[];

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int num_seqs = p.num_seqs;

  // Dynamic shared memory: [stage ring, 1024-aligned][prefix sums of pages].
  const uint32_t dyn_base = smem_u32(dyn_smem);
  const uint32_t ring_off = ((dyn_base + 1023u) & ~1023u) - dyn_base;
  uint8_t* ring = dyn_smem + ring_off;
  int* pref = reinterpret_cast<int*>(ring + kStages * Shape::kStageBytes);

  if (tid == 0) {
    s_abort = 0;
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], HPC);
    }
    fence_mbar_init();
  }
  // With programmatic dependent launch this CTA may start before the kernel
  // ahead of it in the stream has finished.  seq_lens and block tables are
  // only read early when the caller knows that kernel does not write them
  // (the decode-step entry point, whose predecessor is kernel 1).
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
  }
  if (tid == 0) pref[0] = 0;
  __syncthreads();
  if (warp == 0) {
    int carry = 0;
    for (int base = 0; base < num_seqs; base += 32) {
      const int s = base + lane;
      int v = s < num_seqs ? pref[s + 1] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += y;
      }
      if (s < num_seqs) pref[s + 1] = v + carry;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
  }
  __syncthreads();

  const int TP = pref[num_seqs];
  const long long U = static_cast<long long>(p.num_hg) * TP;
  long long chunk = (U + p.n_cta - 1) / p.n_cta;
  if (chunk < kMinPagesPerCta) chunk = kMinPagesPerCta;
  const long long u_begin = static_cast<long long>(blockIdx.x) * chunk;
  const long long u_end = u_begin + chunk < U ? u_begin + chunk : U;

  // q and the pool may still be being written by the kernel before this one.
  if (p.early_prologue) pdl_wait();
  if (blockIdx.x == 0) {
    // Work split for the combine kernel, and zero rows for empty sequences.
    for (int i = tid; i <= num_seqs; i += blockDim.x) p.meta[2 + i] = pref[i];
    if (tid == 0) {
      p.meta[0] = static_cast<int>(chunk);
      p.meta[1] = TP;
    }
    for (int s = 0; s < num_seqs; ++s) {
      if (pref[s + 1] == pref[s]) {
        T* o = static_cast<T*>(p.out) + static_cast<size_t>(s) * p.n_q * D;
        for (int e = tid; e < p.n_q * D; e += blockDim.x) o[e] = Elt<T>::from_f(0.f);
      }
    }
  }
  pdl_trigger();
  if (u_begin >= u_end) return;

  if (warp == 0) {
    // ── producer: one TMA per 64 columns per page ────────────────────────────
    if (lane == 0) prefetch_tmap(&tmap);
    int it = 0;
    for (long long base = u_begin; base < u_end; base += 32) {
      const long long u = base + lane;
      int phys = 0, hg = 0;
      if (u < u_end) {
        hg = static_cast<int>(u / TP);
        const int f = static_cast<int>(u - static_cast<long long>(hg) * TP);
        const int s = upper_bound_pref(pref, num_seqs, f);
        const int j = f - pref[s];
        phys = p.block_tables[static_cast<size_t>(s) * p.max_blocks + j];
        if (phys < 0 || phys >= p.num_blocks) set_error(p.err, kDevErrBlockRange);
      }
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

  // ── consumers: warp h = kv head (hg * HPC + h) ──────────────────────────────
  const int h = warp - 1;
  const int g = lane >> 2;  // MMA row group
  const int c = lane & 3;   // MMA column pair
  const int mi = lane >> 3, r = lane & 7;
  // Per-lane byte offsets inside one [64-column] tile for ldmatrix.
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
    const int ctx = p.seq_lens[s];

    // Q^T as the B operand: b0 = Q[n][ks*16 + 2c..], b1 = Q[n][ks*16 + 8 + 2c..].
    uint32_t qf[NT][KS][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int n = nt * 8 + g;
      const bool valid = n < p.G;
      const T* qrow = qbase + (static_cast<size_t>(s) * p.n_q + kvh * p.G + (valid ? n : 0)) * D;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        qf[nt][ks][0] = valid ? *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 2 * c) : 0u;
        qf[nt][ks][1] = valid ? *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 8 + 2 * c) : 0u;
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

      // S^T = K . Q^T
      float sc[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        uint32_t a[4];
        ldmatrix_x4(a, sbase + (ks >> 2) * Shape::kTileBytes + k_off[ks & 3]);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) Mma<T>::run(sc[nt], a, qf[nt][ks][0], qf[nt][ks][1]);
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
#pragma unroll
        for (int sh = 4; sh < 32; sh <<= 1) {
          mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, sh));
          mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, sh));
        }
        const float mn0 = fmaxf(m_run[nt][0], mx0), mn1 = fmaxf(m_run[nt][1], mx1);
        const float al0 = fast_exp2(m_run[nt][0] - mn0), al1 = fast_exp2(m_run[nt][1] - mn1);
        m_run[nt][0] = mn0;
        m_run[nt][1] = mn1;
        const float p0 = fast_exp2(x0 - mn0), p1 = fast_exp2(x1 - mn1);
        const float p2 = fast_exp2(x2 - mn0), p3 = fast_exp2(x3 - mn1);
        l_run[nt][0] = l_run[nt][0] * al0 + (p0 + p2);
        l_run[nt][1] = l_run[nt][1] * al1 + (p1 + p3);
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
          o[nt][mt][0] *= al0;
          o[nt][mt][1] *= al1;
          o[nt][mt][2] *= al0;
          o[nt][mt][3] *= al1;
        }
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
    }
    if (s_abort) break;

    // Sum each head's l over the 8 row groups.
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
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const float inv0 = 1.f / l_run[nt][0], inv1 = 1.f / l_run[nt][1];
        const int n0 = nt * 8 + 2 * c;
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
          const int d = mt * 16 + g;
          if (n0 < p.G) {
            T* row = obase + (static_cast<size_t>(s) * p.n_q + kvh * p.G + n0) * D;
            row[d] = Elt<T>::from_f(o[nt][mt][0] * inv0);
            row[d + 8] = Elt<T>::from_f(o[nt][mt][2] * inv0);
          }
          if (n0 + 1 < p.G) {
            T* row = obase + (static_cast<size_t>(s) * p.n_q + kvh * p.G + n0 + 1) * D;
            row[d] = Elt<T>::from_f(o[nt][mt][1] * inv1);
            row[d + 8] = Elt<T>::from_f(o[nt][mt][3] * inv1);
          }
        }
      }
    } else {
      // Split sequence: publish this piece for the combine kernel.
      const long long seg_first = static_cast<long long>(hg) * TP + pref[s];
      const int c0 = static_cast<int>(seg_first / chunk);
      const int slot = (static_cast<int>(blockIdx.x) == c0) ? 1 : 0;
      const size_t rec = (static_cast<size_t>(blockIdx.x) * 2 + slot) * HPC * GP +
                         static_cast<size_t>(h) * GP;
      float* ml = p.part_ml + rec * 2;
      float* po = p.part_o + rec * D;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int n0 = nt * 8 + 2 * c;
        if (g == 0) {
          *reinterpret_cast<float4*>(ml + n0 * 2) =
              make_float4(m_run[nt][0], l_run[nt][0], m_run[nt][1], l_run[nt][1]);
        }
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
          const int d = mt * 16 + g;
          po[n0 * D + d] = o[nt][mt][0];
          po[(n0 + 1) * D + d] = o[nt][mt][1];
          po[n0 * D + d + 8] = o[nt][mt][2];
          po[(n0 + 1) * D + d + 8] = o[nt][mt][3];
        }
      }
    }
    u += (j1 - j0);
  }
}

// ── combine: merge the pieces of sequences that were split between CTAs ──────
//
// Grid (num_hg * num_seqs, ceil(HPC*G*D / 256)); one thread per output element.
// Unsplit sequences were written directly by the main kernel and are skipped.
template <typename T>
__global__ void __launch_bounds__(256)
paged_decode_combine_kernel(const DecodeParams p, int hpc, int gp, int D) {
  pdl_wait();  // partials and meta come from the kernel launched just before
  const int seg = blockIdx.x;
  const int s = seg % p.num_seqs;
  const int hg = seg / p.num_seqs;
  const int chunk = p.meta[0];
  const int TP = p.meta[1];
  const int pref_s = p.meta[2 + s];
  const int seg_pages = p.meta[3 + s] - pref_s;
  if (seg_pages <= 0) return;
  const long long first = static_cast<long long>(hg) * TP + pref_s;
  const int c0 = static_cast<int>(first / chunk);
  const int c1 = static_cast<int>((first + seg_pages - 1) / chunk);
  if (c0 == c1) return;
  const int e = blockIdx.y * blockDim.x + threadIdx.x;
  const int G = p.G;
  if (e >= hpc * G * D) return;
  const int h = e / (G * D);
  const int n = (e / D) % G;
  const int d = e % D;
  float M = -INFINITY, num = 0.f, den = 0.f;
  for (int cc = c0; cc <= c1; cc += 4) {
    float m4[4], l4[4], o4[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c = cc + k;
      if (c <= c1) {
        const size_t rec = (static_cast<size_t>(c) * 2 + (c == c0 ? 1 : 0)) * hpc * gp +
                           static_cast<size_t>(h) * gp + n;
        const float2 ml = __ldcg(reinterpret_cast<const float2*>(p.part_ml) + rec);
        m4[k] = ml.x;
        l4[k] = ml.y;
        o4[k] = __ldcg(p.part_o + rec * D + d);
      } else {
        m4[k] = -INFINITY;
        l4[k] = o4[k] = 0.f;
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (m4[k] == -INFINITY) continue;
      if (m4[k] > M) {
        const float r = fast_exp2(M - m4[k]);
        num *= r;
        den *= r;
        M = m4[k];
      }
      const float w = fast_exp2(m4[k] - M);
      num += w * o4[k];
      den += w * l4[k];
    }
  }
  const int kvh = hg * hpc + h;
  static_cast<T*>(p.out)[(static_cast<size_t>(s) * p.n_q + kvh * G + n) * D + d] =
      Elt<T>::from_f(num / den);
}

// ── host side ────────────────────────────────────────────────────────────────

struct DecodeConfig {
  int hpc;  // kv heads per CTA
  int nt;   // 8-wide n-tiles of query heads per kv head
};

static bool pick_config(int n_q, int n_kv, int D, DecodeConfig* cfg) {
  if (D != 64 && D != 128) return false;
  if (n_kv <= 0 || n_q <= 0 || n_q % n_kv) return false;
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

// Workspace layout: [meta: (num_seqs + 3) ints][part_ml][part_o], each 256-aligned.
struct WorkspaceLayout {
  size_t meta, ml, o, total;
};

static WorkspaceLayout workspace_layout(int num_seqs, int D, const DecodeConfig& cfg, int n_cta) {
  WorkspaceLayout w;
  const size_t recs = static_cast<size_t>(n_cta) * 2 * cfg.hpc * 8 * cfg.nt;
  w.meta = 0;
  w.ml = align256(static_cast<size_t>(num_seqs + 3) * sizeof(int));
  w.o = w.ml + align256(recs * 2 * sizeof(float));
  w.total = w.o + align256(recs * D * sizeof(float));
  return w;
}

static size_t workspace_bytes(int num_seqs, int n_kv, int D, const DecodeConfig& cfg, int n_cta) {
  (void)n_kv;
  return workspace_layout(num_seqs, D, cfg, n_cta).total;
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
  using Shape = DecodeShape<D, HPC, T>;
  const size_t smem = 1024 + kStages * Shape::kStageBytes + (p.num_seqs + 1) * sizeof(int);
  static std::once_flag flags[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return fail(VMPS_ERR_CUDA, "device index %d", dev);
  std::call_once(flags[dev], [] {
    cudaFuncSetAttribute(paged_decode_kernel<T, D, HPC, NT>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                         1024 + kStages * Shape::kStageBytes + (kMaxSeqs + 1) * sizeof(int));
  });
  cudaError_t e = launch_pdl(paged_decode_kernel<T, D, HPC, NT>, dim3(p.n_cta),
                             dim3(Shape::kThreads), smem, s, tmap, p);
  if (e != cudaSuccess) {
    return fail(VMPS_ERR_CUDA, "paged_decode_attention: launch failed: %s", cudaGetErrorString(e));
  }
  const int elems = HPC * p.G * D;
  e = launch_pdl(paged_decode_combine_kernel<T>,
                 dim3(p.num_hg * p.num_seqs, (elems + 255) / 256), dim3(256), 0, s, p, HPC,
                 8 * NT, D);
  if (e != cudaSuccess) {
    return fail(VMPS_ERR_CUDA, "paged_decode_attention: combine launch failed: %s",
                cudaGetErrorString(e));
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
  return workspace_bytes(num_seqs > 0 ? num_seqs : 1, n_kv, head_dim, cfg, sms * kCtasPerSm);
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

namespace vmps {

static int decode_enqueue(void* out, const void* q, const void* pool, const int32_t* block_tables,
                          int max_blocks_per_seq, const int32_t* seq_lens, int num_seqs, int n_q,
                          int n_kv, int head_dim, int block_size, int num_blocks, float scale,
                          void* workspace, size_t workspace_bytes_given, int dtype, void* stream,
                          int early_prologue) {
  if (num_seqs < 0 || num_blocks <= 0 || max_blocks_per_seq <= 0) {
    return fail(VMPS_ERR_INVALID_ARG,
                "paged_decode_attention: bad sizes (num_seqs=%d num_blocks=%d max_blocks=%d)",
                num_seqs, num_blocks, max_blocks_per_seq);
  }
  if (num_seqs == 0) return VMPS_OK;
  if (num_seqs > kMaxSeqs) {
    return fail(VMPS_ERR_UNSUPPORTED, "paged_decode_attention: num_seqs %d > %d", num_seqs,
                kMaxSeqs);
  }
  if (dtype != VMPS_DTYPE_F16 && dtype != VMPS_DTYPE_BF16) {
    return fail(VMPS_ERR_INVALID_ARG, "paged_decode_attention: dtype %d", dtype);
  }
  if (block_size != kPageTokens) {
    return fail(VMPS_ERR_UNSUPPORTED, "paged_decode_attention: block_size %d (only 16 is built)",
                block_size);
  }
  DecodeConfig cfg;
  if (!pick_config(n_q, n_kv, head_dim, &cfg)) {
    return fail(VMPS_ERR_UNSUPPORTED,
                "paged_decode_attention: n_q=%d n_kv=%d head_dim=%d not supported "
                "(head_dim 64/128, n_q/n_kv in 1,2,4,8,16)",
                n_q, n_kv, head_dim);
  }
  if (!out || !q || !pool || !block_tables || !seq_lens) {
    return fail(VMPS_ERR_INVALID_ARG, "paged_decode_attention: NULL pointer");
  }
  if (!aligned16(pool) || (reinterpret_cast<uintptr_t>(q) & 3)) {
    return fail(VMPS_ERR_ALIGNMENT, "paged_decode_attention: pool must be 16-byte aligned");
  }
  if (!(scale > 0.f) || !(scale < 1e30f)) {
    return fail(VMPS_ERR_INVALID_ARG, "paged_decode_attention: scale %g", (double)scale);
  }
  int sms = 0;
  if (int rc = device_sm_count(&sms)) return rc;
  const int n_cta = sms * kCtasPerSm;
  const size_t need = workspace_bytes(num_seqs, n_kv, head_dim, cfg, n_cta);
  if (!workspace || workspace_bytes_given < need) {
    return fail(VMPS_ERR_WORKSPACE, "paged_decode_attention: workspace %zu bytes < %zu needed",
                workspace_bytes_given, need);
  }
  if (reinterpret_cast<uintptr_t>(workspace) & 255) {
    return fail(VMPS_ERR_ALIGNMENT, "paged_decode_attention: workspace must be 256-byte aligned");
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
                            4, const_cast<void*>(pool), dims, strides, box,
                            CU_TENSOR_MAP_SWIZZLE_128B)) {
    return rc;
  }

  DecodeParams p;
  p.out = out;
  p.q = q;
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
  const WorkspaceLayout wl = workspace_layout(num_seqs, head_dim, cfg, n_cta);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.meta = reinterpret_cast<int*>(ws + wl.meta);
  p.part_ml = reinterpret_cast<float*>(ws + wl.ml);
  p.part_o = reinterpret_cast<float*>(ws + wl.o);
  p.err = err;
  p.early_prologue = early_prologue;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return dtype == VMPS_DTYPE_F16 ? dispatch_decode<__half>(cfg, head_dim, tmap, p, s)
                                 : dispatch_decode<__nv_bfloat16>(cfg, head_dim, tmap, p, s);
}

}  // namespace vmps

extern "C" int vmps_paged_decode_attention(void* out, const void* q, const void* pool,
                                           const int32_t* block_tables, int max_blocks_per_seq,
                                           const int32_t* seq_lens, int num_seqs, int n_q,
                                           int n_kv, int head_dim, int block_size,
                                           int num_blocks, float scale, void* workspace,
                                           size_t workspace_bytes, int dtype, void* stream) {
  vmps::clear_error();
  return vmps::decode_enqueue(out, q, pool, block_tables, max_blocks_per_seq, seq_lens, num_seqs,
                              n_q, n_kv, head_dim, block_size, num_blocks, scale, workspace,
                              workspace_bytes, dtype, stream, /*early_prologue=*/0);
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
  using namespace vmps;
  clear_error();
  if (q_row_stride != static_cast<int64_t>(n_q) * head_dim) {
    return fail(VMPS_ERR_INVALID_ARG,
                "paged_decode_step: q must be packed [num_seqs][n_q][head_dim] (row stride %lld)",
                (long long)q_row_stride);
  }
  // Validate the attention arguments before anything is enqueued.
  DecodeConfig cfg;
  if (num_seqs > 0 && (block_size != kPageTokens || !pick_config(n_q, n_kv, head_dim, &cfg))) {
    return fail(VMPS_ERR_UNSUPPORTED,
                "paged_decode_step: n_q=%d n_kv=%d head_dim=%d block_size=%d not supported", n_q,
                n_kv, head_dim, block_size);
  }
  int rc = vmps_rope_reshape_and_cache(q, q, q_row_stride, k, k_row_stride, v, v_row_stride,
                                       positions, slot_mapping, inv_freq, pool, num_seqs, n_q,
                                       n_kv, head_dim, block_size, num_blocks, dtype, stream);
  if (rc) return rc;
  return decode_enqueue(out, q, pool, block_tables, max_blocks_per_seq, seq_lens, num_seqs, n_q,
                        n_kv, head_dim, block_size, num_blocks, scale, workspace, workspace_bytes,
                        dtype, stream, /*early_prologue=*/1);
}
