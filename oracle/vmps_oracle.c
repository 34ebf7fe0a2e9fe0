/*
 * vmps_oracle.c -- CPU oracle for the paged decode step (TEST INFRASTRUCTURE).
 *
 * A plain-C restatement of the reference's CPU path for one decode step of
 * PagedAttentionLayer (Nihar0071/vllm_mps), used by the tests as a checker
 * and by bench.py as the timed CPU baseline ("port").  It is never part of
 * the product path.  It follows the same rounding model as
 * oracle/paged_attention_oracle.py and is checked against the same golden
 * fixtures (tests/test_oracle_golden.py):
 *
 *   RoPE   layers/rotary_embedding.py:13-24, 47-53, 55-76 -- cos/sin of the
 *          fp32 angle pos*inv_freq[j], rounded to the model dtype; x*cos and
 *          rotate_half(x)*sin each rounded, then their sum rounded.
 *   write  memory/mps_memory_pool.py:82-102 (+ bounds :257-268) -- rotated K
 *          and V into pool[slot/bs][0|1][slot%bs].
 *   attend layers/paged_attention_layer.py:327-359 -- per query head h the
 *          kv head h/G; scores = round(q.k) then round(s/sqrt(D)); softmax
 *          in fp32 rounded to the dtype; out = round(sum_t p_t v_t).
 *
 * Dtype codes: 0 = fp16, 1 = bf16.  All 16-bit data is passed as raw uint16.
 * Parallelised with OpenMP over (sequence, kv head); `threads` <= 0 uses the
 * OpenMP default.  Returns 0, or -1 on a bad argument.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ── 16-bit conversions (round to nearest even) ─────────────────────────── */

static inline float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: normalise */
      int e = -1;
      do {
        man <<= 1;
        e++;
      } while (!(man & 0x400u));
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ffu) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static inline uint16_t f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t abs = x & 0x7fffffffu;
  if (abs >= 0x7f800000u) { /* inf or nan */
    return (uint16_t)(sign | 0x7c00u | (abs > 0x7f800000u ? 0x200u : 0u));
  }
  if (abs >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to inf */
  if (abs < 0x38800000u) {                                   /* subnormal or zero in fp16 */
    if (abs < 0x33000000u) return (uint16_t)sign;            /* < half of the smallest subnormal */
    const uint32_t e = abs >> 23;
    const uint32_t m = (abs & 0x7fffffu) | 0x800000u;
    const uint32_t shift = 126u - e; /* 14..24 */
    uint32_t r = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (r & 1u))) r++;
    return (uint16_t)(sign | r);
  }
  uint32_t r = abs - 0x38000000u; /* rebias exponent 127 -> 15 */
  const uint32_t rem = r & 0x1fffu;
  r >>= 13;
  if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r++;
  return (uint16_t)(sign | r);
}

static inline float bf16_to_f32(uint16_t h) {
  const uint32_t bits = (uint32_t)h << 16;
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static inline uint16_t f32_to_bf16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u);
  x += 0x7fffu + ((x >> 16) & 1u);
  return (uint16_t)(x >> 16);
}

static inline float to_f(uint16_t h, int dt) { return dt ? bf16_to_f32(h) : f16_to_f32(h); }
static inline uint16_t from_f(float f, int dt) { return dt ? f32_to_bf16(f) : f32_to_f16(f); }
static inline float rnd(float f, int dt) { return to_f(from_f(f, dt), dt); }

/* ── RoPE + write (kernel 1 semantics) ───────────────────────────────────── */

static void rope_row(const uint16_t* x, uint16_t* out, const float* cs, const float* sn, int D,
                     int dt) {
  const int half = D / 2;
  for (int j = 0; j < half; ++j) {
    const float xl = to_f(x[j], dt), xh = to_f(x[j + half], dt);
    const float a_lo = rnd(xl * cs[j], dt), b_lo = rnd(-xh * sn[j], dt);
    const float a_hi = rnd(xh * cs[j], dt), b_hi = rnd(xl * sn[j], dt);
    out[j] = from_f(a_lo + b_lo, dt);
    out[j + half] = from_f(a_hi + b_hi, dt);
  }
}

int vmpso_rope_and_write(uint16_t* q, const uint16_t* k, const uint16_t* v,
                         const int32_t* positions, const int32_t* slot_mapping,
                         const float* inv_freq, uint16_t* pool, int num_seqs, int n_q, int n_kv,
                         int D, int block_size, int num_blocks, int dt) {
  if (D <= 0 || D % 2 || n_kv <= 0 || block_size <= 0) return -1;
  const int half = D / 2;
  float* cs = (float*)malloc(sizeof(float) * half);
  float* sn = (float*)malloc(sizeof(float) * half);
  uint16_t* row = (uint16_t*)malloc(sizeof(uint16_t) * D);
  for (int i = 0; i < num_seqs; ++i) {
    if (inv_freq) {
      for (int j = 0; j < half; ++j) {
        const float ang = (float)positions[i] * inv_freq[j];
        cs[j] = rnd((float)cos((double)ang), dt);
        sn[j] = rnd((float)sin((double)ang), dt);
      }
      for (int h = 0; h < n_q; ++h) {
        uint16_t* x = q + ((size_t)i * n_q + h) * D;
        rope_row(x, row, cs, sn, D, dt);
        memcpy(x, row, sizeof(uint16_t) * D);
      }
    }
    const int32_t slot = slot_mapping[i];
    if (slot < 0) continue;
    const int64_t blk = slot / block_size, off = slot % block_size;
    if (blk >= num_blocks) {
      free(cs);
      free(sn);
      free(row);
      return -1;
    }
    const size_t kv_row = (size_t)n_kv * D;
    uint16_t* kd = pool + ((size_t)(blk * 2 + 0) * block_size + off) * kv_row;
    uint16_t* vd = pool + ((size_t)(blk * 2 + 1) * block_size + off) * kv_row;
    for (int h = 0; h < n_kv; ++h) {
      const uint16_t* kx = k + ((size_t)i * n_kv + h) * D;
      if (inv_freq) {
        rope_row(kx, kd + (size_t)h * D, cs, sn, D, dt);
      } else {
        memcpy(kd + (size_t)h * D, kx, sizeof(uint16_t) * D);
      }
      memcpy(vd + (size_t)h * D, v + ((size_t)i * n_kv + h) * D, sizeof(uint16_t) * D);
    }
  }
  free(cs);
  free(sn);
  free(row);
  return 0;
}

/* ── attention (kernel 2 semantics, reference rounding) ──────────────────── */

int vmpso_paged_attention(uint16_t* out, const uint16_t* q, const uint16_t* pool,
                          const int32_t* block_tables, int max_blocks, const int32_t* seq_lens,
                          int num_seqs, int n_q, int n_kv, int D, int block_size, int num_blocks,
                          int dt, int threads) {
  if (n_kv <= 0 || n_q % n_kv || D <= 0 || block_size <= 0) return -1;
  const int G = n_q / n_kv;
  const float inv_sqrt = (float)(1.0 / sqrt((double)D));
  int bad = 0;
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#endif
#pragma omp parallel reduction(| : bad)
  {
    float* kbuf = NULL;
    float* vbuf = NULL;
    float* sc = NULL;
    size_t cap = 0;
    float* qf = (float*)malloc(sizeof(float) * (size_t)G * D);
    float* acc = (float*)malloc(sizeof(float) * D);
#pragma omp for schedule(dynamic, 1)
    for (int w = 0; w < num_seqs * n_kv; ++w) {
      const int i = w / n_kv, kvh = w % n_kv;
      uint16_t* orow = out + ((size_t)i * n_q + (size_t)kvh * G) * D;
      const int L = seq_lens[i];
      if (L <= 0) {
        memset(orow, 0, sizeof(uint16_t) * (size_t)G * D);
        continue;
      }
      const int pages = (L + block_size - 1) / block_size;
      if (pages > max_blocks) {
        bad = 1;
        continue;
      }
      if ((size_t)L > cap) {
        cap = (size_t)L;
        kbuf = (float*)realloc(kbuf, sizeof(float) * cap * D);
        vbuf = (float*)realloc(vbuf, sizeof(float) * cap * D);
        sc = (float*)realloc(sc, sizeof(float) * cap);
      }
      /* Gather this kv head's history (layers/paged_attention_layer.py:336-343). */
      for (int t = 0; t < L; ++t) {
        const int32_t b = block_tables[(size_t)i * max_blocks + t / block_size];
        if (b < 0 || b >= num_blocks) {
          bad = 1;
          memset(kbuf + (size_t)t * D, 0, sizeof(float) * D);
          memset(vbuf + (size_t)t * D, 0, sizeof(float) * D);
          continue;
        }
        const size_t base = ((size_t)b * 2 * block_size + t % block_size) * n_kv * D + (size_t)kvh * D;
        const uint16_t* kr = pool + base;
        const uint16_t* vr = pool + base + (size_t)block_size * n_kv * D;
        for (int d = 0; d < D; ++d) {
          kbuf[(size_t)t * D + d] = to_f(kr[d], dt);
          vbuf[(size_t)t * D + d] = to_f(vr[d], dt);
        }
      }
      for (int g = 0; g < G; ++g) {
        const uint16_t* qr = q + ((size_t)i * n_q + (size_t)kvh * G + g) * D;
        for (int d = 0; d < D; ++d) qf[d] = to_f(qr[d], dt);
        float mx = -INFINITY;
        for (int t = 0; t < L; ++t) {
          const float* kr = kbuf + (size_t)t * D;
          float s = 0.f;
          for (int d = 0; d < D; ++d) s += qf[d] * kr[d];
          s = rnd(rnd(s, dt) * inv_sqrt, dt); /* :352-353 */
          sc[t] = s;
          if (s > mx) mx = s;
        }
        float sum = 0.f;
        for (int t = 0; t < L; ++t) {
          sc[t] = expf(sc[t] - mx);
          sum += sc[t];
        }
        const float inv = 1.f / sum;
        for (int d = 0; d < D; ++d) acc[d] = 0.f;
        for (int t = 0; t < L; ++t) {
          const float p = rnd(sc[t] * inv, dt); /* softmax output in the dtype (:355) */
          const float* vr = vbuf + (size_t)t * D;
          for (int d = 0; d < D; ++d) acc[d] += p * vr[d];
        }
        for (int d = 0; d < D; ++d) orow[(size_t)g * D + d] = from_f(acc[d], dt);
      }
    }
    free(kbuf);
    free(vbuf);
    free(sc);
    free(qf);
    free(acc);
  }
  return bad ? -1 : 0;
}

/* Threads OpenMP would use for a parallel region (after any override). */
int vmpso_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
