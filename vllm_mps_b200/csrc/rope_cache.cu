// Kernel 1: fused RoPE + reshape-and-cache.
//
// Replaces the per-sequence loop of PagedAttentionLayer._forward_batch that
// rotates Q/K (layers/paged_attention_layer.py:275-286 ->
// layers/rotary_embedding.py:55-76) and writes K/V into the pool slot
// (:317-324 -> memory/mps_memory_pool.py:82-102).  One CTA per sequence;
// every thread moves 16-byte vectors.  The arithmetic reproduces the
// reference's rounding points bit for bit: cos/sin are computed in fp32 and
// rounded to the model dtype (rotary_embedding.py:71-72), then x*cos,
// rotate_half(x)*sin and their sum are each rounded to the model dtype
// (:20-24), which is how PyTorch's CPU kernels evaluate the fp16 expression.
#include "vmps_abi_internal.h"
#include "vmps_common.cuh"

namespace vmps {

struct RopeCacheParams {
  void* q_out;
  const void* q;
  const void* k;
  const void* v;
  int64_t q_stride, k_stride, v_stride;  // elements between sequences
  const int32_t* positions;
  const int32_t* slot_mapping;
  const float* inv_freq;  // D/2 floats, or nullptr for no rotation
  void* pool;
  int n_q, n_kv, block_size;
  int64_t num_slots;  // num_blocks * block_size
  int* err;
};

template <typename T, int D>
__global__ void __launch_bounds__(128) rope_cache_kernel(RopeCacheParams p) {
  constexpr int kHalf = D / 2;
  constexpr int kChunks = kHalf / 8;  // 16-byte chunks per half head
  __shared__ float s_cos[kHalf];
  __shared__ float s_sin[kHalf];

  const int i = blockIdx.x;
  const bool rotate = p.inv_freq != nullptr;
  const int pos = p.positions ? p.positions[i] : 0;
  if (rotate && pos < 0) {
    if (threadIdx.x == 0) set_error(p.err, kDevErrPositionRange);
    return;
  }
  if (rotate) {
    for (int j = threadIdx.x; j < kHalf; j += blockDim.x) {
      // freqs = outer(t, inv_freq): one fp32 product (rotary_embedding.py:49).
      const float ang = static_cast<float>(pos) * p.inv_freq[j];
      double sd, cd;
      sincos(static_cast<double>(ang), &sd, &cd);
      // cos/sin cached in fp32, cast to the model dtype at use (:71-72).
      s_cos[j] = Elt<T>::to_f(Elt<T>::from_f(static_cast<float>(cd)));
      s_sin[j] = Elt<T>::to_f(Elt<T>::from_f(static_cast<float>(sd)));
    }
    __syncthreads();
  }

  const int32_t slot = p.slot_mapping ? p.slot_mapping[i] : -1;
  const bool write = slot >= 0 && slot < p.num_slots;
  if (slot >= p.num_slots && threadIdx.x == 0) set_error(p.err, kDevErrSlotRange);
  const int64_t blk = write ? slot / p.block_size : 0;
  const int64_t off = write ? slot % p.block_size : 0;
  T* pool = static_cast<T*>(p.pool);
  const int64_t kv_row = static_cast<int64_t>(p.n_kv) * D;
  T* k_dst = pool + ((blk * 2 + 0) * p.block_size + off) * kv_row;
  T* v_dst = pool + ((blk * 2 + 1) * p.block_size + off) * kv_row;

  const int rope_units = (p.n_q + p.n_kv) * kChunks;
  const int copy_units = p.n_kv * (D / 8);
  for (int u = threadIdx.x; u < rope_units + copy_units; u += blockDim.x) {
    if (u < rope_units) {
      const int h = u / kChunks;
      const int c = u % kChunks;
      const T* src;
      T* dst;
      if (h < p.n_q) {
        src = static_cast<const T*>(p.q) + i * p.q_stride + h * D;
        dst = static_cast<T*>(p.q_out) + i * p.q_stride + h * D;
      } else {
        const int hk = h - p.n_q;
        src = static_cast<const T*>(p.k) + i * p.k_stride + hk * D;
        dst = write ? k_dst + hk * D : nullptr;
      }
      uint4 lo4 = *reinterpret_cast<const uint4*>(src + c * 8);
      uint4 hi4 = *reinterpret_cast<const uint4*>(src + kHalf + c * 8);
      if (rotate) {
        const T* lo = reinterpret_cast<const T*>(&lo4);
        const T* hi = reinterpret_cast<const T*>(&hi4);
        T out_lo[8], out_hi[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int j = c * 8 + e;
          const float cs = s_cos[j], sn = s_sin[j];
          const float xl = Elt<T>::to_f(lo[e]), xh = Elt<T>::to_f(hi[e]);
          // rotate_half(x) = cat(-x2, x1) (rotary_embedding.py:13-17).
          const float a_lo = Elt<T>::to_f(Elt<T>::from_f(xl * cs));
          const float b_lo = Elt<T>::to_f(Elt<T>::from_f(-xh * sn));
          const float a_hi = Elt<T>::to_f(Elt<T>::from_f(xh * cs));
          const float b_hi = Elt<T>::to_f(Elt<T>::from_f(xl * sn));
          out_lo[e] = Elt<T>::from_f(a_lo + b_lo);
          out_hi[e] = Elt<T>::from_f(a_hi + b_hi);
        }
        lo4 = *reinterpret_cast<const uint4*>(out_lo);
        hi4 = *reinterpret_cast<const uint4*>(out_hi);
      }
      if (dst) {
        *reinterpret_cast<uint4*>(dst + c * 8) = lo4;
        *reinterpret_cast<uint4*>(dst + kHalf + c * 8) = hi4;
      }
    } else if (write) {
      const int cu = u - rope_units;
      const int hv = cu / (D / 8);
      const int c = cu % (D / 8);
      const T* src = static_cast<const T*>(p.v) + i * p.v_stride + hv * D + c * 8;
      *reinterpret_cast<uint4*>(v_dst + hv * D + c * 8) = *reinterpret_cast<const uint4*>(src);
    }
  }
}

template <typename T>
static int launch_rope_cache(const RopeCacheParams& p, int num_seqs, int D, cudaStream_t s) {
  switch (D) {
    case 64:
      rope_cache_kernel<T, 64><<<num_seqs, 128, 0, s>>>(p);
      break;
    case 128:
      rope_cache_kernel<T, 128><<<num_seqs, 128, 0, s>>>(p);
      break;
    case 256:
      rope_cache_kernel<T, 256><<<num_seqs, 128, 0, s>>>(p);
      break;
    default:
      return fail(VMPS_ERR_UNSUPPORTED, "rope_reshape_and_cache: head_dim %d not built", D);
  }
  return check_launch("rope_reshape_and_cache");
}

}  // namespace vmps

extern "C" int vmps_rope_reshape_and_cache(void* q_out, const void* q, int64_t q_row_stride,
                                           const void* k, int64_t k_row_stride, const void* v,
                                           int64_t v_row_stride, const int32_t* positions,
                                           const int32_t* slot_mapping, const float* inv_freq,
                                           void* pool, int num_seqs, int n_q, int n_kv,
                                           int head_dim, int block_size, int num_blocks,
                                           int dtype, void* stream) {
  using namespace vmps;
  clear_error();
  if (num_seqs < 0 || n_q < 0 || n_kv <= 0 || head_dim <= 0 || block_size <= 0 ||
      num_blocks <= 0) {
    return fail(VMPS_ERR_INVALID_ARG,
                "rope_reshape_and_cache: bad sizes (num_seqs=%d n_q=%d n_kv=%d head_dim=%d "
                "block_size=%d num_blocks=%d)",
                num_seqs, n_q, n_kv, head_dim, block_size, num_blocks);
  }
  if (num_seqs == 0) return VMPS_OK;
  if (dtype != VMPS_DTYPE_F16 && dtype != VMPS_DTYPE_BF16) {
    return fail(VMPS_ERR_INVALID_ARG, "rope_reshape_and_cache: dtype %d", dtype);
  }
  if ((n_q > 0 && (!q || !q_out)) || !k || !v || !pool || !slot_mapping ||
      (inv_freq && !positions)) {
    return fail(VMPS_ERR_INVALID_ARG, "rope_reshape_and_cache: NULL pointer");
  }
  if ((n_q > 0 && (!aligned16(q) || !aligned16(q_out))) || !aligned16(k) || !aligned16(v) ||
      !aligned16(pool) || (q_row_stride % 8) || (k_row_stride % 8) || (v_row_stride % 8)) {
    return fail(VMPS_ERR_ALIGNMENT,
                "rope_reshape_and_cache: pointers must be 16-byte aligned and row strides "
                "multiples of 8 elements");
  }
  if (q_row_stride < (int64_t)n_q * head_dim || k_row_stride < (int64_t)n_kv * head_dim ||
      v_row_stride < (int64_t)n_kv * head_dim) {
    return fail(VMPS_ERR_INVALID_ARG, "rope_reshape_and_cache: row stride smaller than a row");
  }
  int* err = nullptr;
  if (int rc = device_error_word(&err)) return rc;
  RopeCacheParams p{q_out,         q,         k,     v,    q_row_stride, k_row_stride,
                    v_row_stride,  positions, slot_mapping, inv_freq, pool, n_q,
                    n_kv,          block_size, (int64_t)num_blocks * block_size, err};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return dtype == VMPS_DTYPE_F16 ? launch_rope_cache<__half>(p, num_seqs, head_dim, s)
                                 : launch_rope_cache<__nv_bfloat16>(p, num_seqs, head_dim, s);
}
