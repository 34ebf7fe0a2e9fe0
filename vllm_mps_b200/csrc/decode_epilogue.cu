// The element-wise work between the GEMMs of a Llama decoder layer, fused so
// a CUDA-graph decode step runs ~8 kernels per layer instead of ~20.
//
// The reference runs these as HuggingFace modules, one PyTorch op each
// (transformers LlamaRMSNorm.forward: x.to(fp32), pow(2).mean(-1),
// x * rsqrt(var + eps), .to(dtype), weight * x; LlamaDecoderLayer.forward:
// residual + x; LlamaMLP.forward: act_fn(gate) * up with act_fn = SiLU).
// Each kernel below keeps those ops' rounding points, so its results are the
// modules' results up to the fp32 summation order of the variance.
//
//  * add_rmsnorm: residual <- round(residual + delta) (delta optional), then
//    out <- round(weight * round(residual * rsqrt(mean(residual^2) + eps))).
//    One CTA per row, 16-byte vector loads, a warp-shuffle + shared-memory
//    reduction of the fp32 sum of squares.
//  * silu_mul: out <- round(round(silu(gate)) * up) for a fused [gate | up]
//    GEMM output row, silu(g) = g / (1 + exp(-g)) in fp32.
//  * embed_rmsnorm: the step's token ids (from the host, or from the previous
//    step's device-side sampling), their embedding rows and the first
//    layer's input RMSNorm in one kernel.
//
// All are HBM-bound at any size (a few FLOPs per byte).
#include <type_traits>

#include "vmps_abi_internal.h"
#include "vmps_common.cuh"

namespace vmps {
namespace {

constexpr int kNormThreads = 256;

// Every kernel here is launched with programmatic dependent launch: it waits for
// the previous kernel's outputs, then at once lets the next kernel launch (a
// decode GEMM then streams its weights while this kernel runs).
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, cudaStream_t s,
                       Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

template <typename T>
__global__ void __launch_bounds__(kNormThreads)
    add_rmsnorm_kernel(T* __restrict__ out, T* __restrict__ residual, const T* __restrict__ delta,
                       const T* __restrict__ weight, int hidden, int64_t out_stride,
                       int64_t res_stride, int64_t delta_stride, float eps) {
  pdl_enter();
  const int row = blockIdx.x;
  T* r = residual + row * res_stride;
  const T* d = delta ? delta + row * delta_stride : nullptr;
  T* o = out + row * out_stride;
  const int n8 = hidden / 8;  // 16-byte vectors per row (hidden % 8 == 0)
  float ss = 0.f;
  // Residual update and the sum of squares (one pass; the row stays in L1/L2).
  for (int v = threadIdx.x; v < n8; v += kNormThreads) {
    uint4 rv = reinterpret_cast<const uint4*>(r)[v];
    T* re = reinterpret_cast<T*>(&rv);
    if (d) {
      const uint4 dv = reinterpret_cast<const uint4*>(d)[v];
      const T* de = reinterpret_cast<const T*>(&dv);
#pragma unroll
      for (int e = 0; e < 8; ++e) re[e] = Elt<T>::from_f(Elt<T>::to_f(re[e]) + Elt<T>::to_f(de[e]));
      reinterpret_cast<uint4*>(r)[v] = rv;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float x = Elt<T>::to_f(re[e]);
      ss = fmaf(x, x, ss);
    }
  }
  __shared__ float part[kNormThreads / 32];
#pragma unroll
  for (int sh = 16; sh > 0; sh >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, sh);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) tot += part[w];
  const float inv = rsqrtf(tot / static_cast<float>(hidden) + eps);
  for (int v = threadIdx.x; v < n8; v += kNormThreads) {
    const uint4 rv = reinterpret_cast<const uint4*>(r)[v];
    const uint4 wv = reinterpret_cast<const uint4*>(weight)[v];
    const T* re = reinterpret_cast<const T*>(&rv);
    const T* we = reinterpret_cast<const T*>(&wv);
    uint4 ov;
    T* oe = reinterpret_cast<T*>(&ov);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const T xn = Elt<T>::from_f(Elt<T>::to_f(re[e]) * inv);
      oe[e] = Elt<T>::from_f(Elt<T>::to_f(we[e]) * Elt<T>::to_f(xn));
    }
    reinterpret_cast<uint4*>(o)[v] = ov;
  }
}

// First kernel of a decode step: each row's input token, its embedding row
// (the residual stream) and the first layer's input RMSNorm.  The token of
// row i is prev[src[i]] when src is given and src[i] >= 0 (the id the
// previous step sampled on the device, so the host need not wait for it),
// else tokens[i].  residual <- table[token] (an exact copy, as an embedding
// lookup); out <- RMSNorm(residual) * weight with add_rmsnorm's rounding
// points.  A src entry at or above n_prev, or a token outside [0, vocab),
// sets kDevErrTokenRange and the row becomes zeros.
template <typename T>
__global__ void __launch_bounds__(kNormThreads)
    embed_rmsnorm_kernel(T* __restrict__ out, T* __restrict__ residual,
                         const T* __restrict__ table, int64_t vocab,
                         const int32_t* __restrict__ tokens, const int32_t* __restrict__ src,
                         const int64_t* __restrict__ prev, int n_prev, const T* __restrict__ weight,
                         int hidden, int64_t out_stride, int64_t res_stride, float eps, int* err) {
  pdl_enter();
  const int row = blockIdx.x;
  int64_t tok = tokens[row];
  if (src) {
    const int s = src[row];
    if (s >= 0) tok = s < n_prev ? prev[s] : int64_t(-1);
  }
  const bool ok = tok >= 0 && tok < vocab;
  if (!ok && threadIdx.x == 0) set_error(err, kDevErrTokenRange);
  const uint4* e = reinterpret_cast<const uint4*>(table + (ok ? tok : 0) * hidden);
  T* r = residual + row * res_stride;
  T* o = out + row * out_stride;
  const int n8 = hidden / 8;
  float ss = 0.f;
  for (int v = threadIdx.x; v < n8; v += kNormThreads) {
    uint4 rv = ok ? e[v] : make_uint4(0u, 0u, 0u, 0u);
    reinterpret_cast<uint4*>(r)[v] = rv;
    const T* re = reinterpret_cast<const T*>(&rv);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float x = Elt<T>::to_f(re[k]);
      ss = fmaf(x, x, ss);
    }
  }
  __shared__ float part[kNormThreads / 32];
#pragma unroll
  for (int sh = 16; sh > 0; sh >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, sh);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) tot += part[w];
  const float inv = rsqrtf(tot / static_cast<float>(hidden) + eps);
  for (int v = threadIdx.x; v < n8; v += kNormThreads) {
    const uint4 rv = reinterpret_cast<const uint4*>(r)[v];
    const uint4 wv = reinterpret_cast<const uint4*>(weight)[v];
    const T* re = reinterpret_cast<const T*>(&rv);
    const T* we = reinterpret_cast<const T*>(&wv);
    uint4 ov;
    T* oe = reinterpret_cast<T*>(&ov);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const T xn = Elt<T>::from_f(Elt<T>::to_f(re[k]) * inv);
      oe[k] = Elt<T>::from_f(Elt<T>::to_f(we[k]) * Elt<T>::to_f(xn));
    }
    reinterpret_cast<uint4*>(o)[v] = ov;
  }
}

template <typename T>
__global__ void silu_mul_kernel(T* __restrict__ out, const T* __restrict__ gate_up, int inter,
                                int64_t out_stride, int64_t in_stride) {
  pdl_enter();
  const int row = blockIdx.y;
  const int v = blockIdx.x * blockDim.x + threadIdx.x;  // 16-byte vector within the row
  if (v >= inter / 8) return;
  const T* g = gate_up + row * in_stride;
  const uint4 gv = reinterpret_cast<const uint4*>(g)[v];
  const uint4 uv = reinterpret_cast<const uint4*>(g + inter)[v];
  const T* ge = reinterpret_cast<const T*>(&gv);
  const T* ue = reinterpret_cast<const T*>(&uv);
  uint4 ov;
  T* oe = reinterpret_cast<T*>(&ov);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float x = Elt<T>::to_f(ge[e]);
    const T s = Elt<T>::from_f(x / (1.f + expf(-x)));
    oe[e] = Elt<T>::from_f(Elt<T>::to_f(s) * Elt<T>::to_f(ue[e]));
  }
  reinterpret_cast<uint4*>(out + row * out_stride)[v] = ov;
}

bool aligned_rows(const void* p, int64_t stride) {
  return aligned16(p) && (stride % 8) == 0;
}

}  // namespace
}  // namespace vmps

using namespace vmps;

extern "C" int vmps_add_rmsnorm(void* out, int64_t out_stride, void* residual, int64_t res_stride,
                                const void* delta, int64_t delta_stride, const void* weight,
                                int rows, int hidden, float eps, int dtype, void* stream) {
  clear_error();
  if (rows < 0 || hidden <= 0 || hidden % 8 || !(eps >= 0.f)) {
    return fail(VMPS_ERR_INVALID_ARG, "add_rmsnorm: rows=%d hidden=%d eps=%g", rows, hidden,
                (double)eps);
  }
  if (rows == 0) return VMPS_OK;
  if (!out || !residual || !weight) return fail(VMPS_ERR_INVALID_ARG, "add_rmsnorm: NULL pointer");
  if (!aligned_rows(out, out_stride) || !aligned_rows(residual, res_stride) || !aligned16(weight) ||
      (delta && !aligned_rows(delta, delta_stride))) {
    return fail(VMPS_ERR_ALIGNMENT,
                "add_rmsnorm: rows must be 16-byte aligned with strides multiples of 8 elements");
  }
  if (dtype != VMPS_DTYPE_F16 && dtype != VMPS_DTYPE_BF16) {
    return fail(VMPS_ERR_INVALID_ARG, "add_rmsnorm: dtype %d", dtype);
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (dtype == VMPS_DTYPE_F16) {
    e = launch_pdl(add_rmsnorm_kernel<__half>, dim3(rows), dim3(kNormThreads), s,
                   static_cast<__half*>(out), static_cast<__half*>(residual),
                   static_cast<const __half*>(delta), static_cast<const __half*>(weight), hidden,
                   out_stride, res_stride, delta_stride, eps);
  } else {
    e = launch_pdl(add_rmsnorm_kernel<__nv_bfloat16>, dim3(rows), dim3(kNormThreads), s,
                   static_cast<__nv_bfloat16*>(out), static_cast<__nv_bfloat16*>(residual),
                   static_cast<const __nv_bfloat16*>(delta),
                   static_cast<const __nv_bfloat16*>(weight), hidden, out_stride, res_stride,
                   delta_stride, eps);
  }
  if (e != cudaSuccess) {
    return fail(VMPS_ERR_CUDA, "add_rmsnorm: launch failed: %s", cudaGetErrorString(e));
  }
  return VMPS_OK;
}

extern "C" int vmps_embed_rmsnorm(void* out, int64_t out_stride, void* residual,
                                  int64_t res_stride, const void* table, int64_t vocab,
                                  const int32_t* tokens, const int32_t* src, const int64_t* prev,
                                  int n_prev, const void* weight, int rows, int hidden, float eps,
                                  int dtype, void* stream) {
  clear_error();
  if (rows < 0 || hidden <= 0 || hidden % 8 || vocab <= 0 || !(eps >= 0.f)) {
    return fail(VMPS_ERR_INVALID_ARG, "embed_rmsnorm: rows=%d hidden=%d vocab=%lld eps=%g", rows,
                hidden, (long long)vocab, (double)eps);
  }
  if (rows == 0) return VMPS_OK;
  if (!out || !residual || !table || !tokens || !weight || (src && (!prev || n_prev < 0))) {
    return fail(VMPS_ERR_INVALID_ARG, "embed_rmsnorm: NULL pointer or n_prev < 0");
  }
  if (!aligned_rows(out, out_stride) || !aligned_rows(residual, res_stride) || !aligned16(table) ||
      !aligned16(weight)) {
    return fail(VMPS_ERR_ALIGNMENT,
                "embed_rmsnorm: rows must be 16-byte aligned with strides multiples of 8 elements");
  }
  if (dtype != VMPS_DTYPE_F16 && dtype != VMPS_DTYPE_BF16) {
    return fail(VMPS_ERR_INVALID_ARG, "embed_rmsnorm: dtype %d", dtype);
  }
  int* err = nullptr;
  if (int rc = device_error_word(&err)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (dtype == VMPS_DTYPE_F16) {
    e = launch_pdl(embed_rmsnorm_kernel<__half>, dim3(rows), dim3(kNormThreads), s,
                   static_cast<__half*>(out), static_cast<__half*>(residual),
                   static_cast<const __half*>(table), vocab, tokens, src, prev, n_prev,
                   static_cast<const __half*>(weight), hidden, out_stride, res_stride, eps, err);
  } else {
    e = launch_pdl(embed_rmsnorm_kernel<__nv_bfloat16>, dim3(rows), dim3(kNormThreads), s,
                   static_cast<__nv_bfloat16*>(out), static_cast<__nv_bfloat16*>(residual),
                   static_cast<const __nv_bfloat16*>(table), vocab, tokens, src, prev, n_prev,
                   static_cast<const __nv_bfloat16*>(weight), hidden, out_stride, res_stride, eps,
                   err);
  }
  if (e != cudaSuccess) {
    return fail(VMPS_ERR_CUDA, "embed_rmsnorm: launch failed: %s", cudaGetErrorString(e));
  }
  return VMPS_OK;
}

extern "C" int vmps_silu_mul(void* out, int64_t out_stride, const void* gate_up,
                             int64_t in_stride, int rows, int inter, int dtype, void* stream) {
  clear_error();
  if (rows < 0 || inter <= 0 || inter % 8) {
    return fail(VMPS_ERR_INVALID_ARG, "silu_mul: rows=%d inter=%d", rows, inter);
  }
  if (rows == 0) return VMPS_OK;
  if (!out || !gate_up) return fail(VMPS_ERR_INVALID_ARG, "silu_mul: NULL pointer");
  if (!aligned_rows(out, out_stride) || !aligned_rows(gate_up, in_stride)) {
    return fail(VMPS_ERR_ALIGNMENT,
                "silu_mul: rows must be 16-byte aligned with strides multiples of 8 elements");
  }
  if (rows > 65535) return fail(VMPS_ERR_UNSUPPORTED, "silu_mul: rows %d > 65535", rows);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid((inter / 8 + 127) / 128, rows);
  cudaError_t e;
  if (dtype == VMPS_DTYPE_F16) {
    e = launch_pdl(silu_mul_kernel<__half>, grid, dim3(128), s, static_cast<__half*>(out),
                   static_cast<const __half*>(gate_up), inter, out_stride, in_stride);
  } else if (dtype == VMPS_DTYPE_BF16) {
    e = launch_pdl(silu_mul_kernel<__nv_bfloat16>, grid, dim3(128), s,
                   static_cast<__nv_bfloat16*>(out), static_cast<const __nv_bfloat16*>(gate_up),
                   inter, out_stride, in_stride);
  } else {
    return fail(VMPS_ERR_INVALID_ARG, "silu_mul: dtype %d", dtype);
  }
  if (e != cudaSuccess) {
    return fail(VMPS_ERR_CUDA, "silu_mul: launch failed: %s", cudaGetErrorString(e));
  }
  return VMPS_OK;
}
