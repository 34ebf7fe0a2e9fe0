/*
 * vmps.h -- C ABI of libvmps_kernels.so, the sm_100a (B200) kernels behind
 * the paged decode-attention step of vllm_mps.
 *
 * The reference (Nihar0071/vllm_mps) has no C ABI: its device code is two
 * Metal shaders held as Python strings and its CPU path is PyTorch code.
 * Each entry point below names the reference interface it replaces.  The
 * Python side binds these symbols with ctypes (vllm_mps_b200/kernels).
 *
 * Conventions shared by every entry point:
 *   - All pointers are device pointers unless stated; the caller owns every
 *     buffer.  The library allocates nothing; besides the device error word
 *     it keeps one fixed scratch array in its own device memory, used only
 *     by vmps_paged_decode_attention_noalloc (its calls must not overlap on
 *     the GPU).
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Work is
 *     only enqueued; calls return before the GPU finishes.
 *   - `dtype` is VMPS_DTYPE_F16 or VMPS_DTYPE_BF16 for every 16-bit tensor
 *     of the call (q, k, v, pool, out).
 *   - The KV pool has the reference layout
 *       pool[num_blocks][2][block_size][n_kv][head_dim]   (dim 1: 0 = K, 1 = V)
 *     (memory/mps_memory_pool.py:62-66), contiguous.
 *   - Return 0 on success or a negative VMPS_ERR_* code; vmps_last_error()
 *     then describes the failure (thread-local).  Arguments are checked on
 *     the host before anything is launched.  Device-side index violations
 *     skip the access and set a bit in the error word (vmps_debug_error_word).
 */
#ifndef VMPS_H_
#define VMPS_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VMPS_OK 0
#define VMPS_ERR_INVALID_ARG (-1)  /* bad pointer, size or shape */
#define VMPS_ERR_UNSUPPORTED (-2)  /* valid but not built (e.g. head_dim 96) */
#define VMPS_ERR_ALIGNMENT (-3)    /* a pointer or stride is not 16-byte aligned */
#define VMPS_ERR_WORKSPACE (-4)    /* workspace missing or too small */
#define VMPS_ERR_CUDA (-5)         /* CUDA runtime/driver error */

#define VMPS_DTYPE_F16 0
#define VMPS_DTYPE_BF16 1

/* Library version string, e.g. "vmps 0.1.0 sm_100a". */
const char* vmps_version(void);

/* Description of the last failure on the calling thread ("" if none). */
const char* vmps_last_error(void);

/*
 * Fused RoPE + reshape-and-cache (kernel 1).
 *
 * Replaces the per-sequence RoPE loop and K/V write loop of
 * PagedAttentionLayer._forward_batch (layers/paged_attention_layer.py:275-286
 * and :317-324), i.e. RotaryEmbedding.forward (layers/rotary_embedding.py:55-76)
 * followed by MPSMemoryPool.write_kv (memory/mps_memory_pool.py:82-102), and
 * Phase 1 of the Metal fused_attention shader (kernels/__init__.py:139-161).
 *
 * For each sequence i in [0, num_seqs):
 *   q_out[i] = rope(q[i], positions[i])                  (n_q heads)
 *   pool[slot / block_size][0][slot % block_size] = rope(k[i], positions[i])
 *   pool[slot / block_size][1][slot % block_size] = v[i]
 * with slot = slot_mapping[i] (= block_table[pos / block_size] * block_size
 * + pos % block_size); a negative slot skips the write.  rope() is the
 * rotate-half form with cos/sin = cos/sin(position * inv_freq[j]) rounded
 * to the model dtype and each product and the sum rounded to the model
 * dtype, as the reference computes it.  inv_freq (head_dim/2 floats) = NULL
 * means "no rotation" (K/V are written as given, q_out = q).
 *
 * q/k/v rows are head-major [heads][head_dim] with a row stride in elements
 * between sequences (so slices of a fused QKV output work).  q_out may equal
 * q (in-place) and uses q_row_stride too.  positions and slot_mapping are
 * int32[num_seqs] on the device.
 */
int vmps_rope_reshape_and_cache(void* q_out, const void* q, int64_t q_row_stride,
                                const void* k, int64_t k_row_stride, const void* v,
                                int64_t v_row_stride, const int32_t* positions,
                                const int32_t* slot_mapping, const float* inv_freq, void* pool,
                                int num_seqs, int n_q, int n_kv, int head_dim, int block_size,
                                int num_blocks, int dtype, void* stream);

/*
 * Workspace needed by vmps_paged_decode_attention / vmps_paged_decode_step
 * on the current device for up to `num_seqs` sequences: split-K partial
 * results of sequences cut between CTAs, and one arrival counter per kv head
 * and sequence (a fixed 1 MiB region, so one workspace serves calls of any
 * shape).  The workspace must be zero-filled once after allocation
 * (vmps_paged_decode_workspace_init); every call leaves the counters at zero
 * again.  Calls sharing a workspace must be ordered (same stream).  Returns 0
 * if the shape is unsupported.
 */
size_t vmps_paged_decode_workspace_bytes(int num_seqs, int n_q, int n_kv, int head_dim,
                                         int dtype);

/* cudaMemsetAsync(workspace, 0, bytes, stream): the one-time initialisation
 * a new workspace needs. */
int vmps_paged_decode_workspace_init(void* workspace, size_t workspace_bytes, void* stream);

/*
 * Paged decode attention (kernel 2), one query token per sequence.
 *
 * Replaces the gather/pad loop, GQA expansion and masked softmax attention of
 * PagedAttentionLayer._forward_batch (layers/paged_attention_layer.py:326-359),
 * MPSMemoryPool.gather_blocks_tensor (memory/mps_memory_pool.py:159-176), and
 * Phases 2-4 of the Metal fused_attention shader (kernels/__init__.py:166-241).
 *
 *   out[i][h][:] = softmax_t( scale * q[i][h] . K_i[t][h / G] ) . V_i[t][h / G]
 * for t < seq_lens[i], G = n_q / n_kv, where K_i[t] / V_i[t] is slot
 * t % block_size of block block_tables[i * max_blocks_per_seq + t / block_size].
 * Computed with fp32 scores, fp32 online softmax and fp32 accumulation;
 * out is rounded once to the model dtype.  q and out are [num_seqs][n_q][head_dim]
 * contiguous (q and the pool 16-byte aligned, out 2-byte aligned:
 * VMPS_ERR_ALIGNMENT otherwise); seq_lens counts the new token; block tables are int32, only
 * the first ceil(seq_len / block_size) entries of a row are read.  A
 * sequence with seq_len 0 gets a zero output row.
 *
 * Supported: head_dim 64 or 128, block_size 16, n_q / n_kv in {1,2,4,8,16},
 * n_kv <= 64, num_seqs <= 4096.  Long sequences are split across CTAs (flash-decoding)
 * and the last piece to finish merges them in the same launch.  The kernel
 * is launched with programmatic dependent launch (it waits for the
 * preceding kernel's writes before reading anything).
 */
int vmps_paged_decode_attention(void* out, const void* q, const void* pool,
                                const int32_t* block_tables, int max_blocks_per_seq,
                                const int32_t* seq_lens, int num_seqs, int n_q, int n_kv,
                                int head_dim, int block_size, int num_blocks, float scale,
                                void* workspace, size_t workspace_bytes, int dtype, void* stream);

/*
 * One decode step of one attention layer in a single kernel launch.
 *
 * Same result as vmps_rope_reshape_and_cache (rotated K and V written to
 * the pool slot) followed by vmps_paged_decode_attention on the rotated q,
 * i.e. PagedAttentionLayer's batched step between its projections
 * (layers/paged_attention_layer.py:275-359) and the whole Metal
 * fused_attention shader (kernels/__init__.py:99-242) with RoPE folded in.
 * q is rotated in registers and left unchanged in memory.  Requirements:
 * seq_lens[i] >= 1 and slot_mapping[i] addresses a slot of the last page of
 * sequence i (as the reference's write_info always does for position
 * seq_len-1); otherwise the write is flagged in the error word (bit 32).
 * The launch may start while the kernel before it on the stream still runs
 * (programmatic dependent launch): the step metadata -- seq_lens, block
 * tables, positions, slot_mapping, inv_freq -- is read before that kernel
 * finishes, so it must not produce them (pool pages are only pulled into L2
 * then, which is coherent with its writes); q/k/v and the pool contents are
 * read after it finishes.
 * q/k/v rows may have any row stride (slices of a fused QKV output).
 */
int vmps_paged_decode_step(void* out, void* q, int64_t q_row_stride, const void* k,
                           int64_t k_row_stride, const void* v, int64_t v_row_stride,
                           const int32_t* positions, const int32_t* slot_mapping,
                           const float* inv_freq, void* pool, const int32_t* block_tables,
                           int max_blocks_per_seq, const int32_t* seq_lens, int num_seqs, int n_q,
                           int n_kv, int head_dim, int block_size, int num_blocks, float scale,
                           void* workspace, size_t workspace_bytes, int dtype, void* stream);

/*
 * Allocation-free variant of vmps_paged_decode_attention.  No counterpart in
 * the reference.  It exists for callers that cannot allocate device memory
 * while running (a C/FFI host without a caching allocator, or a process that
 * has already reserved all free HBM for its KV pool), which therefore cannot
 * pass the workspace the other entry point needs.
 *
 * Same arguments and results as vmps_paged_decode_attention minus the
 * workspace: the split-K scratch is a fixed 8 MiB device array inside the
 * library, held on every GPU that loads the library until exit.  Calls that
 * would need more scratch (vmps_paged_decode_workspace_bytes) return
 * VMPS_ERR_WORKSPACE; on a 148-SM B200 every supported shape with up to 8
 * query heads per kv head fits, 16 query heads per kv head does not.  All calls
 * on a device share the array, so calls that may overlap on the GPU race and
 * must be ordered on one stream.  Every call first clears the merge counters
 * it uses (n_kv * num_seqs ints) with a cudaMemsetAsync on `stream`, so a
 * call that gave up a bounded wait (error bit 8) cannot disturb the next.
 * The first call on a device looks up the array's address
 * (cudaGetSymbolAddress) and caches it; make that first call before any
 * stream capture.  Allocates nothing (no cudaMalloc/cudaFree).
 */
int vmps_paged_decode_attention_noalloc(void* out, const void* q, const void* pool,
                                        const int32_t* block_tables, int max_blocks_per_seq,
                                        const int32_t* seq_lens, int num_seqs, int n_q, int n_kv,
                                        int head_dim, int block_size, int num_blocks, float scale,
                                        int dtype, void* stream);

/*
 * Causal paged prefill attention (kernel 3, tcgen05 tensor cores).  Replaces
 * the reference's prompt processing, which runs the single-token path once
 * per prompt token (layers/paged_attention_layer.py:175-241, driven by
 * benchmarks/batch_size_benchmark.py:49-60): row r of sequence i sits at
 * position q_start_pos[i] + r and attends to the sequence's slots
 * 0..q_start_pos[i] + r, which must already hold K/V (written by
 * vmps_rope_reshape_and_cache for the new rows).
 *
 * q:    [total_q rows][n_q][head_dim], rotated (kernel 1's q_out), row r of
 *       sequence i at cu_q[i] + r; row stride q_row_stride elements
 *       (multiple of 8).  16-byte aligned.
 * out:  [total_q][n_q][head_dim], contiguous, same dtype; rows are written
 *       only for r < q_lens[i].
 * q_start_pos, q_lens, cu_q: int32 [num_seqs] on the device.  max_q_len
 *       bounds q_lens (it sizes the grid; rows past it are not computed and
 *       set error bit 64).
 * block_tables: int32 [num_seqs][max_blocks_per_seq] covering
 *       q_start_pos[i] + q_lens[i] slots.
 * Supported: head_dim 64 or 128, block_size 16, n_q/n_kv in {1,2,4,8,16}.
 * Allocates nothing; no workspace.
 */
int vmps_paged_prefill_attention(void* out, const void* q, int64_t q_row_stride,
                                 const void* pool, const int32_t* block_tables,
                                 int max_blocks_per_seq, const int32_t* q_start_pos,
                                 const int32_t* q_lens, const int32_t* cu_q, int num_seqs,
                                 int total_q, int max_q_len, int n_q, int n_kv, int head_dim,
                                 int block_size, int num_blocks, float scale, int dtype,
                                 void* stream);

/*
 * Element-wise work between the GEMMs of a Llama decoder layer, fused for
 * the CUDA-graph decode step.  No kernel counterpart in the reference, which
 * runs these as HuggingFace modules (LlamaRMSNorm, the residual additions of
 * LlamaDecoderLayer, SiLU(gate) * up of LlamaMLP); the rounding points of
 * those modules are kept.
 *
 * vmps_add_rmsnorm: residual <- residual + delta (delta may be NULL), then
 *   out <- weight * (residual * rsqrt(mean(residual^2) + eps)) for `rows`
 *   rows of `hidden` elements (hidden % 8 == 0; rows 16-byte aligned).
 * vmps_silu_mul: out[:, :inter] <- silu(gate_up[:, :inter]) * gate_up[:, inter:2*inter].
 * vmps_embed_rmsnorm: the step's first kernel (the HF embedding lookup and
 *   the first layer's input LlamaRMSNorm).  Row i's token is prev[src[i]]
 *   when src is non-NULL and src[i] >= 0 (an id the previous step sampled on
 *   the device: a pipelined engine launches step k+1 before it reads step
 *   k's tokens back), else tokens[i]; residual[i] <- table[token] (table:
 *   [vocab, hidden]), out[i] <- RMSNorm(residual[i]) * weight as
 *   vmps_add_rmsnorm with delta NULL.  src[i] >= n_prev or a token outside
 *   [0, vocab) sets error bit 128 and zeroes the row.
 */
int vmps_add_rmsnorm(void* out, int64_t out_row_stride, void* residual, int64_t res_row_stride,
                     const void* delta, int64_t delta_row_stride, const void* weight, int rows,
                     int hidden, float eps, int dtype, void* stream);
int vmps_silu_mul(void* out, int64_t out_row_stride, const void* gate_up,
                  int64_t in_row_stride, int rows, int inter, int dtype, void* stream);
int vmps_embed_rmsnorm(void* out, int64_t out_row_stride, void* residual,
                       int64_t res_row_stride, const void* table, int64_t vocab,
                       const int32_t* tokens, const int32_t* src, const int64_t* prev,
                       int n_prev, const void* weight, int rows, int hidden, float eps,
                       int dtype, void* stream);

/*
 * Decode GEMM for the projections around the attention step at decode batch
 * sizes (replaces the nn.Linear calls of the HF decoder layer that the
 * reference's models/llama_adapter.py:137-207 runs: q/k/v, o, gate/up and
 * down projections).  out[M, N] = x[M, K] . w[N, K]^T, fp32 accumulation,
 * rounded to the 16-bit type.  With silu_mul != 0, w is the fused [gate; up]
 * weight of 2N rows and out[M, N] = silu(x . Wg^T) * (x . Wu^T), each
 * projection rounded first (transformers LlamaMLP).
 * Shapes: M <= 8, N % 8 == 0, K % 64 == 0, K <= 8192; x and w 16-byte
 * aligned, x rows a multiple of 8 elements apart; out 4-byte aligned with an
 * even row stride.  vmps_decode_gemm_supported says whether a shape is
 * built (1) or not (0), so a caller can fall back to its GEMM library.
 * Launched with programmatic dependent launch: the weight stream starts
 * before the wait on the previous kernel in the stream.
 */
int vmps_decode_gemm_supported(int M, int N, int K, int silu_mul);
int vmps_decode_gemm(void* out, int64_t out_row_stride, const void* x, int64_t x_row_stride,
                     const void* w, int M, int N, int K, int silu_mul, int dtype, void* stream);

/*
 * Batch GEMM for the same projections at decode batch sizes 1..256 (the
 * nn.Linear calls of models/llama_adapter.py:137-207 at the engine's batch;
 * no kernel counterpart in the reference): out[M, N] = x[M, K] . w[N, K]^T,
 * fp16 or bf16, fp32 accumulation on the tcgen05 tensor cores, one rounding.
 * Requires N % 128 == 0, K % 64 == 0, x, w and out 16-byte aligned, x and
 * out rows a multiple of 8 elements apart (x rows at least K, out rows at
 * least N).  Narrow shapes split K over a thread-block cluster of up to 4
 * CTAs whose fp32 partials are summed (in a fixed order) through the
 * caller's workspace: vmps_batch_gemm_split returns that cluster size for a
 * shape on the current device (0 = shape not built) and
 * vmps_batch_gemm_workspace_bytes the workspace it needs (0 = none; at most
 * 16 MiB), which must be 16-byte aligned; it needs no initialisation, and
 * calls that may overlap on the GPU need different workspaces (calls on one
 * stream never overlap).  VMPS_ERR_WORKSPACE if it is missing or too small.
 * Launched with programmatic dependent launch: the weight stream starts
 * before the previous kernel has finished.
 */
int vmps_batch_gemm_split(int M, int N, int K);
size_t vmps_batch_gemm_workspace_bytes(int M, int N, int K, int dtype);
int vmps_batch_gemm(void* out, int64_t out_row_stride, const void* x, int64_t x_row_stride,
                    const void* w, int M, int N, int K, void* workspace, size_t workspace_bytes,
                    int dtype, void* stream);

/*
 * Copies `bytes` from `src` to `dst` with the GPU's own loads and stores,
 * as a link of a chain of kernels launched with programmatic dependent
 * launch.  No counterpart in the reference (whose inputs never leave host
 * memory).  `src` may be pinned host memory: this is how a serving loop
 * stages a decode step's inputs from the host without a copy-engine copy
 * between two decode steps, which would cost the second step its early
 * launch.  The copy starts while the kernel before it on the stream still
 * runs and does not wait for it; the launch then completes only after that
 * kernel has, so the kernel after it finds both finished.  Therefore `dst`
 * must not be read or written by the kernel immediately before this one on
 * the stream (earlier kernels have completed).  A fused decode step reads
 * its step metadata before its own PDL wait, so between the
 * stage copy of its inputs and the step itself there must be a kernel that
 * waits before it lets the next one start (another decode step): stage
 * step i+1 just before step i (three staging buffers), and stage the first
 * step of a chain with an ordinary copy.  Both pointers 16-byte aligned,
 * bytes a multiple of 16.
 */
int vmps_stage_copy(void* dst, const void* src, size_t bytes, void* stream);

/*
 * Reads and clears the device error word of the current device (a bitwise OR
 * of index violations the kernels skipped since the last call).  Synchronises
 * `stream`.  Bits: 1 slot out of range, 2 block id out of range, 4 seq_len
 * beyond the block table, 8 an internal wait timed out, 16 negative position,
 * 32 a fused-step slot outside the sequence's last page, 64 prefill query
 * rows outside [0, total_q) or a q_len above max_q_len.
 */
int vmps_debug_error_word(void* stream, int* word_out);

#ifdef __cplusplus
}
#endif

#endif /* VMPS_H_ */
