"""Python bindings of libvmps_kernels.so (the sm_100a kernels of the decode step).

This module replaces the reference's ``vllm_mps.kernels`` (Metal shaders
compiled through ``torch.mps.compile_shader``, kernels/__init__.py:245-406).
It binds the C ABI declared in ``include/vmps.h`` with ctypes and passes raw
device pointers plus the current CUDA stream.  There is no CPU or PyTorch
fallback: if the shared library is missing or a tensor is not on a CUDA
device, the call raises.

Public functions
----------------
* :func:`rope_reshape_and_cache` -- kernel 1 (RoPE on Q/K + K/V write).
* :func:`paged_decode_attention` -- kernel 2 (paged GQA decode attention).
* :func:`fused_attention` / :func:`fused_attention_metal_fast` -- the
  reference's fused entry point (kernels/__init__.py:320-368): write the
  already-rotated new K/V into the slot given by ``write_info`` and attend.
* :func:`gather_kv` -- the reference's padded paged gather
  (kernels/__init__.py:279-312), kept for API compatibility.
"""

from __future__ import annotations

import ctypes
import math
import os
import threading

import torch

_PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(_PKG_DIR, "libvmps_kernels.so")

VMPS_DTYPE_F16 = 0
VMPS_DTYPE_BF16 = 1

_ERRORS = {
    -1: ValueError,        # VMPS_ERR_INVALID_ARG
    -2: NotImplementedError,  # VMPS_ERR_UNSUPPORTED
    -3: ValueError,        # VMPS_ERR_ALIGNMENT
    -4: RuntimeError,      # VMPS_ERR_WORKSPACE
    -5: RuntimeError,      # VMPS_ERR_CUDA
}

#: Symbols every build of the library exports (mirrors include/vmps.h).
EXPORTED_SYMBOLS = (
    "vmps_version",
    "vmps_last_error",
    "vmps_rope_reshape_and_cache",
    "vmps_paged_decode_workspace_bytes",
    "vmps_paged_decode_workspace_init",
    "vmps_paged_decode_attention",
    "vmps_paged_decode_step",
    "vmps_paged_prefill_attention",
    "vmps_add_rmsnorm",
    "vmps_silu_mul",
    "vmps_embed_rmsnorm",
    "vmps_decode_gemm_supported",
    "vmps_decode_gemm",
    "vmps_batch_gemm_split",
    "vmps_batch_gemm_workspace_bytes",
    "vmps_batch_gemm",
    "vmps_stage_copy",
    "vmps_debug_error_word",
)

_lib = None
_lib_lock = threading.Lock()


def load_library(path: str | None = None) -> ctypes.CDLL:
    """Load (once) and return the kernel library, declaring every signature."""
    global _lib
    with _lib_lock:
        if _lib is not None and path is None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise ImportError(
                f"{p} is missing: build it with `python -m vllm_mps_b200.build` "
                "(there is no CPU fallback for the CUDA kernels)")
        lib = ctypes.CDLL(p)
        vp, i32, i64, f32, sz = (ctypes.c_void_p, ctypes.c_int, ctypes.c_int64,
                                 ctypes.c_float, ctypes.c_size_t)
        lib.vmps_version.restype = ctypes.c_char_p
        lib.vmps_version.argtypes = []
        lib.vmps_last_error.restype = ctypes.c_char_p
        lib.vmps_last_error.argtypes = []
        lib.vmps_rope_reshape_and_cache.restype = i32
        lib.vmps_rope_reshape_and_cache.argtypes = [
            vp, vp, i64, vp, i64, vp, i64, vp, vp, vp, vp,
            i32, i32, i32, i32, i32, i32, i32, vp]
        lib.vmps_paged_decode_workspace_bytes.restype = sz
        lib.vmps_paged_decode_workspace_bytes.argtypes = [i32, i32, i32, i32, i32]
        lib.vmps_paged_decode_workspace_init.restype = i32
        lib.vmps_paged_decode_workspace_init.argtypes = [vp, sz, vp]
        lib.vmps_paged_decode_attention.restype = i32
        lib.vmps_paged_decode_attention.argtypes = [
            vp, vp, vp, vp, i32, vp, i32, i32, i32, i32, i32, i32, f32, vp, sz, i32, vp]
        lib.vmps_paged_decode_step.restype = i32
        lib.vmps_paged_decode_step.argtypes = [
            vp, vp, i64, vp, i64, vp, i64, vp, vp, vp, vp, vp, i32, vp,
            i32, i32, i32, i32, i32, i32, f32, vp, sz, i32, vp]
        lib.vmps_paged_prefill_attention.restype = i32
        lib.vmps_paged_prefill_attention.argtypes = [
            vp, vp, i64, vp, vp, i32, vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, i32,
            f32, i32, vp]
        lib.vmps_add_rmsnorm.restype = i32
        lib.vmps_add_rmsnorm.argtypes = [vp, i64, vp, i64, vp, i64, vp, i32, i32, f32, i32, vp]
        lib.vmps_silu_mul.restype = i32
        lib.vmps_silu_mul.argtypes = [vp, i64, vp, i64, i32, i32, i32, vp]
        lib.vmps_embed_rmsnorm.restype = i32
        lib.vmps_embed_rmsnorm.argtypes = [vp, i64, vp, i64, vp, i64, vp, vp, vp, i32, vp, i32,
                                           i32, f32, i32, vp]
        lib.vmps_decode_gemm_supported.restype = i32
        lib.vmps_decode_gemm_supported.argtypes = [i32, i32, i32, i32]
        lib.vmps_decode_gemm.restype = i32
        lib.vmps_decode_gemm.argtypes = [vp, i64, vp, i64, vp, i32, i32, i32, i32, i32, vp]
        lib.vmps_batch_gemm_split.restype = i32
        lib.vmps_batch_gemm_split.argtypes = [i32, i32, i32]
        lib.vmps_batch_gemm_workspace_bytes.restype = ctypes.c_size_t
        lib.vmps_batch_gemm_workspace_bytes.argtypes = [i32, i32, i32, i32]
        lib.vmps_batch_gemm.restype = i32
        lib.vmps_batch_gemm.argtypes = [vp, i64, vp, i64, vp, i32, i32, i32, vp, ctypes.c_size_t,
                                        i32, vp]
        lib.vmps_stage_copy.restype = i32
        lib.vmps_stage_copy.argtypes = [vp, vp, sz, vp]
        lib.vmps_debug_error_word.restype = i32
        lib.vmps_debug_error_word.argtypes = [vp, ctypes.POINTER(ctypes.c_int)]
        if path is None:
            _lib = lib
        return lib


def _check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load_library().vmps_last_error().decode(errors="replace")
        raise _ERRORS.get(rc, RuntimeError)(f"{what}: {msg or 'error %d' % rc}")


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float16:
        return VMPS_DTYPE_F16
    if dtype == torch.bfloat16:
        return VMPS_DTYPE_BF16
    raise TypeError(f"unsupported dtype {dtype} (float16 or bfloat16)")


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(
                f"vllm_mps_b200 kernels need CUDA tensors (got a {t.device} tensor); "
                "there is no CPU fallback")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} and {t.device}")
    return dev


def _int32(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dtype != torch.int32:
        raise TypeError(f"{name} must be int32 (got {t.dtype})")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t


def _check_pool(pool: torch.Tensor):
    if pool.dim() != 5 or pool.shape[1] != 2:
        raise ValueError(f"pool must be (num_blocks, 2, block_size, n_kv, head_dim); got {tuple(pool.shape)}")
    if not pool.is_contiguous():
        raise ValueError("pool must be contiguous")
    return pool.shape[0], pool.shape[2], pool.shape[3], pool.shape[4]


def _rows(t: torch.Tensor, heads: int, d: int, name: str):
    """(B, heads, d) or (B, heads*d) view with unit inner strides -> row stride."""
    if t.dim() == 3:
        if t.shape[1:] != (heads, d) or t.stride(2) != 1 or t.stride(1) != d:
            raise ValueError(f"{name}: expected (B, {heads}, {d}) with packed heads")
        return t.stride(0)
    if t.dim() == 2:
        if t.shape[1] != heads * d or t.stride(1) != 1:
            raise ValueError(f"{name}: expected (B, {heads * d})")
        return t.stride(0)
    raise ValueError(f"{name}: expected 2-D or 3-D tensor")


# ── kernel 1 ─────────────────────────────────────────────────────────────────


def rope_reshape_and_cache(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                           positions: torch.Tensor | None, slot_mapping: torch.Tensor,
                           inv_freq: torch.Tensor | None, pool: torch.Tensor,
                           q_out: torch.Tensor | None = None) -> torch.Tensor:
    """RoPE on q and k, then write rotated k and v into ``pool`` at ``slot_mapping``.

    ``q``: (B, n_q, D) or (B, n_q*D); ``k``/``v``: (B, n_kv, D) or (B, n_kv*D)
    (row strides may be larger, e.g. slices of a fused QKV output).
    ``positions``/``slot_mapping``: int32 (B,).  ``inv_freq``: fp32 (D/2,) or
    None (no rotation).  Returns ``q_out`` (default: ``q`` rotated in place).
    Same semantics as the reference's per-sequence loop
    (layers/paged_attention_layer.py:275-286, :317-324).
    """
    num_blocks, block_size, n_kv, D = _check_pool(pool)
    B = k.shape[0]
    n_q = (q.shape[1] if q.dim() == 3 else q.shape[1] // D) if q is not None else 0
    if q_out is None:
        q_out = q
    dev = _require_cuda(q, k, v, positions, slot_mapping, inv_freq, pool, q_out)
    for t, name in ((q, "q"), (k, "k"), (v, "v"), (q_out, "q_out")):
        if t is not None and t.dtype != pool.dtype:
            raise TypeError(f"{name} dtype {t.dtype} != pool dtype {pool.dtype}")
    qs = _rows(q, n_q, D, "q") if n_q else 0
    if q_out is not q and n_q:
        if _rows(q_out, n_q, D, "q_out") != qs:
            raise ValueError("q_out must have the same row stride as q")
    ks = _rows(k, n_kv, D, "k")
    vs = _rows(v, n_kv, D, "v")
    _int32(slot_mapping, "slot_mapping")
    if positions is not None:
        _int32(positions, "positions")
    if inv_freq is not None:
        if inv_freq.dtype != torch.float32 or inv_freq.numel() != D // 2 or not inv_freq.is_contiguous():
            raise ValueError(f"inv_freq must be contiguous float32 of {D // 2} entries")
    lib = load_library()
    with torch.cuda.device(dev):
        rc = lib.vmps_rope_reshape_and_cache(
            _ptr(q_out), _ptr(q), qs, _ptr(k), ks, _ptr(v), vs, _ptr(positions),
            _ptr(slot_mapping), _ptr(inv_freq), _ptr(pool), B, n_q, n_kv, D, block_size,
            num_blocks, dtype_code(pool.dtype), _stream(dev))
    _check(rc, "rope_reshape_and_cache")
    return q_out


# ── kernel 2 ─────────────────────────────────────────────────────────────────


class DecodeWorkspace:
    """Zero-initialised scratch for the decode kernels, grown on demand.

    Holds the split-K partial results and per-sequence arrival counters of
    one call; the kernel leaves the counters at zero, so one buffer is reused
    across calls on the same stream.  Calls on different streams that may
    overlap need different workspaces.
    """

    def __init__(self) -> None:
        self._buf: dict[torch.device, torch.Tensor] = {}

    def get(self, device: torch.device, num_seqs: int, n_q: int, n_kv: int, d: int,
            dtype: torch.dtype) -> torch.Tensor:
        lib = load_library()
        with torch.cuda.device(device):
            need = lib.vmps_paged_decode_workspace_bytes(num_seqs, n_q, n_kv, d, dtype_code(dtype))
        if need == 0:
            raise NotImplementedError(
                f"paged_decode_attention: n_q={n_q} n_kv={n_kv} head_dim={d} not supported")
        buf = self._buf.get(device)
        if buf is None or buf.numel() < need:
            # Grow geometrically; torch allocations are 512-byte aligned.
            size = max(need, 0 if buf is None else 2 * buf.numel())
            buf = torch.zeros(size, dtype=torch.uint8, device=device)
            self._buf[device] = buf
        return buf


_default_workspace = DecodeWorkspace()


def paged_decode_attention(q: torch.Tensor, pool: torch.Tensor, block_tables: torch.Tensor,
                           seq_lens: torch.Tensor, scale: float | None = None,
                           out: torch.Tensor | None = None,
                           workspace: DecodeWorkspace | torch.Tensor | None = None) -> torch.Tensor:
    """Decode attention of one query token per sequence over its paged K/V.

    ``q``: (B, n_q, D) contiguous; ``pool``: (num_blocks, 2, 16, n_kv, D);
    ``block_tables``: int32 (B, max_blocks) zero-padded; ``seq_lens``: int32
    (B,) counting the new token.  Returns ``out`` (B, n_q, D) in the pool
    dtype.  ``scale`` defaults to ``1/sqrt(D)`` (layers/paged_attention_layer.py:353).
    """
    num_blocks, block_size, n_kv, D = _check_pool(pool)
    if q.dim() != 3 or q.shape[2] != D or not q.is_contiguous():
        raise ValueError(f"q must be contiguous (B, n_q, {D}); got {tuple(q.shape)}")
    B, n_q = q.shape[0], q.shape[1]
    if block_tables.dim() != 2 or block_tables.shape[0] != B:
        raise ValueError("block_tables must be (B, max_blocks)")
    if seq_lens.numel() != B:
        raise ValueError("seq_lens must have B entries")
    if q.dtype != pool.dtype:
        raise TypeError(f"q dtype {q.dtype} != pool dtype {pool.dtype}")
    _int32(block_tables, "block_tables")
    _int32(seq_lens, "seq_lens")
    if out is None:
        out = torch.empty_like(q)
    elif out.shape != q.shape or out.dtype != q.dtype or not out.is_contiguous():
        raise ValueError("out must be a contiguous tensor like q")
    dev = _require_cuda(q, pool, block_tables, seq_lens, out)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if isinstance(workspace, torch.Tensor):
        ws = workspace
    else:
        ws = (workspace or _default_workspace).get(dev, B, n_q, n_kv, D, pool.dtype)
    lib = load_library()
    with torch.cuda.device(dev):
        rc = lib.vmps_paged_decode_attention(
            _ptr(out), _ptr(q), _ptr(pool), _ptr(block_tables), block_tables.shape[1],
            _ptr(seq_lens), B, n_q, n_kv, D, block_size, num_blocks, float(scale),
            _ptr(ws), ws.numel() * ws.element_size(), dtype_code(pool.dtype), _stream(dev))
    _check(rc, "paged_decode_attention")
    return out


def paged_decode_step(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                      positions: torch.Tensor, slot_mapping: torch.Tensor,
                      inv_freq: torch.Tensor | None, pool: torch.Tensor,
                      block_tables: torch.Tensor, seq_lens: torch.Tensor,
                      scale: float | None = None, out: torch.Tensor | None = None,
                      workspace: DecodeWorkspace | torch.Tensor | None = None) -> torch.Tensor:
    """One decode step of one layer in one kernel: RoPE, K/V write, paged attention.

    ``q`` (B, n_q, D) is rotated in registers (left unchanged in memory);
    ``k``/``v`` (B, n_kv, D) (any row stride) are rotated / written to
    ``pool`` at ``slot_mapping``, which must address position ``seq_lens-1``
    of each sequence (its last page).  Returns the attention output
    (B, n_q, D).  Replaces PagedAttentionLayer._forward_batch between its
    projections (layers/paged_attention_layer.py:275-359).
    """
    num_blocks, block_size, n_kv, D = _check_pool(pool)
    if q.dim() == 2:
        q = q.view(q.shape[0], -1, D)
    if q.dim() != 3 or q.shape[2] != D or q.stride(2) != 1 or q.stride(1) != D:
        raise ValueError(f"q must be (B, n_q, {D}) with packed heads")
    B, n_q = q.shape[0], q.shape[1]
    ks = _rows(k, n_kv, D, "k")
    vs = _rows(v, n_kv, D, "v")
    for t, name in ((q, "q"), (k, "k"), (v, "v")):
        if t.dtype != pool.dtype:
            raise TypeError(f"{name} dtype {t.dtype} != pool dtype {pool.dtype}")
    _int32(positions, "positions")
    _int32(slot_mapping, "slot_mapping")
    _int32(block_tables, "block_tables")
    _int32(seq_lens, "seq_lens")
    if block_tables.dim() != 2 or block_tables.shape[0] != B or seq_lens.numel() != B:
        raise ValueError("block_tables must be (B, max_blocks) and seq_lens (B,)")
    if inv_freq is not None and (inv_freq.dtype != torch.float32 or inv_freq.numel() != D // 2):
        raise ValueError(f"inv_freq must be float32 of {D // 2} entries")
    if out is None:
        out = torch.empty((B, n_q, D), dtype=q.dtype, device=q.device)
    dev = _require_cuda(q, k, v, positions, slot_mapping, inv_freq, pool, block_tables,
                        seq_lens, out)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if isinstance(workspace, torch.Tensor):
        ws = workspace
    else:
        ws = (workspace or _default_workspace).get(dev, B, n_q, n_kv, D, pool.dtype)
    lib = load_library()
    with torch.cuda.device(dev):
        rc = lib.vmps_paged_decode_step(
            _ptr(out), _ptr(q), q.stride(0), _ptr(k), ks, _ptr(v), vs, _ptr(positions),
            _ptr(slot_mapping), _ptr(inv_freq), _ptr(pool), _ptr(block_tables),
            block_tables.shape[1], _ptr(seq_lens), B, n_q, n_kv, D, block_size, num_blocks,
            float(scale), _ptr(ws), ws.numel() * ws.element_size(), dtype_code(pool.dtype),
            _stream(dev))
    _check(rc, "paged_decode_step")
    return out


# ── kernel 3 ─────────────────────────────────────────────────────────────────


def paged_prefill_attention(q: torch.Tensor, pool: torch.Tensor, block_tables: torch.Tensor,
                            q_start: torch.Tensor, q_lens: torch.Tensor, cu_q: torch.Tensor,
                            max_q_len: int, scale: float | None = None,
                            out: torch.Tensor | None = None) -> torch.Tensor:
    """Causal attention of prompt rows over their sequences' paged K/V.

    The whole-prompt form of the reference's token-by-token single-token
    path (layers/paged_attention_layer.py:175-241): row r of sequence i is at
    position ``q_start[i] + r`` and attends to slots ``0..q_start[i] + r``,
    whose K/V must already be in ``pool`` (``rope_reshape_and_cache`` writes
    the new rows').  ``q``: (total_q, n_q, D) rotated queries, heads packed
    (rows may be strided); ``q_start``/``q_lens``/``cu_q``: int32 (B,) on the
    device; ``max_q_len`` >= every ``q_lens`` entry (host int, sizes the
    grid).  Returns ``out`` (total_q, n_q, D).
    """
    num_blocks, block_size, n_kv, D = _check_pool(pool)
    if q.dim() == 2:
        q = q.view(q.shape[0], -1, D)
    if q.dim() != 3 or q.shape[2] != D or q.stride(2) != 1 or q.stride(1) != D:
        raise ValueError(f"q must be (total_q, n_q, {D}) with packed heads; got {tuple(q.shape)}")
    total_q, n_q = q.shape[0], q.shape[1]
    B = q_lens.numel()
    if block_tables.dim() != 2 or block_tables.shape[0] != B:
        raise ValueError("block_tables must be (B, max_blocks)")
    if q_start.numel() != B or cu_q.numel() != B:
        raise ValueError("q_start, q_lens and cu_q must have one entry per sequence")
    if q.dtype != pool.dtype:
        raise TypeError(f"q dtype {q.dtype} != pool dtype {pool.dtype}")
    for t, name in ((block_tables, "block_tables"), (q_start, "q_start"), (q_lens, "q_lens"),
                    (cu_q, "cu_q")):
        _int32(t, name)
    if out is None:
        out = torch.empty((total_q, n_q, D), dtype=q.dtype, device=q.device)
    elif out.shape != (total_q, n_q, D) or out.dtype != q.dtype or not out.is_contiguous():
        raise ValueError("out must be a contiguous (total_q, n_q, D) tensor of q's dtype")
    dev = _require_cuda(q, pool, block_tables, q_start, q_lens, cu_q, out)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    lib = load_library()
    with torch.cuda.device(dev):
        rc = lib.vmps_paged_prefill_attention(
            _ptr(out), _ptr(q), q.stride(0), _ptr(pool), _ptr(block_tables),
            block_tables.shape[1], _ptr(q_start), _ptr(q_lens), _ptr(cu_q), B, total_q,
            int(max_q_len), n_q, n_kv, D, block_size, num_blocks, float(scale),
            dtype_code(pool.dtype), _stream(dev))
    _check(rc, "paged_prefill_attention")
    return out


# ── decoder-layer element-wise kernels (CUDA-graph decode step) ─────────────


def _row_stride(t: torch.Tensor, cols: int, name: str) -> int:
    if t.dim() != 2 or t.shape[1] < cols or t.stride(1) != 1:
        raise ValueError(f"{name} must be 2-D (rows, >= {cols}) with unit inner stride")
    return t.stride(0)


def add_rmsnorm(residual: torch.Tensor, weight: torch.Tensor, eps: float,
                delta: torch.Tensor | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """``residual += delta`` in place (when given), then ``out = RMSNorm(residual)``.

    The residual addition and RMSNorm of transformers' LlamaDecoderLayer /
    LlamaRMSNorm in one kernel (same rounding points: the sum rounded to the
    dtype, the variance in fp32, the normalised value rounded before the
    weight product).  ``residual``/``delta``/``out``: (rows, hidden), hidden a
    multiple of 8; ``weight``: (hidden,).  Returns ``out``.
    """
    hidden = weight.numel()
    rs = _row_stride(residual, hidden, "residual")
    if residual.shape[1] != hidden:
        raise ValueError(f"residual has {residual.shape[1]} columns, weight {hidden}")
    for t, name in ((delta, "delta"), (out, "out")):
        if t is not None and (t.shape != residual.shape or t.dtype != residual.dtype):
            raise ValueError(f"{name} must match residual's shape and dtype")
    if weight.dtype != residual.dtype or not weight.is_contiguous():
        raise ValueError("weight must be contiguous with residual's dtype")
    if out is None:
        out = torch.empty_like(residual)
    dev = _require_cuda(residual, weight, delta, out)
    ds = _row_stride(delta, hidden, "delta") if delta is not None else 0
    os_ = _row_stride(out, hidden, "out")
    lib = load_library()
    with torch.cuda.device(dev):
        rc = lib.vmps_add_rmsnorm(_ptr(out), os_, _ptr(residual), rs, _ptr(delta), ds,
                                  _ptr(weight), residual.shape[0], hidden, float(eps),
                                  dtype_code(residual.dtype), _stream(dev))
    _check(rc, "add_rmsnorm")
    return out


def embed_rmsnorm(table: torch.Tensor, weight: torch.Tensor, eps: float, tokens: torch.Tensor,
                  src: torch.Tensor | None = None, prev: torch.Tensor | None = None,
                  residual: torch.Tensor | None = None,
                  out: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Embedding rows of the step's tokens and the first RMSNorm, one kernel.

    Row i's token is ``prev[src[i]]`` when ``src`` is given and ``src[i] >=
    0``, else ``tokens[i]`` (``tokens``/``src`` int32, ``prev`` int64: the
    previous step's sampled ids, still on the device).  ``residual[i] =
    table[token]`` (the embedding lookup) and ``out = RMSNorm(residual) *
    weight`` with :func:`add_rmsnorm`'s rounding.  A ``src`` entry beyond
    ``prev`` or a token outside the table sets bit 128 of the device error
    word and zeroes the row.  Returns ``(residual, out)``.
    """
    vocab, hidden = table.shape
    rows = tokens.numel()
    if tokens.dtype != torch.int32 or not tokens.is_contiguous():
        raise ValueError("tokens must be contiguous int32")
    if (src is None) != (prev is None):
        raise ValueError("src and prev go together")
    if src is not None:
        if src.dtype != torch.int32 or not src.is_contiguous() or src.numel() != rows:
            raise ValueError("src must be contiguous int32 with one entry per token")
        if prev.dtype != torch.int64 or not prev.is_contiguous():
            raise ValueError("prev must be contiguous int64")
    if not table.is_contiguous() or weight.dtype != table.dtype or not weight.is_contiguous() \
            or weight.numel() != hidden:
        raise ValueError("table and weight must be contiguous, same dtype, weight (hidden,)")
    if residual is None:
        residual = torch.empty((rows, hidden), dtype=table.dtype, device=table.device)
    if out is None:
        out = torch.empty_like(residual)
    for t, name in ((residual, "residual"), (out, "out")):
        if t.shape != (rows, hidden) or t.dtype != table.dtype:
            raise ValueError(f"{name} must be ({rows}, {hidden}) {table.dtype}")
    dev = _require_cuda(table, weight, tokens, src, prev, residual, out)
    lib = load_library()
    with torch.cuda.device(dev):
        rc = lib.vmps_embed_rmsnorm(_ptr(out), _row_stride(out, hidden, "out"), _ptr(residual),
                                    _row_stride(residual, hidden, "residual"), _ptr(table), vocab,
                                    _ptr(tokens), _ptr(src), _ptr(prev),
                                    0 if prev is None else prev.numel(), _ptr(weight), rows,
                                    hidden, float(eps), dtype_code(table.dtype), _stream(dev))
    _check(rc, "embed_rmsnorm")
    return residual, out


def silu_mul(gate_up: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """``silu(gate_up[:, :I]) * gate_up[:, I:]`` for a fused [gate | up] GEMM output.

    LlamaMLP's ``act_fn(gate_proj(x)) * up_proj(x)`` after one GEMM of the
    concatenated weights; silu rounded to the dtype before the product, as
    the module does.  ``gate_up``: (rows, 2*I), I a multiple of 8.  Returns
    ``out`` (rows, I).
    """
    if gate_up.dim() != 2 or gate_up.shape[1] % 2:
        raise ValueError("gate_up must be (rows, 2 * inter)")
    rows, inter = gate_up.shape[0], gate_up.shape[1] // 2
    ins = _row_stride(gate_up, 2 * inter, "gate_up")
    if out is None:
        out = torch.empty((rows, inter), dtype=gate_up.dtype, device=gate_up.device)
    elif out.shape != (rows, inter) or out.dtype != gate_up.dtype:
        raise ValueError("out must be (rows, inter) of gate_up's dtype")
    dev = _require_cuda(gate_up, out)
    lib = load_library()
    with torch.cuda.device(dev):
        rc = lib.vmps_silu_mul(_ptr(out), _row_stride(out, inter, "out"), _ptr(gate_up), ins,
                               rows, inter, dtype_code(gate_up.dtype), _stream(dev))
    _check(rc, "silu_mul")
    return out


def decode_gemm_supported(m: int, n: int, k: int, silu_mul: bool = False) -> bool:
    """Whether ``decode_gemm`` is built for this shape (M <= 8, N % 8, K % 64, K <= 8192)."""
    return bool(load_library().vmps_decode_gemm_supported(int(m), int(n), int(k), int(silu_mul)))


def decode_gemm(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None,
                silu_mul: bool = False) -> torch.Tensor:
    """``x @ w.T`` for decode batch sizes (M <= 8), weight-streaming on HBM.

    The projections of a decoder layer at decode time (nn.Linear without
    bias, as transformers' Llama layers call them).  ``x``: (M, K) with unit
    inner stride; ``w``: contiguous (N, K).  With ``silu_mul`` the weight is
    the fused [gate; up] matrix of 2I rows and the result is
    ``silu(x @ Wg.T) * (x @ Wu.T)`` of shape (M, I), each projection rounded
    to the dtype first (LlamaMLP).  Returns ``out``.
    """
    if x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("x must be 2-D (M, K) with unit inner stride")
    if w.dim() != 2 or not w.is_contiguous():
        raise ValueError("w must be a contiguous (N, K) matrix")
    M, K = x.shape
    if w.shape[1] != K:
        raise ValueError(f"x has K={K}, w has K={w.shape[1]}")
    if w.dtype != x.dtype:
        raise TypeError(f"w dtype {w.dtype} != x dtype {x.dtype}")
    if silu_mul and w.shape[0] % 2:
        raise ValueError("silu_mul needs a [gate; up] weight with an even row count")
    N = w.shape[0] // 2 if silu_mul else w.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=x.dtype, device=x.device)
    elif out.shape != (M, N) or out.dtype != x.dtype or out.stride(1) != 1:
        raise ValueError(f"out must be ({M}, {N}) of x's dtype with unit inner stride")
    dev = _require_cuda(x, w, out)
    lib = load_library()
    with torch.cuda.device(dev):
        rc = lib.vmps_decode_gemm(_ptr(out), out.stride(0), _ptr(x), x.stride(0), _ptr(w), M, N, K,
                                  int(bool(silu_mul)), dtype_code(x.dtype), _stream(dev))
    _check(rc, "decode_gemm")
    return out


def batch_gemm_split(m: int, n: int, k: int) -> int:
    """CTAs per output tile (split-K cluster size) ``batch_gemm`` uses for this
    shape on the current device, or 0 when the shape is not built
    (1 <= M <= 256, N % 128 == 0, K % 64 == 0).  Needs a CUDA device."""
    return int(load_library().vmps_batch_gemm_split(int(m), int(n), int(k)))


def batch_gemm_workspace_bytes(m: int, n: int, k: int, dtype: torch.dtype) -> int:
    """Bytes of workspace ``batch_gemm`` needs for this shape (0: none, or not built)."""
    return int(load_library().vmps_batch_gemm_workspace_bytes(int(m), int(n), int(k),
                                                              dtype_code(dtype)))


def batch_gemm(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None,
               workspace: torch.Tensor | None = None) -> torch.Tensor:
    """``x @ w.T`` at decode batch sizes up to 256 on the tcgen05 tensor cores.

    ``x``: (M, K) with unit inner stride and rows a multiple of 8 elements
    apart; ``w``: contiguous (N, K), N % 128 == 0, K % 64 == 0; fp16 or bf16;
    ``out`` rows a multiple of 8 elements apart.  fp32 accumulation, one
    rounding (nn.Linear without bias).  Narrow shapes split K over a
    thread-block cluster (``batch_gemm_split``) whose fp32 partials meet in
    a workspace of ``batch_gemm_workspace_bytes`` bytes: ``workspace`` (a
    device tensor of at least that many bytes), else one from torch's caching
    allocator for this call (stream-ordered, so calls on different streams
    never share it).  Measured slower than cuBLAS at the engine's shapes; the
    engine does not call it.  Returns ``out`` (M, N).
    """
    if x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("x must be 2-D (M, K) with unit inner stride")
    if w.dim() != 2 or not w.is_contiguous():
        raise ValueError("w must be a contiguous (N, K) matrix")
    M, K = x.shape
    N = w.shape[0]
    if w.shape[1] != K:
        raise ValueError(f"x has K={K}, w has K={w.shape[1]}")
    if w.dtype != x.dtype:
        raise TypeError(f"w dtype {w.dtype} != x dtype {x.dtype}")
    if out is None:
        out = torch.empty((M, N), dtype=x.dtype, device=x.device)
    elif out.shape != (M, N) or out.dtype != x.dtype or out.stride(1) != 1:
        raise ValueError(f"out must be ({M}, {N}) of x's dtype with unit inner stride")
    if M == 0:
        return out
    dev = _require_cuda(x, w, out)
    lib = load_library()
    with torch.cuda.device(dev):
        need = int(lib.vmps_batch_gemm_workspace_bytes(M, N, K, dtype_code(x.dtype)))
        if workspace is None and need > 0:
            workspace = torch.empty(need, dtype=torch.uint8, device=dev)
        ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
        rc = lib.vmps_batch_gemm(_ptr(out), out.stride(0), _ptr(x), x.stride(0), _ptr(w), M, N, K,
                                 _ptr(workspace), ws_bytes, dtype_code(x.dtype), _stream(dev))
    _check(rc, "batch_gemm")
    return out


def stage_copy(dst: torch.Tensor, src: torch.Tensor) -> torch.Tensor:
    """Copy ``src`` (pinned host memory or a device tensor) into the CUDA tensor ``dst``
    with a kernel that is one link of a programmatic-dependent-launch chain.

    It overlaps the kernel before it on the current stream and completes only
    after that kernel, so ``dst`` must not be in use by that kernel.  A fused
    decode step reads its lengths and block tables before its own wait: stage
    step i+1 just before step i (three buffers), the first step with an
    ordinary copy (``vmps_stage_copy`` in include/vmps.h).  Both tensors
    contiguous, the same number of bytes (a multiple of 16), 16-byte aligned.
    """
    dev = _require_cuda(dst)
    if src.is_cuda:
        if src.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} and {src.device}")
    elif not src.is_pinned():
        raise ValueError("stage_copy: a host source must be pinned memory")
    if not (dst.is_contiguous() and src.is_contiguous()):
        raise ValueError("stage_copy: tensors must be contiguous")
    nbytes = dst.numel() * dst.element_size()
    if src.numel() * src.element_size() != nbytes:
        raise ValueError("stage_copy: dst and src differ in size")
    lib = load_library()
    with torch.cuda.device(dev):
        rc = lib.vmps_stage_copy(_ptr(dst), _ptr(src), nbytes, _stream(dev))
    _check(rc, "stage_copy")
    return dst


def error_word(device: torch.device | int | None = None) -> int:
    """Read and clear the device error word (bit meanings in include/vmps.h)."""
    dev = torch.device("cuda", device) if isinstance(device, int) else (device or torch.device("cuda"))
    word = ctypes.c_int(0)
    lib = load_library()
    with torch.cuda.device(dev):
        _check(lib.vmps_debug_error_word(_stream(dev), ctypes.byref(word)), "debug_error_word")
    return word.value


# ── reference-named entry points (kernels/__init__.py) ───────────────────────


def fused_attention(pool: torch.Tensor, new_k: torch.Tensor, new_v: torch.Tensor,
                    queries: torch.Tensor, bt_tensor: torch.Tensor, sl_tensor: torch.Tensor,
                    write_info: torch.Tensor, n_heads: int, n_kv_heads: int, d_k: int,
                    block_size: int) -> torch.Tensor:
    """Write the new (already rotated) K/V, then attend; returns (B, n_heads, d_k).

    Same contract as the reference's ``fused_attention_metal_fast``
    (kernels/__init__.py:320-368): ``write_info`` is int32 (B, 2) of
    (block_id, token_pos), ``sl_tensor`` counts the new token, ``bt_tensor``
    is the zero-padded int32 (B, max_blocks) block table.  The write and the
    attention are two launches on one stream, so the new token is always
    visible to the attention (the Metal kernel relied on redundant
    per-threadgroup writes instead, kernels/__init__.py:135-164).
    """
    B = queries.shape[0]
    if pool.shape[3] != n_kv_heads or pool.shape[4] != d_k or pool.shape[2] != block_size:
        raise ValueError("pool shape does not match n_kv_heads / d_k / block_size")
    if queries.shape[1:] != (n_heads, d_k):
        raise ValueError("queries must be (B, n_heads, d_k)")
    _int32(write_info, "write_info")
    slot = (write_info[:, 0] * block_size + write_info[:, 1]).to(torch.int32)
    rope_reshape_and_cache(None, new_k.contiguous(), new_v.contiguous(), None, slot, None, pool)
    return paged_decode_attention(queries.contiguous(), pool, bt_tensor, sl_tensor)


#: The reference's name for the same entry point.
fused_attention_metal_fast = fused_attention


def gather_kv(pool: torch.Tensor, block_tables: torch.Tensor, seq_lens: torch.Tensor,
              max_seq_len: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Padded paged gather ``(B, max_seq_len, n_kv, D)`` of K and V (zeros past seq_len).

    API-compatible with ``gather_kv_metal`` (kernels/__init__.py:279-312).
    Not on the decode hot path (the attention kernel reads pages in place);
    implemented with device-side indexing.
    """
    _require_cuda(pool, block_tables, seq_lens)
    num_blocks, bs, n_kv, D = _check_pool(pool)
    B = block_tables.shape[0]
    t = torch.arange(max_seq_len, device=pool.device)
    page = (t // bs).clamp_max(block_tables.shape[1] - 1)
    blk = block_tables.long().gather(1, page.unsqueeze(0).expand(B, -1))
    off = (t % bs).unsqueeze(0).expand(B, -1)
    k = pool[blk, 0, off]
    v = pool[blk, 1, off]
    valid = (t.unsqueeze(0) < seq_lens.long().unsqueeze(1)).unsqueeze(-1).unsqueeze(-1)
    return k * valid, v * valid
