"""ctypes front end of the C oracle (oracle/vmps_oracle.c) -- TEST INFRASTRUCTURE.

Builds ``oracle/libvmps_oracle.so`` with gcc (OpenMP) and exposes the decode
step on numpy uint16 arrays.  Used by the tests as a second checker and by
``bench.py`` as the timed CPU baseline; never by the product path.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "vmps_oracle.c")
LIB = os.path.join(HERE, "libvmps_oracle.so")
# x86-64-v3 (AVX2/FMA/F16C) so the library built here also runs on the GPU
# box's host CPU.
CFLAGS = ["-O3", "-march=x86-64-v3", "-fopenmp", "-fPIC", "-shared", "-std=c11"]

_lib = None


def build(force: bool = False) -> str:
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(SRC):
        tmp = LIB + ".tmp"
        subprocess.run(["gcc", *CFLAGS, "-o", tmp, SRC, "-lm"], check=True)
        os.replace(tmp, LIB)
    return LIB


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        lib = ctypes.CDLL(LIB)
        vp, i32 = ctypes.c_void_p, ctypes.c_int
        lib.vmpso_rope_and_write.restype = i32
        lib.vmpso_rope_and_write.argtypes = [vp, vp, vp, vp, vp, vp, vp] + [i32] * 7
        lib.vmpso_paged_attention.restype = i32
        lib.vmpso_paged_attention.argtypes = [vp, vp, vp, vp, i32, vp] + [i32] * 8
        lib.vmpso_max_threads.restype = i32
        lib.vmpso_max_threads.argtypes = []
        _lib = lib
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _dt(dtype: str) -> int:
    return {"float16": 0, "bfloat16": 1}[dtype]


def decode_step(q_bits, k_bits, v_bits, positions, seq_lens, block_tables, pool_bits,
                inv_freq, dtype: str, block_size: int = 16, threads: int = 0):
    """Same contract as ``paged_attention_oracle.decode_step`` (pool updated in place)."""
    lib = load()
    q = np.ascontiguousarray(q_bits, dtype=np.uint16).copy()
    k = np.ascontiguousarray(k_bits, dtype=np.uint16)
    v = np.ascontiguousarray(v_bits, dtype=np.uint16)
    B, n_q, D = q.shape
    n_kv = k.shape[1]
    pos = np.ascontiguousarray(positions, dtype=np.int32)
    sl = np.ascontiguousarray(seq_lens, dtype=np.int32)
    bt = np.ascontiguousarray(block_tables, dtype=np.int32)
    slot = np.array([bt[i, p // block_size] * block_size + p % block_size for i, p in enumerate(pos)],
                    dtype=np.int32)
    assert pool_bits.flags["C_CONTIGUOUS"] and pool_bits.dtype == np.uint16
    inv = None if inv_freq is None else np.ascontiguousarray(inv_freq, dtype=np.float32)
    rc = lib.vmpso_rope_and_write(_p(q), _p(k), _p(v), _p(pos), _p(slot), _p(inv), _p(pool_bits),
                                  B, n_q, n_kv, D, block_size, pool_bits.shape[0], _dt(dtype))
    if rc:
        raise IndexError("vmpso_rope_and_write: slot out of range")
    out = np.empty_like(q)
    rc = lib.vmpso_paged_attention(_p(out), _p(q), _p(pool_bits), _p(bt), bt.shape[1], _p(sl), B,
                                   n_q, n_kv, D, block_size, pool_bits.shape[0], _dt(dtype), threads)
    if rc:
        raise IndexError("vmpso_paged_attention: block table out of range")
    return out, q


def max_threads() -> int:
    return load().vmpso_max_threads()
