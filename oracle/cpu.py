"""ctypes loader of the C restatement (``cpu_attention.c``) — test / baseline infrastructure.

Only ``tests/``, ``__graft_entry__`` and ``bench.py``'s CPU-baseline leg use it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle_attn.so")
_lib = None


def build() -> str:
    """Compile ``cpu_attention.c`` with the committed Makefile; returns the .so path."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    """The loaded C oracle (built on first use when missing)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        f32p = ctypes.POINTER(ctypes.c_float)
        u16p = ctypes.POINTER(ctypes.c_uint16)
        i32p = ctypes.POINTER(ctypes.c_int32)
        L.oracle_chunked_attention.argtypes = [f32p, f32p, f32p, f32p] + [ctypes.c_int] * 5 + [
            ctypes.c_float, i32p, ctypes.c_int]
        L.oracle_chunked_attention.restype = ctypes.c_int
        L.oracle_attention_forward.argtypes = [u16p] * 5 + [f32p, f32p, ctypes.c_float, f32p, i32p,
                                                             ctypes.c_float] + [ctypes.c_int] * 5 + [
            f32p, ctypes.c_int]
        L.oracle_attention_forward.restype = ctypes.c_int
        L.oracle_num_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _p(a, t):
    return a.ctypes.data_as(ctypes.POINTER(t))


def chunked_attention(q, k, v, scale, key_len=None, threads=0):
    """C chunked_attention on float32 [B,H,S,D]; key_len int32 [B] or None."""
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    b, h, sq, d = q.shape
    skv = k.shape[2]
    out = np.empty((b, h, sq, d), np.float32)
    kl = None if key_len is None else np.ascontiguousarray(key_len, np.int32)
    rc = lib().oracle_chunked_attention(_p(q, ctypes.c_float), _p(k, ctypes.c_float),
                                        _p(v, ctypes.c_float), _p(out, ctypes.c_float),
                                        b, h, sq, skv, d, float(scale),
                                        None if kl is None else _p(kl, ctypes.c_int32), threads)
    if rc != 0:
        raise MemoryError("oracle_chunked_attention failed")
    return out


def attention_forward(q_bits, k_bits, v_bits, pk_bits, pv_bits, wq, wk, eps, pe,
                      prefix_valid, scale, threads=0):
    """C restatement of the norm -> RoPE -> cat -> chunked_attention -> merge span.

    *_bits are uint16 bf16 bit patterns: q/k/v [B,T,H,D], pk/pv [B,H,P,D].  Returns
    float32 [B,T,H*D]."""
    b, t, h, d = q_bits.shape
    p = pk_bits.shape[2] if pk_bits is not None else 0
    if pk_bits is None:
        pk_bits = np.zeros((b, h, 0, d), np.uint16)
        pv_bits = np.zeros((b, h, 0, d), np.uint16)
    arrs = [np.ascontiguousarray(x, np.uint16) for x in (q_bits, k_bits, v_bits, pk_bits, pv_bits)]
    wq = np.ascontiguousarray(wq, np.float32)
    wk = np.ascontiguousarray(wk, np.float32)
    pe = np.ascontiguousarray(pe, np.float32)
    pvv = None if prefix_valid is None else np.ascontiguousarray(prefix_valid, np.int32)
    out = np.empty((b, t, h * d), np.float32)
    rc = lib().oracle_attention_forward(*[_p(a, ctypes.c_uint16) for a in arrs],
                                        _p(wq, ctypes.c_float), _p(wk, ctypes.c_float),
                                        float(eps), _p(pe, ctypes.c_float),
                                        None if pvv is None else _p(pvv, ctypes.c_int32),
                                        float(scale), b, t, h, p, d, _p(out, ctypes.c_float),
                                        threads)
    if rc != 0:
        raise MemoryError("oracle_attention_forward failed")
    return out


def num_threads() -> int:
    return int(lib().oracle_num_threads())
