"""CPU restatement of the GGML k-quant dequantisation — TEST INFRASTRUCTURE ONLY (the
checker of b200_dequant_q4_k / b200_dequant_q6_k; never called by the product).

The reference's GGUF linears are candle QMatMuls (src/quantized_transformer.rs:14-33)
over GGML super-blocks; candle's k_quants (candle-core 0.11.0, Cargo.lock:383-475) and
GGML define the formats.  Neither is vendored in the reference, so this module restates
the published block layouts and dequantisation formulas, float32 throughout, each product
and difference rounded separately:
  Q4_K: w = (f32(d) * scale_j) * q - (f32(dmin) * min_j), 8 sub-blocks of 32
  Q6_K: w = (f32(d) * scale_j) * (q - 32), 16 sub-blocks of 16

Parity status: pinned against llama.cpp's gguf-py (gguf 0.19.0, `gguf.quants`), an
independent implementation of the same formats, through golden fixtures generated in
this container by tests/golden/make_golden_gguf.py (tests/golden/gguf_kquants.npz).
"""
from __future__ import annotations

import numpy as np

QK_K = 256


def scale_min_q4_k(s: np.ndarray):
    """The 8 (scale, min) 6-bit pairs of Q4_K blocks from their 12 packed bytes [N, 12]:
    pairs 0-3 are the low 6 bits of bytes 0-3 / 4-7; pairs 4-7 take their low 4 bits from
    bytes 8-11 and their top 2 bits from bits 6-7 of bytes 0-3 / 4-7."""
    s = s.astype(np.uint32)
    sc = np.empty((s.shape[0], 8), np.uint32)
    mn = np.empty((s.shape[0], 8), np.uint32)
    for j in range(4):
        sc[:, j] = s[:, j] & 63
        mn[:, j] = s[:, j + 4] & 63
        sc[:, j + 4] = (s[:, j + 8] & 0xF) | ((s[:, j] >> 6) << 4)
        mn[:, j + 4] = (s[:, j + 8] >> 4) | ((s[:, j + 4] >> 6) << 4)
    return sc, mn


def dequantize_q4_k(blocks: np.ndarray) -> np.ndarray:
    """uint8 [N, 144] -> float32 [N, 256]."""
    b = np.ascontiguousarray(blocks, np.uint8).reshape(-1, 144)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)[:, 0]
    dmin = b[:, 2:4].copy().view(np.float16).astype(np.float32)[:, 0]
    sc, mn = scale_min_q4_k(b[:, 4:16])
    d1 = (d[:, None] * sc.astype(np.float32)).astype(np.float32)      # [N, 8]
    m1 = (dmin[:, None] * mn.astype(np.float32)).astype(np.float32)
    qs = b[:, 16:144].reshape(-1, 4, 32)
    q = np.stack([qs & 0xF, qs >> 4], 2).reshape(-1, 8, 32).astype(np.float32)  # sub-block j
    return (d1[:, :, None] * q - m1[:, :, None]).astype(np.float32).reshape(-1, QK_K)


def dequantize_q6_k(blocks: np.ndarray) -> np.ndarray:
    """uint8 [N, 210] -> float32 [N, 256]."""
    b = np.ascontiguousarray(blocks, np.uint8).reshape(-1, 210)
    n = b.shape[0]
    ql = b[:, 0:128].reshape(n, 2, 2, 32)    # [half, low/high 32 bytes, l]
    qh = b[:, 128:192].reshape(n, 2, 32)
    scales = b[:, 192:208].view(np.int8).astype(np.float32)
    d = b[:, 208:210].copy().view(np.float16).astype(np.float32)[:, 0]
    out = np.empty((n, 2, 4, 32), np.float32)
    for g in range(4):
        low = ql[:, :, g & 1, :]
        low = (low >> 4) if g >= 2 else (low & 0xF)
        hi = (qh >> (2 * g)) & 3
        q = (low.astype(np.int32) | (hi.astype(np.int32) << 4)) - 32
        out[:, :, g, :] = q
    ds = (d[:, None] * scales).astype(np.float32)                        # [N, 16]
    q = out.reshape(n, 16, 16)
    return (ds[:, :, None] * q).astype(np.float32).reshape(n, QK_K)
