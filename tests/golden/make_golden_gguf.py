"""Generates tests/golden/gguf_kquants.npz: Q4_K and Q6_K super-blocks and their float32
dequantisation by llama.cpp's gguf-py (gguf 0.19.0, `gguf.quants.dequantize`), the
independent implementation the k-quant oracle (oracle/gguf_ref.py) is pinned against.

Blocks: random bytes with random finite f16 super-scales (positive, negative, zero,
subnormal, large), plus blocks of the product quantizer (b200attn.gguf) on Gaussian
weights.  Run from the repository root: python tests/golden/make_golden_gguf.py
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [ROOT, os.path.join(ROOT, "qwen3-image21_b200")]

import gguf  # noqa: E402

from b200attn import gguf as bq  # noqa: E402


def f16_bytes(vals):
    return np.asarray(vals, np.float16).view(np.uint8).reshape(-1, 2)


def main():
    rng = np.random.default_rng(2024)
    special = [0.0, -0.0, 1.0, -1.0, 6.1e-05, 5.96e-08, 3.0e-06, 65504.0, -2.5, 0.0137]
    n = 48
    q4 = rng.integers(0, 256, size=(n, 144), dtype=np.uint8)
    q6 = rng.integers(0, 256, size=(n, 210), dtype=np.uint8)
    d = np.concatenate([special, rng.standard_normal(n - len(special)) * 0.01])
    dmin = np.concatenate([special[::-1], rng.standard_normal(n - len(special)) * 0.01])
    q4[:, 0:2] = f16_bytes(d)
    q4[:, 2:4] = f16_bytes(dmin)
    q6[:, 208:210] = f16_bytes(d)
    g = torch.Generator().manual_seed(7)
    w = torch.randn(4, 512, generator=g) * 0.02
    q4 = np.concatenate([q4, bq.quantize_q4_k(w).numpy().reshape(-1, 144)])
    q6 = np.concatenate([q6, bq.quantize_q6_k(w).numpy().reshape(-1, 210)])
    want4 = gguf.quants.dequantize(q4.reshape(-1), gguf.GGMLQuantizationType.Q4_K).reshape(-1, 256)
    want6 = gguf.quants.dequantize(q6.reshape(-1), gguf.GGMLQuantizationType.Q6_K).reshape(-1, 256)
    np.savez_compressed(os.path.join(HERE, "gguf_kquants.npz"), q4_k=q4, q4_k_f32=want4.astype(np.float32),
                        q6_k=q6, q6_k_f32=want6.astype(np.float32), weights=w.numpy())
    print("wrote", q4.shape, q6.shape)


if __name__ == "__main__":
    main()
