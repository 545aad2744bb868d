"""GGUF k-quant weights (Q4_K, Q6_K; the Q4_K_M mix) for the denoising loop's linears.

The reference's GGUF model keeps each linear as candle's QMatMul over the file's blocks
(src/quantized_transformer.rs:14-33).  Here a linear is its GGML super-blocks in HBM
(row-major along the input dimension, exactly the file's bytes) and the CUDA library
dequantises a layer's matrices to a bf16 scratch right before its GEMMs
(b200_dequant_q4_k / b200_dequant_q6_k).

Block layouts (GGML, 256 weights per super-block):
  Q4_K (144 B): f16 d | f16 dmin | 12 B packed 6-bit (scale, min) x 8 | 128 B 4-bit quants
  Q6_K (210 B): 128 B low nibbles | 64 B high 2 bits | 16 x int8 scale | f16 d

The quantizer here turns random-init weights into valid blocks: per 32-weight sub-block
(16 for Q6_K) the scale (and min) come from the sub-block's range, the super-block scales
are the largest sub-block values over 63 (Q4_K) or 127 (Q6_K), rounded to f16.  GGML's
own quantizer refines the sub-block scales with a search; the format and the
dequantisation are the same.  `q4_k_m_type` is llama.cpp's Q4_K_M rule: Q6_K for the value
projection and the MLP down-projection of the layers `use_more_bits` picks, Q4_K for the
other block linears.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Tuple

QK_K = 256
BLOCK_BYTES = {"q4_k": 144, "q6_k": 210}


def use_more_bits(layer: int, n_layers: int) -> bool:
    """llama.cpp's use_more_bits: the first and last eighth of the layers and every third
    layer in between."""
    return layer < n_layers // 8 or layer >= 7 * n_layers // 8 or (layer - n_layers // 8) % 3 == 2


def q4_k_m_type(name: str, layer: int, n_layers: int) -> str:
    """Block type of a transformer-block linear under Q4_K_M (attn_v ~ to_v, ffn_down ~
    img_mlp.out)."""
    if name in ("to_v", "out") and use_more_bits(layer, n_layers):
        return "q6_k"
    return "q4_k"


def _f16_bytes(x):
    """f32 tensor [N] -> (f16 values as f32, uint8 [N, 2] little-endian bytes)."""
    import torch
    h = x.to(torch.float16)
    b = h.view(torch.int16).to(torch.int32)
    return h.float(), torch.stack([b & 0xFF, (b >> 8) & 0xFF], -1).to(torch.uint8)


def quantize_q4_k(w):
    """w f32 [rows, cols] (cols % 256 == 0) -> uint8 [rows, cols / 256 * 144]."""
    import torch
    rows, cols = w.shape
    assert cols % QK_K == 0
    x = w.float().reshape(-1, 8, 32)
    n = x.shape[0]
    mn = x.amin(-1).clamp(max=0.0)
    mx = x.amax(-1)
    scale = (mx - mn) / 15.0
    th_min = -mn
    d_h, d_b = _f16_bytes(scale.amax(-1) / 63.0)
    dm_h, dm_b = _f16_bytes(th_min.amax(-1) / 63.0)
    safe = lambda v: torch.where(v > 0, v, torch.ones_like(v))
    sc = torch.where(d_h[:, None] > 0, torch.round(scale / safe(d_h)[:, None]), torch.zeros_like(scale)).clamp(0, 63)
    mq = torch.where(dm_h[:, None] > 0, torch.round(th_min / safe(dm_h)[:, None]), torch.zeros_like(th_min)).clamp(0, 63)
    d1 = d_h[:, None] * sc                                   # f32 products, as dequantised
    m1 = dm_h[:, None] * mq
    q = torch.where(d1[..., None] > 0, torch.round((x + m1[..., None]) / safe(d1)[..., None]),
                    torch.zeros_like(x)).clamp(0, 15).to(torch.int32).reshape(n, 4, 2, 32)
    qs = (q[:, :, 0, :] | (q[:, :, 1, :] << 4)).reshape(n, 128)
    sc, mq = sc.to(torch.int32), mq.to(torch.int32)
    s = torch.zeros(n, 12, dtype=torch.int32, device=w.device)
    s[:, 0:4] = (sc[:, 0:4] & 63) | ((sc[:, 4:8] >> 4) << 6)
    s[:, 4:8] = (mq[:, 0:4] & 63) | ((mq[:, 4:8] >> 4) << 6)
    s[:, 8:12] = (sc[:, 4:8] & 0xF) | ((mq[:, 4:8] & 0xF) << 4)
    out = torch.cat([d_b, dm_b, s.to(torch.uint8), qs.to(torch.uint8)], -1)
    return out.reshape(rows, cols // QK_K * 144).contiguous()


def quantize_q6_k(w):
    """w f32 [rows, cols] (cols % 256 == 0) -> uint8 [rows, cols / 256 * 210]."""
    import torch
    rows, cols = w.shape
    assert cols % QK_K == 0
    x = w.float().reshape(-1, 16, 16)
    n = x.shape[0]
    scale = x.abs().amax(-1) / 31.0
    d_h, d_b = _f16_bytes(scale.amax(-1) / 127.0)
    safe = lambda v: torch.where(v > 0, v, torch.ones_like(v))
    sc = torch.where(d_h[:, None] > 0, torch.round(scale / safe(d_h)[:, None]), torch.zeros_like(scale)).clamp(0, 127)
    ds = d_h[:, None] * sc
    q = torch.where(ds[..., None] > 0, torch.round(x / safe(ds)[..., None]), torch.zeros_like(x))
    q = (q.clamp(-32, 31) + 32).to(torch.int32).reshape(n, 2, 4, 32)   # [half, group, l]
    q1, q2, q3, q4 = q[:, :, 0], q[:, :, 1], q[:, :, 2], q[:, :, 3]
    ql = torch.cat([(q1 & 0xF) | ((q3 & 0xF) << 4), (q2 & 0xF) | ((q4 & 0xF) << 4)], -1)  # [n, 2, 64]
    qh = (q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6)            # [n, 2, 32]
    out = torch.cat([ql.reshape(n, 128).to(torch.uint8), qh.reshape(n, 64).to(torch.uint8),
                     sc.to(torch.int8).view(torch.uint8), d_b], -1)
    return out.reshape(rows, cols // QK_K * 210).contiguous()


def quantize(w, qtype: str):
    return quantize_q4_k(w) if qtype == "q4_k" else quantize_q6_k(w)


@dataclass
class QuantLinear:
    """One linear's weight [out_features, in_features] as GGML super-blocks."""
    blocks: object           # uint8 device tensor [out, in / 256 * block bytes]
    qtype: str               # "q4_k" | "q6_k"
    shape: Tuple[int, int]   # (out_features, in_features)

    def dequant_into(self, out, stream=None):
        """bf16 weight [out_features, in_features] into `out` (a contiguous bf16 buffer)."""
        import b200attn
        return b200attn.dequant(self.blocks, self.qtype, out=out.view(-1), stream=stream).view(self.shape)

    def nbytes(self) -> int:
        return self.blocks.numel()

    def matvec(self, x, out=None, stream=None):
        """x f32 [m, in_features] (m <= 2) -> f32 [m, out_features] = x W^T, the weight
        expanded in registers (b200_kquant_gemv), never written out."""
        import b200attn
        return b200attn.kquant_gemv(x, self.blocks, self.qtype, self.shape[0], out=out,
                                    stream=stream)
