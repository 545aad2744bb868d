"""CPU float32 restatement of the reference's transformer and denoising loop — TEST
INFRASTRUCTURE ONLY (the checker of b200attn.mmdit; never called by the product).

Follows, step by step and in float32 (torch on the CPU):
  TransformerBlock::forward            src/transformer.rs:396-427
  Attention::forward                   src/transformer.rs:163-197
  chunked_attention (dense, one chunk) src/transformer.rs:259-296
  GatedMlp::forward                    src/transformer.rs:326-333
  Modulation / zero_modulation         src/transformer.rs:357-359, 715-727
  FinalLayer::forward                  src/transformer.rs:448-454
  TextEmbedder::forward                src/transformer.rs:496-502 (GELU: candle's tanh form)
  forward_conditioned (both branches)  src/transformer.rs:573-668
  prefix_kv                            src/transformer.rs:674-707 (cache rounded to bf16,
                                       KV_CACHE_DTYPE, src/transformer.rs:24)
  FlowMatchEuler, timestep_embedding   src/scheduler.rs:26-126
  denoise (CFG, Euler)                 src/pipeline.rs:126-197
RoPE tables, positions, rotation, RMSNorm, the joint layout and the block-causal mask come
from oracle.reference (pinned there by the reference's own known-answer tests).

Parity status: the scheduler is pinned by the reference's own tests (src/scheduler.rs:
159-187: first sigma 1, last sigma shift_terminal, strictly decreasing, higher resolution
shifts more), ported in tests/test_mmdit.py; the cached step is pinned against this
module's own uncached full-sequence forward (the reference's claim that the prefix cache
reproduces the full joint pass, src/transformer.rs:8-13).  The block arithmetic itself has
no golden vector in the reference (its golden-tensor script and weights are not shipped).
"""
from __future__ import annotations

import math
from typing import List, Optional, Sequence, Tuple

import numpy as np
import torch
import torch.nn.functional as F

from oracle import reference as ref

HEAD_DIM = 128
AXES = (16, 56, 56)


# ----------------------------------------------------------------------------- scheduler
def calculate_shift(image_seq_len: int, base_seq_len=256, max_seq_len=8192, base_shift=0.5,
                    max_shift=0.9) -> np.float32:
    """calculate_shift (src/scheduler.rs:71-75), float32."""
    f = np.float32
    m = (f(max_shift) - f(base_shift)) / (f(max_seq_len) - f(base_seq_len))
    b = f(base_shift) - m * f(base_seq_len)
    return f(image_seq_len) * m + b


def sigmas(steps: int, image_seq_len: int, shift_terminal: float = 0.02) -> np.ndarray:
    """FlowMatchEuler::new (src/scheduler.rs:26-39): linspace (93-98), exponential time shift
    (78-82, shift exponent 1), stretch to the terminal (85-91); float32 throughout."""
    f = np.float32
    mu = calculate_shift(image_seq_len)
    if steps <= 1:
        lin = [f(1.0)]
    else:
        lo = f(1.0) / f(steps)
        lin = [f(1.0) + (lo - f(1.0)) * f(i) / f(steps - 1) for i in range(steps)]
    e_mu = f(math.exp(float(mu)))
    out = [e_mu / (e_mu + (f(1.0) / t - f(1.0)) ** f(1.0)) for t in lin]
    scale = (f(1.0) - out[-1]) / (f(1.0) - f(shift_terminal))
    return np.array([f(1.0) - (f(1.0) - s) / scale for s in out], np.float32)


def timestep_embedding(t: float, dim: int = 256) -> torch.Tensor:
    """timestep_embedding (src/scheduler.rs:101-126): cos half first, then sin."""
    half = dim // 2
    i = torch.arange(half, dtype=torch.float32)
    e = torch.exp(-math.log(1e4) * (i / half))
    a = (torch.tensor(t, dtype=torch.float32) * 1000.0) * e
    return torch.cat([torch.cos(a), torch.sin(a)])


# ----------------------------------------------------------------------------- the model
class Reference:
    """The transformer in float32 on the CPU with the given weights (a dict of tensors named
    as the reference's VarBuilder paths; bf16 values are used exactly, as float32)."""

    def __init__(self, weights: dict, layers: int, heads: int):
        self.w = {k: v.detach().to("cpu", torch.float32) for k, v in weights.items()}
        self.layers, self.heads = layers, heads
        self.hidden = heads * HEAD_DIM

    def lin(self, x, name):
        return x @ self.w[name + ".weight"].t()

    # -- pieces ------------------------------------------------------------------------
    @staticmethod
    def layer_norm(x, eps=1e-6):
        """fixed_layer_norm (src/transformer.rs:364-372): weight 1, bias 0."""
        mu = x.mean(-1, keepdim=True)
        var = ((x - mu) ** 2).mean(-1, keepdim=True)
        return (x - mu) / torch.sqrt(var + eps)

    @staticmethod
    def rms_norm(x, w, eps=1e-6):
        return x / torch.sqrt((x * x).mean(-1, keepdim=True) + eps) * w

    @staticmethod
    def rope(x, pe):
        """apply_rope on [H, S, D] with pe [S, D] interleaved (cos, sin) pairs."""
        c, s = pe[:, 0::2], pe[:, 1::2]
        x0, x1 = x[..., 0::2], x[..., 1::2]
        out = torch.empty_like(x)
        out[..., 0::2] = x0 * c - x1 * s
        out[..., 1::2] = x0 * s + x1 * c
        return out

    def t_emb(self, sinusoid):
        p = "time_text_embed.timestep_embedder."
        return self.lin(F.silu(self.lin(sinusoid, p + "linear_1")), p + "linear_2")

    def modulation(self, t_emb):
        return self.lin(F.silu(t_emb), "modulation.1")

    def zero_modulation(self):
        """src/transformer.rs:715-727: the t = 0 sinusoid is [1]*128 + [0]*128."""
        z = torch.cat([torch.ones(128), torch.zeros(128)])
        return self.modulation(self.t_emb(z))

    def attention(self, i, x, pe, mask, prefix):
        """Attention::forward (src/transformer.rs:163-197) for one sequence x [S, hidden];
        mask [S, Lk] bool or None; prefix (k, v) [H, P, D] or None.  Returns (out, k, v)."""
        p = f"transformer_blocks.{i}.attn."
        S, H = x.shape[0], self.heads
        q = self.lin(x, p + "to_q").view(S, H, HEAD_DIM)
        k = self.lin(x, p + "to_k").view(S, H, HEAD_DIM)
        v = self.lin(x, p + "to_v").view(S, H, HEAD_DIM).transpose(0, 1)
        q = self.rope(self.rms_norm(q, self.w[p + "norm_q.weight"]).transpose(0, 1), pe)
        k = self.rope(self.rms_norm(k, self.w[p + "norm_k.weight"]).transpose(0, 1), pe)
        ka, va = (k, v) if prefix is None else (torch.cat([prefix[0], k], 1),
                                                 torch.cat([prefix[1], v], 1))
        s = (q * HEAD_DIM ** -0.5) @ ka.transpose(1, 2)
        if mask is not None:
            s = s.masked_fill(~mask[None], float("-inf"))
        o = torch.softmax(s, -1) @ va
        o = o.transpose(0, 1).reshape(S, self.hidden)
        return self.lin(o, p + "to_out.0"), k, v

    def block(self, i, x, mod, pe, mask, prefix):
        """TransformerBlock::forward (src/transformer.rs:396-427); mod [S or 1, 4*hidden]."""
        h = self.hidden
        s1, g1, s2, g2 = (mod[..., j * h:(j + 1) * h] for j in range(4))
        a, k, v = self.attention(i, self.layer_norm(x) * (1 + s1), pe, mask, prefix)
        x = x + torch.tanh(g1) * a
        n = self.layer_norm(x) * (1 + s2)
        p = f"transformer_blocks.{i}.img_mlp."
        m = self.lin(F.silu(self.lin(n, p + "gate_layer")) * self.lin(n, p + "proj"), p + "out")
        return x + torch.tanh(g2) * m, k, v

    def final(self, x, t_emb):
        scale = self.lin(F.silu(t_emb), "norm_out.linear")
        return self.lin(self.layer_norm(x) * (1 + scale), "proj_out")

    def txt_in(self, emb):
        e = self.rms_norm(emb, self.w["txt_in.text_norm.weight"] + 1.0)
        return self.lin(F.gelu(self.lin(e, "txt_in.in_layer"), approximate="tanh"), "txt_in.out_layer")

    # -- forward paths -----------------------------------------------------------------
    def prefix_kv(self, emb, grid, cache_bf16: bool = True):
        """prefix_kv (src/transformer.rs:674-707) for one text-only prompt emb [L, text_dim]."""
        L = emb.shape[0]
        lay = ref.joint_layout(L, None, [], grid)
        pe = torch.from_numpy(ref.embed_nd(lay["img_shapes"], lay["image_pad_mask"])[:L])
        mask = torch.from_numpy(ref.block_causal_mask(lay["image_ids"][:L], None, 1)[0, 0])
        x = self.txt_in(emb)
        mod = self.zero_modulation()
        layers = []
        for i in range(self.layers):
            x, k, v = self.block(i, x, mod, pe, mask, None)
            if cache_bf16:
                k, v = k.to(torch.bfloat16).float(), v.to(torch.bfloat16).float()
            layers.append((k, v))
        return layers

    def forward_cached(self, lat, t: float, cache, text_len: int, grid):
        """forward_conditioned with a filled cache (src/transformer.rs:573-668): lat [T, C]."""
        T = lat.shape[0]
        lay = ref.joint_layout(text_len, None, [], grid)
        pe = torch.from_numpy(ref.embed_nd(lay["img_shapes"], lay["image_pad_mask"])[text_len:])
        t_emb = self.t_emb(timestep_embedding(t))
        mod = self.modulation(t_emb)
        x = self.lin(lat, "img_in")
        for i in range(self.layers):
            x, _, _ = self.block(i, x, mod, pe, None, cache[i])
        return self.final(x, t_emb)

    def forward_uncached(self, lat, t: float, emb, grid):
        """forward_conditioned without a cache (src/transformer.rs:608-668): the whole joint
        sequence [text ; target] with per-token modulation rows (t = 0 for the prefix) and
        the block-causal mask; returns the target rows."""
        L, T = emb.shape[0], lat.shape[0]
        lay = ref.joint_layout(L, None, [], grid)
        pe = torch.from_numpy(ref.embed_nd(lay["img_shapes"], lay["image_pad_mask"]))
        mask = torch.from_numpy(ref.block_causal_mask(lay["image_ids"], None, 1)[0, 0])
        x = torch.cat([self.txt_in(emb), self.lin(lat, "img_in")], 0)
        t_emb = self.t_emb(timestep_embedding(t))
        mod = torch.cat([self.zero_modulation().expand(L, -1), self.modulation(t_emb).expand(T, -1)], 0)
        for i in range(self.layers):
            x, _, _ = self.block(i, x, mod, pe, mask, None)
        return self.final(x, t_emb)[L:]

    def denoise(self, pos_embs: Sequence, neg_embs: Optional[Sequence], grid: Tuple[int, int],
                steps: int, cfg_scale: float, noise):
        """denoise (src/pipeline.rs:126-197) per prompt: noise [n, T, C] packed f32."""
        T = grid[0] * grid[1]
        sig = sigmas(steps, T)
        out = []
        for p in range(noise.shape[0]):
            pos = pos_embs[p].float()
            cache_p = self.prefix_kv(pos, grid)
            neg = None if neg_embs is None else neg_embs[p].float()
            cache_n = None if neg is None else self.prefix_kv(neg, grid)
            lat = noise[p].float().clone()
            for i in range(steps):
                pred = self.forward_cached(lat, float(sig[i]), cache_p, pos.shape[0], grid)
                if neg is not None:
                    pn = self.forward_cached(lat, float(sig[i]), cache_n, neg.shape[0], grid)
                    pred = pn + (pred - pn) * cfg_scale
                dt = sig[i + 1] - sig[i] if i + 1 < steps else -sig[i]
                lat = lat + pred * float(dt)
            out.append(lat)
        return torch.stack(out)
