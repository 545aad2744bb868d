"""The denoising loop around the attention path: the 32-block single-stream MMDiT of
Qwen-Image-2.1 with a per-prompt prefix K/V cache, true CFG and the FlowMatch Euler
scheduler, on one GPU.

It stands in for the reference's Rust pipeline, which keeps calling the attention
library at its two call sites; here it measures that library in context (denoise-step
time) and carries the end-to-end latents check.  Mirrors:

  QwenImageTransformer::forward_conditioned  src/transformer.rs:573-668 (cached step)
  QwenImageTransformer::prefix_kv            src/transformer.rs:674-707
  zero_modulation                            src/transformer.rs:715-727
  TransformerBlock::forward                  src/transformer.rs:396-427
  GatedMlp / Modulation / FinalLayer         src/transformer.rs:326-331, 357-359, 448-454
  TextEmbedder (txt_in)                      src/transformer.rs:480-503
  FlowMatchEuler, timestep_embedding         src/scheduler.rs:26-126
  denoise (CFG + Euler loop)                 src/pipeline.rs:126-197

Unlike the reference, which runs each sequence (prompt x {pos, neg}) as its own forward
call, every sequence of a step goes through each block together: one GEMM per linear over
all sequences' target tokens, one attention launch whose batch rows carry their own prefix
lengths (b200_kv_desc) and RoPE tables (pe_batch_stride).  The residual stream is f32;
GEMM operands are bf16 (cuBLAS through torch); attention, Q/K norm + RoPE and the
elementwise block steps run in this package's CUDA library.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

import b200attn

HEAD_DIM = 128
T_DIM = 256                       # sinusoidal timestep width (src/scheduler.rs:101)
AXES = (16, 56, 56)               # Config::axes_dims_rope (src/transformer.rs:70)
ROPE_THETA = 1e4
# FlowMatch Euler constants (src/scheduler.rs:16-20)
BASE_SHIFT, MAX_SHIFT = 0.5, 0.9
BASE_IMAGE_SEQ_LEN, MAX_IMAGE_SEQ_LEN = 256, 8192
SHIFT_TERMINAL = 0.02


@dataclass(frozen=True)
class MMDiTConfig:
    """Config of src/transformer.rs:48-91 (defaults: Qwen-Image-2.1, 32 x 32 heads x 128)."""
    layers: int = 32
    heads: int = 32
    in_channels: int = 64
    text_dim: int = 4096           # joint_attention_dim
    mlp_ratio: int = 3             # Config::mlp_hidden_size = 3 * hidden

    @property
    def hidden(self) -> int:
        return self.heads * HEAD_DIM

    @property
    def ffn(self) -> int:
        return self.mlp_ratio * self.hidden

    def params(self) -> int:
        h, f = self.hidden, self.ffn
        per_block = 4 * h * h + 3 * h * f + 2 * HEAD_DIM
        return (self.layers * per_block + h * self.in_channels * 2 + h * self.text_dim + h * h
                + h * T_DIM + h * h + 4 * h * h + h * h + h)

    def linear_flops_per_token(self) -> float:
        """GEMM FLOPs of one target token through every block (2 per MAC)."""
        h, f = self.hidden, self.ffn
        return 2.0 * self.layers * (4 * h * h + 3 * h * f)


# ----------------------------------------------------------------------- scheduler
def flow_match_sigmas(steps: int, image_seq_len: int) -> np.ndarray:
    """FlowMatchEuler::new (src/scheduler.rs:26-39) in float32, as the reference computes:
    linspace(1, 1/steps), exponential time shift with mu(image_seq_len), stretched so the
    last sigma is SHIFT_TERMINAL."""
    f = np.float32
    m = (f(MAX_SHIFT) - f(BASE_SHIFT)) / (f(MAX_IMAGE_SEQ_LEN) - f(BASE_IMAGE_SEQ_LEN))
    b = f(BASE_SHIFT) - m * f(BASE_IMAGE_SEQ_LEN)
    mu = f(image_seq_len) * m + b
    if steps <= 1:
        s = np.array([1.0], np.float32)
    else:
        start, end = f(1.0), f(1.0) / f(steps)
        s = np.array([start + (end - start) * f(i) / f(steps - 1) for i in range(steps)], np.float32)
    e_mu = np.exp(mu, dtype=np.float32)
    s = (e_mu / (e_mu + (f(1.0) / s - f(1.0)) ** f(1.0))).astype(np.float32)
    scale = (f(1.0) - s[-1]) / (f(1.0) - f(SHIFT_TERMINAL))
    return (f(1.0) - (f(1.0) - s) / scale).astype(np.float32)


def euler_dt(sigmas: np.ndarray, i: int) -> float:
    """FlowMatchEuler::step's dt (src/scheduler.rs:54-66)."""
    return float(sigmas[i + 1] - sigmas[i]) if i + 1 < len(sigmas) else float(-sigmas[i])


def timestep_embedding(t: float, dim: int = T_DIM) -> np.ndarray:
    """timestep_embedding (src/scheduler.rs:101-126): [cos(1000 t e_i), sin(1000 t e_i)] with
    e_i = exp(-ln(1e4) i / half), float32, cos first."""
    half = dim // 2
    i = np.arange(half, dtype=np.float32)
    e = np.exp(-np.float32(math.log(1e4)) * (i / np.float32(half))).astype(np.float32)
    a = (np.float32(t) * np.float32(1000.0)) * e
    return np.concatenate([np.cos(a), np.sin(a)]).astype(np.float32)


def pack_latents(noise):
    """pack_latents (src/vae.rs:641-646): [B, C, 1, H, W] -> [B, H*W, C]."""
    b, c, _, h, w = noise.shape
    return noise.reshape(b, c, h * w).transpose(1, 2).contiguous()


# ----------------------------------------------------------------------- weights
def weight_shapes(cfg: MMDiTConfig) -> Dict[str, Tuple[int, ...]]:
    """Tensor names and shapes as the reference's VarBuilder paths name them."""
    h, f = cfg.hidden, cfg.ffn
    s = {
        "img_in.weight": (h, cfg.in_channels),
        "txt_in.text_norm.weight": (h,),
        "txt_in.in_layer.weight": (h, cfg.text_dim),
        "txt_in.out_layer.weight": (h, h),
        "time_text_embed.timestep_embedder.linear_1.weight": (h, T_DIM),
        "time_text_embed.timestep_embedder.linear_2.weight": (h, h),
        "modulation.1.weight": (4 * h, h),
        "norm_out.linear.weight": (h, h),
        "proj_out.weight": (cfg.in_channels, h),
    }
    for i in range(cfg.layers):
        p = f"transformer_blocks.{i}."
        for n in ("to_q", "to_k", "to_v"):
            s[p + f"attn.{n}.weight"] = (h, h)
        s[p + "attn.to_out.0.weight"] = (h, h)
        s[p + "attn.norm_q.weight"] = (HEAD_DIM,)
        s[p + "attn.norm_k.weight"] = (HEAD_DIM,)
        s[p + "img_mlp.proj.weight"] = (f, h)
        s[p + "img_mlp.gate_layer.weight"] = (f, h)
        s[p + "img_mlp.out.weight"] = (h, f)
    return s


def random_weights(cfg: MMDiTConfig, seed: int, device="cpu", std: float = 0.02) -> dict:
    """Random-init weights: matrices ~ N(0, std) in bf16; RMSNorm weights 1 + N(0, std) in
    f32 (txt_in.text_norm stores scale - 1, as the checkpoint does: N(0, std)).  Generated
    on `device` from one seeded generator, in name order."""
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    out = {}
    for name, shape in weight_shapes(cfg).items():
        w = torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std
        if name.endswith(("norm_q.weight", "norm_k.weight")):
            out[name] = w + 1.0
        elif name.endswith("text_norm.weight"):
            out[name] = w
        else:
            out[name] = w.to(torch.bfloat16)
    return out


# ----------------------------------------------------------------------- the model
@dataclass
class PrefixCache:
    """Per-layer post-RoPE K and V of every sequence's prefix, [B, H, Pmax, D] bf16 (the
    TextKvCache of src/transformer.rs:14-19, one tensor per layer for the whole batch;
    rows past a sequence's own length hold its padding tokens' finite K/V, which every
    cached step masks through the sequence's descriptor)."""
    k: List
    v: List
    lengths: List[int]

    def offload(self) -> "PrefixCache":
        """set_kv_cache_offload (src/transformer.rs:27-45): keep the cache in pinned host
        memory.  Cached steps then stream each layer's K and V back to the GPU on a copy
        stream, one layer ahead of the attention that reads them."""
        self.k = [t.cpu().pin_memory() for t in self.k]
        self.v = [t.cpu().pin_memory() for t in self.v]
        return self

    @property
    def on_host(self) -> bool:
        return not self.k[0].is_cuda


class MMDiT:
    """The transformer on one GPU with bf16 weights (see module docstring)."""

    def __init__(self, cfg: MMDiTConfig, weights: dict, device="cuda", mlp_chunk_rows: int = 16384,
                 weight_format: str = "bf16", fused_qkv: bool = False, gemm: str = "cublas",
                 prefetch_weights: bool = True):
        """weight_format "bf16" keeps the block linears in bf16; "q4_k_m" stores them as GGUF
        Q4_K / Q6_K super-blocks (llama.cpp's Q4_K_M rule) and dequantises each block's six
        matrices to a bf16 scratch right before its GEMMs; the timestep embedder's two
        linears and the modulation linear become Q4_K too and run as one-row products
        straight from the super-blocks (b200_kquant_gemv), as the reference's GGUF model
        runs them through QMatMul (src/quantized_transformer.rs:37-53, 216-228).  The
        other weights (img_in, txt_in, norm_out, proj_out) stay bf16 / f32 either way, as
        the GGUF files the reference reads store them unquantised.  fused_qkv: a cached step runs the Q/K/V projections with the
        Q/K RMSNorm + RoPE in the GEMM epilogue (b200_qkv_norm_rope_gemm) and then the
        attention kernel alone; otherwise (the default, 1.3 % faster at config 5 while the
        tcgen05 GEMM runs the 12288-wide projection at ~90 % of cuBLAS) three cuBLAS GEMMs
        and b200_attn_fwd.  prefetch_weights (q4_k_m): dequantise block i + 1's linears on a
        side stream while block i computes (two scratch slots); off, each block's are
        dequantised on the compute stream right before its GEMMs."""
        import torch
        if weight_format not in ("bf16", "q4_k_m"):
            raise ValueError(f"unknown weight format {weight_format!r}")
        if gemm not in ("cublas", "b200"):
            raise ValueError(f"unknown GEMM {gemm!r}")
        self.gemm_impl = gemm
        self.cfg, self.device = cfg, torch.device(device)
        self.mlp_chunk_rows = mlp_chunk_rows
        self.weight_format = weight_format
        self.fused_qkv = fused_qkv
        self.prefetch_weights = prefetch_weights
        dev = self.device
        bf = lambda n: weights[n].to(device=dev, dtype=torch.bfloat16).contiguous()
        f32 = lambda n: weights[n].to(device=dev, dtype=torch.float32).contiguous()
        self.img_in = bf("img_in.weight")
        self.proj_out = bf("proj_out.weight")
        self.txt_norm_w = f32("txt_in.text_norm.weight") + 1.0   # ZeroCenterRMSNorm (:487)
        self.txt_in1 = bf("txt_in.in_layer.weight")
        self.txt_in2 = bf("txt_in.out_layer.weight")
        # The timestep path is a few matrix-vector products per step: kept in f32.
        self.t1 = f32("time_text_embed.timestep_embedder.linear_1.weight")
        self.t2 = f32("time_text_embed.timestep_embedder.linear_2.weight")
        self.mod_w = f32("modulation.1.weight")
        self.norm_out_w = f32("norm_out.linear.weight")
        self.blocks = []
        for i in range(cfg.layers):
            p = f"transformer_blocks.{i}."
            self.blocks.append(dict(
                wq=bf(p + "attn.to_q.weight"), wk=bf(p + "attn.to_k.weight"),
                wv=bf(p + "attn.to_v.weight"), wo=bf(p + "attn.to_out.0.weight"),
                nq=f32(p + "attn.norm_q.weight"), nk=f32(p + "attn.norm_k.weight"),
                # [gate_layer ; proj] stacked: one GEMM feeds b200_swiglu.
                wgp=torch.cat([bf(p + "img_mlp.gate_layer.weight"),
                               bf(p + "img_mlp.proj.weight")], 0).contiguous(),
                wmo=bf(p + "img_mlp.out.weight")))
        h = cfg.hidden
        for blk in self.blocks:  # [to_q ; to_k ; to_v] stacked: one GEMM for the fused path
            blk["wqkv"] = torch.cat([blk.pop("wq"), blk.pop("wk"), blk.pop("wv")], 0).contiguous()
            blk["wq"], blk["wk"], blk["wv"] = (blk["wqkv"][j * h:(j + 1) * h] for j in range(3))
        self.q_time = None
        if weight_format == "q4_k_m":
            from b200attn import gguf as bq
            self.q_time = {k: bq.QuantLinear(bq.quantize(w, "q4_k"), "q4_k", tuple(w.shape))
                           for k, w in (("t1", self.t1), ("t2", self.t2), ("mod", self.mod_w))}
            del self.t1, self.t2, self.mod_w
            # reference names of the block linears (the fused gate_up is one GGUF tensor in
            # ComfyUI-style files, src/quantized_transformer.rs:160-166, output [gate; up])
            names = dict(wq="to_q", wk="to_k", wv="to_v", wo="to_out", wgp="gate_up", wmo="out")
            for i, blk in enumerate(self.blocks):
                del blk["wqkv"]
                for key, name in names.items():
                    w = blk.pop(key)
                    qtype = bq.q4_k_m_type(name, i, cfg.layers)
                    blk["q_" + key] = bq.QuantLinear(bq.quantize(w.float(), qtype), qtype, tuple(w.shape))
                    del w
        self._bufs = {}
        # When a list, every attention call of the block loop appends its (start, end) CUDA
        # events (the attention kernel; with fused_qkv off, the b200_attn_fwd span of Q/K
        # norm + RoPE prologue and attention kernel).
        self.attn_marks = None

    # -- small helpers -------------------------------------------------------------
    def _buf(self, name, shape, dtype):
        import torch
        t = self._bufs.get(name)
        n = int(np.prod(shape))
        if t is None or t.numel() < n or t.dtype != dtype:
            t = torch.empty(n, dtype=dtype, device=self.device)
            self._bufs[name] = t
        return t[:n].view(*shape)

    def _copy_stream(self):
        """The model's host<->device copy stream (created once)."""
        import torch
        if getattr(self, "_copy", None) is None:
            self._copy = torch.cuda.Stream(self.device)
        return self._copy

    def _staging(self, tag: str, shape):
        """Two (K, V) device staging slots of `shape` bf16, kept across calls."""
        import torch
        return [(self._buf(f"stage_{tag}_k{j}", tuple(shape), torch.bfloat16),
                 self._buf(f"stage_{tag}_v{j}", tuple(shape), torch.bfloat16)) for j in range(2)]

    def _linear_f32(self, x, name):
        """x f32 [k] @ W^T for the timestep / modulation linears: f32 weights, or (q4_k_m)
        the Q4_K super-blocks through b200_kquant_gemv."""
        if self.q_time is not None:
            return self.q_time[name].matvec(x.reshape(1, -1).contiguous())[0]
        return x @ {"t1": self.t1, "t2": self.t2, "mod": self.mod_w}[name].t()

    def _time_proj(self, e):
        import torch.nn.functional as F
        return self._linear_f32(F.silu(self._linear_f32(e, "t1")), "t2")

    def time_embed(self, t: float):
        """QwenTimestepProj (src/transformer.rs:112-114) of timestep_embedding(t) -> f32 [hidden]."""
        import torch
        return self._time_proj(torch.from_numpy(timestep_embedding(t)).to(self.device))

    def zero_time_embed(self):
        """t_emb of the t = 0 sinusoid [1]*128 + [0]*128 (src/transformer.rs:715-727)."""
        import torch
        e = torch.cat([torch.ones(T_DIM // 2), torch.zeros(T_DIM // 2)]).to(self.device)
        return self._time_proj(e)

    def modulation(self, t_emb):
        """Modulation::forward (src/transformer.rs:357-359): [4 * hidden] f32, chunks
        (scale1, gate1, scale2, gate2)."""
        import torch.nn.functional as F
        return self._linear_f32(F.silu(t_emb), "mod")

    def final_scale(self, t_emb):
        """FinalLayer's scale (src/transformer.rs:450): linear(silu(t_emb))."""
        import torch.nn.functional as F
        return F.silu(t_emb) @ self.norm_out_w.t()

    def block_weights(self, i: int, slot: int = 0, stream=None) -> dict:
        """Block i's bf16 weights: the stored tensors, or (q4_k_m) its six linears
        dequantised into this model's scratch slot `slot` on `stream` (valid until the slot
        is filled again)."""
        import torch
        blk = self.blocks[i]
        if self.weight_format == "bf16":
            return blk
        out = dict(nq=blk["nq"], nk=blk["nk"])
        h = self.cfg.hidden
        wqkv = self._buf(f"dq{slot}_wqkv", (3 * h, h), torch.bfloat16)
        for j, key in enumerate(("wq", "wk", "wv")):
            out[key] = blk["q_" + key].dequant_into(wqkv[j * h:(j + 1) * h], stream=stream)
        out["wqkv"] = wqkv
        for key in ("wo", "wgp", "wmo"):
            ql = blk["q_" + key]
            out[key] = ql.dequant_into(self._buf(f"dq{slot}_" + key, ql.shape, torch.bfloat16),
                                       stream=stream)
        return out

    def _dq_stream(self):
        """Side stream that dequantises the next block's weights during this block."""
        import torch
        if getattr(self, "_dq", None) is None:
            self._dq = torch.cuda.Stream(self.device)
        return self._dq

    def weight_bytes(self) -> int:
        """HBM bytes of the block linears (the 99 % of the parameters they hold)."""
        total = 0
        for blk in self.blocks:
            if self.weight_format == "bf16":
                total += sum(blk[k].numel() * 2 for k in ("wqkv", "wo", "wgp", "wmo"))
            else:
                total += sum(blk["q_" + k].nbytes() for k in ("wq", "wk", "wv", "wo", "wgp", "wmo"))
        return total

    def effective_weights(self, weights: dict) -> dict:
        """`weights` with each block linear replaced by the values this model multiplies by
        (the bf16 dequantisation for q4_k_m), as float32 CPU tensors: what a float32
        reference of this model must use."""
        import torch
        out = {k: v.detach().float().cpu() for k, v in weights.items()}
        if self.weight_format == "bf16":
            return out
        for key, name in (("t1", "time_text_embed.timestep_embedder.linear_1.weight"),
                          ("t2", "time_text_embed.timestep_embedder.linear_2.weight"),
                          ("mod", "modulation.1.weight")):
            ql = self.q_time[key]
            out[name] = ql.dequant_into(torch.empty(ql.shape, dtype=torch.bfloat16,
                                                    device=self.device)).float().cpu()
        names = dict(wq="attn.to_q", wk="attn.to_k", wv="attn.to_v", wo="attn.to_out.0",
                     wmo="img_mlp.out")
        f = self.cfg.ffn
        for i in range(self.cfg.layers):
            w = self.block_weights(i)
            p = f"transformer_blocks.{i}."
            for key, name in names.items():
                out[p + name + ".weight"] = w[key].float().cpu()
            gp = w["wgp"].float().cpu()
            out[p + "img_mlp.gate_layer.weight"] = gp[:f].clone()
            out[p + "img_mlp.proj.weight"] = gp[f:].clone()
        return out

    def _gemm(self, a, w, name, out=None):
        """a [R, K] bf16 @ w[N, K]^T -> bf16 [R, N]: cuBLAS, or this package's tcgen05 GEMM
        (gemm="b200")."""
        import torch
        if out is None:
            out = self._buf(name, (a.shape[0], w.shape[0]), torch.bfloat16)
        if self.gemm_impl == "b200":
            b200attn.gemm(a, w, out=out)
        else:
            torch.mm(a, w.t(), out=out)
        return out

    # -- the block loop -----------------------------------------------------------
    def _run_blocks(self, x, B: int, T: int, mod, pe, prefix: Optional[PrefixCache], desc,
                    row_limit=None, kv_out: Optional[PrefixCache] = None, final_scale=None):
        """x f32 [B*T, hidden] (updated in place) through every block; mod f32 [4*hidden]
        (one row for every token).  Returns LN(x) * (1 + final_scale) bf16 when final_scale
        is given (FinalLayer), else None."""
        import torch
        cfg = self.cfg
        h, H, R = cfg.hidden, cfg.heads, B * T
        m = mod.view(1, 4 * h)
        scale1, gate1, scale2, gate2 = (m[:, j * h:(j + 1) * h] for j in range(4))
        y = self._buf("y", (R, h), torch.bfloat16)
        attn = self._buf("attn", (B, T, h), torch.bfloat16)
        ws_need = 2 * B * H * T * HEAD_DIM * 2 + b200attn.SPLIT_WORKSPACE_BYTES + 4096
        ws = self._buf("ws", (ws_need,), torch.uint8)
        b200attn.residual_adaln(x, None, None, scale1, y, rows_per_mod=R)      # norm1 of block 0
        # A host-resident cache streams in one layer ahead: layer i's K/V land in staging
        # slot i % 2 on the copy stream while layer i - 1 computes; a slot is refilled only
        # after the attention that read it.
        staged = None
        cur = torch.cuda.current_stream(self.device)
        if prefix is not None and prefix.on_host:
            copy_stream = self._copy_stream()
            staged = self._staging("in", prefix.k[0].shape)
            landed = [torch.cuda.Event() for _ in range(2)]
            consumed = [torch.cuda.Event() for _ in range(2)]

            def stage(layer):
                sl = layer % 2
                if layer < 2:
                    copy_stream.wait_stream(cur)  # earlier work on the slots is ordered first
                else:
                    copy_stream.wait_event(consumed[sl])  # layer - 2 has read this slot
                with torch.cuda.stream(copy_stream):
                    staged[sl][0].copy_(prefix.k[layer], non_blocking=True)
                    staged[sl][1].copy_(prefix.v[layer], non_blocking=True)
                    landed[sl].record(copy_stream)

            stage(0)
        # A host-resident prefix pass (prefix_fill(offload=True)) writes each layer's K/V
        # into device staging slot i % 2 and drains it to the pinned host cache on the copy
        # stream while the next layer computes; a slot is rewritten only after its drain.
        sink = None
        if kv_out is not None and kv_out.on_host:
            sink_stream = self._copy_stream()
            sink = self._staging("out", kv_out.k[0].shape)
            computed = [torch.cuda.Event() for _ in range(2)]
            drained = [None, None]
        # Q4_K_M weights: block i + 1's six linears are dequantised into the other scratch
        # slot on a side stream while block i computes (the dequantisation reads HBM, the
        # block's GEMMs keep the tensor cores busy); a slot is refilled only after the
        # block that read it is done.
        quant = self.weight_format == "q4_k_m" and self.prefetch_weights
        if quant:
            dq = self._dq_stream()
            w_ready = [torch.cuda.Event(), torch.cuda.Event()]
            w_free = [None, None]
            dq.wait_stream(cur)  # earlier work on the scratch slots is ordered first

            def fetch(layer):
                sl = layer % 2
                if w_free[sl] is not None:
                    dq.wait_event(w_free[sl])
                with torch.cuda.stream(dq):
                    w = self.block_weights(layer, sl, stream=dq)
                    w_ready[sl].record(dq)
                return w

            nxt = fetch(0)
        for i in range(len(self.blocks)):
            if quant:
                blk = nxt
                cur.wait_event(w_ready[i % 2])
                if i + 1 < len(self.blocks):
                    nxt = fetch(i + 1)
            else:
                blk = self.block_weights(i)
            pk = pv = None
            if staged is not None:
                if i + 1 < len(self.blocks):
                    stage(i + 1)
                cur.wait_event(landed[i % 2])
                pk, pv = staged[i % 2]
            elif prefix is not None:
                pk, pv = prefix.k[i], prefix.v[i]
            fused = self.fused_qkv and kv_out is None and row_limit is None and H % 2 == 0
            if fused:   # projections + Q/K norm + RoPE in one GEMM, then the attention kernel
                q_rot, k_rot, v = b200attn.qkv_norm_rope_gemm(
                    y, blk["wqkv"], B, T, H, blk["nq"], blk["nk"], pe,
                    q_rot=self._buf("q_rot", (B, H, T, HEAD_DIM), torch.bfloat16),
                    k_rot=self._buf("k_rot", (B, H, T, HEAD_DIM), torch.bfloat16),
                    v=self._buf("v", (B, T, H, HEAD_DIM), torch.bfloat16))
            else:
                q = self._gemm(y, blk["wq"], "q").view(B, T, H, HEAD_DIM)
                k = self._gemm(y, blk["wk"], "k").view(B, T, H, HEAD_DIM)
                v = self._gemm(y, blk["wv"], "v").view(B, T, H, HEAD_DIM)
            if self.attn_marks is not None:
                ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                ev[0].record()
            if fused:
                b200attn.joint_attention(
                    q_rot, k_rot, v, pk, pv, desc=desc, out=attn,
                    workspace=ws[:b200attn.SPLIT_WORKSPACE_BYTES])
            else:
                k_dst = v_dst = None
                if sink is not None:
                    if drained[i % 2] is not None:
                        cur.wait_event(drained[i % 2])  # layer i - 2 has left this slot
                    k_dst, v_dst = sink[i % 2]
                elif kv_out is not None:
                    k_dst, v_dst = kv_out.k[i], kv_out.v[i]
                b200attn.attention_forward(
                    q, k, v, pk, pv, blk["nq"], blk["nk"], pe, desc=desc,
                    out=attn, workspace=ws, row_limit=row_limit, k_rot_out=k_dst, v_out=v_dst)
                if sink is not None:
                    sl = i % 2
                    computed[sl].record(cur)
                    sink_stream.wait_event(computed[sl])
                    with torch.cuda.stream(sink_stream):
                        kv_out.k[i].copy_(k_dst, non_blocking=True)
                        kv_out.v[i].copy_(v_dst, non_blocking=True)
                        drained[sl] = torch.cuda.Event()
                        drained[sl].record(sink_stream)
            if staged is not None:
                consumed[i % 2].record(cur)
            if self.attn_marks is not None:
                ev[1].record()
                self.attn_marks.append(ev)
            o = self._gemm(attn.view(R, h), blk["wo"], "o")
            b200attn.residual_adaln(x, o, gate1, scale2, y, rows_per_mod=R)    # attn residual, norm2
            mo = self._buf("mo", (R, h), torch.bfloat16)
            for r0 in range(0, R, self.mlp_chunk_rows):
                r1 = min(R, r0 + self.mlp_chunk_rows)
                gp = self._gemm(y[r0:r1], blk["wgp"], "gp")
                hh = b200attn.swiglu(gp, self._buf("h", (r1 - r0, cfg.ffn), torch.bfloat16))
                self._gemm(hh, blk["wmo"], "mo", out=mo[r0:r1])
            last = i + 1 == len(self.blocks)
            if quant:
                # (the residual kernel below reads no weights; the slot is free after mo)
                w_free[i % 2] = torch.cuda.Event()
                w_free[i % 2].record(cur)
            if last and sink is not None:
                for ev in drained:  # the host cache is complete when the pass is
                    if ev is not None:
                        cur.wait_event(ev)
            if not last:
                b200attn.residual_adaln(x, mo, gate2, scale1, y, rows_per_mod=R)  # next norm1
            elif final_scale is not None:
                b200attn.residual_adaln(x, mo, gate2, final_scale.view(1, h), y, rows_per_mod=R)
                return y
            else:
                b200attn.residual_adaln(x, mo, gate2, None, None, rows_per_mod=R)
        return None

    # -- prefix fill ---------------------------------------------------------------
    def text_embed(self, emb):
        """TextEmbedder::forward (src/transformer.rs:496-502): RMSNorm(w + 1) -> in_layer ->
        GELU (tanh) -> out_layer.  emb [R, text_dim] -> f32 [R, hidden]."""
        import torch
        import torch.nn.functional as F
        e = emb.float()
        e = e * torch.rsqrt(e.pow(2).mean(-1, keepdim=True) + 1e-6) * self.txt_norm_w
        a = F.gelu((e.to(torch.bfloat16) @ self.txt_in1.t()).float(), approximate="tanh")
        return (a.to(torch.bfloat16) @ self.txt_in2.t()).float()

    def prefix_fill(self, text_embs: Sequence, offload: bool = False) -> PrefixCache:
        """prefix_kv (src/transformer.rs:674-707) for a batch of text-only prompts of ragged
        lengths, in one pass: the prompts are padded to Pmax rows, each row's descriptor
        limits its keys to its own length, and the text rows' causal mask
        (build_block_causal_mask over image_ids = -1) is the row-limit list 1..Pmax.  The
        attention writes post-RoPE K and V straight into the cache layout.

        offload=True (set_kv_cache_offload, src/transformer.rs:27-45, which moves each
        layer's entry to the CPU as it is computed): the cache is allocated in pinned host
        memory up front and each layer's K/V goes through one of two reused device staging
        slots, drained to the host on a copy stream while the next layer computes, so the
        device never holds more than two layers of it."""
        import torch
        cfg = self.cfg
        B = len(text_embs)
        lengths = [int(e.shape[0]) for e in text_embs]
        P = max(lengths)
        emb = torch.zeros((B, P, cfg.text_dim), dtype=torch.bfloat16, device=self.device)
        for b, e in enumerate(text_embs):
            emb[b, :lengths[b]] = e.to(self.device, torch.bfloat16)
        x = self.text_embed(emb.view(B * P, cfg.text_dim)).contiguous()
        shape = (B, cfg.heads, P, HEAD_DIM)
        if offload:
            alloc = lambda: torch.empty(shape, dtype=torch.bfloat16).pin_memory()
        else:
            alloc = lambda: torch.zeros(shape, dtype=torch.bfloat16, device=self.device)
        cache = PrefixCache(k=[alloc() for _ in range(cfg.layers)],
                            v=[alloc() for _ in range(cfg.layers)], lengths=lengths)
        lay = b200attn.joint_layout(P, None, [], (0, 0))
        pe = torch.from_numpy(b200attn.rope_pe(lay["img_shapes"], lay["image_pad_mask"], AXES,
                                               ROPE_THETA)[:P]).to(self.device)
        limits = torch.from_numpy(b200attn.block_causal_limits(lay["image_ids"][:P])).to(self.device)
        desc = torch.tensor([[0, n] for n in lengths], dtype=torch.int32, device=self.device)
        mod = self.modulation(self.zero_time_embed())
        self._run_blocks(x, B, P, mod, pe, None, desc, row_limit=limits, kv_out=cache)
        return cache

    def target_pe(self, lengths: Sequence[int], grid: Tuple[int, int]):
        """RoPE rows of the target tokens of each sequence, f32 [B, T, D]: the target's frame
        position is its prompt's length (src/rope.rs:146-160), so rows differ per prompt."""
        import torch
        rows = []
        for n in lengths:
            lay = b200attn.joint_layout(n, None, [], grid)
            pe = b200attn.rope_pe(lay["img_shapes"], lay["image_pad_mask"], AXES, ROPE_THETA)
            rows.append(pe[n:])
        return torch.from_numpy(np.stack(rows)).to(self.device).contiguous()

    # -- one cached step --------------------------------------------------------------
    def step(self, lat, t: float, cache: PrefixCache, pe, desc):
        """The cached forward_conditioned of every sequence at timestep t: lat [B, T, C]
        (bf16 or f32) -> velocity f32 [B, T, C]."""
        import torch
        cfg = self.cfg
        B, T, C = lat.shape
        x = self._buf("x", (B * T, cfg.hidden), torch.float32)
        x_in = self._gemm(lat.reshape(B * T, C).to(torch.bfloat16), self.img_in, "x_in")
        x.copy_(x_in)
        t_emb = self.time_embed(t)
        y = self._run_blocks(x, B, T, self.modulation(t_emb), pe, cache, desc,
                             final_scale=self.final_scale(t_emb))
        out = self._buf("pred", (B * T, C), torch.bfloat16)
        torch.mm(y, self.proj_out.t(), out=out)
        return out.view(B, T, C).float()


def cached_desc(cache: PrefixCache, target_len: int, device):
    """Key descriptors of a cached step: each sequence sees its own prefix and every target
    key (src/transformer.rs:642-649 with key_valid None)."""
    import torch
    return torch.tensor([[n, target_len] for n in cache.lengths], dtype=torch.int32, device=device)


def denoise(model: MMDiT, pos_embs: Sequence, neg_embs: Optional[Sequence], grid: Tuple[int, int],
            steps: int, cfg_scale: float, noise, step_callback=None, offload_cache: bool = False):
    """denoise (src/pipeline.rs:126-197) for a batch of prompts: noise f32 [n_prompts, T, C]
    (packed), one prefix cache for every positive and negative prompt, `steps` Euler steps
    with true CFG (neg + scale * (pos - neg)) when neg_embs is given.  Latents stay f32;
    the transformer reads them as bf16.  offload_cache keeps the prefix cache in pinned host
    memory (set_kv_cache_offload).  Returns the final packed latents f32 [n, T, C]."""
    import torch
    n = noise.shape[0]
    T = grid[0] * grid[1]
    embs = list(pos_embs)
    if neg_embs is not None:  # sequence order: p0 pos, p0 neg, p1 pos, p1 neg, ...
        embs = [e for pair in zip(pos_embs, neg_embs) for e in pair]
    cache = model.prefix_fill(embs, offload=offload_cache)
    pe = model.target_pe(cache.lengths, grid)
    desc = cached_desc(cache, T, model.device)
    sigmas = flow_match_sigmas(steps, T)
    lat = noise.to(model.device, torch.float32).clone()
    for i in range(steps):
        x_in = lat.repeat_interleave(2, 0) if neg_embs is not None else lat
        pred = model.step(x_in, float(sigmas[i]), cache, pe, desc)
        if neg_embs is not None:
            pos, neg = pred[0::2], pred[1::2]
            pred = neg + (pos - neg) * cfg_scale
        lat = lat + pred * euler_dt(sigmas, i)
        if step_callback is not None:
            step_callback(i)
    return lat
