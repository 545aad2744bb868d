"""CPU restatement of the reference's joint-attention path — TEST INFRASTRUCTURE ONLY.

This module is the checker for the CUDA path.  Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline leg may import it; the product library never calls it.

Parity status: the RoPE tables / positions, the rotation formula and the joint layout are
pinned by the reference's own unit tests (``src/rope.rs:278-316``, ``src/rope.rs:351-361``,
``src/joint_layout.rs:133-164``), ported as known-answer tests in ``tests/golden``.  The
attention arithmetic (``chunked_attention``) has no golden vector in the reference: it is
restated from its call sites over candle 0.11.0 (``candle-core`` matmul,
``candle-nn::ops::softmax_last_dim``; ``Cargo.lock`` pins both), and the reference itself
cannot be built here (Rust, no cargo) — attention parity is anchored on this restatement.

Every function cites the reference file:line it follows.  Arrays are numpy; float math is
done in float32 like the reference's F32 path unless a function says otherwise.
"""
from __future__ import annotations

import math
from typing import List, Optional, Sequence, Tuple

import numpy as np

# src/rope.rs:43-47 — table rows cover positions -1024..8191; row = position + 1024
# (src/rope.rs:177).
TABLE_NEG = 1024
TABLE_POS = 8192
TABLE_OFFSET = 1024

# src/transformer.rs:206
ATTENTION_SCORE_BUDGET_BYTES = 256 << 20


# ----------------------------------------------------------------------------- layout
def joint_layout(text_len: int, text_image_mask: Optional[Sequence[bool]],
                 cond_shapes: Sequence[Tuple[int, int]], target: Tuple[int, int]):
    """JointLayout::new (src/joint_layout.rs:52-103).

    Returns dict(pieces, image_pad_mask, image_ids, img_shapes, prefix_len, target_len).
    Raises ValueError for the reference's ``bail!`` cases.
    """
    tokens_per_slot = 4  # src/joint_layout.rs:10
    slots = list(text_image_mask) if text_image_mask is not None else [False] * text_len
    if len(slots) != text_len:
        raise ValueError(f"text_image_mask has {len(slots)} entries for {text_len} prompt tokens")
    pieces = []
    i = next_image = 0
    while i < text_len:
        if not slots[i]:
            n = 0
            while i + n < text_len and not slots[i + n]:
                n += 1
            pieces.append(("text", i, n))
            i += n
            continue
        if next_image >= len(cond_shapes):
            raise ValueError("prompt has more image slots than condition images")
        h, w = cond_shapes[next_image]
        needed = h * w // tokens_per_slot
        if (h * w) % tokens_per_slot != 0 or sum(1 for s in slots[i:i + needed] if s) != needed:
            raise ValueError(f"condition image {next_image} needs {needed} consecutive image slots")
        pieces.append(("cond", next_image))
        next_image += 1
        i += needed
    if next_image != len(cond_shapes):
        raise ValueError("more condition images than slots")
    pieces.append(("target",))
    img_shapes = [(1, h, w) for (h, w) in cond_shapes] + [(1, target[0], target[1])]
    image_pad_mask: List[bool] = []
    image_ids: List[int] = []
    for p in pieces:
        if p[0] == "text":
            n, ident = p[2], -1
        elif p[0] == "cond":
            h, w = cond_shapes[p[1]]
            n, ident = h * w, p[1]
        else:
            n, ident = target[0] * target[1], len(cond_shapes)
        image_pad_mask += [ident >= 0] * n
        image_ids += [ident] * n
    target_len = target[0] * target[1]
    return dict(pieces=pieces, image_pad_mask=image_pad_mask, image_ids=image_ids,
                img_shapes=img_shapes, prefix_len=len(image_ids) - target_len,
                target_len=target_len)


# ----------------------------------------------------------------------------- RoPE
def rope_positions(img_shapes: Sequence[Tuple[int, int, int]],
                   image_pad_mask: Sequence[bool]) -> np.ndarray:
    """EmbedNd::forward position rules (src/rope.rs:118-172) -> int64 [S, 3] (f, h, w)."""
    seq_len = len(image_pad_mask)
    is_img = [bool(x) for x in image_pad_mask]
    fr: List[int] = []
    hi: List[int] = []
    wi: List[int] = []
    cursor = 0
    position = 0
    for (frame, height, width) in img_shapes:
        block_tokens = frame * height * width
        block_start = seq_len
        for p in range(cursor, seq_len):
            if is_img[p]:
                block_start = p
                break
        for _ in range(block_start - cursor):  # text tokens advance all axes
            fr.append(position); hi.append(position); wi.append(position)
            position += 1
        cursor = block_start
        fr += [position] * block_tokens  # frame frozen at the running position
        position += max(height, width)
        h_start = -(height - height // 2)
        w_start = -(width - width // 2)
        for h in range(height):
            for w in range(width):
                hi.append(h_start + h)
                wi.append(w_start + w)
        cursor += block_tokens
    for _ in range(cursor, seq_len):
        fr.append(position); hi.append(position); wi.append(position)
        position += 1
    return np.stack([np.array(fr, np.int64), np.array(hi, np.int64), np.array(wi, np.int64)], 1)


def rope_tables(theta: float = 1e4, axes_dim: Sequence[int] = (16, 56, 56)):
    """EmbedNd::new_with_mode (src/rope.rs:37-88): per axis (cos, sin) tables
    [9216, dim/2] float32, row = position + 1024.  Angles follow the reference:
    inv_freq = exp(i * (-2 ln(theta)/dim)) in f32, angle = position * inv_freq in f32."""
    pos = np.arange(0, TABLE_POS, dtype=np.float32)
    neg = -np.arange(1, TABLE_NEG + 1, dtype=np.float32)[::-1]
    idx = np.concatenate([neg, pos]).astype(np.float32)
    out = []
    for dim in axes_dim:
        half = dim // 2
        coef = np.float32(-2.0 * math.log(theta) / dim)
        inv_freq = np.exp(np.arange(half, dtype=np.float32) * coef).astype(np.float32)
        ang = (idx[:, None] * inv_freq[None, :]).astype(np.float32)
        out.append((np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)))
    return out


def embed_nd(img_shapes, image_pad_mask, theta: float = 1e4,
             axes_dim: Sequence[int] = (16, 56, 56)) -> np.ndarray:
    """EmbedNd::forward (src/rope.rs:104-211) -> pe [S, sum(axes)] float32 with
    interleaved (cos_i, sin_i) pairs: 8 frame pairs, then 28 height, then 28 width."""
    pos = rope_positions(img_shapes, image_pad_mask)
    tabs = rope_tables(theta, axes_dim)
    parts = []
    for axis, (c, s) in enumerate(tabs):
        row = pos[:, axis] + TABLE_OFFSET
        if row.min(initial=0) < 0 or row.max(initial=0) >= c.shape[0]:
            raise IndexError("RoPE position outside the reference table range")
        parts.append(np.stack([c[row], s[row]], -1))  # [S, half, 2]
    cat = np.concatenate(parts, 1)
    return cat.reshape(cat.shape[0], -1).astype(np.float32)


def apply_rope(x: np.ndarray, pe: np.ndarray) -> np.ndarray:
    """apply_rope / rope_i (src/rope.rs:222-228, formula pinned by src/rope.rs:324-349):
    x [B,H,S,D]; pair i: (x0 c - x1 s, x0 s + x1 c)."""
    s_len, d = x.shape[-2], x.shape[-1]
    f = pe.reshape(s_len, d // 2, 2)
    c, s = f[..., 0], f[..., 1]
    xr = x.reshape(*x.shape[:-1], d // 2, 2)
    x0, x1 = xr[..., 0], xr[..., 1]
    o0 = x0 * c - x1 * s
    o1 = x0 * s + x1 * c
    return np.stack([o0, o1], -1).reshape(x.shape).astype(np.float32)


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """candle_nn::RmsNorm as built at src/transformer.rs:141-145 (eps 1e-6):
    x / sqrt(mean(x^2) + eps) * w over the last axis, float32."""
    x = x.astype(np.float32)
    ms = np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32)
    return (x / np.sqrt(ms + np.float32(eps)) * w.astype(np.float32)).astype(np.float32)


# ----------------------------------------------------------------------------- masks
def key_valid(txt_mask: Optional[np.ndarray], layout: dict, seq_txt: int, seq_img: int):
    """QwenImageTransformer::key_valid (src/transformer.rs:738-745): [B, len] uint8 — the
    text mask on text positions, 1 on condition and target tokens."""
    if txt_mask is None:
        return None
    b = txt_mask.shape[0]
    total = len(layout["image_ids"])
    out = np.ones((b, total), np.uint8)
    pos = 0
    for p in layout["pieces"]:
        if p[0] == "text":
            out[:, pos:pos + p[2]] = txt_mask[:, p[1]:p[1] + p[2]]
            pos += p[2]
        elif p[0] == "cond":
            pos += int(np.prod(layout["img_shapes"][p[1]][1:]))
        else:
            pos += seq_img
    return out


def block_causal_mask(image_ids: Sequence[int], key_valid_: Optional[np.ndarray], batch: int):
    """build_block_causal_mask (src/attention_mask.rs:18-66): [B,1,S,S] bool,
    causal OR (same image block AND q_image_id >= 0), times key_valid."""
    ids = np.asarray(image_ids, np.int64)
    s = ids.shape[0]
    same = (ids[:, None] == ids[None, :]) & (ids[:, None] >= 0)
    causal = np.arange(s)[:, None] >= np.arange(s)[None, :]
    allowed = (causal | same)[None, None]
    if key_valid_ is not None:
        return allowed & (key_valid_[:, None, None, :] != 0)
    return np.broadcast_to(allowed, (batch, 1, s, s)).copy()


def block_causal_limits_from_mask(mask2d: np.ndarray):
    """Per-row key limits of a dense [S,S] mask whose rows are leading runs of keys
    (build_block_causal_mask without key_valid); None if a row is not a leading run."""
    out = []
    for row in mask2d.astype(bool):
        n = int(row.sum())
        if not row[:n].all():
            return None
        out.append(n)
    return np.asarray(out, np.int32)


def key_valid_to_desc(kv: np.ndarray, prefix_len: int, target_len: int):
    """Descriptor form of a cached step's key_valid [B, P+T]: (prefix_valid, target_valid)
    per row; None if padding is not a prefix suffix (then no descriptor exists)."""
    out = []
    for row in kv:
        pre = row[:prefix_len].astype(bool)
        pv = int(pre.sum())
        if not pre[:pv].all() or not row[prefix_len:prefix_len + target_len].astype(bool).all():
            return None
        out.append((pv, target_len))
    return out


# ----------------------------------------------------------------------------- attention
def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 to the nearest bfloat16 (ties to even), returned as float32."""
    x = np.ascontiguousarray(x, np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) << 16
    out = (r & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
    return np.where(np.isnan(x), x, out)


def chunked_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float,
                      mask: Optional[np.ndarray] = None, p_dtype: str = "f32") -> np.ndarray:
    """chunked_attention (src/transformer.rs:259-296), the non-FA CPU path.

    q [B,H,Sq,D], k/v [B,H,Skv,D]; mask bool [B,1,Sq|1,Skv] (True = attend).  The query
    chunk holds ATTENTION_SCORE_BUDGET_BYTES of f32 scores (line 273); q is scaled first
    (275); scores + additive -inf mask (284-287); softmax in f32 (292); P cast to the v
    dtype (``p_dtype`` "bf16" rounds it like the reference's BF16 run); P @ v (293).
    """
    b, h, sq, _ = q.shape
    skv = k.shape[2]
    rows = max(1, min(sq, ATTENTION_SCORE_BUDGET_BYTES // (b * h * skv * 4)))
    qs = (q.astype(np.float32) * np.float32(scale)).astype(np.float32)
    kt = np.swapaxes(k.astype(np.float32), 2, 3)
    vf = v.astype(np.float32)
    outs = []
    for start in range(0, sq, rows):
        n = min(rows, sq - start)
        w = np.matmul(qs[:, :, start:start + n], kt).astype(np.float32)
        if mask is not None:
            m = mask if mask.shape[2] == 1 else mask[:, :, start:start + n]
            w = w + np.where(m, np.float32(0), np.float32(-np.inf))
        mx = w.max(-1, keepdims=True)
        e = np.exp(w - mx).astype(np.float32)
        p = (e / e.sum(-1, keepdims=True, dtype=np.float32)).astype(np.float32)
        if p_dtype == "bf16":
            p = bf16_round(p)
        outs.append(np.matmul(p, vf).astype(np.float32))
    return np.concatenate(outs, 2)


def attention_forward(q_raw, k_raw, v_raw, norm_q_w, norm_k_w, pe, prefix=None,
                      desc=None, scale=None, eps=1e-6):
    """Attention::forward from the norm to the head merge (src/transformer.rs:179-193).

    q_raw/k_raw/v_raw [B,T,H,D] (the projections, as float32 values of the bf16 inputs);
    prefix = (pk, pv) [B,H,P,D] post-RoPE cache; desc = list of (prefix_valid,
    target_valid) per batch row, or None (no mask).  Returns (out [B,T,H*D], k_rot
    [B,H,T,D], v [B,H,T,D]) in float32.
    """
    b, t, h, d = q_raw.shape
    if scale is None:
        scale = d ** -0.5
    q = np.transpose(rms_norm(q_raw, norm_q_w, eps), (0, 2, 1, 3))
    k = np.transpose(rms_norm(k_raw, norm_k_w, eps), (0, 2, 1, 3))
    v = np.transpose(v_raw.astype(np.float32), (0, 2, 1, 3))
    q = apply_rope(q, pe)
    k = apply_rope(k, pe)
    if prefix is not None:
        k_all = np.concatenate([prefix[0].astype(np.float32), k], 2)
        v_all = np.concatenate([prefix[1].astype(np.float32), v], 2)
        p_len = prefix[0].shape[2]
    else:
        k_all, v_all, p_len = k, v, 0
    mask = None
    if desc is not None:
        mask = np.zeros((b, 1, 1, p_len + t), bool)
        for i, (pv_, tv_) in enumerate(desc):
            mask[i, 0, 0, :pv_] = True
            mask[i, 0, 0, p_len:p_len + tv_] = True
    o = chunked_attention(q, k_all, v_all, scale, mask)
    out = np.transpose(o, (0, 2, 1, 3)).reshape(b, t, h * d)
    return out, k, v


def attention_flops(b: int, h: int, sq: int, lk_valid: int, d: int = 128) -> float:
    """Algorithmic FLOPs of one attention call: QK^T plus PV, 4*B*H*Sq*Lk*D."""
    return 4.0 * b * h * sq * lk_valid * d


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    """||a-b|| / ||b|| in float64 (the parity metric, with max-abs)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
