"""Generates the golden fixtures in tests/golden (run: python tests/golden/make_golden.py).

- rope_kat.json     — the reference's RoPE known-answer case (src/rope.rs:278-316): a
                      2-token prompt followed by a 1x2x2 image block.  Expected rows are the
                      closed form the reference test uses (``reference_cos_sin``,
                      rope.rs:256-268: cos/sin of coord * theta^(-2i/dim) in f64, cast to
                      f32) at the positions that test states (text advances all axes;
                      the image frame is frozen at 2 and h, w in {-1, 0}).
- layout_kat.json   — the expected values asserted by src/joint_layout.rs:133-164.
- attn_small.npz    — a seeded small attention case (bf16 inputs as uint16 bit patterns,
                      ragged prefix) with its expected float32 output from the CPU oracle
                      (oracle/reference.py, the float32 path of the reference).  The
                      reference cannot run here (Rust/candle without cargo), so this
                      fixture pins the CUDA path to the restatement, not to candle.
"""
from __future__ import annotations

import json
import math
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import reference as ref  # noqa: E402  (test infrastructure)


def rope_kat():
    axes, theta = [16, 56, 56], 10000.0

    def cos_sin(coord):
        row = []
        for axis, dim in enumerate(axes):
            for i in range(dim // 2):
                ang = coord[axis] * theta ** (-2.0 * i / dim)
                row += [float(np.float32(math.cos(ang))), float(np.float32(math.sin(ang)))]
        return row

    coords = [(0, 0, 0), (1, 1, 1), (2, -1, -1), (2, -1, 0), (2, 0, -1), (2, 0, 0)]
    return dict(source="src/rope.rs:278-316", axes=axes, theta=theta, img_shapes=[[1, 2, 2]],
                image_pad_mask=[0, 0, 1, 1, 1, 1], positions=[list(c) for c in coords],
                rows=[cos_sin(c) for c in coords], tol=1e-3)


def layout_kat():
    cases = [
        dict(source="src/joint_layout.rs:133-139", text_len=3, text_image_mask=None,
             cond_shapes=[], target=[2, 2], image_ids=[-1, -1, -1, 0, 0, 0, 0],
             prefix_len=3, target_len=4),
        dict(source="src/joint_layout.rs:141-156", text_len=4,
             text_image_mask=[False, True, True, False], cond_shapes=[[2, 4]], target=[2, 2],
             image_ids=[-1] + [0] * 8 + [-1] + [1] * 4, prefix_len=10, target_len=4),
        dict(source="src/joint_layout.rs:158-164", text_len=2, text_image_mask=[True, True],
             cond_shapes=[[2, 2], [2, 2]], target=[2, 2],
             image_ids_prefix8=[0, 0, 0, 0, 1, 1, 1, 1]),
    ]
    return cases


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    r = ref.bf16_round(x.astype(np.float32))
    return (r.view(np.uint32) >> 16).astype(np.uint16)


def bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def attn_small():
    rng = np.random.default_rng(20261201)
    B, T, H, D, P = 2, 40, 3, 128, 24
    q = to_bf16_bits(rng.standard_normal((B, T, H, D), dtype=np.float32))
    k = to_bf16_bits(rng.standard_normal((B, T, H, D), dtype=np.float32))
    v = to_bf16_bits(rng.standard_normal((B, T, H, D), dtype=np.float32))
    pk = to_bf16_bits(rng.standard_normal((B, H, P, D), dtype=np.float32))
    pv = to_bf16_bits(rng.standard_normal((B, H, P, D), dtype=np.float32))
    wq = (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    wk = (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    # a 24-token prompt followed by a 5x8 target grid
    lay = ref.joint_layout(P, None, [], (5, 8))
    pe_all = ref.embed_nd(lay["img_shapes"], lay["image_pad_mask"])
    pe = pe_all[P:]
    desc = [(19, T), (24, T)]
    out, krot, _ = ref.attention_forward(bits_to_f32(q), bits_to_f32(k),
                                         bits_to_f32(v), wq, wk, pe,
                                         prefix=(bits_to_f32(pk), bits_to_f32(pv)), desc=desc)
    return dict(q=q, k=k, v=v, prefix_k=pk, prefix_v=pv, norm_q_w=wq, norm_k_w=wk, pe=pe,
                desc=np.asarray(desc, np.int32), out=out.astype(np.float32),
                k_rot=krot.astype(np.float32))


def main():
    with open(os.path.join(HERE, "rope_kat.json"), "w") as f:
        json.dump(rope_kat(), f)
    with open(os.path.join(HERE, "layout_kat.json"), "w") as f:
        json.dump(layout_kat(), f, indent=1)
    np.savez_compressed(os.path.join(HERE, "attn_small.npz"), **attn_small())


if __name__ == "__main__":
    main()
