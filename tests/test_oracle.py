"""The CPU oracle pinned against the reference's own known-answer tests and checked
against independent formulations (no GPU)."""
import json
import math
import os

import numpy as np
import pytest

from oracle import cpu as ocpu
from oracle import reference as ref

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


# --------------------------------------------------------------- RoPE KATs (src/rope.rs)
def test_embed_nd_matches_reference_formula():
    """Port of rope::tests::test_embed_nd_matches_reference_formula (src/rope.rs:278-316)."""
    kat = load("rope_kat.json")
    shapes = [tuple(s) for s in kat["img_shapes"]]
    pe = ref.embed_nd(shapes, kat["image_pad_mask"], kat["theta"], kat["axes"])
    assert pe.shape == (6, 128)
    assert np.all((np.abs(np.abs(pe[0]) - 1) < 1e-4) | (np.abs(pe[0]) < 1e-4))
    want = np.asarray(kat["rows"], np.float32)
    assert np.max(np.abs(pe - want)) < kat["tol"]
    pos = ref.rope_positions(shapes, kat["image_pad_mask"])
    assert pos.tolist() == kat["positions"]


def test_apply_rope_matches_complex_multiply():
    """Port of rope::tests::test_apply_rope_matches_reference (src/rope.rs:351-361)."""
    rng = np.random.default_rng(0)
    x = rng.standard_normal((1, 3, 5, 16)).astype(np.float32)
    ang = (3.0 * rng.standard_normal((5, 8))).astype(np.float32)
    freqs = np.stack([np.cos(ang), np.sin(ang)], 2).reshape(5, 16)
    got = ref.apply_rope(x, freqs)
    xc = x.reshape(1, 3, 5, 8, 2)
    z = (xc[..., 0] + 1j * xc[..., 1]) * (np.cos(ang) + 1j * np.sin(ang))
    want = np.stack([z.real, z.imag], -1).reshape(x.shape)
    assert np.max(np.abs(got - want)) < 1e-5


def test_rope_positions_grid_centering():
    """h, w run over [-(n - n//2), n//2) for odd and even grids (src/rope.rs:153-158); the
    running position advances by max(h, w) after a block (rope.rs:150)."""
    lay = ref.joint_layout(3, None, [], (3, 4))
    pos = ref.rope_positions(lay["img_shapes"], lay["image_pad_mask"])
    assert pos[:3].tolist() == [[0, 0, 0], [1, 1, 1], [2, 2, 2]]
    assert set(pos[3:, 0]) == {3}
    assert sorted(set(pos[3:, 1])) == [-2, -1, 0]
    assert sorted(set(pos[3:, 2])) == [-2, -1, 0, 1]


# --------------------------------------------------------------- layout KATs
@pytest.mark.parametrize("case", load("layout_kat.json"), ids=lambda c: c["source"])
def test_joint_layout_kat(case):
    cs = [tuple(s) for s in case["cond_shapes"]]
    lay = ref.joint_layout(case["text_len"], case["text_image_mask"], cs, tuple(case["target"]))
    if "image_ids" in case:
        assert lay["image_ids"] == case["image_ids"]
        assert (lay["prefix_len"], lay["target_len"]) == (case["prefix_len"], case["target_len"])
    else:
        assert lay["image_ids"][:8] == case["image_ids_prefix8"]


def test_joint_layout_errors():
    with pytest.raises(ValueError):
        ref.joint_layout(2, [True, False], [], (2, 2))  # slot without image
    with pytest.raises(ValueError):
        ref.joint_layout(2, [True, True], [(4, 4)], (2, 2))  # needs 4 slots, has 2
    with pytest.raises(ValueError):
        ref.joint_layout(3, [False, False, False], [(2, 2)], (2, 2))  # image without slots


# --------------------------------------------------------------- attention oracle
def _softmax_attention_f64(q, k, v, scale, kvalid=None):
    s = np.einsum("bhqd,bhkd->bhqk", q.astype(np.float64), k.astype(np.float64)) * scale
    if kvalid is not None:
        for b, n in enumerate(kvalid):
            s[b, :, :, n:] = -np.inf
    s -= s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    return np.einsum("bhqk,bhkd->bhqd", p, v.astype(np.float64))


@pytest.mark.parametrize("sq,skv", [(1, 1), (7, 33), (128, 300), (200, 129)])
def test_chunked_attention_matches_softmax(sq, skv):
    rng = np.random.default_rng(sq * 1000 + skv)
    q = rng.standard_normal((2, 3, sq, 128)).astype(np.float32)
    k = rng.standard_normal((2, 3, skv, 128)).astype(np.float32)
    v = rng.standard_normal((2, 3, skv, 128)).astype(np.float32)
    got = ref.chunked_attention(q, k, v, 128 ** -0.5)
    want = _softmax_attention_f64(q, k, v, 128 ** -0.5)
    assert ref.rel_l2(got, want) < 1e-5


def test_chunked_attention_matches_torch_sdpa():
    """A third, independent implementation: torch's scaled_dot_product_attention (CPU,
    float64) with the same boolean key mask."""
    import torch
    rng = np.random.default_rng(17)
    q = rng.standard_normal((2, 3, 40, 128)).astype(np.float32)
    k = rng.standard_normal((2, 3, 90, 128)).astype(np.float32)
    v = rng.standard_normal((2, 3, 90, 128)).astype(np.float32)
    mask = np.zeros((2, 1, 1, 90), bool)
    mask[0, ..., :61] = True
    mask[1, ..., :90] = True
    got = ref.chunked_attention(q, k, v, 128 ** -0.5, mask)
    t = lambda x: torch.from_numpy(x).double()
    want = torch.nn.functional.scaled_dot_product_attention(
        t(q), t(k), t(v), attn_mask=torch.from_numpy(mask), scale=128 ** -0.5).numpy()
    assert ref.rel_l2(got, want) < 1e-5


def test_chunked_attention_chunking_is_exact(monkeypatch):
    """The 256 MiB query chunk bounds memory only (src/transformer.rs:201-205): the result
    matches the unchunked one up to the GEMM's summation order."""
    rng = np.random.default_rng(1)
    q = rng.standard_normal((1, 2, 50, 128)).astype(np.float32)
    k = rng.standard_normal((1, 2, 70, 128)).astype(np.float32)
    v = rng.standard_normal((1, 2, 70, 128)).astype(np.float32)
    whole = ref.chunked_attention(q, k, v, 0.088)
    monkeypatch.setattr(ref, "ATTENTION_SCORE_BUDGET_BYTES", 2 * 70 * 4 * 7)
    chunked = ref.chunked_attention(q, k, v, 0.088)
    assert ref.rel_l2(chunked, whole) < 1e-6


def test_masked_attention_and_desc():
    rng = np.random.default_rng(2)
    q = rng.standard_normal((2, 2, 9, 128)).astype(np.float32)
    k = rng.standard_normal((2, 2, 20, 128)).astype(np.float32)
    v = rng.standard_normal((2, 2, 20, 128)).astype(np.float32)
    mask = np.zeros((2, 1, 1, 20), bool)
    mask[0, ..., :13] = True
    mask[1, ..., :20] = True
    got = ref.chunked_attention(q, k, v, 0.1, mask)
    want = _softmax_attention_f64(q, k, v, 0.1, [13, 20])
    assert ref.rel_l2(got, want) < 1e-5
    kv = np.ones((2, 20), np.uint8)
    kv[0, 10:15] = 0  # prefix of 15 with 5 padded keys at its end
    assert ref.key_valid_to_desc(kv, 15, 5) == [(10, 5), (15, 5)]
    kv[1, 3] = 0
    assert ref.key_valid_to_desc(kv, 15, 5) is None


def test_block_causal_mask_matches_definition():
    """src/attention_mask.rs:3 — (q >= kv) OR (same image block AND q_image_id >= 0)."""
    lay = ref.joint_layout(4, [False, True, True, False], [(2, 4)], (2, 2))
    ids = lay["image_ids"]
    m = ref.block_causal_mask(ids, None, 1)[0, 0]
    for qi in range(len(ids)):
        for ki in range(len(ids)):
            assert m[qi, ki] == ((qi >= ki) or (ids[qi] == ids[ki] and ids[qi] >= 0))


def test_c_oracle_matches_numpy_oracle():
    rng = np.random.default_rng(3)
    q = rng.standard_normal((1, 2, 70, 128)).astype(np.float32)
    k = rng.standard_normal((1, 2, 150, 128)).astype(np.float32)
    v = rng.standard_normal((1, 2, 150, 128)).astype(np.float32)
    got = ocpu.chunked_attention(q, k, v, 128 ** -0.5, np.array([111], np.int32))
    mask = np.zeros((1, 1, 1, 150), bool)
    mask[..., :111] = True
    want = ref.chunked_attention(q, k, v, 128 ** -0.5, mask)
    assert ref.rel_l2(got, want) < 1e-5


def test_c_oracle_full_span_matches_golden():
    """The C restatement of the whole norm -> RoPE -> cat -> attention span reproduces the
    committed golden case (ragged prefix, two batch rows)."""
    g = np.load(os.path.join(GOLDEN, "attn_small.npz"))
    out = ocpu.attention_forward(g["q"], g["k"], g["v"], g["prefix_k"], g["prefix_v"],
                                 g["norm_q_w"], g["norm_k_w"], 1e-6, g["pe"], g["desc"][:, 0],
                                 128 ** -0.5)
    assert ref.rel_l2(out, g["out"]) < 1e-5


def test_bf16_round_ties_to_even():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, np.inf], np.float32)
    r = ref.bf16_round(x)
    assert r.tolist() == [1.0, 1.0, 1.015625, -2.5, np.inf]
    assert math.isnan(ref.bf16_round(np.array([np.nan], np.float32))[0])
