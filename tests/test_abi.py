"""The C-ABI library without a GPU: it loads, exports every symbol include/*.h
declares, its host-side mirrors reproduce the reference's known answers and the oracle,
and its entry points reject bad arguments before touching a device."""
import ctypes
import json
import os
import re

import numpy as np
import pytest

import b200attn
from oracle import reference as ref

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")


def declared_functions():
    names = set()
    for hdr in sorted(f for f in os.listdir(os.path.join(ROOT, "include")) if f.endswith(".h")):
        src = open(os.path.join(ROOT, "include", hdr)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names |= set(re.findall(r"\b(b200_[a-z0-9_]+)\s*\(", src))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    names = declared_functions()
    assert len(names) >= 10
    lib = b200attn.lib()
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/ but not exported"
    assert set(names) <= set(b200attn.EXPORTED) | {"b200_attn_fwd_noalloc"}
    hdr = open(os.path.join(ROOT, "include", "b200_attn.h")).read()
    version = int(re.search(r"#define B200_ATTN_ABI_VERSION (\d+)", hdr).group(1))
    assert lib.b200_abi_version() == version


def test_strerror():
    assert b200attn.strerror(0) == "ok"
    for code in range(-6, 0):
        assert b200attn.strerror(code) != "unknown status"


@pytest.mark.parametrize("case", json.load(open(os.path.join(GOLDEN, "layout_kat.json"))),
                         ids=lambda c: c["source"])
def test_joint_layout_kat_through_abi(case):
    cs = [tuple(s) for s in case["cond_shapes"]]
    lay = b200attn.joint_layout(case["text_len"], case["text_image_mask"], cs, tuple(case["target"]))
    if "image_ids" in case:
        assert lay["image_ids"].tolist() == case["image_ids"]
        assert (lay["prefix_len"], lay["target_len"]) == (case["prefix_len"], case["target_len"])
    else:
        assert lay["image_ids"][:8].tolist() == case["image_ids_prefix8"]


def test_joint_layout_errors_through_abi():
    with pytest.raises(b200attn.B200Error):
        b200attn.joint_layout(2, [True, False], [], (2, 2))
    with pytest.raises(b200attn.B200Error):
        b200attn.joint_layout(2, [True, True], [(4, 4)], (2, 2))
    with pytest.raises(b200attn.B200Error):
        b200attn.joint_layout(3, [False] * 3, [(2, 2)], (2, 2))


def test_rope_kat_through_abi():
    kat = json.load(open(os.path.join(GOLDEN, "rope_kat.json")))
    pe = b200attn.rope_pe(kat["img_shapes"], kat["image_pad_mask"], kat["axes"], kat["theta"])
    assert np.max(np.abs(pe - np.asarray(kat["rows"], np.float32))) < kat["tol"]
    pos = b200attn.rope_positions(kat["img_shapes"], kat["image_pad_mask"])
    assert pos.tolist() == kat["positions"]


@pytest.mark.parametrize("text,cond,target", [
    (512, [], (64, 64)),                       # config 2 layout (1024^2 T2I)
    (256, [], (32, 32)),                       # config 1 layout (512^2)
    (40, [(4, 6), (8, 8)], (6, 10)),           # two condition images in the prompt
])
def test_rope_pe_matches_oracle(text, cond, target):
    slots = [False] * text
    p = 2
    for (h, w) in cond:  # place each image's slots after a couple of text tokens
        n = h * w // 4
        slots[p:p + n] = [True] * n
        p += n + 2
    lay = ref.joint_layout(text, slots, cond, target)
    want = ref.embed_nd(lay["img_shapes"], lay["image_pad_mask"])
    got = b200attn.rope_pe(lay["img_shapes"], lay["image_pad_mask"])
    # both build the tables in f32; one-ulp differences of inv_freq grow with the
    # position (angles up to ~600 rad here), well inside the reference KAT's 1e-3
    assert np.max(np.abs(got - want)) < 1e-4
    assert np.array_equal(b200attn.rope_positions(lay["img_shapes"], lay["image_pad_mask"]),
                          ref.rope_positions(lay["img_shapes"], lay["image_pad_mask"]))
    lay2 = b200attn.joint_layout(text, slots, cond, target)
    assert lay2["image_ids"].tolist() == lay["image_ids"]


def test_rope_pe_rejects_positions_outside_table():
    # a 9000-token prompt runs past the reference's 8191 table end
    with pytest.raises(b200attn.B200Error):
        b200attn.rope_pe([(1, 2, 2)], [0] * 9000 + [1] * 4)


def test_key_valid_to_desc_through_abi():
    kv = np.ones((2, 20), np.uint8)
    kv[0, 10:15] = 0
    assert b200attn.key_valid_to_desc(kv, 15, 5).tolist() == [[10, 5], [15, 5]]
    kv[1, 3] = 0
    with pytest.raises(b200attn.B200Error):
        b200attn.key_valid_to_desc(kv, 15, 5)


def test_entry_points_reject_bad_arguments_without_device():
    lib = b200attn.lib()
    a = b200attn.AttnArgs()
    a.batch, a.heads, a.head_dim, a.target_len = 1, 1, 64, 8
    assert lib.b200_attn_fwd(ctypes.byref(a), None) == b200attn.ERR_UNSUPPORTED
    a.head_dim = 128
    assert lib.b200_attn_fwd(ctypes.byref(a), None) == b200attn.ERR_INVALID  # null tensors
    a.target_len = 0
    assert lib.b200_attn_fwd(ctypes.byref(a), None) == b200attn.OK  # nothing to do
    assert lib.b200_attn_fwd(None, None) == b200attn.ERR_INVALID
    assert lib.b200_chunked_attention(None, None, None, None, 1, 1, 4, 4, 96, 0.1, None, None,
                                      None) == b200attn.ERR_UNSUPPORTED
    assert lib.b200_chunked_attention(None, None, None, None, 1, 1, 4, 4, 128, 0.1, None, None,
                                      None) == b200attn.ERR_INVALID
    assert lib.b200_norm_rope(None, None, 1, 1, 1, 128, None, 1e-6, None, None) == b200attn.ERR_INVALID
    # misaligned (but non-null) pointers are refused before any device access
    assert lib.b200_chunked_attention(8, 16, 32, 48, 1, 1, 4, 4, 128, 0.1, None, None,
                                      None) == b200attn.ERR_INVALID
    # the [B,S,H,D] (flash_attn) contract: same checks before any launch
    assert lib.b200_flash_attention(None, None, None, None, 1, 4, 4, 1, 128, 0.1, None, None,
                                    None) == b200attn.ERR_INVALID
    assert lib.b200_flash_attention(16, 16, 16, 16, 1, 4, 4, 1, 64, 0.1, None, None,
                                    None) == b200attn.ERR_UNSUPPORTED
    assert lib.b200_flash_attention(16, 16, 16, 16, 1, 4, 0, 1, 128, 0.1, None, None,
                                    None) == b200attn.ERR_INVALID
    assert lib.b200_flash_attention(16, 16, 16, 16, 1, 0, 4, 1, 128, 0.1, None, None,
                                    None) == b200attn.OK  # nothing to do
    assert lib.b200_flash_attention(16, 16, 16, 16, 1, 4, 4, 1, 128, -1.0, None, None,
                                    None) == b200attn.ERR_INVALID
    # b200_flash_attention_ex: bf16 and f16 pass the checks, any other element type (f32,
    # an unknown code) is refused before anything else is looked at
    for dt in (b200attn.DTYPE_F32, 7, -1):
        assert lib.b200_flash_attention_ex(16, 16, 16, 16, 1, 4, 4, 1, 128, 0.1, None, dt, None,
                                           None) == b200attn.ERR_UNSUPPORTED
    for dt in (b200attn.DTYPE_BF16, b200attn.DTYPE_F16):
        assert lib.b200_flash_attention_ex(None, None, None, None, 1, 4, 4, 1, 128, 0.1, None, dt,
                                           None, None) == b200attn.ERR_INVALID
        assert lib.b200_flash_attention_ex(16, 16, 16, 16, 1, 4, 4, 1, 64, 0.1, None, dt, None,
                                           None) == b200attn.ERR_UNSUPPORTED
        assert lib.b200_flash_attention_ex(16, 16, 16, 16, 1, 0, 4, 1, 128, 0.1, None, dt, None,
                                           None) == b200attn.OK  # nothing to do


def test_workspace_bytes():
    a = b200attn.AttnArgs()
    a.batch, a.heads, a.head_dim, a.target_len = 1, 32, 128, 4096
    n = b200attn.workspace_bytes(a)
    split = b200attn.SPLIT_WORKSPACE_BYTES
    assert n == 2 * 32 * 4096 * 128 * 2 + split
    a.k_rot_out = 256
    assert b200attn.workspace_bytes(a) == 32 * 4096 * 128 * 2 + split
    # the header constant matches the binding's
    hdr = open(os.path.join(ROOT, "include", "b200_attn.h")).read()
    assert f"B200_ATTN_SPLIT_WORKSPACE_BYTES {split}u" in hdr


@pytest.mark.parametrize("text,cond", [(3, []), (40, [(4, 6), (8, 8)]), (9, [(2, 2), (2, 2)])])
def test_block_causal_limits_match_the_reference_mask(text, cond):
    """b200_block_causal_limits == the leading-run lengths of build_block_causal_mask
    (src/attention_mask.rs:18-66) over the prefix of the joint layout."""
    slots = [False] * text
    p = 1
    for (h, w) in cond:
        slots[p:p + h * w // 4] = [True] * (h * w // 4)
        p += h * w // 4 + 1
    lay = ref.joint_layout(text, slots, cond, (2, 2))
    ids = lay["image_ids"]
    want = ref.block_causal_limits_from_mask(ref.block_causal_mask(ids, None, 1)[0, 0])
    assert want is not None
    assert np.array_equal(b200attn.block_causal_limits(ids), want)
    assert np.all(np.diff(want) >= 0)  # non-decreasing: the kernel relies on it


def test_tp_entry_points_reject_bad_arguments():
    lib = b200attn.lib()
    h = ctypes.c_void_p()
    uid = (ctypes.c_uint8 * b200attn.TP_ID_BYTES)()
    assert lib.b200_tp_unique_id(None) == b200attn.ERR_INVALID
    assert lib.b200_tp_init(None, uid, 1, 0, 0) == b200attn.ERR_INVALID
    assert lib.b200_tp_init(ctypes.byref(h), None, 1, 0, 0) == b200attn.ERR_INVALID
    assert lib.b200_tp_init(ctypes.byref(h), uid, 2, 2, 0) == b200attn.ERR_INVALID  # rank >= n
    assert lib.b200_tp_init(ctypes.byref(h), uid, 0, 0, 0) == b200attn.ERR_INVALID
    assert lib.b200_tp_init_from_nccl(ctypes.byref(h), None, 0) == b200attn.ERR_INVALID
    assert lib.b200_tp_out_proj_allreduce(None, None, 1, 0, None) == b200attn.ERR_INVALID
    assert lib.b200_tp_wait(None, None) == b200attn.ERR_INVALID
    assert lib.b200_tp_destroy(None) == b200attn.ERR_INVALID
    assert lib.b200_tp_rank(None) == b200attn.ERR_INVALID
    assert lib.b200_tp_size(None) == b200attn.ERR_INVALID


def test_tp_unique_id_is_fresh():
    """Group ids come from NCCL at run time (no link-time NCCL dependency); two calls give
    two groups."""
    try:
        a, b = b200attn.tp_unique_id(), b200attn.tp_unique_id()
    except b200attn.B200Error as e:
        pytest.skip(f"NCCL not loadable here: {e}")
    assert len(a) == b200attn.TP_ID_BYTES and a != b
