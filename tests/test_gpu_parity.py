"""Parity of the CUDA path (through the C ABI) with the CPU oracle.

Tolerances (bf16 output against the reference's f32 path):
relative L2 <= 5e-3 and max-abs <= 2e-2.  Small cases compare every element with the
oracle; the full-size configurations compare whole heads (every query row) with the C
oracle and check size-independent properties (softmax weights sum to one, linearity in
V)."""
import os

import numpy as np
import pytest

import b200attn
from oracle import reference as ref

pytestmark = pytest.mark.gpu

REL_L2 = 5e-3
MAX_ABS = 2e-2
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _torch():
    import torch
    return torch


def bf16(t):
    return t.to(_torch().bfloat16)


def f32np(t):
    return t.float().cpu().numpy()


def check(got, want, rel=REL_L2, mx=MAX_ABS):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert np.isfinite(got).all()
    r = ref.rel_l2(got, want)
    m = float(np.max(np.abs(got - want))) if got.size else 0.0
    assert r <= rel and m <= mx, f"rel_l2={r:.3e} max_abs={m:.3e}"
    return r, m


def make_case(B, T, H, P, seed, device, pv=None, layout_text=None):
    torch = _torch()
    g = torch.Generator().manual_seed(seed)
    q = bf16(torch.randn(B, T, H, 128, generator=g))
    k = bf16(torch.randn(B, T, H, 128, generator=g))
    v = bf16(torch.randn(B, T, H, 128, generator=g))
    pk = bf16(torch.randn(B, H, P, 128, generator=g)) if P else None
    pvv = bf16(torch.randn(B, H, P, 128, generator=g)) if P else None
    wq = (1 + 0.1 * torch.randn(128, generator=g)).float()
    wk = (1 + 0.1 * torch.randn(128, generator=g)).float()
    # target grid as close to square as T allows, behind a `text`-token prompt
    hgt = int(np.sqrt(T))
    while T % hgt:
        hgt -= 1
    text = P if layout_text is None else layout_text
    lay = ref.joint_layout(text, None, [], (hgt, T // hgt))
    pe = ref.embed_nd(lay["img_shapes"], lay["image_pad_mask"])[text:]
    desc = None
    if pv is not None:
        desc = np.array([(x, T) for x in pv], np.int32)
    dev = dict(q=q.to(device), k=k.to(device), v=v.to(device),
               pk=None if pk is None else pk.to(device), pv=None if pvv is None else pvv.to(device),
               wq=wq.to(device), wk=wk.to(device), pe=torch.from_numpy(pe).to(device),
               desc=None if desc is None else torch.from_numpy(desc).to(device))
    host = dict(q=f32np(q), k=f32np(k), v=f32np(v), pk=None if pk is None else f32np(pk),
                pv=None if pvv is None else f32np(pvv), wq=wq.numpy(), wk=wk.numpy(), pe=pe,
                desc=None if desc is None else [tuple(x) for x in desc])
    return dev, host


def run_gpu(d, **kw):
    return b200attn.attention_forward(d["q"], d["k"], d["v"], d["pk"], d["pv"], d["wq"], d["wk"],
                                      d["pe"], desc=d["desc"], **kw)


def run_oracle(h):
    prefix = None if h["pk"] is None else (h["pk"], h["pv"])
    return ref.attention_forward(h["q"], h["k"], h["v"], h["wq"], h["wk"], h["pe"], prefix, h["desc"])


# ------------------------------------------------------------------ prologue
def test_norm_rope_matches_oracle(cuda):
    torch = _torch()
    d, h = make_case(2, 300, 3, 0, 11, cuda)
    y = b200attn.norm_rope(d["q"], d["wq"], 1e-6, d["pe"])
    torch.cuda.synchronize()
    want = ref.apply_rope(np.transpose(ref.rms_norm(h["q"], h["wq"]), (0, 2, 1, 3)), h["pe"])
    # one bf16 rounding of the f32 result: <= 2^-8 relative per element
    assert np.max(np.abs(f32np(y) - want) / (np.abs(want) + 1e-3)) < 2 ** -8 + 1e-6
    check(f32np(y), want, rel=3e-3)


@pytest.mark.parametrize("B,T,H", [(1, 77, 40), (2, 33, 64), (1, 5, 33), (3, 17, 8)])
def test_norm_rope_head_counts(cuda, B, T, H):
    """Head counts past one warp's 32 rows per token (the kernel walks them 32 at a time)
    and below it; ragged token counts."""
    torch = _torch()
    d, h = make_case(B, T, H, 0, 4200 + T + H, cuda)
    y = b200attn.norm_rope(d["k"], d["wk"], 1e-6, d["pe"])
    torch.cuda.synchronize()
    want = ref.apply_rope(np.transpose(ref.rms_norm(h["k"], h["wk"]), (0, 2, 1, 3)), h["pe"])
    assert np.max(np.abs(f32np(y) - want) / (np.abs(want) + 1e-3)) < 2 ** -8 + 1e-6


# ------------------------------------------------------------------ plain attention
@pytest.mark.parametrize("B,H,sq,skv", [
    (1, 1, 128, 128), (1, 2, 256, 256), (2, 3, 1, 1), (1, 2, 37, 300), (2, 1, 300, 129),
    (1, 4, 500, 1000), (1, 1, 257, 2000),
])
def test_chunked_attention_matches_oracle(cuda, B, H, sq, skv):
    torch = _torch()
    g = torch.Generator().manual_seed(B * 7 + H * 13 + sq + skv)
    q = bf16(torch.randn(B, H, sq, 128, generator=g))
    k = bf16(torch.randn(B, H, skv, 128, generator=g))
    v = bf16(torch.randn(B, H, skv, 128, generator=g))
    out = b200attn.chunked_attention(q.to(cuda), k.to(cuda), v.to(cuda), 128 ** -0.5)
    torch.cuda.synchronize()
    want = ref.chunked_attention(f32np(q), f32np(k), f32np(v), 128 ** -0.5)
    check(f32np(out), want)


@pytest.mark.parametrize("B,H,sq,skv,lens", [
    (1, 2, 256, 256, None), (2, 3, 37, 300, None), (1, 4, 500, 1000, None),
    (2, 2, 300, 4608, [4608, 4581]),   # config-2-like key count, one row's tail padded
    (3, 1, 129, 200, [1, 128, 200]),
])
def test_flash_attention_bshd_matches_oracle(cuda, B, H, sq, skv, lens):
    """The flash_attn contract on token-major [B,S,H,D] tensors against the oracle's
    chunked_attention on the same values transposed to [B,H,S,D]."""
    torch = _torch()
    g = torch.Generator().manual_seed(B * 11 + H * 7 + sq + skv)
    q = bf16(torch.randn(B, sq, H, 128, generator=g))
    k = bf16(torch.randn(B, skv, H, 128, generator=g))
    v = bf16(torch.randn(B, skv, H, 128, generator=g))
    key_len = None if lens is None else torch.tensor(lens, dtype=torch.int32, device=cuda)
    out = b200attn.flash_attention(q.to(cuda), k.to(cuda), v.to(cuda), 128 ** -0.5,
                                   key_len=key_len)
    torch.cuda.synchronize()
    mask = None
    if lens is not None:
        mask = np.zeros((B, 1, 1, skv), bool)
        for b, n in enumerate(lens):
            mask[b, ..., :n] = True
    t = lambda x: np.transpose(f32np(x), (0, 2, 1, 3))
    want = ref.chunked_attention(t(q), t(k), t(v), 128 ** -0.5, mask)
    check(np.transpose(f32np(out), (0, 2, 1, 3)), want)


@pytest.mark.parametrize("B,H,sq,skv,lens", [
    (1, 2, 256, 256, None), (2, 3, 37, 300, None),
    (2, 2, 300, 4608, [4608, 4581]),
    (3, 1, 129, 200, [1, 128, 200]),
])
def test_flash_attention_f16_matches_oracle(cuda, B, H, sq, skv, lens):
    """The FA2 branch in the type the reference casts to (IEEE half, src/transformer.rs:
    244-251): f16 q/k/v in, f16 out, against the oracle on the same f16 values."""
    torch = _torch()
    g = torch.Generator().manual_seed(B * 13 + H * 5 + sq + skv)
    q = torch.randn(B, sq, H, 128, generator=g).half()
    k = torch.randn(B, skv, H, 128, generator=g).half()
    v = torch.randn(B, skv, H, 128, generator=g).half()
    key_len = None if lens is None else torch.tensor(lens, dtype=torch.int32, device=cuda)
    out = b200attn.flash_attention(q.to(cuda), k.to(cuda), v.to(cuda), 128 ** -0.5,
                                   key_len=key_len)
    torch.cuda.synchronize()
    assert out.dtype == torch.float16
    mask = None
    if lens is not None:
        mask = np.zeros((B, 1, 1, skv), bool)
        for b, n in enumerate(lens):
            mask[b, ..., :n] = True
    t = lambda x: np.transpose(f32np(x), (0, 2, 1, 3))
    want = ref.chunked_attention(t(q), t(k), t(v), 128 ** -0.5, mask)
    # f16 carries 3 more mantissa bits than bf16: the same bar, met with room to spare
    r, _ = check(np.transpose(f32np(out), (0, 2, 1, 3)), want)
    assert r < 1.5e-3
    # the bf16 entry point on the same values (rounded to bf16) agrees to bf16 precision
    out_bf = b200attn.flash_attention(bf16(q.float()).to(cuda), bf16(k.float()).to(cuda),
                                      bf16(v.float()).to(cuda), 128 ** -0.5, key_len=key_len)
    torch.cuda.synchronize()
    check(f32np(out_bf), f32np(out), rel=1e-2, mx=3e-2)


def test_flash_attention_rejects_other_dtypes(cuda):
    torch = _torch()
    q = torch.zeros(1, 16, 1, 128, device=cuda, dtype=torch.float32)
    with pytest.raises(b200attn.B200Error) as e:
        b200attn.flash_attention(q, q, q, 0.1, out=torch.empty(1, 16, 1, 128, device=cuda,
                                                                 dtype=torch.float16))
    assert e.value.status == b200attn.ERR_UNSUPPORTED


def test_chunked_attention_key_mask(cuda):
    torch = _torch()
    g = torch.Generator().manual_seed(5)
    B, H, sq, skv = 3, 2, 200, 400
    q = bf16(torch.randn(B, H, sq, 128, generator=g))
    k = bf16(torch.randn(B, H, skv, 128, generator=g))
    v = bf16(torch.randn(B, H, skv, 128, generator=g))
    mask = torch.zeros(B, 1, 1, skv, dtype=torch.bool)
    for b, n in enumerate([1, 129, 400]):
        mask[b, ..., :n] = True
    out = b200attn.chunked_attention(q.to(cuda), k.to(cuda), v.to(cuda), 128 ** -0.5, mask=mask.to(cuda))
    torch.cuda.synchronize()
    want = ref.chunked_attention(f32np(q), f32np(k), f32np(v), 128 ** -0.5, mask.numpy())
    check(f32np(out), want)
    bad = mask.clone()
    bad[0, ..., 5] = True  # hole -> not a leading run of keys
    with pytest.raises(b200attn.B200Error):
        b200attn.chunked_attention(q.to(cuda), k.to(cuda), v.to(cuda), 128 ** -0.5, mask=bad.to(cuda))


def test_no_valid_key_gives_nan_like_the_reference(cuda):
    """A batch row whose key length is 0: the reference's softmax over an all -inf row is
    NaN, and so is every output of that row; the other rows are unaffected.  Through both
    the [B,H,S,D] and the [B,S,H,D] entry points."""
    torch = _torch()
    g = torch.Generator().manual_seed(23)
    B, H, sq, skv = 3, 2, 70, 200
    q = bf16(torch.randn(B, H, sq, 128, generator=g))
    k = bf16(torch.randn(B, H, skv, 128, generator=g))
    v = bf16(torch.randn(B, H, skv, 128, generator=g))
    lens = [0, 57, 200]
    key_len = torch.tensor(lens, dtype=torch.int32, device=cuda)
    out = b200attn.chunked_attention(q.to(cuda), k.to(cuda), v.to(cuda), 128 ** -0.5,
                                     key_len=key_len)
    t = lambda x: x.transpose(1, 2).contiguous().to(cuda)
    out_fa = b200attn.flash_attention(t(q), t(k), t(v), 128 ** -0.5, key_len=key_len)
    torch.cuda.synchronize()
    mask = np.zeros((B, 1, 1, skv), bool)
    for b, n in enumerate(lens):
        mask[b, ..., :n] = True
    with np.errstate(invalid="ignore"):
        want = ref.chunked_attention(f32np(q), f32np(k), f32np(v), 128 ** -0.5, mask)
    got = f32np(out)
    got_fa = np.transpose(f32np(out_fa), (0, 2, 1, 3))
    for arr in (got, got_fa):
        assert np.isnan(arr[0]).all() and np.isnan(want[0]).all()
        check(arr[1:], want[1:])


def test_chunked_attention_scale_and_large_logits(cuda):
    """Logits far above 1 exercise the running-max rescale of O."""
    torch = _torch()
    g = torch.Generator().manual_seed(9)
    q = bf16(4 * torch.randn(1, 2, 256, 128, generator=g))
    k = bf16(4 * torch.randn(1, 2, 1024, 128, generator=g))
    v = bf16(torch.randn(1, 2, 1024, 128, generator=g))
    out = b200attn.chunked_attention(q.to(cuda), k.to(cuda), v.to(cuda), 0.25)
    torch.cuda.synchronize()
    want = ref.chunked_attention(f32np(q), f32np(k), f32np(v), 0.25)
    check(f32np(out), want)


# ------------------------------------------------------------------ the full span
def test_golden_fixture(cuda):
    torch = _torch()
    g = np.load(os.path.join(GOLDEN, "attn_small.npz"))

    def t(name):
        a = g[name]
        if a.dtype == np.uint16:
            return torch.from_numpy(a.astype(np.int16)).view(torch.bfloat16).to(cuda)
        return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)

    B, T, H, _ = g["q"].shape
    k_rot = torch.empty(B, H, T, 128, dtype=torch.bfloat16, device=cuda)
    v_out = torch.empty(B, H, T, 128, dtype=torch.bfloat16, device=cuda)
    out = b200attn.attention_forward(t("q"), t("k"), t("v"), t("prefix_k"), t("prefix_v"),
                                     t("norm_q_w"), t("norm_k_w"), t("pe"), desc=t("desc"),
                                     k_rot_out=k_rot, v_out=v_out)
    torch.cuda.synchronize()
    check(f32np(out), g["out"])
    check(f32np(k_rot), g["k_rot"], rel=3e-3)
    v_ref = np.transpose((g["v"].astype(np.uint32) << 16).view(np.float32), (0, 2, 1, 3))
    assert np.array_equal(f32np(v_out), v_ref)


@pytest.mark.parametrize("B,T,H,P,pv", [
    (1, 1024, 32, 256, None),         # config 1 (512^2): 1024 queries over 256 + 1024 keys
    (1, 200, 4, 300, [263]),          # ragged prefix (config 3 shape in miniature)
    (2, 130, 2, 0, None),             # no prefix cache
    (2, 77, 3, 129, [1, 129]),        # one valid prefix key; full prefix
    (1, 64, 2, 40, [0]),              # every prefix key padded
])
def test_attention_forward_matches_oracle(cuda, B, T, H, P, pv):
    torch = _torch()
    d, h = make_case(B, T, H, P, 1000 + T + P, cuda, pv=pv)
    out = run_gpu(d)
    torch.cuda.synchronize()
    want, _, _ = run_oracle(h)
    check(f32np(out), want)


def test_attention_forward_is_deterministic_and_status_clear(cuda):
    torch = _torch()
    d, _ = make_case(1, 1024, 8, 256, 77, cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    a = run_gpu(d, status=status)
    b = run_gpu(d, status=status)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert int(status.item()) == 0


def test_attention_forward_replays_in_a_cuda_graph(cuda):
    """b200_attn_fwd captured in a CUDA graph (as the benchmark replays a step) gives the
    eager call's output on every replay, with new inputs copied into the captured buffers
    (the tail split's counters reset themselves between replays)."""
    torch = _torch()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    H = (sms + 3 + 1) // 2  # T = 512: 2 query blocks per head, a last wave to split
    d, h = make_case(1, 512, H, 256, 91, cuda, pv=[200])
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = torch.empty(1, 512, H * 128, dtype=torch.bfloat16, device=cuda)
    args = b200attn.make_args(d["q"], d["k"], d["v"], d["pk"], d["pv"], d["wq"], d["wk"], d["pe"],
                              out, d["desc"])
    ws = torch.empty(b200attn.workspace_bytes(args), dtype=torch.uint8, device=cuda)
    eager = run_gpu(d, workspace=ws, status=status).clone()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        run_gpu(d, out=out, workspace=ws, status=status, stream=side)
    torch.cuda.current_stream().wait_stream(side)
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
    d2, h2 = make_case(1, 512, H, 256, 92, cuda, pv=[200])
    for name in ("q", "k", "v", "pk", "pv", "wq", "wk"):
        d[name].copy_(d2[name])
    graph.replay()
    torch.cuda.synchronize()
    check(f32np(out), run_oracle(h2)[0])
    assert int(status.item()) == 0


# ------------------------------------------------------------------ full sizes
def _bits(x):
    """bf16 bit patterns (uint16) of a float32 array holding bf16 values."""
    return (np.ascontiguousarray(x, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def _whole_heads_check(out, h, heads):
    """Every query row of the given heads against the C oracle (OpenMP, all host cores):
    norm -> RoPE -> [prefix ; keys] -> chunked_attention -> merge, f32."""
    from oracle import cpu as ocpu
    sel = lambda x: _bits(x[:, :, heads])
    pk = None if h["pk"] is None else _bits(h["pk"][:, heads])
    pv = None if h["pv"] is None else _bits(h["pv"][:, heads])
    prefix_valid = None if h["desc"] is None else np.array([d[0] for d in h["desc"]], np.int32)
    want = ocpu.attention_forward(sel(h["q"]), sel(h["k"]), sel(h["v"]), pk, pv, h["wq"], h["wk"],
                                  1e-6, h["pe"], prefix_valid, 128 ** -0.5)
    b, t = want.shape[:2]
    got = f32np(out).reshape(b, t, -1, 128)[:, :, heads].reshape(b, t, -1)
    return check(got, want)


@pytest.mark.parametrize("T,P,pv,heads", [
    (4096, 512, None, list(range(32))),       # config 2 (1024^2 T2I): every head
    (4096, 10624, [10587], list(range(32))),  # config 3 (edit, 37 padded keys): every head
    # config 4 (2048^2, all 32 heads on one GPU: 132 key tiles): the first and last heads
    # (the last items of the grid are the tail-split ones) and some in between
    (16384, 512, None, [0, 1, 9, 16, 23, 29, 30, 31]),
])
def test_full_size_configs(cuda, T, P, pv, heads):
    """Full-size configurations: whole heads (every query row) against the C oracle, plus
    size-independent properties."""
    torch = _torch()
    d, h = make_case(1, T, 32, P, 2000 + P, cuda, pv=pv, layout_text=512)
    out = run_gpu(d)
    torch.cuda.synchronize()
    _whole_heads_check(out, h, heads)
    # linearity in V (size independent): attn(2 v) == 2 attn(v) exactly in bf16
    d2 = dict(d)
    d2["v"] = d["v"] * 2
    d2["pv"] = d["pv"] * 2
    out2 = run_gpu(d2)
    torch.cuda.synchronize()
    assert torch.equal(out2, out * 2)
    # constant V rows -> every output equals that constant (weights sum to one)
    d3 = dict(d)
    d3["v"] = torch.full_like(d["v"], 0.75)
    d3["pv"] = torch.full_like(d["pv"], 0.75)
    out3 = run_gpu(d3)
    torch.cuda.synchronize()
    assert float((out3.float() - 0.75).abs().max()) < 4e-3


# ------------------------------------------------------------------ tail split
def _check_heads(out, h, heads):
    """Oracle on a subset of heads (heads are independent)."""
    sub = dict(h)
    for key in ("q", "k", "v"):
        sub[key] = h[key][:, :, heads]
    for key in ("pk", "pv"):
        sub[key] = None if h[key] is None else h[key][:, heads]
    want, _, _ = run_oracle(sub)
    b, t = want.shape[:2]
    got = f32np(out).reshape(b, t, -1, 128)[:, :, heads].reshape(b, t, -1)
    check(got, want)


@pytest.mark.parametrize("T,P,pv,extra", [
    (512, 512, None, 3),     # 2 query blocks per head; last wave of 3-4 items split 4 ways
    (256, 512, [0], 2),      # 2 key tiles cut into 3 pieces: one piece has no tile
    (512, 300, [263], 5),    # ragged prefix inside split pieces
])
def test_tail_split_matches_oracle(cuda, T, P, pv, extra):
    torch = _torch()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    nqb = (T + 255) // 256
    H = (sms + extra + nqb - 1) // nqb  # items = H * nqb lands just past a full wave
    d, h = make_case(1, T, H, P, 3000 + T + P + extra, cuda, pv=pv)
    ws = torch.empty(b200attn.SPLIT_WORKSPACE_BYTES, dtype=torch.uint8, device=cuda)
    q_rot, k_rot = b200attn.qk_norm_rope(d["q"], d["k"], d["wq"], d["wk"], 1e-6, d["pe"])
    out_split = b200attn.joint_attention(q_rot, k_rot, d["v"], d["pk"], d["pv"], desc=d["desc"],
                                         workspace=ws)
    out_again = b200attn.joint_attention(q_rot, k_rot, d["v"], d["pk"], d["pv"], desc=d["desc"],
                                         workspace=ws)
    out_plain = b200attn.joint_attention(q_rot, k_rot, d["v"], d["pk"], d["pv"], desc=d["desc"])
    out_fwd = run_gpu(d)  # b200_attn_fwd with its full workspace (split region included)
    torch.cuda.synchronize()
    assert torch.equal(out_split, out_again)  # arrival counters reset themselves
    assert torch.equal(out_fwd, out_split)
    check(f32np(out_split), f32np(out_plain), rel=2e-3, mx=1e-2)  # merge vs single pass
    _check_heads(out_split, h, [0, H - 3, H - 2, H - 1])  # the last items are the split ones


def test_prefix_fill_tail_split_rows_without_keys(cuda):
    """Causal prefix fill whose last partial wave is split by key tiles: a piece can hold
    rows that see none of its keys (rows 0..127 of a first query block in the piece of keys
    128..255).  Such rows contribute nothing to the merge; the output stays finite and
    matches the oracle."""
    torch = _torch()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    T, nqb = 512, 2
    H = (sms + 4 + nqb - 1) // nqb          # items = 2H lands 4 past a full wave: split 2
    lay = ref.joint_layout(T, None, [], (0, 0))
    limits = b200attn.block_causal_limits(lay["image_ids"][:T])
    pe = ref.embed_nd(lay["img_shapes"], lay["image_pad_mask"])[:T]
    g = torch.Generator().manual_seed(77)
    q, k, v = (bf16(torch.randn(1, T, H, 128, generator=g)) for _ in range(3))
    w = torch.ones(128)
    out = b200attn.attention_forward(q.to(cuda), k.to(cuda), v.to(cuda), None, None, w.to(cuda),
                                     w.to(cuda), torch.from_numpy(pe).to(cuda),
                                     row_limit=torch.from_numpy(limits).to(cuda))
    torch.cuda.synchronize()
    got = f32np(out).reshape(1, T, H, 128)
    assert np.isfinite(got).all()
    heads = [0, H - 2, H - 1]               # the last heads' items are the split ones
    mask = ref.block_causal_mask(lay["image_ids"][:T], None, 1)
    qh = ref.apply_rope(np.transpose(ref.rms_norm(f32np(q[:, :, heads]), w.numpy()), (0, 2, 1, 3)), pe)
    kh = ref.apply_rope(np.transpose(ref.rms_norm(f32np(k[:, :, heads]), w.numpy()), (0, 2, 1, 3)), pe)
    vh = np.transpose(f32np(v[:, :, heads]), (0, 2, 1, 3))
    want = np.transpose(ref.chunked_attention(qh, kh, vh, 128 ** -0.5, mask), (0, 2, 1, 3))
    check(got[:, :, heads].reshape(1, T, -1), want.reshape(1, T, -1))


# ------------------------------------------------------------------ prefix fill (block-causal)
@pytest.mark.parametrize("cond,pad", [([], 0), ([(8, 16), (16, 16)], 7), ([(16, 16)], 0)])
def test_prefix_fill_block_causal_matches_oracle(cuda, cond, pad):
    """The prefix-only pass (src/transformer.rs:674-707): the prefix attends to itself under
    the block-causal mask times key_valid; its post-RoPE K and V fill the cache."""
    torch = _torch()
    slots, lead = [], 10
    for (hh, ww) in cond:
        slots += [False] * lead + [True] * (hh * ww // 4)
    slots += [False] * 150
    lay = ref.joint_layout(len(slots), slots, cond, (2, 2))
    P, H = lay["prefix_len"], 4
    ids = lay["image_ids"][:P]
    limits = b200attn.block_causal_limits(ids)
    pe = ref.embed_nd(lay["img_shapes"], lay["image_pad_mask"])[:P]
    g = torch.Generator().manual_seed(P + pad)
    q, k, v = (bf16(torch.randn(1, P, H, 128, generator=g)) for _ in range(3))
    w = torch.ones(128)
    pv = P - pad  # padded prompt tokens sit at the end of the prompt
    desc = torch.tensor([[0, pv]], dtype=torch.int32, device=cuda) if pad else None
    k_rot = torch.empty(1, H, P, 128, dtype=torch.bfloat16, device=cuda)
    v_out = torch.empty(1, H, P, 128, dtype=torch.bfloat16, device=cuda)
    out = b200attn.attention_forward(q.to(cuda), k.to(cuda), v.to(cuda), None, None, w.to(cuda),
                                     w.to(cuda), torch.from_numpy(pe).to(cuda), desc=desc,
                                     row_limit=torch.from_numpy(limits).to(cuda),
                                     k_rot_out=k_rot, v_out=v_out)
    torch.cuda.synchronize()
    kv = np.ones((1, P), np.uint8)
    kv[0, pv:] = 0
    mask = ref.block_causal_mask(ids, kv if pad else None, 1)
    qh = ref.apply_rope(np.transpose(ref.rms_norm(f32np(q), w.numpy()), (0, 2, 1, 3)), pe)
    kh = ref.apply_rope(np.transpose(ref.rms_norm(f32np(k), w.numpy()), (0, 2, 1, 3)), pe)
    vh = np.transpose(f32np(v), (0, 2, 1, 3))
    want = np.transpose(ref.chunked_attention(qh, kh, vh, 128 ** -0.5, mask), (0, 2, 1, 3))
    check(f32np(out), want.reshape(1, P, H * 128))
    check(f32np(k_rot), kh, rel=3e-3)
    assert np.array_equal(f32np(v_out), vh)
