"""The tcgen05 GEMM (b200_gemm): C = A·Bᵀ against a float32 torch reference, with ragged
M and K, a column slice of a larger weight as B (the head-sharded to_out), bf16 stores and
f32 red-add accumulation; argument checks without a GPU."""
import pytest
import torch

import b200attn


def _rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm())


def test_gemm_rejects_bad_arguments():
    L = b200attn.lib()
    args = lambda m=128, n=256, k=64, lda=64, ldb=64, ldc=256, mode=0, a=16, c=16: (
        a, lda, 16, ldb, c, ldc, m, n, k, mode, None, None)
    assert L.b200_gemm(*args(n=100)) == b200attn.ERR_INVALID        # N % 32
    assert L.b200_gemm(*args(k=60, lda=64, ldb=64)) == b200attn.ERR_INVALID  # K % 8
    assert L.b200_gemm(*args(lda=32)) == b200attn.ERR_INVALID        # lda < K
    assert L.b200_gemm(*args(ldc=100)) == b200attn.ERR_INVALID       # ldc < N
    assert L.b200_gemm(*args(mode=7)) == b200attn.ERR_INVALID
    assert L.b200_gemm(*args(a=8)) == b200attn.ERR_INVALID           # misaligned A
    assert L.b200_gemm(*args(m=0)) == b200attn.OK


def test_owner_steps_reject_bad_arguments():
    """The owners' reduce steps validate every argument before touching memory (the
    addresses below are never dereferenced); rows = 0 with valid arguments is a no-op."""
    import ctypes
    L = b200attn.lib()
    INV, OK = b200attn.ERR_INVALID, b200attn.OK
    dst = (ctypes.c_void_p * 2)(4096, 8192)

    def rr(slots=16, n_src=2, slot_rows=8, rows=0, cols=64, ld=64, x=16, ldx=64, gate=16,
           scale=16, rpm=1 << 62, ms=0, eps=1e-6, n_dst=2, row0=0, dst_ld=64):
        return L.b200_reduce_residual_adaln_gather(slots, n_src, slot_rows, rows, cols, ld, x,
                                                   ldx, gate, scale, rpm, ms, eps, dst, n_dst,
                                                   row0, dst_ld, None)
    assert rr() == OK
    assert rr(cols=60, ld=64, ldx=64, dst_ld=64) == INV       # cols % 8
    assert rr(cols=8200, ld=8200, ldx=8200, dst_ld=8200) == INV  # > 8192 columns
    assert rr(slot_rows=4, rows=8) == INV                     # rows beyond a slot
    assert rr(ldx=62) == INV                                  # f32 rows not 16-byte vectors
    assert rr(x=8) == INV                                     # misaligned residual rows
    assert rr(gate=None) == INV
    assert rr(ms=6) == INV                                    # modulation stride % 4
    assert rr(eps=-1.0) == INV
    assert rr(n_dst=9) == INV                                 # more owners than supported
    assert rr(dst_ld=32) == INV                               # dst rows narrower than cols

    def nv(mc_part=16, part_ld=64, mc_out=32, out_ld=64, row0=0, rows=0, cols=64, x=None,
           ldx=0, gate=None, scale=None, rpm=1 << 62, ms=0, eps=1e-6):
        return L.b200_reduce_nvls(mc_part, part_ld, mc_out, out_ld, row0, rows, cols, x, ldx,
                                  gate, scale, rpm, ms, eps, None)
    assert nv() == OK                                          # plain sum, no rows
    assert nv(x=16, ldx=64, gate=16, scale=16) == OK          # with the residual step
    assert nv(cols=60, part_ld=64, out_ld=64) == INV
    assert nv(mc_part=8) == INV                                # misaligned multicast address
    assert nv(part_ld=32) == INV
    assert nv(row0=-1) == INV
    assert nv(x=16, ldx=62, gate=16, scale=16) == INV
    assert nv(x=16, ldx=64, gate=None, scale=16) == INV
    assert nv(x=16, ldx=64, gate=16, scale=16, eps=-1.0) == INV


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (300, 512, 200), (1000, 96, 520),
                                   (4096, 4096, 4096), (16384, 4096, 512), (77, 12288, 4096)])
def test_gemm_bf16_matches_reference(cuda, m, n, k):
    g = torch.Generator(device=cuda).manual_seed(m + n + k)
    a = torch.randn(m, k, generator=g, device=cuda).bfloat16()
    b = torch.randn(n, k, generator=g, device=cuda).bfloat16()
    st = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = b200attn.gemm(a, b, status=st)
    want = a.float() @ b.float().t()
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    assert _rel(out.float(), want) < 4e-3        # bf16 rounding of the output
    assert (out.float() - want).abs().max() < 2e-2 * want.abs().max()


@pytest.mark.gpu
def test_gemm_column_slice_and_red_add(cuda):
    """B = columns [h0*128, h1*128) of a [hidden, H*128] weight (row stride H*128): the
    head-sharded to_out partial; two red-add calls accumulate into an f32 sub-view."""
    g = torch.Generator(device=cuda).manual_seed(5)
    T, H, hidden, h0, h1 = 640, 8, 1024, 2, 5
    attn = torch.randn(T, (h1 - h0) * 128, generator=g, device=cuda).bfloat16()
    w_out = (0.02 * torch.randn(hidden, H * 128, generator=g, device=cuda)).bfloat16()
    w_cols = w_out[:, h0 * 128:h1 * 128]
    assert w_cols.stride(0) == H * 128
    big = torch.zeros(T, hidden + 64, dtype=torch.float32, device=cuda)
    c = big[:, :hidden]
    for _ in range(2):
        b200attn.gemm(attn, w_cols, out=c, mode=b200attn.GEMM_RED_F32)
    want = 2 * (attn.float() @ w_cols.float().t())
    torch.cuda.synchronize()
    assert _rel(c, want) < 1e-5
    assert big[:, hidden:].abs().max() == 0      # nothing written past N


@pytest.mark.gpu
@pytest.mark.parametrize("world,T", [(2, 1000), (4, 640), (3, 257)])
def test_scatter_gather_emulated_ranks(cuda, world, T):
    """The reduce-scatter / all-gather pair of the head-sharded to_out, with `world` ranks
    emulated on one GPU (each rank's owner buffer is a local tensor): every rank's output
    equals the sum of all ranks' partial products."""
    g = torch.Generator(device=cuda).manual_seed(world + T)
    H, hidden = 2 * world, 512
    attn = torch.randn(T, H * 128, generator=g, device=cuda).bfloat16()
    w_out = (0.02 * torch.randn(hidden, H * 128, generator=g, device=cuda)).bfloat16()
    rows_per = -(-T // world)
    slots = [torch.zeros(world * rows_per, hidden, dtype=torch.bfloat16, device=cuda) for _ in range(world)]
    outs = [torch.zeros(world * rows_per, hidden, dtype=torch.bfloat16, device=cuda) for _ in range(world)]
    hs = H // world
    for r in range(world):   # each rank's GEMM: its heads' columns, scattered to the owners
        b200attn.gemm_scatter(attn[:, r * hs * 128:(r + 1) * hs * 128].contiguous(),
                              w_out[:, r * hs * 128:(r + 1) * hs * 128],
                              [t.data_ptr() for t in slots], r, rows_per, hidden)
    for q in range(world):   # each owner sums its slots and broadcasts its rows
        mine = max(0, min(rows_per, T - q * rows_per))
        b200attn.reduce_gather(slots[q], world, rows_per, mine, hidden, hidden,
                               [t.data_ptr() for t in outs], q * rows_per, hidden)
    torch.cuda.synchronize()
    want = attn.float() @ w_out.float().t()
    for q in range(world):
        assert _rel(outs[q][:T].float(), want) < 5e-3
        assert torch.equal(outs[q], outs[0])   # identical on every rank


@pytest.mark.gpu
@pytest.mark.parametrize("world,T,hidden,per_mod", [(2, 1000, 512, None), (4, 640, 3072, 160),
                                                    (3, 257, 2048, 100)])
def test_scatter_residual_adaln_emulated_ranks(cuda, world, T, hidden, per_mod):
    """The head-sharded to_out with the gated residual and the next modulated LayerNorm
    fused into the owners' step (src/transformer.rs:411-418), `world` ranks emulated on one
    GPU: each owner's rows of x become x + tanh(gate) * attn_out in place, and every rank
    receives LN(x) * (1 + scale) for all rows.  per_mod = rows sharing one modulation row
    (one per batch item); None = one row for all tokens."""
    g = torch.Generator(device=cuda).manual_seed(world * 7 + T)
    H = 2 * world
    attn = torch.randn(T, H * 128, generator=g, device=cuda).bfloat16()
    w_out = (0.02 * torch.randn(hidden, H * 128, generator=g, device=cuda)).bfloat16()
    x = torch.randn(T, hidden, generator=g, device=cuda)
    n_mod = 1 if per_mod is None else -(-T // per_mod)
    gate = torch.randn(n_mod, hidden, generator=g, device=cuda)
    scale = 0.5 * torch.randn(n_mod, hidden, generator=g, device=cuda)
    rows_per = -(-T // world)
    slots = [torch.zeros(world * rows_per, hidden, dtype=torch.bfloat16, device=cuda) for _ in range(world)]
    outs = [torch.zeros(world * rows_per, hidden, dtype=torch.bfloat16, device=cuda) for _ in range(world)]
    x_own = [x[q * rows_per:(q + 1) * rows_per].clone() for q in range(world)]
    hs = H // world
    for r in range(world):
        b200attn.gemm_scatter(attn[:, r * hs * 128:(r + 1) * hs * 128].contiguous(),
                              w_out[:, r * hs * 128:(r + 1) * hs * 128],
                              [t.data_ptr() for t in slots], r, rows_per, hidden)
    for q in range(world):
        mine = max(0, min(rows_per, T - q * rows_per))
        b200attn.reduce_residual_adaln_gather(
            slots[q], world, rows_per, mine, hidden, hidden, x_own[q], gate, scale,
            [t.data_ptr() for t in outs], q * rows_per, hidden, rows_per_mod=per_mod,
            mod_stride=hidden if per_mod else 0)
    torch.cuda.synchronize()
    m = torch.zeros(T, dtype=torch.long, device=cuda) if per_mod is None else \
        torch.arange(T, device=cuda) // per_mod
    x_want = x + torch.tanh(gate[m]) * (attn.float() @ w_out.float().t())
    y_want = torch.nn.functional.layer_norm(x_want, (hidden,), eps=1e-6) * (1 + scale[m])
    assert _rel(torch.cat(x_own)[:T], x_want) < 2e-3   # bf16 partials summed in f32
    for q in range(world):
        assert _rel(outs[q][:T].float(), y_want) < 6e-3
        assert torch.equal(outs[q], outs[0])


@pytest.mark.gpu
@pytest.mark.parametrize("B,T,H,C", [(1, 256, 2, 256), (3, 200, 4, 512), (2, 4096, 32, 4096)])
def test_qkv_norm_rope_gemm_matches_unfused(cuda, B, T, H, C):
    """The fused Q/K/V projection (RMSNorm + RoPE in the epilogue) against the float32
    reference of the same span, and the unfused path (bf16 GEMMs + b200_qk_norm_rope)."""
    import numpy as np
    from oracle import reference as ref
    g = torch.Generator(device=cuda).manual_seed(B * T + H)
    x = torch.randn(B * T, C, generator=g, device=cuda).bfloat16()
    w = (torch.randn(3 * H * 128, C, generator=g, device=cuda) * C ** -0.5).bfloat16()
    nq = 1 + 0.1 * torch.randn(128, generator=g, device=cuda)
    nk = 1 + 0.1 * torch.randn(128, generator=g, device=cuda)
    pes = []
    for b in range(B):   # a different text length per batch row: different frame position
        lay = ref.joint_layout(17 + 5 * b, None, [], (T // 8, 8) if T % 8 == 0 else (T, 1))
        pes.append(ref.embed_nd(lay["img_shapes"], lay["image_pad_mask"])[17 + 5 * b:])
    pe = torch.from_numpy(np.stack(pes)).to(cuda)
    st = torch.zeros(1, dtype=torch.int32, device=cuda)
    qr, kr, v = b200attn.qkv_norm_rope_gemm(x, w, B, T, H, nq, nk, pe, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    # float32 reference of to_q/to_k/to_v -> norm -> RoPE
    y = (x.float() @ w.float().t()).view(B, T, 3, H, 128)
    def norm_rope(t, wn):
        t = t / torch.sqrt((t * t).mean(-1, keepdim=True) + 1e-6) * wn
        c, s_ = pe[:, :, None, 0::2], pe[:, :, None, 1::2]
        o = torch.empty_like(t)
        o[..., 0::2] = t[..., 0::2] * c - t[..., 1::2] * s_
        o[..., 1::2] = t[..., 0::2] * s_ + t[..., 1::2] * c
        return o.transpose(1, 2)
    want_q, want_k, want_v = norm_rope(y[:, :, 0], nq), norm_rope(y[:, :, 1], nk), y[:, :, 2]
    assert _rel(qr.float(), want_q) < 5e-3 and _rel(kr.float(), want_k) < 5e-3
    assert _rel(v.float(), want_v) < 5e-3
    # the unfused path on the same inputs (bf16 rounding of the raw projections in between)
    q0 = (x @ w[:H * 128].t()).view(B, T, H, 128)
    k0 = (x @ w[H * 128:2 * H * 128].t()).view(B, T, H, 128)
    for b in range(B):
        uq, uk = b200attn.qk_norm_rope(q0[b:b + 1], k0[b:b + 1], nq, nk, 1e-6, pe[b])
        assert _rel(qr[b:b + 1].float(), uq.float()) < 5e-3
        assert _rel(kr[b:b + 1].float(), uk.float()) < 5e-3
