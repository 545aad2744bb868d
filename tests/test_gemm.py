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
