"""The denoising loop around the attention path (b200attn.mmdit) against the float32 oracle
(oracle/mmdit_ref.py).

CPU: the scheduler known answers of the reference's own tests (src/scheduler.rs:159-187),
the product's scheduler / timestep embedding against the oracle's, and the oracle's cached
step against its uncached full-sequence pass.  GPU: the elementwise block kernels against
torch float32, the batched prefix fill and cached step against the oracle per sequence, and
20-step end-to-end latents with true CFG (rel L2 <= 2e-2, the end-to-end bound)."""
import numpy as np
import pytest
import torch

from b200attn import mmdit
from oracle import mmdit_ref as M

TINY = mmdit.MMDiTConfig(layers=2, heads=2, text_dim=256)
GRID = (16, 16)
# std 0.1 makes the attention branch carry most of the output at this width (about 70 % of
# the velocity changes when it is zeroed), so the end-to-end check is sensitive to it.
STD = 0.1


def rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm())


# ----------------------------------------------------------------------------- CPU
@pytest.mark.parametrize("seq_len", [64, 1024, 4096])
def test_schedule_endpoints_kat(seq_len):
    """src/scheduler.rs:159-178: first sigma 1, last sigma shift_terminal, decreasing."""
    for s in (M.sigmas(20, seq_len), mmdit.flow_match_sigmas(20, seq_len)):
        assert len(s) == 20
        assert abs(s[0] - 1.0) < 1e-5
        assert abs(s[-1] - 0.02) < 1e-4
        assert np.all(np.diff(s) < 0)


def test_higher_resolution_shifts_more_kat():
    """src/scheduler.rs:180-187."""
    for f in (M.sigmas, mmdit.flow_match_sigmas):
        assert f(20, 4096)[10] > f(20, 256)[10]


@pytest.mark.parametrize("steps,seq_len", [(20, 4096), (20, 256), (8, 1024), (2, 4096), (50, 16384)])
def test_product_schedule_matches_oracle(steps, seq_len):
    a, b = mmdit.flow_match_sigmas(steps, seq_len), M.sigmas(steps, seq_len)
    np.testing.assert_allclose(a, b, rtol=0, atol=2e-7)
    dts = [mmdit.euler_dt(a, i) for i in range(steps)]
    assert abs(sum(dts) + 1.0) < 1e-6   # the Euler steps integrate t from 1 to 0


def test_single_step_schedule_is_undefined_like_the_reference():
    """With one step the stretch divides 0 by 0 (src/scheduler.rs:85-91: last sigma 1): the
    reference yields NaN, and so do both restatements."""
    assert np.isnan(M.sigmas(1, 4096)).all() and np.isnan(mmdit.flow_match_sigmas(1, 4096)).all()


def test_timestep_embedding():
    z = mmdit.timestep_embedding(0.0)
    assert np.array_equal(z, np.concatenate([np.ones(128), np.zeros(128)]).astype(np.float32))
    for t in (0.02, 0.37, 1.0):
        np.testing.assert_allclose(mmdit.timestep_embedding(t), M.timestep_embedding(t).numpy(),
                                   atol=1e-4)


def test_weights_are_seeded_and_named():
    w1 = mmdit.random_weights(TINY, 3)
    w2 = mmdit.random_weights(TINY, 3)
    assert list(w1) == list(mmdit.weight_shapes(TINY))
    assert all(torch.equal(w1[k], w2[k]) for k in w1)
    assert sum(t.numel() for t in w1.values()) == TINY.params()
    full = mmdit.MMDiTConfig()
    assert 7.0e9 < full.params() < 7.2e9   # 7.1 B parameters: hidden 4096, MLP 3x


def test_oracle_cached_step_equals_uncached_pass():
    """The prefix cache reproduces the full joint pass (src/transformer.rs:8-13): with a
    float32 cache the cached step equals the uncached forward over [text ; target] with the
    block-causal mask and per-token modulation; the bf16 cache (KV_CACHE_DTYPE) stays close."""
    R = M.Reference(mmdit.random_weights(TINY, 0, std=STD), TINY.layers, TINY.heads)
    g = torch.Generator().manual_seed(1)
    emb, lat = torch.randn(40, 256, generator=g), torch.randn(256, 64, generator=g)
    full = R.forward_uncached(lat, 0.7, emb, GRID)
    cached = R.forward_cached(lat, 0.7, R.prefix_kv(emb, GRID, cache_bf16=False), 40, GRID)
    assert rel(cached, full) < 1e-5
    cached16 = R.forward_cached(lat, 0.7, R.prefix_kv(emb, GRID), 40, GRID)
    assert rel(cached16, full) < 1e-2


# ----------------------------------------------------------------------------- GPU
def _embs(lengths, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(n, TINY.text_dim, generator=g).to(torch.bfloat16) for n in lengths]


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols,rows_per_mod", [(64, 256, 64), (96, 4096, 32), (40, 8192, 40),
                                                    (33, 1000, 11), (1, 4, 1)])
def test_residual_adaln_matches_torch(cuda, rows, cols, rows_per_mod):
    import b200attn
    g = torch.Generator().manual_seed(rows + cols)
    n_mod = (rows + rows_per_mod - 1) // rows_per_mod
    x = torch.randn(rows, cols, generator=g) * 3 + 0.5
    y = torch.randn(rows, cols, generator=g).to(torch.bfloat16)
    mod = torch.randn(n_mod, 4 * cols, generator=g)
    gate, scale = mod[:, :cols], mod[:, cols:2 * cols]
    idx = torch.arange(rows) // rows_per_mod
    want_x = x + torch.tanh(gate[idx]) * y.float()
    ln = (want_x - want_x.mean(-1, keepdim=True)) / torch.sqrt(want_x.var(-1, unbiased=False, keepdim=True) + 1e-6)
    want = ln * (1 + scale[idx])
    xd, md = x.to(cuda), mod.to(cuda)
    out = torch.empty(rows, cols, dtype=torch.bfloat16, device=cuda)
    b200attn.residual_adaln(xd, y.to(cuda), md[:, :cols], md[:, cols:2 * cols], out, rows_per_mod)
    torch.cuda.synchronize()
    assert rel(xd.cpu(), want_x) < 1e-6
    assert (out.float().cpu() - want).abs().max() <= 2e-2 * (1 + want.abs().max())
    assert rel(out.float().cpu(), want) < 5e-3
    # norm only (no residual) and residual only (no norm)
    x2 = x.to(cuda)
    b200attn.residual_adaln(x2, None, None, md[:, cols:2 * cols], out, rows_per_mod)
    ln0 = (x - x.mean(-1, keepdim=True)) / torch.sqrt(x.var(-1, unbiased=False, keepdim=True) + 1e-6)
    assert rel(out.float().cpu(), ln0 * (1 + scale[idx])) < 5e-3
    assert torch.equal(x2.cpu(), x)
    b200attn.residual_adaln(x2, y.to(cuda), md[:, :cols], None, None, rows_per_mod)
    assert rel(x2.cpu(), want_x) < 1e-6


@pytest.mark.gpu
@pytest.mark.parametrize("rows,ffn", [(7, 8), (300, 768), (2048, 12288)])
def test_swiglu_matches_torch(cuda, rows, ffn):
    import b200attn
    g = torch.Generator().manual_seed(ffn)
    gp = (torch.randn(rows, 2 * ffn, generator=g) * 4).to(torch.bfloat16)
    h = b200attn.swiglu(gp.to(cuda)).float().cpu()
    gf = gp.float()
    want = torch.nn.functional.silu(gf[:, :ffn]) * gf[:, ffn:]
    assert (h - want).abs().max() <= 1e-2 * (1 + want.abs().max())
    assert rel(h, want) < 5e-3


def test_block_ops_reject_bad_arguments():
    import b200attn
    L = b200attn.lib()
    assert L.b200_residual_adaln(None, None, None, None, None, 4, 256, 4, 0, 1e-6, None) == b200attn.ERR_INVALID
    assert L.b200_residual_adaln(16, None, None, 16, 16, 4, 254, 4, 0, 1e-6, None) == b200attn.ERR_INVALID
    assert L.b200_residual_adaln(16, None, None, 16, 16, 4, 16384, 4, 0, 1e-6, None) == b200attn.ERR_INVALID
    assert L.b200_residual_adaln(16, None, None, 16, 16, 0, 256, 4, 0, 1e-6, None) == b200attn.OK
    assert L.b200_swiglu(16, 16, 4, 12, None) == b200attn.ERR_INVALID
    assert L.b200_swiglu(None, 16, 4, 16, None) == b200attn.ERR_INVALID
    assert L.b200_swiglu(16, 16, 0, 16, None) == b200attn.OK


@pytest.fixture(scope="module")
def tiny(request):
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    w = mmdit.random_weights(TINY, 0, std=STD)
    return w, mmdit.MMDiT(TINY, w, device="cuda:0", mlp_chunk_rows=300), \
        M.Reference(w, TINY.layers, TINY.heads)


@pytest.mark.gpu
def test_prefix_fill_matches_oracle(tiny):
    """One batched prefix pass over ragged prompts == the oracle's prefix_kv per prompt."""
    _, model, R = tiny
    lengths = [40, 72, 1, 57]
    embs = _embs(lengths, 5)
    cache = model.prefix_fill(embs)
    torch.cuda.synchronize()
    for b, n in enumerate(lengths):
        want = R.prefix_kv(embs[b].float(), GRID)
        for i in range(TINY.layers):
            k = cache.k[i][b, :, :n].float().cpu()
            v = cache.v[i][b, :, :n].float().cpu()
            assert rel(k, want[i][0]) < 1.5e-2, (b, i)   # bf16 GEMM operands: ~7e-3
            assert rel(v, want[i][1]) < 1.5e-2, (b, i)
            # rows past the prompt hold the padding tokens' K/V: finite, and masked by the
            # sequence's descriptor in every later step
            assert torch.isfinite(cache.k[i][b].float()).all() and torch.isfinite(cache.v[i][b].float()).all()


@pytest.mark.gpu
def test_cached_step_matches_oracle(tiny):
    """One cached step of a batch of ragged prompts == the oracle per sequence."""
    _, model, R = tiny
    lengths = [40, 72, 57]
    embs = _embs(lengths, 6)
    g = torch.Generator().manual_seed(9)
    lat = torch.randn(len(lengths), 256, 64, generator=g)
    cache = model.prefix_fill(embs)
    pe = model.target_pe(lengths, GRID)
    desc = mmdit.cached_desc(cache, 256, model.device)
    got = model.step(lat.to("cuda:0"), 0.55, cache, pe, desc).cpu()
    for b, n in enumerate(lengths):
        want = R.forward_cached(lat[b], 0.55, R.prefix_kv(embs[b].float(), GRID), n, GRID)
        assert rel(got[b], want) < 1.5e-2, b   # bf16 GEMM operands: ~8e-3
        assert (got[b] - want).abs().max() < 5e-2 * (1 + want.abs().max())


@pytest.mark.gpu
def test_host_offloaded_cache_gives_the_same_step(tiny):
    """set_kv_cache_offload: with the prefix cache in pinned host memory, streamed back a
    layer ahead of the attention, the cached step is bit-identical to the device cache's."""
    _, model, _ = tiny
    lengths = [33, 64]
    embs = _embs(lengths, 8)
    g = torch.Generator().manual_seed(12)
    lat = torch.randn(len(lengths), 256, 64, generator=g).to("cuda:0")
    cache = model.prefix_fill(embs)
    pe = model.target_pe(lengths, GRID)
    desc = mmdit.cached_desc(cache, 256, model.device)
    on_device = model.step(lat, 0.4, cache, pe, desc).clone()
    host = mmdit.PrefixCache(k=[t.clone() for t in cache.k], v=[t.clone() for t in cache.v],
                             lengths=list(cache.lengths)).offload()
    assert host.on_host and not cache.on_host
    slots = None
    for _ in range(2):  # the model's staging slots are reused across calls
        streamed = model.step(lat, 0.4, host, pe, desc)
        torch.cuda.synchronize()
        assert torch.equal(streamed, on_device)
        now = [t.data_ptr() for pair in model._staging("in", host.k[0].shape) for t in pair]
        assert slots is None or now == slots
        slots = now


@pytest.mark.gpu
def test_prefix_fill_offload_streams_each_layer_to_host():
    """prefix_fill(offload=True): each layer's K/V leaves the GPU as it is computed (two
    device staging slots), so the fill's peak device memory grows by a small part of the
    cache instead of the whole cache; the host cache equals the device-filled one bit for
    bit, and the offloaded fill then drives the same cached step."""
    cfg = mmdit.MMDiTConfig(layers=16, heads=2, text_dim=256)
    model = mmdit.MMDiT(cfg, mmdit.random_weights(cfg, 3, std=STD), device="cuda:0")
    lengths = [1500, 1100]
    embs = _embs(lengths, 21)
    dev_cache = model.prefix_fill(embs)          # also sizes the model's work buffers
    torch.cuda.synchronize()
    cache_bytes = sum(t.numel() * 2 for t in dev_cache.k + dev_cache.v)

    def peak_growth(fn):
        torch.cuda.synchronize()
        base = torch.cuda.memory_allocated()
        torch.cuda.reset_peak_memory_stats()
        out = fn()
        torch.cuda.synchronize()
        return out, torch.cuda.max_memory_allocated() - base

    again, grow_dev = peak_growth(lambda: model.prefix_fill(embs))
    host = model.prefix_fill(embs, offload=True)   # sizes the two staging slots
    host_again, grow_off = peak_growth(lambda: model.prefix_fill(embs, offload=True))
    assert host.on_host and all(t.is_pinned() for t in host.k + host.v)
    assert grow_dev >= cache_bytes
    assert grow_off <= cache_bytes // 4, (grow_off, cache_bytes)
    for i in range(cfg.layers):
        assert torch.equal(host.k[i], dev_cache.k[i].cpu()) and torch.equal(host.v[i], dev_cache.v[i].cpu())
        assert torch.equal(host_again.k[i], host.k[i])   # staging slots reused across fills
    del again
    g = torch.Generator().manual_seed(22)
    lat = torch.randn(len(lengths), 256, 64, generator=g).to("cuda:0")
    pe = model.target_pe(lengths, GRID)
    desc = mmdit.cached_desc(dev_cache, 256, model.device)
    want = model.step(lat, 0.3, dev_cache, pe, desc).clone()
    got = model.step(lat, 0.3, host, pe, desc)
    torch.cuda.synchronize()
    assert torch.equal(got, want)


@pytest.mark.gpu
def test_denoise_20_steps_with_cfg_matches_oracle(tiny):
    """End-to-end: 2 prompts x {pos, neg}, 20 FlowMatch Euler steps, true CFG 2.5 —
    final latents within rel L2 2e-2 of the float32 oracle.  (bf16 GEMM operands alone put
    this model about 1e-2 from float32; zeroing the attention moves the latents by ~40 %.)"""
    _, model, R = tiny
    pos = _embs([40, 72], 11)
    neg = _embs([33, 50], 12)
    g = torch.Generator().manual_seed(13)
    noise = mmdit.pack_latents(torch.randn(2, 64, 1, *GRID, generator=g))
    got = mmdit.denoise(model, pos, neg, GRID, 20, 2.5, noise).cpu()
    want = R.denoise(pos, neg, GRID, 20, 2.5, noise)
    for p in range(2):
        assert rel(got[p], want[p]) <= 2e-2, p
    assert rel(got, noise) > 0.1   # the loop moved the latents


@pytest.mark.gpu
def test_batch_rows_are_independent(tiny):
    """A sequence's velocity does not depend on the other sequences of its batch."""
    _, model, _ = tiny
    lengths = [40, 72]
    embs = _embs(lengths, 21)
    g = torch.Generator().manual_seed(22)
    lat = torch.randn(2, 256, 64, generator=g).to("cuda:0")
    cache = model.prefix_fill(embs)
    both = model.step(lat, 0.3, cache, model.target_pe(lengths, GRID),
                      mmdit.cached_desc(cache, 256, model.device)).cpu()
    one = model.prefix_fill(embs[1:])
    alone = model.step(lat[1:], 0.3, one, model.target_pe(lengths[1:], GRID),
                       mmdit.cached_desc(one, 256, model.device)).cpu()
    assert rel(both[1:], alone) < 5e-3


@pytest.mark.gpu
def test_fused_qkv_step_matches_unfused(tiny):
    """The cached step with the Q/K/V projections fused with norm + RoPE (one tcgen05 GEMM)
    equals the unfused step (three GEMMs + b200_attn_fwd) up to bf16 rounding."""
    w, _, R = tiny
    lengths = [40, 72]
    embs = _embs(lengths, 41)
    g = torch.Generator().manual_seed(42)
    lat = torch.randn(2, 256, 64, generator=g).to("cuda:0")
    outs = []
    for fused in (False, True):
        model = mmdit.MMDiT(TINY, w, device="cuda:0", fused_qkv=fused)
        cache = model.prefix_fill(embs)
        outs.append(model.step(lat, 0.4, cache, model.target_pe(lengths, GRID),
                               mmdit.cached_desc(cache, 256, model.device)).cpu())
    assert rel(outs[1], outs[0]) < 1e-2
    for b, n in enumerate(lengths):
        want = R.forward_cached(lat[b].cpu(), 0.4, R.prefix_kv(embs[b].float(), GRID), n, GRID)
        assert rel(outs[1][b], want) < 1.5e-2


@pytest.mark.gpu
def test_tcgen05_gemm_model_matches_cublas_model(tiny):
    """The model with its block linears on the tcgen05 GEMM equals the cuBLAS model up to
    bf16 rounding of the GEMM outputs."""
    w, _, _ = tiny
    lengths = [40, 72]
    embs = _embs(lengths, 51)
    g = torch.Generator().manual_seed(52)
    lat = torch.randn(2, 256, 64, generator=g).to("cuda:0")
    outs = []
    for impl in ("cublas", "b200"):
        model = mmdit.MMDiT(TINY, w, device="cuda:0", gemm=impl, mlp_chunk_rows=300)
        cache = model.prefix_fill(embs)
        outs.append(model.step(lat, 0.6, cache, model.target_pe(lengths, GRID),
                               mmdit.cached_desc(cache, 256, model.device)).cpu())
    assert rel(outs[1], outs[0]) < 1e-2
