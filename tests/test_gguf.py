"""GGUF k-quant weights: the CPU oracle against llama.cpp's gguf-py dequantisation (golden
fixture tests/golden/gguf_kquants.npz), the product quantizer's blocks, the Q4_K_M type
rule, and on the GPU the CUDA dequantisation (bit-exact in bf16) and the denoising loop
with Q4_K_M weights against the float32 oracle."""
import os

import numpy as np
import pytest
import torch

import b200attn
from b200attn import gguf as bq
from b200attn import mmdit
from oracle import gguf_ref as G
from oracle import mmdit_ref as M

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FIX = np.load(os.path.join(ROOT, "tests", "golden", "gguf_kquants.npz"))


def _rel(a, b):
    return float((a.double() - b.double()).norm() / b.double().norm())


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even (finite inputs)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


# ----------------------------------------------------------------------------- CPU
@pytest.mark.parametrize("qtype", ["q4_k", "q6_k"])
def test_oracle_matches_gguf_py_fixture(qtype):
    deq = G.dequantize_q4_k if qtype == "q4_k" else G.dequantize_q6_k
    got = deq(FIX[qtype])
    want = FIX[qtype + "_f32"]
    assert got.shape == want.shape == (FIX[qtype].shape[0], 256)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("qtype,bound", [("q4_k", 0.1), ("q6_k", 0.03)])
def test_quantizer_round_trip(qtype, bound):
    g = torch.Generator().manual_seed(3)
    w = torch.randn(64, 1024, generator=g) * 0.02
    w[3] = 0.0                                  # an all-zero row (zero super-scales)
    w[5, :256] = torch.linspace(-1, 1, 256)     # a large-range block
    blocks = bq.quantize(w, qtype)
    assert blocks.dtype == torch.uint8
    assert blocks.shape == (64, 1024 // 256 * bq.BLOCK_BYTES[qtype])
    deq = G.dequantize_q4_k if qtype == "q4_k" else G.dequantize_q6_k
    back = torch.from_numpy(deq(blocks.numpy())).reshape(64, 1024)
    assert torch.isfinite(back).all()
    assert float((back - w).norm() / w.norm()) < bound
    assert back[3].abs().max() == 0
    assert float((back[5, :256] - w[5, :256]).abs().max()) < (0.15 if qtype == "q4_k" else 0.02)


def test_q4_k_m_rule():
    more = [i for i in range(32) if bq.use_more_bits(i, 32)]
    assert more == [0, 1, 2, 3, 6, 9, 12, 15, 18, 21, 24, 27, 28, 29, 30, 31]
    assert bq.q4_k_m_type("to_v", 0, 32) == "q6_k" and bq.q4_k_m_type("to_v", 4, 32) == "q4_k"
    assert bq.q4_k_m_type("out", 6, 32) == "q6_k" and bq.q4_k_m_type("to_q", 0, 32) == "q4_k"
    assert bq.q4_k_m_type("gate_up", 31, 32) == "q4_k"


def test_dequant_rejects_bad_arguments():
    L = b200attn.lib()
    assert L.b200_dequant_q4_k(16, 16, -1, None) == b200attn.ERR_INVALID
    assert L.b200_dequant_q4_k(None, 16, 4, None) == b200attn.ERR_INVALID
    assert L.b200_dequant_q4_k(8, 16, 4, None) == b200attn.ERR_INVALID    # blocks not 16-aligned
    assert L.b200_dequant_q6_k(16, 8, 4, None) == b200attn.ERR_INVALID    # out not 16-aligned
    assert L.b200_dequant_q6_k(17, 16, 4, None) == b200attn.ERR_INVALID   # odd blocks address
    assert L.b200_dequant_q6_k(16, 16, 0, None) == b200attn.OK


def test_kquant_gemv_rejects_bad_arguments():
    L = b200attn.lib()
    Q4 = b200attn.KQUANT_TYPES["q4_k"]
    assert L.b200_kquant_gemv(16, 256, 16, Q4, 16, 64, 0, 64, 256, None) == b200attn.OK  # m = 0
    assert L.b200_kquant_gemv(16, 256, 16, Q4, 16, 64, 3, 64, 256, None) == b200attn.ERR_INVALID
    assert L.b200_kquant_gemv(16, 300, 16, Q4, 16, 64, 2, 64, 300, None) == b200attn.ERR_INVALID
    assert L.b200_kquant_gemv(16, 256, 16, 7, 16, 64, 2, 64, 256, None) == b200attn.ERR_INVALID
    assert L.b200_kquant_gemv(16, 128, 16, Q4, 16, 64, 2, 64, 256, None) == b200attn.ERR_INVALID
    assert L.b200_kquant_gemv(16, 256, 8, Q4, 16, 64, 2, 64, 256, None) == b200attn.ERR_INVALID
    assert L.b200_kquant_gemv(None, 256, 16, Q4, 16, 64, 2, 64, 256, None) == b200attn.ERR_INVALID


# ----------------------------------------------------------------------------- GPU
@pytest.mark.gpu
@pytest.mark.parametrize("qtype", ["q4_k", "q6_k"])
@pytest.mark.parametrize("m,n,k,pad", [(1, 4096, 4096, 0), (2, 33, 256, 0), (1, 96, 8192, 64),
                                       (2, 1000, 2048, 0), (2, 64, 12288, 256), (1, 40, 768, 0)])
def test_kquant_gemv_matches_dequantized_matmul(cuda, qtype, m, n, k, pad):
    """The fused few-row product straight from the super-blocks equals x times the
    dequantised bf16 weight (the oracle's f32 dequantisation rounded to bf16), summed in
    float64, to f32 accumulation accuracy: ragged row counts, x rows wider than k (pad),
    k split into several shared-memory chunks of 8 super-blocks (k = 8192, 12288) or ending
    in a partial one (k = 768: 3 blocks, whose Q6_K rows are only 2-byte aligned)."""
    g = torch.Generator(device=cuda).manual_seed(m * 1000 + n)
    w = torch.randn(n, k, generator=g, device=cuda) * 0.02
    blocks = bq.quantize(w, qtype)
    x_full = torch.randn(m, k + pad, generator=g, device=cuda)
    x = x_full[:, :k]
    got = bq.QuantLinear(blocks, qtype, (n, k)).matvec(x)
    torch.cuda.synchronize()
    deq = G.dequantize_q4_k if qtype == "q4_k" else G.dequantize_q6_k
    w_bf16 = torch.from_numpy(deq(blocks.cpu().numpy()).reshape(n, k)).bfloat16().double()
    want = x.cpu().double() @ w_bf16.t()
    assert got.shape == (m, n)
    assert _rel(got.cpu(), want) <= 1e-5


@pytest.mark.gpu
@pytest.mark.parametrize("qtype", ["q4_k", "q6_k"])
def test_cuda_dequant_bit_exact_on_fixture(cuda, qtype):
    blocks = torch.from_numpy(FIX[qtype]).to(cuda)
    out = b200attn.dequant(blocks, qtype)
    torch.cuda.synchronize()
    got = out.cpu().view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(got, bf16_bits(FIX[qtype + "_f32"]).reshape(-1))


@pytest.mark.gpu
@pytest.mark.parametrize("qtype", ["q4_k", "q6_k"])
def test_cuda_dequant_bit_exact_at_size(cuda, qtype):
    """A 4096 x 12288 matrix (the config-5 MLP down-projection shape): every weight equals
    the oracle's dequantisation rounded to bf16."""
    g = torch.Generator(device=cuda).manual_seed(11)
    w = torch.randn(4096, 12288, generator=g, device=cuda) * 0.02
    blocks = bq.quantize(w, qtype)
    out = bq.QuantLinear(blocks, qtype, (4096, 12288)).dequant_into(
        torch.empty(4096, 12288, dtype=torch.bfloat16, device=cuda))
    torch.cuda.synchronize()
    deq = G.dequantize_q4_k if qtype == "q4_k" else G.dequantize_q6_k
    want = bf16_bits(deq(blocks.cpu().numpy()))
    got = out.cpu().view(torch.int16).numpy().view(np.uint16).reshape(want.shape)
    assert np.array_equal(got, want)


TINY = mmdit.MMDiTConfig(layers=2, heads=2, text_dim=256)
GRID = (16, 16)


@pytest.mark.gpu
def test_q4_k_m_model_matches_oracle(cuda):
    """The denoising loop with Q4_K_M block linears, 20 CFG steps end to end, against the
    float32 oracle run on the same (dequantised) weights."""
    w = mmdit.random_weights(TINY, 0, std=0.1)
    model = mmdit.MMDiT(TINY, w, device=cuda, weight_format="q4_k_m")
    # with 2 layers use_more_bits picks layer 1 only (the last eighth)
    assert model.blocks[1]["q_wv"].qtype == "q6_k" and model.blocks[1]["q_wmo"].qtype == "q6_k"
    assert model.blocks[0]["q_wv"].qtype == "q4_k" and model.blocks[1]["q_wq"].qtype == "q4_k"
    R = M.Reference(model.effective_weights(w), TINY.layers, TINY.heads)
    g = torch.Generator().manual_seed(31)
    pos = [torch.randn(n, 256, generator=g).to(torch.bfloat16) for n in (40, 72)]
    neg = [torch.randn(n, 256, generator=g).to(torch.bfloat16) for n in (33, 50)]
    noise = mmdit.pack_latents(torch.randn(2, 64, 1, *GRID, generator=g))
    got = mmdit.denoise(model, pos, neg, GRID, 20, 2.5, noise).cpu()
    want = R.denoise(pos, neg, GRID, 20, 2.5, noise)
    for p in range(2):
        assert _rel(got[p], want[p]) <= 2e-2, p
    # the quantised model is a different model from the bf16 one
    ref_bf16 = M.Reference(w, TINY.layers, TINY.heads).denoise(pos, neg, GRID, 20, 2.5, noise)
    assert _rel(want, ref_bf16) > 1e-2
