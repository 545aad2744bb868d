"""b200_attn_fwd_noalloc: the entry point for callers that cannot allocate device memory
when they call (its scratch is a fixed array inside the library).  Checked through the C
ABI against b200_attn_fwd with a caller workspace and against the CPU oracle, on two
calls in a row — the second call reuses the scratch the first one left behind, with a
different shape and inputs.

This file is collected last so that a run stopping at the first failure has already run
every other test; it also passes alone in a fresh process."""
import ctypes

import numpy as np
import pytest

import b200attn
from oracle import cpu as ocpu
from oracle import reference as ref

pytestmark = pytest.mark.gpu

REL_L2 = 5e-3
MAX_ABS = 2e-2
SCRATCH_BYTES = 64 << 20  # B200_NOALLOC_SCRATCH_BYTES


def _lib():
    L = b200attn.lib()
    L.b200_attn_fwd_noalloc.argtypes = [ctypes.POINTER(b200attn.AttnArgs), ctypes.c_void_p]
    L.b200_attn_fwd_noalloc.restype = ctypes.c_int
    return L


def _case(device, seed, B, T, H, P, pv):
    import torch
    g = torch.Generator().manual_seed(seed)
    bf = lambda *s: torch.randn(*s, generator=g).to(torch.bfloat16).to(device)
    d = dict(q=bf(B, T, H, 128), k=bf(B, T, H, 128), v=bf(B, T, H, 128),
             pk=bf(B, H, P, 128), pv=bf(B, H, P, 128),
             wq=(1 + 0.1 * torch.randn(128, generator=g)).float().to(device),
             wk=(1 + 0.1 * torch.randn(128, generator=g)).float().to(device))
    hgt = int(np.sqrt(T))
    while T % hgt:
        hgt -= 1
    lay = ref.joint_layout(P, None, [], (hgt, T // hgt))
    pe = ref.embed_nd(lay["img_shapes"], lay["image_pad_mask"])[P:]
    d["pe"] = torch.from_numpy(pe).to(device)
    d["desc"] = torch.tensor([[x, T] for x in pv], dtype=torch.int32, device=device)
    return d


def _noalloc(d, out, k_rot_out=None):
    import torch
    args = b200attn.make_args(d["q"], d["k"], d["v"], d["pk"], d["pv"], d["wq"], d["wk"], d["pe"],
                              out, desc=d["desc"], k_rot_out=k_rot_out)
    stream = torch.cuda.current_stream().cuda_stream
    return _lib().b200_attn_fwd_noalloc(ctypes.byref(args), stream)


def test_noalloc_matches_workspace_entry_point_twice(cuda):
    import torch
    cases = [  # (seed, B, T, H, P, prefix_valid per row, pass k_rot_out)
        (101, 1, 1024, 32, 256, [256], False),
        (102, 2, 300, 4, 130, [77, 130], True),
    ]
    for seed, B, T, H, P, pv, with_k in cases:
        d = _case(cuda, seed, B, T, H, P, pv)
        want = b200attn.attention_forward(d["q"], d["k"], d["v"], d["pk"], d["pv"], d["wq"], d["wk"],
                                          d["pe"], desc=d["desc"])
        out = torch.full_like(want, float("nan"))
        k_rot = torch.empty(B, H, T, 128, dtype=torch.bfloat16, device=cuda) if with_k else None
        assert _noalloc(d, out, k_rot) == b200attn.OK
        torch.cuda.synchronize()
        got, ref_out = out.float().cpu().numpy(), want.float().cpu().numpy()
        assert np.isfinite(got).all()
        assert ref.rel_l2(got, ref_out) <= REL_L2
        assert float(np.max(np.abs(got - ref_out))) <= MAX_ABS
        # and directly against the CPU oracle (the f32 restatement of the reference span)
        bits = lambda t: t.cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
        oracle_out = ocpu.attention_forward(
            bits(d["q"]), bits(d["k"]), bits(d["v"]), bits(d["pk"]), bits(d["pv"]),
            d["wq"].cpu().numpy(), d["wk"].cpu().numpy(), 1e-6, d["pe"].cpu().numpy(),
            np.array(pv, np.int32), 128 ** -0.5)
        assert ref.rel_l2(got, oracle_out) <= REL_L2
        assert float(np.max(np.abs(got - oracle_out))) <= MAX_ABS
        if with_k:
            want_k = b200attn.norm_rope(d["k"], d["wk"], 1e-6, d["pe"])
            torch.cuda.synchronize()
            assert torch.equal(k_rot, want_k)


def test_noalloc_rejects_problems_over_its_limit(cuda):
    import torch
    d = _case(cuda, 103, 1, 64, 2, 64, [64])
    out = torch.empty(1, 64, 2 * 128, dtype=torch.bfloat16, device=cuda)
    args = b200attn.make_args(d["q"], d["k"], d["v"], d["pk"], d["pv"], d["wq"], d["wk"], d["pe"], out)
    # claim a problem whose scratch (post-RoPE Q and K) exceeds the fixed array: the call
    # must refuse before launching anything
    args.batch, args.heads, args.target_len = 4, 32, 4096
    assert b200attn.workspace_bytes(args) > SCRATCH_BYTES
    stream = torch.cuda.current_stream().cuda_stream
    assert _lib().b200_attn_fwd_noalloc(ctypes.byref(args), stream) == b200attn.ERR_WORKSPACE
    torch.cuda.synchronize()
