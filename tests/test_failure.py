"""Device-side failure detection without a GPU fault: a bounded wait on a barrier that
nothing completes gives up, raises the CTA abort flag, reports through the caller's status
words, and leaves the context usable (the attention kernel's protocol)."""
import time

import pytest

import b200attn


def test_wait_selftest_rejects_bad_arguments():
    L = b200attn.lib()
    assert L.b200_wait_selftest(None, 1000, None) == b200attn.ERR_INVALID
    assert L.b200_wait_selftest(16, 0, None) == b200attn.ERR_INVALID
    assert L.b200_wait_selftest(16, 2000001, None) == b200attn.ERR_INVALID
    assert L.b200_wait_selftest(18, 1000, None) == b200attn.ERR_INVALID   # misaligned


@pytest.mark.gpu
def test_bounded_wait_runs_out_and_context_survives(cuda):
    import torch
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    status = b200attn.wait_selftest(limit_us=20000)   # 20 ms
    dt = time.perf_counter() - t0
    assert status == [1, 1]            # the wait ran out; the second waiter left on the flag
    assert dt < 1.0
    # the context is still usable: a small attention call right after
    q, k, v = (torch.randn(1, 64, 2, 128, device=cuda).bfloat16() for _ in range(3))
    w = torch.ones(128, device=cuda)
    pe = torch.zeros(64, 128, device=cuda)
    pe[:, 0::2] = 1.0
    st = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = b200attn.attention_forward(q, k, v, None, None, w, w, pe, status=st)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all() and int(st.item()) == 0
