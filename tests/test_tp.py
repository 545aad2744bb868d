"""The head-sharding communicator of include/b200_tp.h through its Python binding.

One GPU: a single-rank group sums to the identity, on bf16 and f32, on a side stream; a
rank whose peer never joins gives up after its timeout with B200_ERR_DEVICE_TIMEOUT (the
failure is made on the host: the second rank is never started; nothing runs on the GPU).
Two GPUs: head-sharded attention layers whose `to_out` partials are summed through the
C-ABI communicator match the single-GPU layer."""
import os
import socket
import subprocess
import sys
import textwrap

import numpy as np
import pytest

import b200attn

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_single_rank_group_sums_to_identity(cuda):
    import torch
    comm = b200attn.TpComm(b200attn.tp_unique_id(), 1, 0, timeout_ms=20000)
    try:
        assert (comm.rank, comm.size) == (0, 1)
        s = torch.cuda.Stream()
        g = torch.Generator(device=cuda).manual_seed(5)
        for dt in (torch.bfloat16, torch.float32):
            x = torch.randn(4096, 257, generator=g, device=cuda).to(dt)
            want = x.clone()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                comm.allreduce_(x, stream=s)
            comm.wait(stream=s)
            assert torch.equal(x, want)
        with pytest.raises(ValueError):
            comm.allreduce_(torch.zeros(4, 4, dtype=torch.int32, device=cuda))
    finally:
        comm.close()


_LONE_RANK = textwrap.dedent("""
    import sys, time
    sys.path[:0] = [{root!r}, {pkg!r}]
    import torch
    import b200attn
    torch.cuda.set_device(0)
    uid = b200attn.tp_unique_id()
    t0 = time.monotonic()
    try:
        b200attn.TpComm(uid, 2, 0, timeout_ms=3000)
        print("JOINED")
    except b200attn.B200Error as e:
        print("STATUS", e.status, round(time.monotonic() - t0, 2))
""")


def test_join_gives_up_when_the_peer_never_joins(cuda):
    src = _LONE_RANK.format(root=ROOT, pkg=os.path.join(ROOT, "qwen3-image21_b200"))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", CUDA_VISIBLE_DEVICES=os.environ.get(
        "CUDA_VISIBLE_DEVICES", "0").split(",")[0])
    res = subprocess.run([sys.executable, "-c", src], capture_output=True, text=True,
                         timeout=180, env=env)
    line = [ln for ln in res.stdout.splitlines() if ln.startswith(("STATUS", "JOINED"))]
    assert line, res.stdout + res.stderr
    parts = line[-1].split()
    assert parts[0] == "STATUS" and int(parts[1]) == b200attn.ERR_DEVICE_TIMEOUT, line
    assert float(parts[2]) < 60.0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, result_path):
    import torch
    import torch.distributed as dist

    from b200attn import dist as bdist
    from oracle import reference as ref

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    # gloo carries only the group id; the sums go through the C-ABI communicator
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    comm = b200attn.TpComm.from_group(timeout_ms=30000)
    try:
        T, P, H, hidden = 512, 256, 8, 1024
        g = torch.Generator().manual_seed(11)
        bf = lambda *s: torch.randn(*s, generator=g).to(torch.bfloat16).to(dev)
        q, k, v = bf(1, T, H, 128), bf(1, T, H, 128), bf(1, T, H, 128)
        pk, pv = bf(1, H, P, 128), bf(1, H, P, 128)
        w_out = (0.02 * torch.randn(hidden, H * 128, generator=g)).to(torch.bfloat16).to(dev)
        lay = ref.joint_layout(P, None, [], (16, 32))
        pe = torch.from_numpy(ref.embed_nd(lay["img_shapes"], lay["image_pad_mask"])[P:]).to(dev)
        w = torch.ones(128, device=dev)
        h0, h1 = bdist.head_shard(H, world, rank)
        out = bdist.head_sharded_attention_layer(
            q[:, :, h0:h1].contiguous(), k[:, :, h0:h1].contiguous(), v[:, :, h0:h1].contiguous(),
            pk[:, h0:h1].contiguous(), pv[:, h0:h1].contiguous(), w, w, pe, w_out, h0, h1,
            comm=comm)
        comm.wait()
        if rank == 0:
            full = b200attn.attention_forward(q, k, v, pk, pv, w, w, pe)
            want = torch.matmul(full.view(T, H * 128), w_out.t()).view(1, T, hidden)
            a, b = out.float().cpu().numpy(), want.float().cpu().numpy()
            with open(result_path, "w") as f:
                f.write(str(float(np.linalg.norm(a - b) / np.linalg.norm(b))))
        dist.barrier()
    finally:
        comm.close()
        dist.destroy_process_group()


def test_two_rank_head_sharding_through_the_c_abi_communicator(tmp_path):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    result = tmp_path / "rel.txt"
    mp.spawn(_rank, args=(2, _free_port(), str(result)), nprocs=2, join=True)
    assert float(result.read_text()) <= 5e-3
