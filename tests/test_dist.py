"""Multi-GPU host logic on CPU: data-parallel assignment, head sharding, and the
head-sharded to_out partial sums all-reduced over world_size-2 gloo ranks."""
import os
import socket

import pytest

from b200attn import dist as bdist


def test_dp_assign_covers_every_sequence_once():
    seqs = bdist.cfg_pairs(8)  # 8 prompts x {pos, neg} = 16 sequences (config 5)
    assert len(seqs) == 16 and seqs[0] == (0, "pos") and seqs[1] == (0, "neg")
    for world in (1, 2, 4, 8):
        got = [s for r in range(world) for s in bdist.dp_assign(seqs, world, r)]
        assert sorted(got) == sorted(seqs)
    with pytest.raises(ValueError):
        bdist.dp_assign(seqs, 2, 2)


@pytest.mark.parametrize("heads,world", [(32, 1), (32, 2), (32, 4), (32, 8), (30, 4), (5, 3)])
def test_head_shard_partitions_heads(heads, world):
    ranges = [bdist.head_shard(heads, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == heads
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0
    sizes = [h1 - h0 for h0, h1 in ranges]
    assert max(sizes) - min(sizes) <= 1


def test_out_proj_path_follows_the_measured_crossover():
    assert bdist.out_proj_path(1) == "local"
    assert [bdist.out_proj_path(n) for n in (2, 4, 8)] == ["scatter", "scatter", "nvls"]
    assert [bdist.out_proj_path(n, residual=True) for n in (2, 4, 8)] == \
        ["scatter", "scatter", "nvls"]
    # a fused path won at every rank count measured
    assert all(bdist.prefer_fused_out_proj(n, residual=r) for n in (2, 4, 8) for r in (0, 1))
    assert not bdist.prefer_fused_out_proj(1)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_path):
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        torch.manual_seed(0)
        heads, d, t, hidden = 8, 128, 16, 256
        attn = torch.randn(t, heads * d)        # every rank knows the full tensors here,
        w_out = torch.randn(hidden, heads * d)  # but uses only its own heads' slice
        h0, h1 = bdist.head_shard(heads, world, rank)
        part = bdist.out_proj_partial(attn[:, h0 * d:h1 * d], w_out, h0, h1, d)
        bdist.allreduce_sum_(part)
        full = attn @ w_out.t()
        err = float((part - full).abs().max() / full.abs().max())
        worst = bdist.max_over_ranks(err)
        slowest = bdist.max_over_ranks(float(rank + 1))
        if rank == 0:
            with open(result_path, "w") as f:
                f.write(f"{worst} {slowest}")
    finally:
        dist.destroy_process_group()


def test_gloo_head_sharded_out_proj_allreduce(tmp_path):
    import torch.multiprocessing as mp
    world = 2
    result = tmp_path / "result.txt"
    mp.spawn(_worker, args=(world, _free_port(), str(result)), nprocs=world, join=True)
    worst, slowest = map(float, result.read_text().split())
    assert worst < 1e-5          # partial sums over the head shards == the full to_out
    assert slowest == float(world)  # the max over ranks reaches every rank's value
