"""Multi-GPU plumbing around the joint-attention path (one process per GPU).

Two ways the path is partitioned inside one node:

- **Data parallel** — independent generations (seeds, prompts, and the positive and
  negative branches of true CFG) are assigned to ranks; nothing crosses GPUs on the data
  path.  The reference runs one generation per GPU worker (src/server.rs:123-155); its
  CFG branches are two sequential forward calls (src/pipeline.rs:154-197).
- **Head sharding** (>= 2048^2) — rank r owns heads [h0, h1): its to_q/to_k/to_v column
  slices, its slice of every layer's prefix cache, and rows [h0*D, h1*D) of to_out's input
  dimension.  Attention is local; the to_out partial sums of all ranks are added by one
  NCCL all-reduce per layer (the reference's to_out is src/transformer.rs:196).

torch.distributed (NCCL on GPUs, gloo in the CPU tests) is the plumbing.
"""
from __future__ import annotations

import os
from typing import List, Optional, Sequence, Tuple


def env_rank() -> Tuple[int, int, int]:
    """(rank, world_size, local_rank) from the torchrun environment (1 process: 0, 1, 0)."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def dp_assign(items: Sequence, world: int, rank: int) -> List:
    """Round-robin data-parallel assignment: rank r takes items r, r + world, ...
    Every item lands on exactly one rank."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world / rank")
    return list(items[rank::world])


def cfg_pairs(prompts: int) -> List[Tuple[int, str]]:
    """The sequences of a true-CFG batch: (prompt index, 'pos'|'neg') — two per prompt,
    kept adjacent so that a rank owning both branches combines them locally."""
    return [(p, branch) for p in range(prompts) for branch in ("pos", "neg")]


def head_shard(heads: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous head range [h0, h1) of `rank`; sizes differ by at most one head."""
    if world < 1 or not 0 <= rank < world or heads < world:
        raise ValueError("bad heads / world / rank")
    base, extra = divmod(heads, world)
    h0 = rank * base + min(rank, extra)
    return h0, h0 + base + (1 if rank < extra else 0)


def out_proj_partial(attn_local, w_out, h0: int, h1: int, head_dim: int = 128):
    """This rank's share of to_out: attn_local [T, (h1-h0)*D] times the matching input
    columns of w_out [hidden_out, H*D] -> a full-width partial [T, hidden_out]."""
    import torch
    w_cols = w_out[:, h0 * head_dim:h1 * head_dim]
    return torch.matmul(attn_local, w_cols.t())


def allreduce_sum_(t, group=None):
    """In-place sum of `t` over the ranks of `group` (NCCL on GPUs, gloo on CPU)."""
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return t


def max_over_ranks(value: float, device=None, group=None) -> float:
    """The largest `value` of any rank (multi-GPU times are the max over ranks)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def head_sharded_attention_layer(q, k, v, prefix_k, prefix_v, norm_q_w, norm_k_w, pe, w_out,
                                 h0: int, h1: int, desc=None, workspace=None, group=None,
                                 stream=None):
    """One layer of head-sharded joint attention on this rank's heads [h0, h1).

    q, k, v: bf16 [B, T, h1-h0, D] (this rank's column slice of the projections);
    prefix_k/v: bf16 [B, h1-h0, P, D]; w_out: bf16 [hidden, H*D] (full to_out weight).
    Returns the all-reduced to_out output [B, T, hidden] (identical on every rank).
    """
    import b200attn
    b, t, hl, d = q.shape
    attn = b200attn.attention_forward(q, k, v, prefix_k, prefix_v, norm_q_w, norm_k_w, pe,
                                      desc=desc, workspace=workspace, stream=stream)
    partial = out_proj_partial(attn.reshape(b * t, hl * d), w_out, h0, h1, d)
    allreduce_sum_(partial, group)
    return partial.reshape(b, t, -1)
