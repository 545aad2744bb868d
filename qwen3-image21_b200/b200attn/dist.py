"""Multi-GPU plumbing around the joint-attention path (one process per GPU).

Two ways the path is partitioned inside one node:

- **Data parallel** — independent generations (seeds, prompts, and the positive and
  negative branches of true CFG) are assigned to ranks; nothing crosses GPUs on the data
  path.  The reference runs one generation per GPU worker (src/server.rs:123-155); its
  CFG branches are two sequential forward calls (src/pipeline.rs:154-197).
- **Head sharding** (>= 2048^2) — rank r owns heads [h0, h1): its to_q/to_k/to_v column
  slices, its slice of every layer's prefix cache, and rows [h0*D, h1*D) of to_out's input
  dimension.  Attention is local; the to_out partial sums of all ranks are added either by
  one NCCL all-reduce per layer after a cuBLAS GEMM (`out_proj_partial` +
  `allreduce_sum_`), or by the out-projection GEMM itself (`ScatterOutProj`): its epilogue
  stores every partial tile straight into the rank that owns those rows (a reduce-scatter
  overlapped with the GEMM, over NVLink), and a second kernel sums each owner's slots and
  broadcasts the rows.  (The
  reference's to_out is src/transformer.rs:196.)

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


def allreduce_sum_(t, group=None, comm=None, stream=None):
    """In-place sum of `t` over the ranks of `group` (NCCL on GPUs, gloo on CPU), or over
    `comm` (a b200attn.TpComm: the C-ABI communicator, b200_tp_out_proj_allreduce on
    `stream`) when one is given."""
    if comm is not None:
        return comm.allreduce_(t, stream=stream)
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
                                 stream=None, comm=None):
    """One layer of head-sharded joint attention on this rank's heads [h0, h1).

    q, k, v: bf16 [B, T, h1-h0, D] (this rank's column slice of the projections);
    prefix_k/v: bf16 [B, h1-h0, P, D]; w_out: bf16 [hidden, H*D] (full to_out weight).
    Returns the all-reduced to_out output [B, T, hidden] (identical on every rank).  The
    sum goes through `comm` (b200attn.TpComm) when given, else torch.distributed.
    """
    import b200attn
    b, t, hl, d = q.shape
    attn = b200attn.attention_forward(q, k, v, prefix_k, prefix_v, norm_q_w, norm_k_w, pe,
                                      desc=desc, workspace=workspace, stream=stream)
    partial = out_proj_partial(attn.reshape(b * t, hl * d), w_out, h0, h1, d)
    allreduce_sum_(partial, group, comm=comm, stream=stream)
    return partial.reshape(b, t, -1)


def out_proj_path(world: int, residual: bool = False) -> str:
    """How to sum the head-sharded to_out partials at this rank count: "scatter"
    (ScatterOutProj: peer stores from the GEMM epilogue, owners' sum and broadcast),
    "nvls" (NvlsOutProj: owners' sum in the NVSwitch) or "nccl" (cuBLAS + all-reduce).

    Measured on B200 boxes, config 4 (one block: attention + to_out + the sum), ms:
      2 ranks: scatter 2.18-2.28, NCCL 2.27-2.32, NVLS 2.58;
               with residual + norm2: scatter 2.25-2.37, NVLS 2.59, NCCL RS/AG 2.67
      4 ranks: scatter 1.46, NCCL 1.47 (NVLS not measured; by bytes moved it is between)
      8 ranks: NVLS 0.975, scatter 0.986-0.987, NCCL 0.991-0.993;
               with residual + norm2: NVLS 0.981, scatter 0.985-0.989, NCCL RS/AG 1.063
    At 2 ranks NVLS moves more bytes than peer stores ((1 + 1/N) against 2 (N-1)/N
    partials each way); at 8 fewer."""
    if world <= 1:
        return "local"
    if world >= 8:
        return "nvls"
    if residual:
        return "scatter"
    return "scatter" if world <= 4 else "nccl"


def prefer_fused_out_proj(world: int, residual: bool = False) -> bool:
    """Whether one of this library's fused paths (scatter or NVLS) beats cuBLAS + NCCL at
    this rank count (out_proj_path)."""
    return out_proj_path(world, residual) in ("scatter", "nvls")


class ScatterOutProj:
    """Head-sharded to_out fused with the reduction of its partial sums across ranks.

    Rows of the output are split into `world` equal blocks; rank q owns block q.  Per rank,
    two sets (alternating calls) of two symmetric-memory buffers: `slots` bf16
    [world * rows_per, hidden] (rank s's partial of this rank's block lands in slot s) and
    `out` bf16 [world * rows_per, hidden] (the full result).  A call:
      b200_gemm_scatter: attn_local · w_cols^T, each tile stored into its owner's slot for
                         this rank (plain stores over NVLink as tiles finish)
      barrier (every slot written)
      b200_reduce_gather_bf16: this rank sums its block's slots in a fixed order and writes
                         the bf16 rows into every rank's `out`
      barrier (every block written)
    and returns this rank's `out` [T, hidden].  Alternating the buffer sets makes a leading
    barrier unnecessary: the previous use of a set ended before the previous call's last
    barrier, which every rank has passed.  The returned view stays valid until the call
    after next.  Barriers time out after `timeout_ms`.
    """

    def __init__(self, rows: int, hidden: int, device, group=None, timeout_ms: int = 10000):
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem
        group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.rows_per = -(-rows // self.world)
        self.rows, self.hidden, self.timeout_ms = rows, hidden, timeout_ms
        self.sets = []
        for _ in range(2):
            slots = symm_mem.empty(self.world * self.rows_per, hidden, dtype=torch.bfloat16,
                                   device=device)
            out = symm_mem.empty(self.world * self.rows_per, hidden, dtype=torch.bfloat16,
                                 device=device)
            h_slots = symm_mem.rendezvous(slots, group)
            h_out = symm_mem.rendezvous(out, group)
            self.sets.append(dict(slots=slots, out=out, h=h_out,
                                  slot_ptrs=[int(p) for p in h_slots.buffer_ptrs],
                                  out_ptrs=[int(p) for p in h_out.buffer_ptrs]))
        self.calls = 0

    def own_rows(self, t: int):
        """(first row, row count) of the output block this rank owns for t rows."""
        r0 = self.rank * self.rows_per
        return r0, max(0, min(self.rows_per, t - r0))

    def __call__(self, attn_local, w_out, h0: int, h1: int, head_dim: int = 128, status=None,
                 residual=None, eps: float = 1e-6):
        """attn_local [t, (h1-h0)*head_dim] bf16 -> the full to_out product [t, hidden] bf16
        on every rank.  With residual=(x_own, gate, scale) — x_own f32 [own rows, hidden],
        this rank's rows of the residual stream (own_rows), gate / scale f32 [hidden] —
        the owners apply x_own += tanh(gate) * sum and return LN(x) * (1 + scale) instead,
        all-gathered (src/transformer.rs:411-418: the attention residual and norm2)."""
        import b200attn
        t = attn_local.shape[0]
        if t > self.rows or w_out.shape[0] != self.hidden:
            raise ValueError("shape does not fit the buffers")
        st = self.sets[self.calls % 2]
        self.calls += 1
        w_cols = w_out[:, h0 * head_dim:h1 * head_dim]
        b200attn.gemm_scatter(attn_local, w_cols, st["slot_ptrs"], self.rank, self.rows_per,
                              self.hidden, status=status)
        st["h"].barrier(channel=0, timeout_ms=self.timeout_ms)
        r0, mine = self.own_rows(t)
        if residual is None:
            b200attn.reduce_gather(st["slots"], self.world, self.rows_per, mine, self.hidden,
                                   self.hidden, st["out_ptrs"], r0, self.hidden)
        else:
            x_own, gate, scale = residual
            if x_own.shape[0] < mine or x_own.shape[1] != self.hidden:
                raise ValueError("x_own must hold this rank's rows of the residual stream")
            b200attn.reduce_residual_adaln_gather(
                st["slots"], self.world, self.rows_per, mine, self.hidden, self.hidden, x_own,
                gate, scale, st["out_ptrs"], r0, self.hidden, eps=eps)
        st["h"].barrier(channel=0, timeout_ms=self.timeout_ms)
        return st["out"][:t]


class NvlsOutProj:
    """Head-sharded to_out with the sum of the partials done by the NVSwitch (NVLS).

    Each rank's GEMM writes its full partial [T, hidden] into its own symmetric buffer
    (local stores only); after a barrier, owner q reads rows [q*rows_per, ...) of all
    ranks' partials summed in the switch (b200_reduce_nvls: multimem.ld_reduce through the
    partial buffers' multicast address), optionally applies the block's residual and
    norm2, and writes each row once to the output buffers' multicast address, which puts
    it in every rank's output; a second barrier ends the call.  Per GPU the links carry
    (1 + 1/N) partials each way, against 2 (N-1)/N for ScatterOutProj's peer stores, so
    this path is for N >= 4.  Same call contract, buffer alternation and returned view as
    ScatterOutProj.  Raises RuntimeError when the buffers have no multicast address (no
    NVSwitch multicast on this system)."""

    def __init__(self, rows: int, hidden: int, device, group=None, timeout_ms: int = 10000):
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem
        group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.rows_per = -(-rows // self.world)
        self.rows, self.hidden, self.timeout_ms = rows, hidden, timeout_ms
        self.sets = []
        for _ in range(2):
            part = symm_mem.empty(self.world * self.rows_per, hidden, dtype=torch.bfloat16,
                                  device=device)
            out = symm_mem.empty(self.world * self.rows_per, hidden, dtype=torch.bfloat16,
                                 device=device)
            h_part = symm_mem.rendezvous(part, group)
            h_out = symm_mem.rendezvous(out, group)
            mc_part, mc_out = int(h_part.multicast_ptr), int(h_out.multicast_ptr)
            if not mc_part or not mc_out:
                raise RuntimeError("symmetric memory has no multicast address on this system")
            for h, t in ((h_part, part), (h_out, out)):
                # the multicast address must map the tensor from its first element
                if int(h.buffer_ptrs[self.rank]) != t.data_ptr() or int(getattr(h, "offset", 0)):
                    raise RuntimeError("symmetric tensor does not start its buffer")
            self.sets.append(dict(part=part, out=out, h=h_out, mc_part=mc_part, mc_out=mc_out))
        self.calls = 0

    def own_rows(self, t: int):
        """(first row, row count) of the output block this rank owns for t rows."""
        r0 = self.rank * self.rows_per
        return r0, max(0, min(self.rows_per, t - r0))

    def __call__(self, attn_local, w_out, h0: int, h1: int, head_dim: int = 128, status=None,
                 residual=None, eps: float = 1e-6):
        """As ScatterOutProj.__call__ (residual=(x_own, gate, scale) folds in the block's
        attention residual and norm2, src/transformer.rs:411-421)."""
        import b200attn
        t = attn_local.shape[0]
        if t > self.rows or w_out.shape[0] != self.hidden:
            raise ValueError("shape does not fit the buffers")
        st = self.sets[self.calls % 2]
        self.calls += 1
        w_cols = w_out[:, h0 * head_dim:h1 * head_dim]
        b200attn.gemm(attn_local, w_cols, out=st["part"][:t], status=status)
        st["h"].barrier(channel=0, timeout_ms=self.timeout_ms)
        r0, mine = self.own_rows(t)
        if residual is None:
            b200attn.reduce_nvls(st["mc_part"], self.hidden, st["mc_out"], self.hidden, r0, mine,
                                 self.hidden)
        else:
            x_own, gate, scale = residual
            if x_own.shape[0] < mine or x_own.shape[1] != self.hidden:
                raise ValueError("x_own must hold this rank's rows of the residual stream")
            b200attn.reduce_nvls(st["mc_part"], self.hidden, st["mc_out"], self.hidden, r0, mine,
                                 self.hidden, x=x_own, gate=gate, scale=scale, eps=eps)
        st["h"].barrier(channel=0, timeout_ms=self.timeout_ms)
        return st["out"][:t]
