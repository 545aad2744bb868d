#!/usr/bin/env python
"""Benchmark of the B200 joint-attention path (one JSON line on rank 0).

A step is the attention of one cached denoising step across all 32 MMDiT blocks at
1024^2 text-to-image (config 2): per block, 4096 image-token queries attend over the
block's 512-token prefix KV cache plus the step's 4096 image keys, 32 heads x 128, bf16.
Each block call is the public path's two launches — the Q/K RMSNorm+RoPE prologue and
the tcgen05 attention kernel (exactly what b200_attn_fwd launches) — with CUDA events
around the attention launch for the roofline.  ``e2e`` runs the same step through
b200_attn_fwd with host (pinned) q/k/v copied in and the output copied out per block.

Multi-GPU (torchrun, one process per GPU): independent generations, data-parallel, no
collective on the data path (weak scaling); the barrier and a max-reduction of the
timings use NCCL.  ``--impl reference`` times the CPU restatement of the reference's
chunked attention (the reference is Rust/candle and cannot be built here) on the host.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "qwen3-image21_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

HEADS, HEAD_DIM = 32, 128
CONFIGS = {
    # target grid, prefix length, valid prefix keys, blocks per step, condition images
    "c1": dict(grid=(32, 32), P=256, pv=None, layers=32, cond=[], name="512^2 T2I (config 1)"),
    "c2": dict(grid=(64, 64), P=512, pv=None, layers=32, cond=[], name="1024^2 T2I (config 2)"),
    # two 64x64-latent condition images fill 2 x 1024 prompt slots (4 latent tokens per slot)
    # plus 2432 other prompt tokens: a 10624-token prefix with its last 37 keys padded
    "c3": dict(grid=(64, 64), P=10624, pv=10587, layers=32, cond=[(64, 64), (64, 64)],
               name="1024^2 edit, 2 refs (config 3)"),
    # 2048^2: heads sharded 32/N per GPU, to_out partial sums all-reduced (one block per step)
    "c4": dict(grid=(128, 128), P=512, pv=None, layers=1, cond=[], hidden=4096,
               name="2048^2 T2I, head-sharded (config 4)"),
}


def prompt_layout(cfg):
    """(text_len, image-slot mask, condition shapes) whose joint prefix has cfg['P'] tokens."""
    cond = cfg["cond"]
    image_tokens = sum(h * w for h, w in cond)
    other = cfg["P"] - image_tokens
    if not cond:
        return other, None, []
    slots = []
    lead = min(100, other // (len(cond) + 1))
    used = 0
    for h, w in cond:
        slots += [False] * lead + [True] * (h * w // 4)
        used += lead
    slots += [False] * (other - used)
    return len(slots), slots, cond
METRIC = "attn TFLOP/s at 1024^2 (config 2), 32 blocks per denoising step"
FALLBACK_PEAKS = dict(bf16_tflops=1590.0, bf16_tflops_sustained=1400.0, hbm_gbs=6650.0)


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="c2")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--layers", type=int, default=None,
                    help="blocks per step (default 32; fewer only for profiling runs)")
    ap.add_argument("--cpu-heads", type=int, default=4, help="heads in the CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


def flops_per_call(cfg, heads=HEADS):
    t = cfg["grid"][0] * cfg["grid"][1]
    lk = (cfg["pv"] if cfg["pv"] is not None else cfg["P"]) + t
    return 4.0 * heads * t * lk * HEAD_DIM


def profile_traffic(kernel: str, workload: str):
    """DRAM bytes per launch of `kernel` from the committed ncu summary, or None."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d[kernel][workload]["dram_bytes_per_launch"]
    except (OSError, KeyError, ValueError):
        return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu_id, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in (self.out or "").strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) != 8:
                continue
            try:
                rows.append(dict(sm=float(parts[0]), max=float(parts[1]), power=float(parts[2]),
                                 hw=parts[4], hwt=parts[5], swt=parts[6], pcap=parts[7]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        busy = [r for r in rows if r["power"] > 300] or rows
        reasons = set()
        for r in busy:
            for key, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"),
                              ("swt", "sw_thermal_slowdown"), ("pcap", "sw_power_cap")):
                if r[key].lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in busy),
                "sm_max_mhz": max(r["max"] for r in rows), "reasons": sorted(reasons),
                "samples": len(busy), "power_w_max": max(r["power"] for r in rows)}


# --------------------------------------------------------------------------- reference
def run_reference(args, rank):
    """The CPU restatement of the reference's chunked attention, timed on the host."""
    if rank != 0:
        return
    import numpy as np
    from oracle import cpu as ocpu  # CPU baseline leg (test / baseline infrastructure)
    cfg = CONFIGS[args.config]
    heads = max(1, min(args.cpu_heads, HEADS))
    t = cfg["grid"][0] * cfg["grid"][1]
    rng = np.random.default_rng(7)
    bits = lambda shape: (rng.standard_normal(shape, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)
    q, k, v = (bits((1, t, heads, HEAD_DIM)) for _ in range(3))
    pk, pv = (bits((1, heads, cfg["P"], HEAD_DIM)) for _ in range(2))
    w = np.ones(HEAD_DIM, np.float32)
    pe = np.tile(np.array([1.0, 0.0], np.float32), (t, HEAD_DIM // 2))
    prefix_valid = None if cfg["pv"] is None else np.array([cfg["pv"]], np.int32)
    threads = os.cpu_count() or 1

    def one():
        ocpu.attention_forward(q, k, v, pk, pv, w, w, 1e-6, pe, prefix_valid, HEAD_DIM ** -0.5, threads)

    for _ in range(args.warmup):
        one()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one()
    dt = (time.perf_counter() - t0) / max(args.steps, 1)
    value = flops_per_call(cfg, heads) / dt / 1e12
    sample = f"1 of 32 blocks, {heads} of 32 heads of {cfg['name']} per step (oracle C port, f32)"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1))",
        "config": {"workload": f"{cfg['name']} sample", "T": t, "P": cfg["P"], "heads": heads,
                   "head_dim": HEAD_DIM},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline(cfg, heads):
    """Oracle C port on this host's cores: one block, `heads` heads of the workload."""
    import numpy as np
    from oracle import cpu as ocpu  # CPU baseline leg (test / baseline infrastructure)
    t = cfg["grid"][0] * cfg["grid"][1]
    rng = np.random.default_rng(3)
    bits = lambda shape: (rng.standard_normal(shape, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)
    q, k, v = (bits((1, t, heads, HEAD_DIM)) for _ in range(3))
    pk, pv = (bits((1, heads, cfg["P"], HEAD_DIM)) for _ in range(2))
    w = np.ones(HEAD_DIM, np.float32)
    pe = np.tile(np.array([1.0, 0.0], np.float32), (t, HEAD_DIM // 2))
    prefix_valid = None if cfg["pv"] is None else np.array([cfg["pv"]], np.int32)
    threads = os.cpu_count() or 1
    ocpu.attention_forward(q[:, :128], k[:, :128], v[:, :128], pk, pv, w, w, 1e-6, pe[:128],
                           prefix_valid, HEAD_DIM ** -0.5, threads)  # warm the thread pool
    t0 = time.perf_counter()
    ocpu.attention_forward(q, k, v, pk, pv, w, w, 1e-6, pe, prefix_valid, HEAD_DIM ** -0.5, threads)
    dt = time.perf_counter() - t0
    return {"value": flops_per_call(cfg, heads) / dt / 1e12, "unit": "TFLOP/s", "cores": threads,
            "kind": "port",
            "sample": f"1 of 32 blocks, {heads} of 32 heads of {cfg['name']} ({dt:.1f} s, f32 C port "
                      f"of chunked_attention, OpenMP)"}


# --------------------------------------------------------------------------- B200 arm
def main():
    args = parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return

    import numpy as np
    import torch
    import torch.distributed as dist

    import b200attn
    from b200attn import dist as bdist

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    cfg = CONFIGS[args.config]
    if args.config == "c4":
        run_head_sharded(args, cfg, rank, world, dev)
        return
    gh, gw = cfg["grid"]
    T, P, L = gh * gw, cfg["P"], args.layers or cfg["layers"]

    # ---- synthetic workload (independent generation per rank), resident in HBM
    g = torch.Generator(device=dev).manual_seed(1234 + 2 + 1000 * rank)
    randn = lambda *shape: torch.randn(*shape, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    text_len, slots, cond = prompt_layout(cfg)
    lay = b200attn.joint_layout(text_len, slots, cond, (gh, gw))
    assert lay["prefix_len"] == P
    pe = torch.from_numpy(b200attn.rope_pe(lay["img_shapes"], lay["image_pad_mask"])[P:]).to(dev)
    ones = torch.ones(HEAD_DIM, device=dev, dtype=torch.float32)
    layers = []
    for _ in range(L):
        layers.append(dict(q=randn(1, T, HEADS, HEAD_DIM), k=randn(1, T, HEADS, HEAD_DIM),
                           v=randn(1, T, HEADS, HEAD_DIM), pk=randn(1, HEADS, P, HEAD_DIM),
                           pv=randn(1, HEADS, P, HEAD_DIM)))
    desc = None
    if cfg["pv"] is not None:
        desc = torch.tensor([[cfg["pv"], T]], dtype=torch.int32, device=dev)
    q_rot = torch.empty(1, HEADS, T, HEAD_DIM, dtype=torch.bfloat16, device=dev)
    k_rot = torch.empty_like(q_rot)
    out = torch.empty(1, T, HEADS * HEAD_DIM, dtype=torch.bfloat16, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    split_ws = torch.empty(b200attn.SPLIT_WORKSPACE_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step(marks=None):
        for li, ly in enumerate(layers):
            b200attn.qk_norm_rope(ly["q"], ly["k"], ones, ones, 1e-6, pe, q_rot, k_rot, stream=stream)
            if marks is not None:
                marks[li][0].record(stream)
            b200attn.joint_attention(q_rot, k_rot, ly["v"], ly["pk"], ly["pv"], desc=desc, out=out,
                                     workspace=split_ws, status=status, stream=stream)
            if marks is not None:
                marks[li][1].record(stream)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        step()
    barrier()
    marks = [[[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(L)]
             for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    with ClockSampler(uuid) as clocks:
        barrier()
        start.record(stream)
        for s in range(args.steps):
            step(marks[s])
        end.record(stream)
        barrier()
    ms_total = start.elapsed_time(end)
    attn_ms = [m[0].elapsed_time(m[1]) for st in marks for m in st]
    if int(status.item()) != 0:
        raise RuntimeError(f"device wait ran out during the bench (status {int(status.item())})")

    # ---- end to end through the public API with host buffers
    e2e_ms = None
    h2d = L * 3 * T * HEADS * HEAD_DIM * 2
    d2h = L * T * HEADS * HEAD_DIM * 2
    if args.e2e_steps > 0:
        nslot = 4
        host_in = [dict(q=ly["q"].cpu().pin_memory(), k=ly["k"].cpu().pin_memory(),
                        v=ly["v"].cpu().pin_memory()) for ly in layers[:nslot]]
        host_out = torch.empty(T, HEADS * HEAD_DIM, dtype=torch.bfloat16).pin_memory()
        dq = torch.empty_like(layers[0]["q"])
        dk = torch.empty_like(dq)
        dv = torch.empty_like(dq)
        ws = torch.empty(2 * T * HEADS * HEAD_DIM * 2 + b200attn.SPLIT_WORKSPACE_BYTES + 512,
                         dtype=torch.uint8, device=dev)

        def e2e_step():
            for li, ly in enumerate(layers):
                hi = host_in[li % nslot]
                dq.copy_(hi["q"], non_blocking=True)
                dk.copy_(hi["k"], non_blocking=True)
                dv.copy_(hi["v"], non_blocking=True)
                b200attn.attention_forward(dq, dk, dv, ly["pk"], ly["pv"], ones, ones, pe, desc=desc,
                                           out=out, workspace=ws, status=status, stream=stream)
                host_out.copy_(out[0], non_blocking=True)

        e2e_step()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.e2e_steps):
            e2e_step()
        e1.record(stream)
        barrier()
        e2e_ms = e0.elapsed_time(e1) / args.e2e_steps

    # ---- max over ranks
    vals = torch.tensor([ms_total, e2e_ms or 0.0], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms_total, e2e_ms_max = float(vals[0]), float(vals[1])
    ms_step = ms_total / args.steps
    step_flops = flops_per_call(cfg) * L
    value = step_flops * world / (ms_step / 1e3) / 1e12

    if rank == 0:
        pk_d, src = peaks()
        peak = float(pk_d.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
        attn_avg_ms = sum(attn_ms) / len(attn_ms)
        achieved = flops_per_call(cfg) / (attn_avg_ms / 1e3) / 1e12
        traffic = profile_traffic("joint_attn_kernel", args.config)
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline(cfg, max(1, min(args.cpu_heads, HEADS)))
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) q/k/v and prefix cache, weight-1 norms)",
            "config": {"workload": cfg["name"] + ", attention of 32 blocks per step",
                       "T": T, "P": P, "prefix_valid": cfg["pv"] if cfg["pv"] is not None else P,
                       "heads": HEADS, "head_dim": HEAD_DIM, "blocks_per_step": L, "batch": 1,
                       "parallelism": f"dp{world} (independent generations)",
                       "l2": "inputs exceed L2 (3.3 GB of per-block q/k/v/prefix per step)"},
            "pct_bf16_peak": 100.0 * value / world / peak,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "kernel": "joint_attn_kernel", "peak_source": f"{src} bf16_tflops_sustained",
                         "launch_ms": attn_avg_ms},
            "cpu_baseline": cpu,
            "e2e": None if e2e_ms is None else {
                "value": step_flops * world / (e2e_ms_max / 1e3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": e2e_ms_max,
                "path": "b200_attn_fwd with pinned-host q/k/v in and output out per block"},
            "clocks": clocks.summary(),
            "gpu_launches": args.steps * L * 2,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_head_sharded(args, cfg, rank, world, dev):
    """Config 4: each rank runs the attention of its 32/N heads, its share of to_out, and
    one NCCL all-reduce of the partial sums; a step is one block (strong scaling)."""
    import torch
    import torch.distributed as dist

    import b200attn
    from b200attn import dist as bdist

    gh, gw = cfg["grid"]
    T, P, hidden = gh * gw, cfg["P"], cfg["hidden"]
    h0, h1 = bdist.head_shard(HEADS, world, rank)
    hl = h1 - h0
    g = torch.Generator(device=dev).manual_seed(4321 + rank)
    randn = lambda *shape: torch.randn(*shape, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    q, k, v = randn(1, T, hl, HEAD_DIM), randn(1, T, hl, HEAD_DIM), randn(1, T, hl, HEAD_DIM)
    pk, pv = randn(1, hl, P, HEAD_DIM), randn(1, hl, P, HEAD_DIM)
    gw_ = torch.Generator(device=dev).manual_seed(99)  # to_out weights identical on every rank
    w_out = (0.02 * torch.randn(hidden, HEADS * HEAD_DIM, generator=gw_, device=dev)).to(torch.bfloat16)
    lay = b200attn.joint_layout(P, None, [], (gh, gw))
    pe = torch.from_numpy(b200attn.rope_pe(lay["img_shapes"], lay["image_pad_mask"])[P:]).to(dev)
    ones = torch.ones(HEAD_DIM, device=dev, dtype=torch.float32)
    q_rot = torch.empty(1, hl, T, HEAD_DIM, dtype=torch.bfloat16, device=dev)
    k_rot = torch.empty_like(q_rot)
    attn = torch.empty(1, T, hl * HEAD_DIM, dtype=torch.bfloat16, device=dev)
    split_ws = torch.empty(b200attn.SPLIT_WORKSPACE_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step(mark=None):
        b200attn.qk_norm_rope(q, k, ones, ones, 1e-6, pe, q_rot, k_rot, stream=stream)
        if mark is not None:
            mark[0].record(stream)
        b200attn.joint_attention(q_rot, k_rot, v, pk, pv, out=attn, workspace=split_ws,
                                 stream=stream)
        if mark is not None:
            mark[1].record(stream)
        part = bdist.out_proj_partial(attn.view(T, hl * HEAD_DIM), w_out, h0, h1, HEAD_DIM)
        bdist.allreduce_sum_(part)
        return part

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        step()
    barrier()
    marks = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    with ClockSampler(uuid) as clocks:
        barrier()
        e0.record(stream)
        for s_ in range(args.steps):
            step(marks[s_])
        e1.record(stream)
        barrier()
    ms_step = bdist.max_over_ranks(e0.elapsed_time(e1) / args.steps, device=dev)
    attn_ms = bdist.max_over_ranks(sum(m[0].elapsed_time(m[1]) for m in marks) / args.steps, device=dev)
    attn_flops = 4.0 * HEADS * T * (P + T) * HEAD_DIM
    proj_flops = 2.0 * T * HEADS * HEAD_DIM * hidden
    if rank == 0:
        pk_d, src = peaks()
        peak = float(pk_d.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
        achieved = attn_flops * hl / HEADS / (attn_ms / 1e3) / 1e12
        line = {
            "metric": "block TFLOP/s at 2048^2, head-sharded (attention + to_out + all-reduce)",
            "value": (attn_flops + proj_flops) / (ms_step / 1e3) / 1e12, "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) q/k/v and prefix cache, N(0,0.02) to_out)",
            "config": {"workload": cfg["name"] + ", one block per step", "T": T, "P": P,
                       "heads_per_gpu": hl, "head_dim": HEAD_DIM, "hidden": hidden,
                       "parallelism": f"heads/{world} + NCCL all-reduce of to_out partials",
                       "l2": "inputs exceed L2"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": None, "kernel": "joint_attn_kernel",
                         "peak_source": f"{src} bf16_tflops_sustained", "launch_ms": attn_ms},
            "cpu_baseline": None, "e2e": None, "clocks": clocks.summary(),
            "gpu_launches": args.steps * 2,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
