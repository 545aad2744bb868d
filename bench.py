#!/usr/bin/env python
"""Benchmark of the B200 joint-attention path (one JSON line on rank 0).

A step is the attention of one cached denoising step across all 32 MMDiT blocks at
1024^2 text-to-image (config 2): per block, 4096 image-token queries attend over the
block's 512-token prefix KV cache plus the step's 4096 image keys, 32 heads x 128, bf16.
Each block call is the public b200_attn_fwd (two launches: the Q/K RMSNorm+RoPE prologue
and the tcgen05 attention kernel); the timed region replays the step's 32 calls as one CUDA
graph (``--no-graph``: called one by one).  Right after it, under the same clock sampling,
the same step runs with the two launches called separately and CUDA events around every
attention launch: the roofline's kernel time.  ``e2e`` runs the step through b200_attn_fwd
with host (pinned) q/k/v copied in and the output copied out per block.

Multi-GPU (torchrun, one process per GPU): independent generations, data-parallel, no
collective on the data path (weak scaling); the barrier and a max-reduction of the
timings use NCCL.  ``--impl reference`` times the CPU restatement of the reference's
chunked attention (the reference is Rust/candle and cannot be built here) on the host.

Other workloads (``--config``): c1 and c3 are the same step at 512^2 and for a 1024^2
edit with a 10 624-token prefix; c4 is one head-sharded block at 2048^2 (attention of
32/N heads per rank, its share of to_out, the cross-rank sum — fused over NVLink or NCCL —
strong scaling); c5 is the 20-step denoising loop of 8 prompts x CFG (every block linear,
the attention, the Euler update; Q4_K_M weights by default; ms per step, strong scaling).
Each prints its own metric, and ``--impl reference`` prints the matching CPU arm.
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
    # the full 32-block denoising loop: 8 prompts (text lengths ~ U[64, 512]) x true CFG
    # = 16 sequences at 1024^2, data-parallel over ranks by prompt (pos/neg stay together)
    "c5": dict(grid=(64, 64), prompts=8, len_range=(64, 512), layers=32, cfg_scale=4.0,
               denoise_steps=20, name="1024^2 denoising loop, 8 prompts x CFG (config 5)"),
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


def attn_metric(config: str) -> str:
    """Metric name of the attention-step configs; config 2 is the headline."""
    if config == "c2":
        return METRIC
    return f"attn TFLOP/s, {CONFIGS[config]['name']}, 32 blocks per denoising step"
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
    ap.add_argument("--no-graph", action="store_true",
                    help="configs 1-3: launch the step's calls one by one instead of replaying "
                         "them as one CUDA graph")
    ap.add_argument("--weights", choices=["q4_k_m", "bf16"], default="q4_k_m",
                    help="config 5: block linears as GGUF Q4_K_M blocks (the config) or bf16")
    ap.add_argument("--prompts", type=int, default=None,
                    help="config 5: prompts in the batch (default 8; fewer only for profiling)")
    ap.add_argument("--gemm", choices=["cublas", "b200"], default="cublas",
                    help="config 5: the block linears' GEMM (cuBLAS or the tcgen05 kernel)")
    ap.add_argument("--fused-qkv", action="store_true",
                    help="config 5: Q/K/V projections with norm + RoPE in the GEMM epilogue")
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
def attn_step_config(cfg, L, world):
    """The `config` of the attention-step configs (1-3), shared by both arms."""
    T = cfg["grid"][0] * cfg["grid"][1]
    return {"workload": cfg["name"] + ", attention of 32 blocks per step",
            "T": T, "P": cfg["P"], "prefix_valid": cfg["pv"] if cfg["pv"] is not None else cfg["P"],
            "heads": HEADS, "head_dim": HEAD_DIM, "blocks_per_step": L, "batch": 1,
            "parallelism": f"dp{world} (independent generations)",
            "l2": "inputs exceed L2 (3.3 GB of per-block q/k/v/prefix per step)"}


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
        "impl": "reference", "metric": attn_metric(args.config), "value": value, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1))",
        "config": attn_step_config(cfg, args.layers or cfg["layers"], args.gpus),
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
        if args.config == "c5":
            run_reference_denoise(args, rank)
        elif args.config == "c4":
            run_reference_head_sharded(args, rank)
        else:
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
    if args.config == "c5":
        run_denoise(args, cfg, rank, world, dev)
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

    fwd_ws = torch.empty(2 * T * HEADS * HEAD_DIM * 2 + b200attn.SPLIT_WORKSPACE_BYTES + 512,
                         dtype=torch.uint8, device=dev)

    def step(s):
        """One denoising step's attention through the public call (b200_attn_fwd: the
        norm/RoPE prologue, then the attention kernel), block after block."""
        for ly in layers:
            b200attn.attention_forward(ly["q"], ly["k"], ly["v"], ly["pk"], ly["pv"], ones, ones,
                                       pe, desc=desc, out=out, workspace=fwd_ws, status=status,
                                       stream=s)

    def step_marked(marks):
        """The same step as b200_attn_fwd's two launches called one by one, with CUDA events
        around every attention launch (the roofline's kernel time)."""
        for li, ly in enumerate(layers):
            b200attn.qk_norm_rope(ly["q"], ly["k"], ones, ones, 1e-6, pe, q_rot, k_rot, stream=stream)
            marks[li][0].record(stream)
            b200attn.joint_attention(q_rot, k_rot, ly["v"], ly["pk"], ly["pv"], desc=desc, out=out,
                                     workspace=split_ws, status=status, stream=stream)
            marks[li][1].record(stream)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        step(stream)
    barrier()
    graph = None
    if not args.no_graph:
        # The whole step as one CUDA graph: the host work of the 32 calls (argument checks,
        # tensor maps) happens once at capture, and replay launches the kernels back to back.
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            step(side)
        stream.wait_stream(side)
        for _ in range(args.warmup):
            graph.replay()
        barrier()
    n_marked = max(1, min(args.steps, 20))
    marks = [[[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(L)]
             for _ in range(n_marked)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    with ClockSampler(uuid) as clocks:
        barrier()
        start.record(stream)
        for _ in range(args.steps):
            if graph is not None:
                graph.replay()
            else:
                step(stream)
        end.record(stream)
        barrier()
        # the attention kernel's launch time, same kernels and inputs, under the same clocks
        for s in range(n_marked):
            step_marked(marks[s])
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
        # Host q/k/v in, host output out, per block.  Copies run on their own streams
        # (host-to-device and device-to-host in parallel over PCIe), double-buffered
        # against the attention on `stream`: block i's inputs land while block i-1
        # computes and block i-2's output drains.
        nslot = 4
        host_in = [dict(q=ly["q"].cpu().pin_memory(), k=ly["k"].cpu().pin_memory(),
                        v=ly["v"].cpu().pin_memory()) for ly in layers[:nslot]]
        host_out = [torch.empty(T, HEADS * HEAD_DIM, dtype=torch.bfloat16).pin_memory()
                    for _ in range(2)]
        dev_in = [dict(q=torch.empty_like(layers[0]["q"]), k=torch.empty_like(layers[0]["q"]),
                       v=torch.empty_like(layers[0]["q"])) for _ in range(2)]
        dev_out = [torch.empty_like(out) for _ in range(2)]
        ws = torch.empty(2 * T * HEADS * HEAD_DIM * 2 + b200attn.SPLIT_WORKSPACE_BYTES + 512,
                         dtype=torch.uint8, device=dev)
        h2d_stream = torch.cuda.Stream(dev)
        d2h_stream = torch.cuda.Stream(dev)
        # per slot, the last recording: inputs landed / attention done / output home
        landed, computed, drained = ([torch.cuda.Event() for _ in range(2)] for _ in range(3))

        def e2e_step():
            for li, ly in enumerate(layers):
                sl = li % 2
                hi, di = host_in[li % nslot], dev_in[sl]
                with torch.cuda.stream(h2d_stream):
                    h2d_stream.wait_event(computed[sl])  # the slot's previous block is done
                    for name in ("q", "k", "v"):
                        di[name].copy_(hi[name], non_blocking=True)
                    landed[sl].record(h2d_stream)
                stream.wait_event(landed[sl])
                stream.wait_event(drained[sl])  # the slot's previous output is home
                b200attn.attention_forward(di["q"], di["k"], di["v"], ly["pk"], ly["pv"], ones,
                                           ones, pe, desc=desc, out=dev_out[sl], workspace=ws,
                                           status=status, stream=stream)
                computed[sl].record(stream)
                with torch.cuda.stream(d2h_stream):
                    d2h_stream.wait_event(computed[sl])
                    host_out[sl].copy_(dev_out[sl][0], non_blocking=True)
                    drained[sl].record(d2h_stream)
            stream.wait_event(drained[(len(layers) - 1) % 2])  # the last output is home

        e2e_step()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        h2d_stream.wait_event(e0)
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
            "metric": attn_metric(args.config), "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) q/k/v and prefix cache, weight-1 norms)",
            "config": attn_step_config(cfg, L, world),
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
                "path": ("b200_attn_fwd with pinned-host q/k/v in and output out per block; "
                         "copies on their own streams, double-buffered against the attention")},
            "clocks": clocks.summary(),
            "gpu_launches": args.steps * L * 2,
            "launch": ("one CUDA graph per step (32 b200_attn_fwd calls captured once, replayed)"
                       if graph is not None else "b200_attn_fwd called block by block"),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


C4_METRIC = "block TFLOP/s at 2048^2, head-sharded (attention + to_out + all-reduce)"


def c4_config(cfg, world):
    """The `config` of config 4, shared by both arms."""
    return {"workload": cfg["name"] + ", one block per step",
            "T": cfg["grid"][0] * cfg["grid"][1], "P": cfg["P"],
            "heads_per_gpu": HEADS // world, "head_dim": HEAD_DIM, "hidden": cfg["hidden"],
            "parallelism": f"heads/{world}; to_out partials summed over the ranks",
            "l2": "inputs exceed L2"}


def run_reference_head_sharded(args, rank):
    """Config 4 on the host cores: the C port of chunked_attention for a sample of heads and
    their share of to_out (numpy f32 GEMM), at the B200 arm's metric (block TFLOP/s)."""
    if rank != 0:
        return
    value, dt, n, threads, sample = c4_cpu_sample(args.cpu_heads, args.warmup, args.steps)
    print(json.dumps({
        "impl": "reference", "metric": C4_METRIC, "value": value, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": n, "warmup": args.warmup, "ms_per_step": dt * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1))", "config": c4_config(CONFIGS["c4"], args.gpus),
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def c4_cpu_sample(cpu_heads, warmup, steps):
    """The oracle C port of chunked_attention on a bounded sample of config 4 plus the
    sample's share of to_out (numpy f32 GEMM); returns (TFLOP/s, s per step, steps,
    threads, description)."""
    import numpy as np
    from oracle import cpu as ocpu  # CPU baseline leg (test / baseline infrastructure)
    cfg = CONFIGS["c4"]
    heads = max(1, min(cpu_heads, HEADS))
    t = cfg["grid"][0] * cfg["grid"][1]
    t_s = 2048  # query rows of the sample (of 16384), all keys
    rng = np.random.default_rng(9)
    bits = lambda shape: (rng.standard_normal(shape, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)
    q = bits((1, t_s, heads, HEAD_DIM))
    k, v = (bits((1, t, heads, HEAD_DIM)) for _ in range(2))
    pk, pv = (bits((1, heads, cfg["P"], HEAD_DIM)) for _ in range(2))
    w = np.ones(HEAD_DIM, np.float32)
    pe = np.tile(np.array([1.0, 0.0], np.float32), (t, HEAD_DIM // 2))
    w_out = (0.02 * rng.standard_normal((cfg["hidden"], heads * HEAD_DIM))).astype(np.float32)
    threads = os.cpu_count() or 1

    def one():
        # a t_s-token slice of the call (its queries, keys and values) against the prefix
        o = ocpu.attention_forward(q, k[:, :t_s], v[:, :t_s], pk, pv, w, w, 1e-6, pe[:t_s],
                                   None, HEAD_DIM ** -0.5, threads)
        return np.asarray(o, np.float32).reshape(t_s, heads * HEAD_DIM) @ w_out.T

    for _ in range(min(warmup, 1)):
        one()
    n = max(1, min(steps, 3))
    t0 = time.perf_counter()
    for _ in range(n):
        one()
    dt = (time.perf_counter() - t0) / n
    flops = 4.0 * heads * t_s * (t_s + cfg["P"]) * HEAD_DIM + 2.0 * t_s * heads * HEAD_DIM * cfg["hidden"]
    sample = (f"{heads} of 32 heads, {t_s} of {t} query rows against {t_s} + {cfg['P']} keys, "
              f"with their to_out share (oracle C port + numpy f32 GEMM), per step")
    return flops / dt / 1e12, dt, n, threads, sample


def run_head_sharded(args, cfg, rank, world, dev):
    """Config 4: each rank runs the attention of its 32/N heads and its share of to_out; a
    step is one block (strong scaling).  Two ways to sum the to_out partials are timed
    back to back: the fused one — the tcgen05 out-projection GEMM whose epilogue stores
    every partial tile into the rank owning its rows, then the owners' sum and broadcast
    (ScatterOutProj) — and a cuBLAS GEMM followed by an NCCL all-reduce.  `value` is the
    path dist.prefer_fused_out_proj picks for this rank count (both are reported).  On one
    GPU the step is the attention and a plain tcgen05 GEMM."""
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
    w_cols = w_out[:, h0 * HEAD_DIM:h1 * HEAD_DIM]
    lay = b200attn.joint_layout(P, None, [], (gh, gw))
    pe = torch.from_numpy(b200attn.rope_pe(lay["img_shapes"], lay["image_pad_mask"])[P:]).to(dev)
    ones = torch.ones(HEAD_DIM, device=dev, dtype=torch.float32)
    q_rot = torch.empty(1, hl, T, HEAD_DIM, dtype=torch.bfloat16, device=dev)
    k_rot = torch.empty_like(q_rot)
    attn = torch.empty(1, T, hl * HEAD_DIM, dtype=torch.bfloat16, device=dev)
    split_ws = torch.empty(b200attn.SPLIT_WORKSPACE_BYTES, dtype=torch.uint8, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    fused = None
    fused_note = "plain tcgen05 GEMM (one GPU)"
    if world > 1:
        try:
            fused = bdist.ScatterOutProj(T, hidden, dev)
            fused_note = ("tcgen05 GEMM whose epilogue reduce-scatters over NVLink + "
                          "owner sum / broadcast kernel")
        except RuntimeError as e:
            fused_note = f"no symmetric memory ({e}); fused path = NCCL path"
    use_fused = world == 1 or (fused is not None and bdist.prefer_fused_out_proj(world))
    out_bf16 = torch.empty(T, hidden, dtype=torch.bfloat16, device=dev)

    def attention(mark=None):
        b200attn.qk_norm_rope(q, k, ones, ones, 1e-6, pe, q_rot, k_rot, stream=stream)
        if mark is not None:
            mark[0].record(stream)
        b200attn.joint_attention(q_rot, k_rot, v, pk, pv, out=attn, workspace=split_ws,
                                 status=status, stream=stream)
        if mark is not None:
            mark[1].record(stream)
        return attn.view(T, hl * HEAD_DIM)

    def step_fused(mark=None):
        a = attention(mark)
        if fused is not None:
            return fused(a, w_out, h0, h1, status=status)
        if world == 1:
            return b200attn.gemm(a, w_cols, out=out_bf16, status=status)
        return step_nccl_tail(a)

    def step_nccl_tail(a):
        part = bdist.out_proj_partial(a, w_out, h0, h1, HEAD_DIM)
        bdist.allreduce_sum_(part)
        return part

    def step_nccl(mark=None):
        return step_nccl_tail(attention(mark))

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def timed(fn, steps, marks=None):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        e0.record(stream)
        for s_ in range(steps):
            fn(marks[s_] if marks is not None else None)
        e1.record(stream)
        barrier()
        return e0.elapsed_time(e1) / steps

    for _ in range(args.warmup):
        step_fused()
        step_nccl()
    barrier()
    marks = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    with ClockSampler(uuid) as clocks:
        ms_fused = timed(step_fused, args.steps, marks)
    attn_ms = sum(m[0].elapsed_time(m[1]) for m in marks) / args.steps
    ms_nccl = timed(step_nccl, args.steps)
    if int(status.item()) != 0:
        raise RuntimeError(f"device wait ran out during the bench (status {int(status.item())})")
    # ---- end to end through the public calls with host buffers: this rank's q/k/v of a
    # block copied in (host-to-device stream), b200_attn_fwd + to_out + the sum of the
    # partials on the compute stream, the block's output copied out (device-to-host
    # stream), double-buffered across steps.
    e2e = None
    if args.e2e_steps > 0:
        host_in = dict(q=q.cpu().pin_memory(), k=k.cpu().pin_memory(), v=v.cpu().pin_memory())
        dev_in = [dict(q=torch.empty_like(q), k=torch.empty_like(k), v=torch.empty_like(v))
                  for _ in range(2)]
        host_out = [torch.empty(T, hidden, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
        gemm_out = [torch.empty(T, hidden, dtype=torch.bfloat16, device=dev) for _ in range(2)]
        fwd_ws = torch.empty(2 * T * hl * HEAD_DIM * 2 + b200attn.SPLIT_WORKSPACE_BYTES + 512,
                             dtype=torch.uint8, device=dev)
        h2d_s, d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        landed, computed, drained = ([torch.cuda.Event() for _ in range(2)] for _ in range(3))

        def e2e_step(i):
            sl = i % 2
            di = dev_in[sl]
            with torch.cuda.stream(h2d_s):
                h2d_s.wait_event(computed[sl])
                for name in ("q", "k", "v"):
                    di[name].copy_(host_in[name], non_blocking=True)
                landed[sl].record(h2d_s)
            stream.wait_event(landed[sl])
            stream.wait_event(drained[sl])
            a = b200attn.attention_forward(di["q"], di["k"], di["v"], pk, pv, ones, ones, pe,
                                           out=attn, workspace=fwd_ws, status=status,
                                           stream=stream).view(T, hl * HEAD_DIM)
            if fused is not None and use_fused:
                res = fused(a, w_out, h0, h1, status=status)
            elif world == 1:
                res = b200attn.gemm(a, w_cols, out=gemm_out[sl], status=status)
            else:
                res = step_nccl_tail(a)
            res.record_stream(d2h_s)  # the copy-out stream still reads it
            computed[sl].record(stream)
            with torch.cuda.stream(d2h_s):
                d2h_s.wait_event(computed[sl])
                host_out[sl].copy_(res.view(T, hidden), non_blocking=True)
                drained[sl].record(d2h_s)

        for i in range(2):
            e2e_step(i)
        barrier()
        n_e2e = max(args.e2e_steps, 2)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        h2d_s.wait_event(e0)
        for i in range(n_e2e):
            e2e_step(i)
        stream.wait_event(drained[(n_e2e - 1) % 2])
        e1.record(stream)
        barrier()
        e2e = dict(ms=e0.elapsed_time(e1) / n_e2e, h2d=3 * T * hl * HEAD_DIM * 2,
                   d2h=T * hidden * 2)
    ms_fused = bdist.max_over_ranks(ms_fused, device=dev)
    ms_nccl = bdist.max_over_ranks(ms_nccl, device=dev)
    e2e_ms = bdist.max_over_ranks(e2e["ms"], device=dev) if e2e else None
    ms_step = ms_fused if use_fused else ms_nccl
    attn_ms = bdist.max_over_ranks(attn_ms, device=dev)
    attn_flops = 4.0 * HEADS * T * (P + T) * HEAD_DIM
    proj_flops = 2.0 * T * HEADS * HEAD_DIM * hidden
    if rank == 0:
        pk_d, src = peaks()
        peak = float(pk_d.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
        achieved = attn_flops * hl / HEADS / (attn_ms / 1e3) / 1e12
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            value_c, _, _, threads_c, sample_c = c4_cpu_sample(args.cpu_heads, 1, 1)
            cpu = {"value": value_c, "unit": "TFLOP/s", "cores": threads_c, "kind": "port",
                   "sample": sample_c}
        line = {
            "metric": C4_METRIC,
            "value": (attn_flops + proj_flops) / (ms_step / 1e3) / 1e12, "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) q/k/v and prefix cache, N(0,0.02) to_out)",
            "config": c4_config(cfg, world),
            "sum_of_partials": (fused_note if use_fused else
                                "cuBLAS + NCCL all-reduce (faster than the fused path at this "
                                "rank count)"),
            "nccl_path": {"ms_per_step": ms_nccl,
                          "value": (attn_flops + proj_flops) / (ms_nccl / 1e3) / 1e12,
                          "how": "cuBLAS to_out partial + NCCL all-reduce (bf16)"},
            "fused_path": {"ms_per_step": ms_fused, "how": fused_note},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak,
                         # captured with all 32 heads on one GPU; a rank's launch moves its
                         # heads' share (traffic grows in proportion to the heads)
                         "traffic": (None if profile_traffic("joint_attn_kernel", "c4") is None
                                     else profile_traffic("joint_attn_kernel", "c4") * hl / HEADS),
                         "kernel": "joint_attn_kernel",
                         "peak_source": f"{src} bf16_tflops_sustained", "launch_ms": attn_ms},
            "cpu_baseline": cpu, "clocks": clocks.summary(),
            "e2e": None if e2e is None else {
                "value": (attn_flops + proj_flops) / (e2e_ms / 1e3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"],
                "ms_per_step": e2e_ms,
                "path": ("b200_attn_fwd + to_out + sum of partials with this rank's pinned-host "
                         "q/k/v in and the block output out; copies on their own streams, "
                         "double-buffered")},
            "gpu_launches": args.steps * (4 if world > 1 and use_fused else 2 if world > 1 else 3),
        }
        print(json.dumps(line), flush=True)
    del fused
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# --------------------------------------------------------------------------- config 5
C5_METRIC = "denoise-step ms at 1024^2 (config 5: 16 sequences = 8 prompts x CFG, 32 blocks)"


def c5_workload(cfg):
    """Seeded prompt lengths (pos, neg) of the 8 prompts, uniform in [64, 512]."""
    import numpy as np
    rng = np.random.default_rng(5)
    lo, hi = cfg["len_range"]
    return [(int(a), int(b)) for a, b in rng.integers(lo, hi + 1, size=(cfg["prompts"], 2))]


def c5_config(cfg, args, world):
    """The `config` of config 5, shared by both arms."""
    mcfg_ = None
    try:
        from b200attn import mmdit
        mcfg_ = mmdit.MMDiTConfig()
    except ImportError:
        pass
    return {"workload": cfg["name"], "T": cfg["grid"][0] * cfg["grid"][1],
            "prompts": cfg["prompts"], "sequences": 2 * cfg["prompts"],
            "prompt_lengths": c5_workload(cfg),
            "blocks": args.layers or cfg["layers"], "hidden": getattr(mcfg_, "hidden", 4096),
            "ffn": getattr(mcfg_, "ffn", 12288), "weights": args.weights,
            "cfg_scale": cfg["cfg_scale"],
            "gemm": args.gemm + (" + fused QKV/norm/RoPE" if args.fused_qkv else ""),
            "parallelism": f"dp{world} by prompt (pos/neg pairs together)",
            "l2": "every step streams GBs of weights and activations (> L2)"}


def c5_flops(model_cfg, lengths, T):
    """GEMM + attention FLOPs of one cached step of the given sequences."""
    lin = model_cfg.linear_flops_per_token() * T * len(lengths)
    lin += 2.0 * T * len(lengths) * model_cfg.hidden * model_cfg.in_channels * 2  # img_in, proj_out
    attn = sum(4.0 * model_cfg.heads * T * (n + T) * HEAD_DIM for n in lengths) * model_cfg.layers
    return lin, attn


def run_denoise(args, cfg, rank, world, dev):
    """Config 5: every rank runs the denoising loop of its prompts (both CFG branches),
    batched through each block; a step is one Euler step of this rank's sequences.  Strong
    scaling: the 8 prompts are split over the ranks; value = max over ranks of ms/step."""
    import torch
    import torch.distributed as dist

    from b200attn import dist as bdist
    from b200attn import mmdit

    gh, gw = cfg["grid"]
    T = gh * gw
    mcfg = mmdit.MMDiTConfig(layers=args.layers or cfg["layers"])
    if args.prompts:
        cfg = dict(cfg, prompts=args.prompts)
    pairs = c5_workload(cfg)
    mine = bdist.dp_assign(list(range(cfg["prompts"])), world, rank)
    lengths = [n for p in mine for n in pairs[p]]          # p0 pos, p0 neg, p1 pos, ...
    weights = mmdit.random_weights(mcfg, 2024, device=dev, std=0.02)   # same on every rank
    model = mmdit.MMDiT(mcfg, weights, device=dev, weight_format=args.weights,
                        fused_qkv=args.fused_qkv, gemm=args.gemm)
    del weights
    torch.cuda.empty_cache()
    wbytes = model.weight_bytes()
    g = torch.Generator(device=dev).manual_seed(77)
    embs = [torch.randn(n, mcfg.text_dim, generator=g, device=dev).to(torch.bfloat16)
            for p in range(cfg["prompts"]) for n in pairs[p]]
    embs = [embs[2 * p + j] for p in mine for j in range(2)]
    noise = torch.randn(cfg["prompts"], T, mcfg.in_channels, generator=g, device=dev)[mine]
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    # prefix fill (once per prompt, outside the step) and the step's fixed inputs
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    cache = model.prefix_fill(embs)
    f1.record(stream)
    pe = model.target_pe(cache.lengths, (gh, gw))
    desc = mmdit.cached_desc(cache, T, dev)
    sig = mmdit.flow_match_sigmas(cfg["denoise_steps"], T)
    lat = noise.clone()

    def step(i):
        nonlocal lat
        k = i % cfg["denoise_steps"]
        pred = model.step(lat.repeat_interleave(2, 0), float(sig[k]), cache, pe, desc)
        pos, neg = pred[0::2], pred[1::2]
        lat = lat + (neg + (pos - neg) * cfg["cfg_scale"]) * mmdit.euler_dt(sig, k)

    for i in range(args.warmup):
        step(i)
    barrier()
    prefix_ms = f0.elapsed_time(f1)
    model.attn_marks = []
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    with ClockSampler(uuid) as clocks:
        barrier()
        e0.record(stream)
        for i in range(args.steps):
            step(args.warmup + i)
        e1.record(stream)
        barrier()
    marks, model.attn_marks = model.attn_marks, None
    ms_rank = e0.elapsed_time(e1) / args.steps
    attn_ms_rank = sum(a.elapsed_time(b) for a, b in marks) / args.steps
    if not torch.isfinite(lat).all():
        raise RuntimeError("non-finite latents in the denoising loop")

    # ---- end to end: the public denoise() call from host prompt embeddings and noise to
    # host latents, prefix fill included, over the full 20-step schedule
    e2e = None
    if args.e2e_steps > 0:
        host_embs = [e.cpu().pin_memory() for e in embs]
        host_noise = noise.cpu().pin_memory()
        n_steps = cfg["denoise_steps"]
        barrier()
        e0.record(stream)
        out = mmdit.denoise(model, host_embs[0::2], host_embs[1::2], (gh, gw), n_steps,
                            cfg["cfg_scale"], host_noise)
        host_lat = out.cpu()
        e1.record(stream)
        barrier()
        e2e_rank = e0.elapsed_time(e1) / n_steps
        h2d = sum(e.numel() * 2 for e in host_embs) + host_noise.numel() * 4
        e2e = dict(ms=e2e_rank, h2d=h2d, d2h=host_lat.numel() * 4, steps=n_steps)

    vals = torch.tensor([ms_rank, attn_ms_rank, prefix_ms, e2e["ms"] if e2e else 0.0],
                        dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms_step, attn_ms, prefix_ms_max, e2e_ms = (float(v) for v in vals)
    all_lengths = [n for p in range(cfg["prompts"]) for n in pairs[p]]
    lin_f, attn_f = c5_flops(mcfg, all_lengths, T)
    my_lin, my_attn = c5_flops(mcfg, lengths, T)
    if rank == 0:
        pk_d, src = peaks()
        peak = float(pk_d.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
        attn_achieved = my_attn / (attn_ms_rank / 1e3) / 1e12
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline_denoise(cfg, all_lengths)
        line = {
            "metric": C5_METRIC, "value": ms_step, "unit": "ms", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init N(0,0.02) weights"
                    + (" quantised to GGUF Q4_K_M" if args.weights == "q4_k_m" else " in bf16")
                    + ", seeded N(0,1) prompt embeddings and noise)",
            "config": c5_config(cfg, args, world),
            "weight_bytes": {"block_linears": wbytes, "note": "7.1 B parameters"},
            "step_tflops": (lin_f + attn_f) / (ms_step / 1e3) / 1e12,
            "pct_bf16_peak": 100.0 * (lin_f + attn_f) / world / (ms_step / 1e3) / 1e12 / peak,
            "attention_ms_per_step": attn_ms, "attention_share": attn_ms / ms_step,
            "prefix_fill_ms": prefix_ms_max,
            "roofline": {"bound": "tensor", "achieved": attn_achieved, "peak": peak,
                         "unit": "TFLOP/s", "frac": attn_achieved / peak, "traffic": None,
                         "kernel": "b200_attn_fwd span (norm_rope + joint_attn_kernel) in the loop",
                         "peak_source": f"{src} bf16_tflops_sustained"},
            "cpu_baseline": cpu,
            "e2e": None if e2e is None else {
                "value": e2e_ms, "unit": "ms", "h2d_bytes_per_step": e2e["h2d"] // e2e["steps"],
                "d2h_bytes_per_step": e2e["d2h"] // e2e["steps"],
                "path": "mmdit.denoise(): host embeddings + noise in, prefix fill, 20 steps, "
                        "host latents out; ms per step"},
            "clocks": clocks.summary(),
            # per block: 2 residual/norm kernels, 2 attention launches, 1 swiglu per MLP
            # chunk, 6 dequantisations (q4_k_m); plus block 0's norm1 (GEMMs are cuBLAS,
            # not counted)
            "gpu_launches": args.steps * (mcfg.layers * (4 + (6 if args.weights == "q4_k_m" else 0)
                                                         + -(-T * len(lengths) // model.mlp_chunk_rows)) + 1),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _denoise_cpu_sample(cfg, length):
    """Seconds of one cached block of one sequence at full width on the host's cores, with
    the float32 oracle (a 1-block model; weights N(0, 0.02))."""
    import torch
    from b200attn import mmdit
    from oracle import mmdit_ref as M  # CPU baseline leg (test / baseline infrastructure)
    torch.set_num_threads(os.cpu_count() or 1)
    gh, gw = cfg["grid"]
    one = mmdit.MMDiTConfig(layers=1)
    R = M.Reference(mmdit.random_weights(one, 1), one.layers, one.heads)
    g = torch.Generator().manual_seed(3)
    emb = torch.randn(length, one.text_dim, generator=g)
    lat = torch.randn(gh * gw, one.in_channels, generator=g)
    cache = R.prefix_kv(emb, (gh, gw))
    R.forward_cached(lat[:256], 0.5, cache, length, (16, 16))  # warm the thread pool
    t0 = time.perf_counter()
    R.forward_cached(lat, 0.5, cache, length, (gh, gw))
    return time.perf_counter() - t0


def cpu_baseline_denoise(cfg, lengths):
    """The float32 oracle on the host: one block of one mean-length sequence, scaled to a
    step of 16 sequences x 32 blocks."""
    n = int(round(sum(lengths) / len(lengths)))
    dt = _denoise_cpu_sample(cfg, n)
    ms = dt * 1e3 * len(lengths) * CONFIGS["c5"]["layers"]
    return {"value": ms, "unit": "ms", "cores": os.cpu_count() or 1, "kind": "port",
            "sample": f"1 of 32 blocks of 1 of {len(lengths)} sequences (prompt {n} tokens, "
                      f"{dt:.1f} s, float32 torch oracle), scaled x{len(lengths) * 32}"}


def run_reference_denoise(args, rank):
    """Config 5 on the host cores with the float32 oracle (bounded sample, see above)."""
    if rank != 0:
        return
    cfg = CONFIGS["c5"]
    lengths = [n for pair in c5_workload(cfg) for n in pair]
    n = int(round(sum(lengths) / len(lengths)))
    for _ in range(min(args.warmup, 1)):
        _denoise_cpu_sample(cfg, n)
    samples = [_denoise_cpu_sample(cfg, n) for _ in range(max(1, min(args.steps, 3)))]
    ms = statistics.median(samples) * 1e3 * len(lengths) * cfg["layers"]
    sample = (f"1 of 32 blocks of 1 of {len(lengths)} sequences per step (prompt {n} tokens, "
              f"float32 torch oracle), scaled x{len(lengths) * 32}")
    print(json.dumps({
        "impl": "reference", "metric": C5_METRIC, "value": ms, "unit": "ms",
        "n_gpus": args.gpus, "steps": len(samples), "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (random-init weights, seeded embeddings and noise)",
        "config": c5_config(cfg, args, args.gpus),
        "cpu_baseline": {"value": ms, "unit": "ms", "cores": os.cpu_count() or 1, "kind": "port",
                         "sample": sample},
        "e2e": {"value": ms, "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


if __name__ == "__main__":
    main()
