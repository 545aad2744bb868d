#!/usr/bin/env python
"""Benchmark of the B200 joint-attention path (one JSON line on rank 0).

A step is the attention of one cached denoising step across all 32 MMDiT blocks at
1024^2 text-to-image (config 2): per block, 4096 image-token queries attend over the
block's 512-token prefix KV cache plus the step's 4096 image keys, 32 heads x 128, bf16.
Each block call is the public b200_attn_fwd (two launches: the Q/K RMSNorm+RoPE prologue
and the tcgen05 attention kernel); the timed region replays the step's 32 calls as one CUDA
graph (``--no-graph``: called one by one).  Right after it, under the same clock sampling,
the same step runs with the two launches called separately and CUDA events around every
attention launch: the roofline's kernel time, against the measured burst bf16 peak (the
timed loop is well under a second).  ``e2e`` runs the step through b200_attn_fwd with host
(pinned) q/k/v copied in and the output copied out per block, beside the measured host-link
bandwidth that bounds it.  On one GPU, ``library_baseline`` times FlashAttention-2 (the
reference's flash_attention branch kernel) and torch SDPA's cuDNN and flash backends on the
same problem.  The default (config 2) line also carries ``denoise``: config 5's denoise-step
ms at this GPU count (the metric's second half; strong scaling over the ranks).

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
    ap.add_argument("--cpu-heads", type=int, default=32, help="heads in the CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-library", action="store_true",
                    help="configs 1-3: skip the library attention kernels (FA2, cuDNN SDPA)")
    ap.add_argument("--no-denoise", action="store_true",
                    help="config 2: skip the config-5 denoise-step leg")
    ap.add_argument("--no-graph", action="store_true",
                    help="configs 1-3: launch the step's calls one by one instead of replaying "
                         "them as one CUDA graph")
    ap.add_argument("--weights", choices=["q4_k_m", "bf16"], default="q4_k_m",
                    help="config 5: block linears as GGUF Q4_K_M blocks (the config) or bf16")
    ap.add_argument("--prompts", type=int, default=None,
                    help="config 5: prompts in the batch (default 8; fewer only for profiling)")
    ap.add_argument("--gemm", choices=["cublas", "b200"], default="cublas",
                    help="config 5: the block linears' GEMM (cuBLAS or the tcgen05 kernel)")
    ap.add_argument("--dequant-sweep", action="store_true",
                    help="config 5: time Q4_K dequantisation + GEMM against the bf16 GEMM "
                         "for one block's gate_up linear over M = 16 ... 65536 rows, then exit")
    ap.add_argument("--fused-qkv", action="store_true",
                    help="config 5: Q/K/V projections with norm + RoPE in the GEMM epilogue")
    ap.add_argument("--no-weight-prefetch", action="store_true",
                    help="config 5 (q4_k_m): dequantise each block's weights on the compute "
                         "stream instead of one block ahead on a side stream")
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


def _cpu_inputs(cfg, heads, seed):
    """bf16 bit patterns of one block's q/k/v ([1,T,heads,D]) and prefix K/V, the weight-1
    norms, the layout's real RoPE table (the oracle's EmbedNd restatement) and the valid
    prefix length, for the CPU legs."""
    import numpy as np
    from oracle import reference as oref  # CPU baseline leg (test / baseline infrastructure)
    t = cfg["grid"][0] * cfg["grid"][1]
    rng = np.random.default_rng(seed)
    bits = lambda shape: (rng.standard_normal(shape, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)
    q, k, v = (bits((1, t, heads, HEAD_DIM)) for _ in range(3))
    pk, pv = (bits((1, heads, cfg["P"], HEAD_DIM)) for _ in range(2))
    w = np.ones(HEAD_DIM, np.float32)
    text_len, slots, cond = prompt_layout(cfg)
    lay = oref.joint_layout(text_len, slots, cond, cfg["grid"])
    pe = np.ascontiguousarray(oref.embed_nd(lay["img_shapes"], lay["image_pad_mask"])[cfg["P"]:],
                              np.float32)
    prefix_valid = None if cfg["pv"] is None else np.array([cfg["pv"]], np.int32)
    return q, k, v, pk, pv, w, pe, prefix_valid


def run_reference(args, rank):
    """The CPU restatement of the reference's chunked attention, timed on the host: each
    step is one whole block (all 32 heads) of the workload, all host threads."""
    if rank != 0:
        return
    from oracle import cpu as ocpu  # CPU baseline leg (test / baseline infrastructure)
    cfg = CONFIGS[args.config]
    heads = max(1, min(args.cpu_heads, HEADS))
    q, k, v, pk, pv, w, pe, prefix_valid = _cpu_inputs(cfg, heads, 7)
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
    sample = (f"1 of 32 blocks ({heads} of 32 heads) of {cfg['name']} per step, real RoPE table "
              f"(oracle C port of chunked_attention, f32, OpenMP)")
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
    from oracle import cpu as ocpu  # CPU baseline leg (test / baseline infrastructure)
    q, k, v, pk, pv, w, pe, prefix_valid = _cpu_inputs(cfg, heads, 3)
    threads = os.cpu_count() or 1
    ocpu.attention_forward(q[:, :128], k[:, :128], v[:, :128], pk, pv, w, w, 1e-6, pe[:128],
                           prefix_valid, HEAD_DIM ** -0.5, threads)  # warm the thread pool
    t0 = time.perf_counter()
    ocpu.attention_forward(q, k, v, pk, pv, w, w, 1e-6, pe, prefix_valid, HEAD_DIM ** -0.5, threads)
    dt = time.perf_counter() - t0
    return {"value": flops_per_call(cfg, heads) / dt / 1e12, "unit": "TFLOP/s", "cores": threads,
            "kind": "port",
            "sample": f"1 of 32 blocks ({heads} of 32 heads) of {cfg['name']}, real RoPE table "
                      f"({dt:.1f} s, f32 C port of chunked_attention, OpenMP)"}


# --------------------------------------------------------------------------- library bar
def library_baseline(layers, T, P, pv, dev, reps=3):
    """Library attention kernels on the same problem, timed like joint_attn_kernel (CUDA
    events around every launch, one launch per block over `layers`' distinct inputs, which
    exceed L2): FlashAttention-2 (flash_attn 2.8, the kernel family of the reference's
    flash_attention branch, src/transformer.rs:243-254, candle_flash_attn) on token-major
    [B,S,H,D], and torch's scaled_dot_product_attention with the cuDNN and the flash backends
    forced on head-major [B,H,S,D].  Inputs are post-RoPE Q/K and the prefix-concatenated
    K/V in the layout each library wants (built before timing).  `fa2_branch_span` adds the
    copies the reference's FA2 branch makes around the kernel: the prefix `cat` of K and V
    (src/transformer.rs:186-189), the transposes to [B,S,H,D] (:247-249) and the output's
    transposes back to [B,S,H*D] (:253, :193).  The prefix mask (ragged valid keys) is not
    expressible in these calls without a materialised mask, so configs with padded prefix
    keys use all P keys here (slightly more work than the B200 kernel does)."""
    import torch
    import torch.nn.functional as F
    flops = 4.0 * HEADS * T * (P + T) * HEAD_DIM
    scale = HEAD_DIM ** -0.5
    g = torch.Generator(device=dev).manual_seed(55)
    rnd = lambda *s: torch.randn(*s, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    data = []
    for _ in range(layers):
        q = rnd(1, HEADS, T, HEAD_DIM)
        k = rnd(1, HEADS, T, HEAD_DIM)
        v_tm = rnd(1, T, HEADS, HEAD_DIM)
        pk, pvv = rnd(1, HEADS, P, HEAD_DIM), rnd(1, HEADS, P, HEAD_DIM)
        k_all = torch.cat([pk, k], 2)
        v_all = torch.cat([pvv, v_tm.transpose(1, 2)], 2)
        data.append(dict(q=q, k=k, v_tm=v_tm, pk=pk, pv=pvv, k_all=k_all, v_all=v_all,
                         q_tm=q.transpose(1, 2).contiguous(), k_tm=k_all.transpose(1, 2).contiguous(),
                         vv_tm=v_all.transpose(1, 2).contiguous()))
    stream = torch.cuda.current_stream(dev)

    def timed(fn):
        for d in data[:3]:
            fn(d)
        torch.cuda.synchronize(dev)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(reps * len(data))]
        i = 0
        for _ in range(reps):
            for d in data:
                ev[i][0].record(stream)
                fn(d)
                ev[i][1].record(stream)
                i += 1
        torch.cuda.synchronize(dev)
        ms = sum(a.elapsed_time(b) for a, b in ev) / len(ev)
        return {"launch_ms": ms, "tflops": flops / (ms / 1e3) / 1e12}

    out = {"problem": f"B=1, H={HEADS}, Sq={T}, Lk={P + T}, D={HEAD_DIM}, bf16, non-causal",
           "note": ("kernel = one library attention launch on inputs already in its layout; "
                    "fa2_branch_span = prefix cat + transposes + FA2 + output transposes")}
    if pv is not None:
        out["note"] += f"; all {P} prefix keys attended (the B200 kernel masks to {pv})"
    try:
        from flash_attn import flash_attn_func
        out["flash_attn2"] = timed(lambda d: flash_attn_func(d["q_tm"], d["k_tm"], d["vv_tm"],
                                                             softmax_scale=scale, causal=False))

        def fa2_span(d):
            k_all = torch.cat([d["pk"], d["k"]], 2)
            v_all = torch.cat([d["pv"], d["v_tm"].transpose(1, 2)], 2)
            o = flash_attn_func(d["q"].transpose(1, 2).contiguous(), k_all.transpose(1, 2).contiguous(),
                                v_all.transpose(1, 2).contiguous(), softmax_scale=scale, causal=False)
            return o.transpose(1, 2).contiguous().transpose(1, 2).reshape(1, T, HEADS * HEAD_DIM)

        out["fa2_branch_span"] = timed(fa2_span)
        out["flash_attn_version"] = __import__("flash_attn").__version__
    except Exception as e:  # library kernel unavailable on this GPU / build
        out["flash_attn2"] = {"unavailable": f"{type(e).__name__}: {str(e)[:160]}"}
    from torch.nn.attention import SDPBackend, sdpa_kernel
    for name, backend in (("sdpa_cudnn", SDPBackend.CUDNN_ATTENTION),
                          ("sdpa_flash", SDPBackend.FLASH_ATTENTION)):
        try:
            with sdpa_kernel(backend):
                out[name] = timed(lambda d: F.scaled_dot_product_attention(
                    d["q"], d["k_all"], d["v_all"], scale=scale))
        except Exception as e:
            out[name] = {"unavailable": f"{type(e).__name__}: {str(e)[:160]}"}
    out["cudnn_version"] = torch.backends.cudnn.version()
    del data
    torch.cuda.empty_cache()
    return out


def host_link_gbs(dev, nbytes=1 << 30):
    """Pinned host -> device and device -> host copy bandwidth (GB/s) of one `nbytes` copy
    each (best of 3), the bound of an e2e step that streams its inputs over the host link."""
    import torch
    h = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    d = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    res = {}
    for name, dst, src in (("h2d", d, h), ("d2h", h, d)):
        best = None
        for _ in range(3):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            dst.copy_(src, non_blocking=True)
            e1.record()
            torch.cuda.synchronize(dev)
            ms = e0.elapsed_time(e1)
            best = ms if best is None else min(best, ms)
        res[name] = nbytes / (best / 1e3) / 1e9
    del h, d
    return res


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
    if args.config == "c5" and args.dequant_sweep:
        dequant_sweep(dev)
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
    vals = torch.tensor([ms_total, e2e_ms or 0.0, sum(attn_ms) / len(attn_ms)],
                        dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms_total, e2e_ms_max, attn_avg_ms = float(vals[0]), float(vals[1]), float(vals[2])
    ms_step = ms_total / args.steps
    step_flops = flops_per_call(cfg) * L
    value = step_flops * world / (ms_step / 1e3) / 1e12
    clock_summary = clocks.summary()
    # release this workload before the other legs
    del layers, graph, fwd_ws, split_ws, q_rot, k_rot, out
    if args.e2e_steps > 0:
        del host_in, host_out, dev_in, dev_out, ws
    torch.cuda.empty_cache()

    # ---- the library attention kernels on the same problem, and the host link (1 GPU)
    lib_bar = link = None
    if world == 1 and not args.no_library:
        lib_bar = library_baseline(min(L, 8), T, P, cfg["pv"], dev)
        link = host_link_gbs(dev)
    # ---- config 5's denoise-step time at this GPU count (every rank takes part)
    den = None
    if args.config == "c2" and not args.no_denoise:
        den = run_denoise(args, CONFIGS["c5"], rank, world, dev, leg=True)

    if rank == 0:
        pk_d, src = peaks()
        peak = float(pk_d.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
        peak_sus = float(pk_d.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
        achieved = flops_per_call(cfg) / (attn_avg_ms / 1e3) / 1e12
        traffic = profile_traffic("joint_attn_kernel", args.config)
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline(cfg, max(1, min(args.cpu_heads, HEADS)))
        if lib_bar is not None:
            lib_bar["joint_attn_kernel"] = {"launch_ms": attn_avg_ms, "tflops": achieved}
        e2e = None
        if e2e_ms is not None:
            e2e = {"value": step_flops * world / (e2e_ms_max / 1e3) / 1e12, "unit": "TFLOP/s",
                   "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                   "ms_per_step": e2e_ms_max,
                   "path": ("b200_attn_fwd with pinned-host q/k/v in and output out per block; "
                            "copies on their own streams, double-buffered against the attention"),
                   "h2d_gbs": h2d / (e2e_ms_max / 1e3) / 1e9}
            if link is not None:
                e2e["host_link_gbs"] = link
                e2e["host_link_bound_ms"] = 1e3 * max(h2d / (link["h2d"] * 1e9),
                                                      d2h / (link["d2h"] * 1e9))
        line = {
            "metric": attn_metric(args.config), "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": ("synthetic (seeded N(0,1) q/k/v and prefix cache, weight-1 norms; each "
                     "block's q/k/v are generated once and the same tensors are attended every "
                     "step: 3.3 GB per step, which L2 cannot hold across steps)"),
            "config": attn_step_config(cfg, L, world),
            "pct_bf16_peak": 100.0 * value / world / peak,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "kernel": "joint_attn_kernel",
                         "peak_source": (f"{src} bf16_tflops (burst: the kernel's timed loop "
                                         f"runs well under a second)"),
                         "frac_of_sustained": achieved / peak_sus,
                         "launch_ms": attn_avg_ms},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "clocks": clock_summary,
            "gpu_launches": args.steps * L * 2,
            "launch": ("one CUDA graph per step (32 b200_attn_fwd calls captured once, replayed)"
                       if not args.no_graph else "b200_attn_fwd called block by block"),
        }
        if lib_bar is not None:
            line["library_baseline"] = lib_bar
        if den is not None:
            line["denoise"] = den
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
    nvls = None
    nvls_note = "one GPU"
    if world > 1:
        try:
            nvls = bdist.NvlsOutProj(T, hidden, dev)
            nvls_note = ("tcgen05 GEMM into this rank's buffer + owners' sum in the NVSwitch "
                         "(multimem.ld_reduce) and broadcast (multimem.st)")
        except RuntimeError as e:
            nvls_note = f"unavailable: {e}"
    path = bdist.out_proj_path(world)
    if path == "nvls" and nvls is None:
        path = "scatter"
    if path == "scatter" and fused is None:
        path = "nccl"
    use_fused = world == 1 or path in ("scatter", "nvls")
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

    def step_nvls(mark=None):
        return nvls(attention(mark), w_out, h0, h1, status=status)

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
        if nvls is not None:
            step_nvls()
    barrier()
    marks = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    with ClockSampler(uuid) as clocks:
        ms_fused = timed(step_fused, args.steps, marks)
    attn_ms = sum(m[0].elapsed_time(m[1]) for m in marks) / args.steps
    ms_nccl = timed(step_nccl, args.steps)
    ms_nvls = timed(step_nvls, args.steps) if nvls is not None else None
    # ---- the block's next steps fused into the owners' step: x += tanh(gate1) * to_out and
    # norm2(x) * (1 + scale2) (src/transformer.rs:411-421).  Timed against the same work
    # done after the gather / all-reduce by the residual_adaln kernel over all T rows.
    res_ms = None
    if fused is not None:
        x_full = torch.randn(T, hidden, generator=g, device=dev, dtype=torch.float32)
        gate = torch.randn(1, hidden, generator=g, device=dev, dtype=torch.float32)
        scale = 0.5 * torch.randn(1, hidden, generator=g, device=dev, dtype=torch.float32)
        r0, mine = fused.own_rows(T)
        x_own = x_full[r0:r0 + mine].clone()
        y_full = torch.empty(T, hidden, dtype=torch.bfloat16, device=dev)

        def step_res_owner(mark=None):
            return fused(attention(), w_out, h0, h1, status=status,
                         residual=(x_own, gate, scale))

        def step_res_after(tail):
            def run(mark=None):
                y = tail(attention())
                b200attn.residual_adaln(x_full, y, gate, scale, y_full, rows_per_mod=T,
                                        stream=stream)
                return y_full
            return run

        legs = {}
        if nvls is not None:
            x_nv = x_full[r0:r0 + mine].clone()
            legs["nvls_owner_step"] = lambda mark=None: nvls(
                attention(), w_out, h0, h1, status=status, residual=(x_nv, gate, scale))
        legs.update(owner_step=step_res_owner,
                    fused_then_residual_adaln=step_res_after(
                        lambda a: fused(a, w_out, h0, h1, status=status)),
                    nccl_then_residual_adaln=step_res_after(step_nccl_tail))
        if T % world == 0:
            # The same split with library collectives: reduce-scatter the partials, the
            # residual and norm2 on this rank's rows, all-gather the normalised rows.
            rows_n = T // world
            x_n = x_full[rank * rows_n:(rank + 1) * rows_n].clone()
            rs = torch.empty(rows_n, hidden, dtype=torch.bfloat16, device=dev)
            y_n = torch.empty(rows_n, hidden, dtype=torch.bfloat16, device=dev)

            def step_res_nccl_owner(mark=None):
                part = bdist.out_proj_partial(attention(), w_out, h0, h1, HEAD_DIM)
                dist.reduce_scatter_tensor(rs, part)
                b200attn.residual_adaln(x_n, rs, gate, scale, y_n, rows_per_mod=T,
                                        stream=stream)
                dist.all_gather_into_tensor(y_full, y_n)
                return y_full

            legs["nccl_reduce_scatter_owner_all_gather"] = step_res_nccl_owner
        for fn in legs.values():
            for _ in range(2):
                fn()
        res_ms = {name: timed(fn, args.steps) for name, fn in legs.items()}
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
            if path == "nvls":
                res = nvls(a, w_out, h0, h1, status=status)
            elif fused is not None and use_fused:
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
    if ms_nvls is not None:
        ms_nvls = bdist.max_over_ranks(ms_nvls, device=dev)
    e2e_ms = bdist.max_over_ranks(e2e["ms"], device=dev) if e2e else None
    ms_step = ms_nvls if path == "nvls" else ms_fused if use_fused else ms_nccl
    attn_ms = bdist.max_over_ranks(attn_ms, device=dev)
    if res_ms is not None:
        res_ms = {k: bdist.max_over_ranks(v, device=dev) for k, v in res_ms.items()}
    attn_flops = 4.0 * HEADS * T * (P + T) * HEAD_DIM
    proj_flops = 2.0 * T * HEADS * HEAD_DIM * hidden
    if rank == 0:
        pk_d, src = peaks()
        peak = float(pk_d.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
        peak_sus = float(pk_d.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
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
            "sum_of_partials": (nvls_note if path == "nvls" else fused_note if use_fused else
                                "cuBLAS + NCCL all-reduce (faster than the fused paths at "
                                "this rank count)"),
            "nccl_path": {"ms_per_step": ms_nccl,
                          "value": (attn_flops + proj_flops) / (ms_nccl / 1e3) / 1e12,
                          "how": "cuBLAS to_out partial + NCCL all-reduce (bf16)"},
            "fused_path": {"ms_per_step": ms_fused, "how": fused_note},
            "nvls_path": {"ms_per_step": ms_nvls, "how": nvls_note},
            "with_residual_norm2": None if res_ms is None else dict(
                res_ms, how=("step + x += tanh(gate1) * to_out + norm2 * (1 + scale2): in the "
                             "owners' reduce step (owner_step); vs a residual_adaln kernel over "
                             "all rows after the sum; vs NCCL reduce-scatter, residual_adaln on "
                             "this rank's rows and NCCL all-gather (ms per step, max over "
                             "ranks)")),
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak,
                         # captured with all 32 heads on one GPU; a rank's launch moves its
                         # heads' share (traffic grows in proportion to the heads)
                         "traffic": (None if profile_traffic("joint_attn_kernel", "c4") is None
                                     else profile_traffic("joint_attn_kernel", "c4") * hl / HEADS),
                         "kernel": "joint_attn_kernel",
                         "peak_source": f"{src} bf16_tflops (burst: a sub-second timed loop)",
                         "frac_of_sustained": achieved / peak_sus, "launch_ms": attn_ms},
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
    del nvls
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# --------------------------------------------------------------------------- config 5
C5_METRIC = "denoise-step ms at 1024^2 (config 5: 16 sequences = 8 prompts x CFG, 32 blocks)"
DENOISE_LEG_STEPS = 10   # timed steps of the default line's config-5 leg (at most --steps)
DENOISE_LEG_WARMUP = 3


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


def dequant_sweep(dev, ms=(1, 2, 16, 64, 256, 1024, 4096, 16384, 65536), reps=20):
    """Config 5's largest linear (gate_up: [2 x 12288, 4096], Q4_K) at M token rows: the
    large-M path (dequantise into a bf16 scratch, then cuBLAS) against cuBLAS on a resident
    bf16 weight, the fused few-row product (b200_kquant_gemv, M <= 2: the path of the
    timestep and modulation linears), and the floor of a fused dequantising GEMM (its Q4_K
    bytes at the measured copy bandwidth, or its FLOPs at the burst bf16 peak, whichever is
    larger).  The Q4_K bytes (57 MB) fit in L2 across repetitions.  One JSON line."""
    import torch
    import b200attn
    from b200attn import gguf
    from b200attn.mmdit import MMDiTConfig
    mc = MMDiTConfig()
    n, k = 2 * mc.ffn, mc.hidden
    g = torch.Generator(device=dev).manual_seed(11)
    w = (0.02 * torch.randn(n, k, generator=g, device=dev)).to(torch.bfloat16)
    blocks = gguf.quantize(w, "q4_k")
    ql = gguf.QuantLinear(blocks, "q4_k", (n, k))
    scratch = torch.empty(n, k, dtype=torch.bfloat16, device=dev)
    w_dq = ql.dequant_into(scratch).clone()
    pk_d, _src = peaks()
    hbm = float(pk_d.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    peak = float(pk_d.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    stream = torch.cuda.current_stream(dev)

    def timed(fn):
        """Device time per call: `reps` calls captured in one CUDA graph and replayed (the
        Python launch cost of a call exceeds these kernels' run time)."""
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for _ in range(3):
                fn()
        stream.wait_stream(side)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            for _ in range(reps):
                fn()
        graph.replay()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        graph.replay()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        del graph
        return e0.elapsed_time(e1) / reps

    rows = []
    for m in ms:
        x = torch.randn(m, k, generator=g, device=dev).to(torch.bfloat16)
        y = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
        t_dq_gemm = timed(lambda: torch.matmul(x, ql.dequant_into(scratch).t(), out=y))
        t_gemm = timed(lambda: torch.matmul(x, w_dq.t(), out=y))
        t_dq = timed(lambda: ql.dequant_into(scratch))
        floor_ms = max(blocks.numel() / (hbm * 1e9), 2.0 * m * n * k / (peak * 1e12)) * 1e3
        t_gemv = None
        if m <= b200attn.KQUANT_GEMV_MAX_ROWS:
            xf = x.float()
            yf = torch.empty(m, n, dtype=torch.float32, device=dev)
            t_gemv = round(timed(lambda: ql.matvec(xf, out=yf)), 4)
        rows.append({"m": m, "fused_gemv_ms": t_gemv, "dequant_then_gemm_ms": round(t_dq_gemm, 4),
                     "bf16_gemm_ms": round(t_gemm, 4), "dequant_ms": round(t_dq, 4),
                     "fused_floor_ms": round(floor_ms, 4),
                     "overhead_vs_bf16": round(t_dq_gemm / t_gemm - 1.0, 3),
                     "over_fused_floor": round(t_dq_gemm / floor_ms, 2)})
    print(json.dumps({"dequant_sweep": {
        "linear": f"gate_up [{n}, {k}] Q4_K ({blocks.numel()} bytes)", "rows": rows,
        "how": "CUDA events around a CUDA graph of 20 calls (after 3 warm-up calls); GEMM = "
               "cuBLAS (torch.matmul) bf16"}}),
        flush=True)


def run_denoise(args, cfg, rank, world, dev, leg=False):
    """Config 5: every rank runs the denoising loop of its prompts (both CFG branches),
    batched through each block; a step is one Euler step of this rank's sequences.  Strong
    scaling: the 8 prompts are split over the ranks; value = max over ranks of ms/step.

    leg=True is the config-5 leg of the default (config 2) line: DENOISE_LEG_WARMUP warm-up
    and min(--steps, DENOISE_LEG_STEPS) timed steps, no e2e or CPU sample; returns the
    max-over-ranks figures as a dict (on every rank) instead of printing a line."""
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
                        fused_qkv=args.fused_qkv, gemm=args.gemm,
                        prefetch_weights=not args.no_weight_prefetch)
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

    n_warm = DENOISE_LEG_WARMUP if leg else args.warmup
    n_steps_timed = min(args.steps, DENOISE_LEG_STEPS) if leg else args.steps
    for i in range(n_warm):
        step(i)
    barrier()
    prefix_ms = f0.elapsed_time(f1)
    model.attn_marks = []
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    with ClockSampler(uuid) as clocks:
        barrier()
        e0.record(stream)
        for i in range(n_steps_timed):
            step(n_warm + i)
        e1.record(stream)
        barrier()
    marks, model.attn_marks = model.attn_marks, None
    ms_rank = e0.elapsed_time(e1) / n_steps_timed
    attn_ms_rank = sum(a.elapsed_time(b) for a, b in marks) / n_steps_timed
    if not torch.isfinite(lat).all():
        raise RuntimeError("non-finite latents in the denoising loop")
    if leg:
        vals = torch.tensor([ms_rank, attn_ms_rank, prefix_ms], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(vals, op=dist.ReduceOp.MAX)
        del model, cache
        torch.cuda.empty_cache()
        ms_step, attn_ms, prefix_ms_max = (float(v) for v in vals)
        all_lengths = [n for p in range(cfg["prompts"]) for n in pairs[p]]
        lin_f, attn_f = c5_flops(mcfg, all_lengths, T)
        return {"metric": C5_METRIC, "ms_per_step": ms_step, "unit": "ms", "n_gpus": world,
                "steps": n_steps_timed, "warmup": n_warm, "higher_is_better": False,
                "scaling": "strong", "sequences_per_rank": len(lengths),
                "weights": args.weights, "step_tflops": (lin_f + attn_f) / (ms_step / 1e3) / 1e12,
                "attention_ms_per_step": attn_ms, "prefix_fill_ms": prefix_ms_max,
                "clocks": clocks.summary(),
                "note": ("config 5: 8 prompts x CFG = 16 sequences split over the ranks by "
                         "prompt, 32 blocks, random N(0,0.02) weights; the speed-up over 1 GPU "
                         "is this ms_per_step against the N=1 line's")}

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
