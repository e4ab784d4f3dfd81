#!/usr/bin/env python
"""Benchmark of the FP8 MoE decode path ("config 2").

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one decode step of one MoE layer for a batch of B tokens (default 1):
router GEMV, softmax top-8, grouping by expert, fused gate/up+SiLU, down and
the slot-order combine, with hidden 2048, 128 experts, top-8, expert
intermediate 768, FP8 e4m3 weights with one fp32 scale per 128x128 block,
bf16 activations in and out, fp32 accumulation.  Weights are random-init
N(0, 0.02) quantized on the device; activations N(0, 1) (synthetic data).

L2: each step reads a different one of 8 layer replicas (8 x 604 MB of
experts), so every step streams its weights from HBM.

value   tokens/s over all ranks, device-timed (CUDA events around a CUDA graph of
        exactly K steps, inputs resident in HBM).
e2e     the same through the public C ABI with host buffers, inside the timed
        region: every step's input comes from pinned host memory and its output
        goes back to pinned host memory.  At N = 1 the decode entry point takes
        the host buffers itself (a staging kernel reads x over the bus after the
        previous step, the step stores out into host memory); expert-parallel
        ranks copy in and out with stream-ordered copies.
roofline  the dominant kernel: at N = 1 and B <= 16 the whole step is one
        decode_kernel launch, so its algorithmic bytes over the device-timed
        step give the achieved bandwidth, against the measured HBM copy
        bandwidth of MEASURED_PEAKS.json; gate_up_kernel and gemv_config1 time
        the stand-alone gate/up and dense GEMV kernels in back-to-back launches.
grouped_experts_config5  config 5's routed experts (hidden 4096, 256 experts,
        top-8, intermediate 2048) at batches 32 / 128 / 1024: the tensor-core
        grouped GEMM against the CUDA-core expert kernels on the same routing.
cpu_baseline  the reference's host expert path restated in C++ with AVX-512
        (oracle/cpu_baseline.cpp) on this box's host cores (all of them, and one
        thread), rank 0, N=1 only; the CPU model is reported beside it.

With N > 1 (torchrun) the experts of every layer are sharded over the ranks
(expert parallelism, expert e on rank e / (E / N)); each rank decodes its own
batch of tokens (weak scaling), dispatching every token's slots to the ranks
that own their experts and taking the outputs back.  By default each rank runs
the whole step as one kernel launch whose dispatch and return are stores into
the peers' mailboxes over NVLink (--ep-step fused); --ep-step chain runs it as
a chain of kernels, --ep-transport nccl with NCCL all-to-alls.  Rank 0 prints
one line; times are the max over ranks.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "FP8 expert GEMV HBM GB/s vs B200 peak; MoE decode tokens/s at 1/2/4/8 GPU"
H, E, K_TOP, I = 2048, 128, 8, 768
LAYERS = 8
WORKLOAD = "config2: MoE expert decode, hidden 2048, 128 experts top-8, intermediate 768, FP8 e4m3 128x128 block scales"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--layers", type=int, default=8,
                    help="layer replicas rotated through (8 x 604 MB keeps every step out of L2)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--ep-transport", choices=["peer", "nccl"], default="peer",
                    help="expert-parallel all-to-alls: kernels storing into peer mailboxes over NVLink, or NCCL")
    ap.add_argument("--ep-step", choices=["chain", "fused"], default="fused",
                    help="with peer transport: the chain of kernels, or one launch per rank and step")
    ap.add_argument("--cpu-seconds", type=float, default=12.0,
                    help="CPU work of the cpu_baseline / reference sample")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--quick", action="store_true", help="skip the extra per-config measurements")
    ap.add_argument("--profile", type=int, default=0, metavar="N",
                    help="run N eager decode steps of the workload and exit (a small driver for ncu)")
    ap.add_argument("--profile-mlp", type=int, default=0, metavar="B",
                    help="with --profile: run N config-3 MLP steps at batch B instead (tensor-core path)")
    ap.add_argument("--profile-attn", type=int, default=0, metavar="B",
                    help="with --profile: run N config-4 decode attention launches (context 4096) at batch B instead")
    ap.add_argument("--profile-tiled", type=int, default=0, metavar="B",
                    help="with --profile: run N grouped tensor-core expert steps (config-5 shapes, 32 experts) "
                         "at batch B instead")
    return ap.parse_args()


def config_dict(batch, layers=LAYERS, world=1):
    """The workload's keys, identical for both arms."""
    return {"workload": WORKLOAD, "hidden": H, "experts": E, "top_k": K_TOP, "inter": I,
            "batch_per_gpu": batch, "scale_blocks": "128x128", "layers_rotated": layers,
            "l2": f"inputs larger than L2: each step reads a different layer's experts ({layers} x 604 MB)",
            "parallelism": f"ep{world}" if world > 1 else "single"}


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def load_peaks():
    for p in (os.path.join(ROOT, "MEASURED_PEAKS.json"),):
        if os.path.exists(p):
            d = json.load(open(p))
            return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def load_traffic():
    """DRAM traffic per launch of the dominant kernel from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "roofline_traffic.json")
    if os.path.exists(p):
        try:
            return json.load(open(p))
        except Exception:
            return None
    return None


# ---- clocks --------------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index  # nvidia-smi -i accepts an index or a GPU UUID
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.result = None
        if not self.proc:
            return
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out = ""
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if sm:
            self.result = {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx),
                           "reasons": sorted(reasons), "samples": len(sm)}


# ---- the reference arm (CPU) ---------------------------------------------------------------

def cpu_layer(seed=1):
    """One config-2 layer in host memory: bf16 router and 128 FP8 records.

    The CPU kernels' time does not depend on the weight values, so the records
    hold random finite e4m3 codes (bit 3 cleared: never the NaN codes 0x7f /
    0xff) and block scales of the size N(0, 0.02) weights give (amax / 448).
    """
    import numpy as np

    import oracle as O
    from homelab_b200.records import record_layout
    geo, stride = record_layout(H, I, 1)
    rng = np.random.default_rng(seed)
    recs = (rng.integers(0, 256, size=(E, stride), dtype=np.uint8) & 0xF7).astype(np.uint8)
    for e in range(E):
        for (so, n, k) in ((geo.gate_scale, I, H), (geo.up_scale, I, H), (geo.down_scale, H, I)):
            ns = O.scale_count(n, k, O.SCALE_128X128)
            recs[e, so:so + 4 * ns] = np.full(ns, 0.08 / 448, dtype=np.float32).view(np.uint8)
    router = O.bf16_from_f32(rng.standard_normal(E * H, dtype=np.float32) * 0.02).reshape(E, H)
    ptrs = (C.c_void_p * E)(*[recs[e].ctypes.data for e in range(E)])
    g = O.Fp8Record()
    for f, _ in O.Fp8Record._fields_:
        setattr(g, f, getattr(geo, f))
    return recs, router, ptrs, g


def time_cpu(batch, seconds, threads=None):
    """Best-of-5 per-step time of the CPU baseline (expert_bench.rs:58-80 method)."""
    import numpy as np

    import oracle as O
    recs, router, ptrs, geo = cpu_layer()
    pool = O.CpuPool(threads or os.cpu_count() or 1)
    xs = [O.bf16_to_f32(O.normal_bf16(900 + i, batch * H)).reshape(batch, H) for i in range(16)]
    pool.moe_layer(xs[0], router, K_TOP, ptrs, geo)  # warm-up
    t0 = time.perf_counter()
    pool.moe_layer(xs[1], router, K_TOP, ptrs, geo)
    one = max(time.perf_counter() - t0, 1e-6)
    reps = max(1, int(seconds / 5 / one))
    best = float("inf")
    for r in range(5):
        t0 = time.perf_counter()
        for i in range(reps):
            pool.moe_layer(xs[(r * reps + i) % len(xs)], router, K_TOP, ptrs, geo)
        best = min(best, (time.perf_counter() - t0) / reps)
    threads_used = pool.threads
    pool.close()
    sample = f"{5 * reps} steps of the config-2 layer at batch {batch} (best of 5 rounds of {reps})"
    return best, threads_used, sample, 5 * reps


def run_reference(args, rank, world):
    if rank != 0:
        return
    steps = args.steps
    per, threads, sample, n = time_cpu(args.batch, args.cpu_seconds)
    per1, _, sample1, _ = time_cpu(args.batch, args.cpu_seconds / 3, threads=1)
    tok_s = args.batch / per
    line = {
        "impl": "reference", "metric": METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": steps, "warmup": args.warmup, "ms_per_step": per * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_dict(args.batch, LAYERS, world),
        "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "cpu_model": cpu_model(), "value_1_thread": args.batch / per1,
                         "sample": sample + "; the reference's host expert path (oominf-cpu) restated in "
                                             "C++ with AVX-512, FP8 decode, whole layer on the CPU; one thread: "
                                   + sample1},
        "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---- our arm -------------------------------------------------------------------------------

def run_ours(args, rank, world, local_rank):
    import torch

    import homelab_b200 as hb
    from homelab_b200.backend import Gpu
    from homelab_b200.records import ExpertBank, weight_bytes

    dist = None
    if world > 1:
        import torch.distributed as dist
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    gpu = Gpu(local_rank)
    B = args.batch
    if args.profile and args.profile_attn:
        # a small ncu driver: config-4 attention alone (B x 16.8 MB of cache)
        import torch as _t
        Bq, ctx, NH, NKV, D = args.profile_attn, 4096, 32, 8, 128
        g = _t.Generator(device=dev)
        g.manual_seed(3)
        kc = _t.randn((Bq, ctx, NKV, D), generator=g, device=dev).to(_t.bfloat16)
        vc = _t.randn((Bq, ctx, NKV, D), generator=g, device=dev).to(_t.bfloat16)
        q = _t.randn((Bq, NH, D), generator=g, device=dev).to(_t.bfloat16)
        o = _t.empty((Bq, NH, D), dtype=_t.bfloat16, device=dev)
        ws = gpu.attention_workspace(Bq, NH, NKV, D, ctx)
        for _ in range(args.profile):
            gpu.attention_decode(q, kc, vc, o, ctx, 1.0 / D ** 0.5, ws, NKV)
        _t.cuda.synchronize()
        assert gpu.device_error() == 0
        return None, None
    if args.profile and args.profile_tiled:
        # a small ncu driver: the 32-expert grouped case alone (805 MB of records)
        measure_experts_config5(gpu, dev, torch.cuda.current_stream(dev), batches=(args.profile_tiled,),
                                steps=args.profile, experts=32, forms=("tcgen05_grouped",), warm=0)
        torch.cuda.synchronize()
        assert gpu.device_error() == 0
        return None, None

    # ---- weights: 8 layer replicas; with N > 1 every rank holds E/N of each layer's experts ----
    LAYERS = args.layers
    epr = E // world
    layers = []
    gen = torch.Generator(device=dev)
    for li in range(LAYERS):
        bank = ExpertBank(epr, H, I, hb.SCALE_128X128, dev)
        bank.fill_random(gpu, seed=1000 * (rank + 1) + li)
        gen.manual_seed(77 + li)  # the router is replicated: the same on every rank
        router = (torch.randn((E, H), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
        L = hb.MoeLayer(hidden=H, experts=E, top_k=K_TOP, router_w=router.data_ptr(), recs=bank.addrs.data_ptr())
        L.geo = bank.geo
        layers.append((bank, router, L))
    NX = 64
    gen.manual_seed(5 + rank)
    xs = (torch.randn((NX, B, H), generator=gen, device=dev)).to(torch.bfloat16)
    out = torch.empty((B, H), dtype=torch.bfloat16, device=dev)
    if world == 1:
        ws = gpu.moe_decode_workspace(layers[0][2], B)

        def step(i, x=None, o=None):
            gpu.moe_decode(layers[i % LAYERS][2], xs[i % NX] if x is None else x, B, out if o is None else o, ws)
    else:
        # expert parallelism: route locally, all-to-all dispatch, local experts, all-to-all return, combine
        from homelab_b200.ep import EpDecodeLayer, EpGpuOps, EpMoeLayer, EpPeerMailboxes, EpPeerMoeLayer
        ops = EpGpuOps(dev)
        if args.ep_transport == "peer":
            mailboxes = EpPeerMailboxes(dist.group.WORLD, H, K_TOP, B, torch.bfloat16, dev)
            if args.ep_step == "fused" and B <= 16:  # the one-launch step per rank
                ep_layers = [EpDecodeLayer(mailboxes, rank, H, E, K_TOP, router, bank.addrs, bank.geo, B)
                             for (bank, router, _) in layers]
            else:
                ep_layers = [EpPeerMoeLayer(ops, mailboxes, rank, H, E, K_TOP, I, router, bank.addrs, bank.geo, B)
                             for (bank, router, _) in layers]
        else:
            ep_layers = [EpMoeLayer(ops, dist.group.WORLD, H, E, K_TOP, I, router, bank.addrs, bank.geo, B)
                         for (bank, router, _) in layers]

        def step(i, x=None, o=None):
            ep_layers[i % LAYERS].forward(xs[i % NX] if x is None else x, B, out if o is None else o)
    torch.cuda.synchronize()

    if args.profile:
        if args.profile_mlp:
            profile_mlp(gpu, dev, args.profile_mlp, args.profile)
        else:
            for i in range(args.profile):
                step(i)
        torch.cuda.synchronize()
        assert gpu.device_error() == 0
        return None, None

    # ---- warm-up (eager) ----
    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize()
    assert gpu.device_error() == 0

    K = args.steps
    G = min(K, 2000)  # steps per captured graph
    reps, rem = divmod(K, G)
    s = torch.cuda.Stream(dev)

    # the decode entry points (single GPU, and the one-launch expert-parallel step) read and write
    # pinned host buffers themselves
    host_io = world == 1 or (args.ep_transport == "peer" and args.ep_step == "fused" and B <= 16)

    def capture(n, e2e=False, xh=None, oh=None, xdev=None):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for i in range(n):
                if e2e and host_io:
                    step(i, xh[i % NX], oh[i % NX])
                elif e2e:
                    xdev.copy_(xh[i % NX], non_blocking=True)
                    step(i, xdev, out)
                    oh[i % NX].copy_(out, non_blocking=True)
                else:
                    step(i)
        return g

    class Eager:
        """Replays n steps eagerly (used where the steps cannot be captured)."""

        def __init__(self, n, e2e=False, xh=None, oh=None, xdev=None):
            self.n, self.e2e, self.xh, self.oh, self.xdev = n, e2e, xh, oh, xdev

        def replay(self):
            with torch.cuda.stream(s):
                for i in range(self.n):
                    if self.e2e and host_io:
                        step(i, self.xh[i % NX], self.oh[i % NX])
                    elif self.e2e:
                        self.xdev.copy_(self.xh[i % NX], non_blocking=True)
                        step(i, self.xdev, out)
                        self.oh[i % NX].copy_(out, non_blocking=True)
                    else:
                        step(i)

    graphs_ok = True
    if world > 1:
        # NCCL collectives inside a CUDA graph: try once, fall back to eager steps
        try:
            torch.cuda.synchronize()
            gt = capture(2)
            gt.replay()
            torch.cuda.synchronize()
            del gt
        except Exception:
            graphs_ok = False
        if dist:
            flag = torch.tensor([1 if graphs_ok else 0], device=dev)
            dist.all_reduce(flag, op=dist.ReduceOp.MIN)
            graphs_ok = bool(flag.item())
    if not graphs_ok:
        capture = Eager  # noqa: F811

    def timed(graphs_and_counts, sampler_index):
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s):
            ev0.record(s)
            for g, c in graphs_and_counts:
                for _ in range(c):
                    g.replay()
            ev1.record(s)
        ev1.synchronize()
        torch.cuda.synchronize()
        ms = ev0.elapsed_time(ev1)
        if dist:
            tt = torch.tensor([ms], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            ms = float(tt.item())
        return ms

    g_main = capture(G)
    g_rem = capture(rem) if rem else None
    plan = [(g_main, reps)] + ([(g_rem, 1)] if g_rem else [])
    # untimed graph warm-up, then the timed region under the clock sampler
    for g, _ in plan:
        g.replay()
    torch.cuda.synchronize()
    try:
        smi_id = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        smi_id = str(local_rank)
    with ClockSampler(smi_id) as cs:
        # keep the GPU busy ~0.5 s before the timed region so the sampler sees load
        t_end = time.time() + 0.5
        while time.time() < t_end:
            g_main.replay()
            torch.cuda.synchronize()
        ms = timed(plan, local_rank)
    clocks = cs.result
    assert gpu.device_error() == 0
    tok_s = world * B * K / (ms / 1e3)

    # ---- e2e: host buffers, copies inside the timed region ----
    xh = xs.cpu().pin_memory()
    oh = torch.empty((NX, B, H), dtype=torch.bfloat16).pin_memory()
    xdev = torch.empty((B, H), dtype=torch.bfloat16, device=dev)
    ge_main = capture(G, True, xh, oh, xdev)
    ge_rem = capture(rem, True, xh, oh, xdev) if rem else None
    eplan = [(ge_main, reps)] + ([(ge_rem, 1)] if ge_rem else [])
    for g, _ in eplan:
        g.replay()
    torch.cuda.synchronize()
    ms_e2e = timed(eplan, local_rank)
    e2e = world * B * K / (ms_e2e / 1e3)
    del ge_main, ge_rem

    # ---- roofline: at N = 1 and B <= 16 the step is one launch (decode_kernel), so its
    # algorithmic bytes over the device-timed step are that kernel's achieved bandwidth;
    # the stand-alone gate/up kernel is timed beside it ----
    step_bytes = E * H * 2 + 8 * B * weight_bytes(layers[0][0].geo) + 2 * B * H * 2
    chain_env = os.environ.get("OOMB_DECODE_CHAIN") == "1"
    fused = world == 1 and B <= 16 and not chain_env     # one decode_kernel launch a step
    tiled = world == 1 and B > 16 and not chain_env      # route, 2 splits, 3 grouped GEMMs, SwiGLU, combine
    roof = measure_gate_up(gpu, layers, dev, s, B, LAYERS)
    gemv1 = measure_gemv_config1(gpu, dev, s)
    del layers
    torch.cuda.empty_cache()
    peak, peak_kind = load_peaks()
    traffic = load_traffic()
    extras = world == 1 and not args.quick
    mlp3 = measure_mlp_config3(gpu, dev, s) if extras else None
    experts5 = measure_experts_config5(gpu, dev, s) if extras else None
    staging = measure_staging(dev) if extras else None
    attn4 = measure_attention_config4(gpu, dev, s, peak=peak) if extras else None
    layers4 = measure_layers_config4(gpu, dev, s, peak=peak) if extras else None
    offload5 = measure_offload_config5(gpu, dev, s) if extras else None
    fp8_peak = measure_fp8_peak(dev, s) if extras else None
    if fp8_peak and "tflops" in fp8_peak and experts5:
        for v in experts5.values():
            v["tcgen05_grouped"]["frac_of_fp8_peak"] = v["tcgen05_grouped"]["tflops"] / fp8_peak["tflops"]

    ep5 = None
    if world > 1 and not args.quick:
        ep5 = measure_ep_config5(gpu, dev, s, rank, world)
    result = None
    if rank == 0:
        result = {
            "metric": METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": dict(config_dict(B, LAYERS, world),
                           **({"expert_parallel": f"{E // world} experts per GPU, " + (
                               ("one launch per rank and step: " if args.ep_step == "fused" and B <= 16 else
                                "chain of kernels: ") + "dispatch and return stored by the kernels into peer "
                               "mailboxes over NVLink (CUDA IPC)"
                               if args.ep_transport == "peer" else "NCCL all-to-all dispatch and combine"),
                               "step_capture": "cuda graph" if graphs_ok else "eager"} if world > 1 else {})),
            "roofline": roofline_line(fused, step_bytes, ms / K, roof, peak, peak_kind, traffic),
            "gate_up_kernel": {"kernel": "stream_kernel<2> (gate/up+SiLU over the 8 experts of a step, "
                                         "back-to-back stand-alone launches)",
                               "achieved_gbs": roof["gbs"], "frac": roof["gbs"] / peak, "launch_us": roof["us"],
                               "algorithmic_bytes_per_launch": roof["bytes"]},
            "step_hbm_gbs": step_bytes * K / (ms / 1e3) / 1e9 / 1.0 if world == 1 else None,
            "gemv_config1": {"workload": "config1: 4096x4096 e4m3, 128x128 scales, x bf16 batch 1, bf16 out",
                             "achieved_gbs": gemv1["gbs"], "frac": gemv1["gbs"] / peak, "launch_us": gemv1["us"],
                             "algorithmic_bytes_per_launch": gemv1["bytes"]},
            "batched_dense_config3": mlp3,
            "grouped_experts_config5": experts5,
            "offload_staging_config5": staging,
            "attention_config4": attn4,
            "decode_layers_config4": layers4,
            "offload_overlap_config5": offload5,
            "fp8_tensor_peak": fp8_peak,
            "ep_config5": ep5,
            "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": B * H * 2,
                    "d2h_bytes_per_step": B * H * 2},
            # per step: one decode_kernel up to 16 tokens; from 17 tokens the grouped
            # tensor-core path (route, split x, gate, up, SwiGLU, split h, down, combine);
            # the chain route, gate/up, down, combine with OOMB_DECODE_CHAIN=1;
            # expert-parallel over peer memory: one launch per rank (fused), or router
            # logits, top-k, dispatch, group, gate/up, down, return, combine; over NCCL:
            # logits, top-k, meta, group, gate/up, down, scatter, combine (NCCL's own
            # kernels not counted)
            "gpu_launches": (1 if fused or (world > 1 and args.ep_transport == "peer" and args.ep_step == "fused"
                                           and B <= 16)
                             else 8 if tiled else (4 if world == 1 else 8)) * K,
            "clocks": clocks,
        }
    return result, roof


def roofline_line(fused, step_bytes, ms_per_step, gate_up, peak, peak_kind, traffic):
    """The roofline object of the step's dominant kernel: the one-launch decode
    kernel when the step is one launch, else the gate/up kernel."""
    if fused:
        kernel = "decode_kernel"
        us = ms_per_step * 1e3
        gbs = step_bytes / (us * 1e-6) / 1e9
        desc = "decode_kernel (the whole step in one launch: router, top-k, grouping, gate/up, down, combine)"
        nbytes = step_bytes
    else:
        kernel = "stream_kernel<2"
        us, gbs, nbytes = gate_up["us"], gate_up["gbs"], gate_up["bytes"]
        desc = "stream_kernel<2> (gate/up+SiLU over the 8 experts of a step)"
    t = traffic.get("bytes_per_launch") if traffic and str(traffic.get("kernel", "")).startswith(kernel) else None
    return {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
            "peak_kind": peak_kind, "traffic": t, "kernel": desc, "algorithmic_bytes_per_launch": nbytes,
            "launch_us": us}


def measure_gate_up(gpu, layers, dev, s, B, LAYERS, launches=400):
    """Average duration of back-to-back gate/up launches over 8 fixed experts per launch.

    The routing tables are written before the loop (OOMB_TABLES_READY), so each
    launch streams its experts' weights while the previous launch drains, as
    the down projection does behind gate/up in the decode step."""
    import numpy as np
    import torch

    from homelab_b200.records import scale_bytes
    rng = np.random.default_rng(3)
    tables = []
    for li in range(LAYERS):
        bank = layers[li][0]
        ne = bank.experts
        ids = np.sort(rng.choice(ne, min(8 * B, ne), replace=False)).astype(np.int32)
        recs = bank.addrs[torch.from_numpy(ids).long().to(dev)].contiguous()
        off = torch.arange(0, len(ids) + 1, dtype=torch.int32, device=dev)
        tok = torch.zeros(len(ids), dtype=torch.int32, device=dev)
        tables.append((recs, off, tok, len(ids)))
    x = torch.randn((B, H), device=dev).to(torch.bfloat16)
    h = torch.empty((8 * B, I), dtype=torch.float32, device=dev)
    geo = layers[0][0].geo

    def one(i):
        recs, off, tok, n = tables[i % LAYERS]
        gpu.moe_gate_up(recs, off, tok, n, x, h, geo, 1, tables_ready=True)

    for i in range(16):
        one(i)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(launches):
            one(i)
    g.replay()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    best = float("inf")
    for _ in range(3):
        with torch.cuda.stream(s):
            ev0.record(s)
            g.replay()
            ev1.record(s)
        ev1.synchronize()
        best = min(best, ev0.elapsed_time(ev1) / launches)
    n_e = tables[0][3]
    nbytes = n_e * (2 * I * H + 2 * scale_bytes(I, H, geo.layout)) + n_e * H * 2 + n_e * I * 4
    us = best * 1e3
    return {"gbs": nbytes / (us * 1e-6) / 1e9, "bytes": nbytes, "us": us}


def profile_mlp(gpu, dev, B, steps):
    """`steps` eager config-3 MLP steps at batch B (one weight copy): an ncu driver."""
    import torch

    import homelab_b200 as hb
    H, F = 4096, 14336
    gen = torch.Generator(device=dev)
    gen.manual_seed(13)
    mats = []
    for (n, k) in ((2 * F, H), (H, F)):
        w = (torch.randn((n, k), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
        mats.append(gpu.quantize_fp8(w.view(torch.int16), n, k, hb.SCALE_128X128))
        del w
    x = torch.randn((B, H), generator=gen, device=dev).to(torch.bfloat16)
    gu = torch.empty((B, 2 * F), dtype=torch.float32, device=dev)
    hh = torch.empty((B, F), dtype=torch.bfloat16, device=dev)
    y = torch.empty((B, H), dtype=torch.bfloat16, device=dev)
    ws1 = gpu.gemm_fp8_workspace(B, 2 * F, H) if B >= 2 else None
    ws2 = gpu.gemm_fp8_workspace(B, H, F) if B >= 2 else None
    for _ in range(steps):
        gpu.gemm_fp8(x, mats[0][0], mats[0][1], gu, B, 2 * F, H, hb.SCALE_128X128, ws1)
        gpu.silu_mul_rows(gu, hh, B, F)
        gpu.gemm_fp8(hh, mats[1][0], mats[1][1], y, B, H, F, hb.SCALE_128X128, ws2)


def measure_mlp_config3(gpu, dev, s, batches=(1, 4, 16, 64), steps=24):
    """Llama-3-8B MLP, fused gate/up FP8 W [2 x 14336, 4096] +
    SwiGLU + down FP8 W [4096, 14336], 128x128 block scales, x bf16 [B, 4096].
    Two weight copies alternate (352 MB, beyond L2).  One tcgen05 workspace per
    shape: batches of 2+ tokens run on the tensor cores, one token on the
    CUDA-core stream (the GEMV -> tcgen05 crossover)."""
    import torch

    import homelab_b200 as hb
    H, F = 4096, 14336
    gen = torch.Generator(device=dev)
    gen.manual_seed(13)
    mats = []
    for c in range(2):
        pair = []
        for (n, k) in ((2 * F, H), (H, F)):
            w = (torch.randn((n, k), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
            pair.append(gpu.quantize_fp8(w.view(torch.int16), n, k, hb.SCALE_128X128))
            del w
        mats.append(pair)
    torch.cuda.empty_cache()
    wbytes = 2 * F * H + H * F + ((2 * F // 128) * (H // 128) + (H // 128) * (F // 128)) * 4
    out = {}
    for B in batches:
        x = torch.randn((B, H), generator=gen, device=dev).to(torch.bfloat16)
        gu = torch.empty((B, 2 * F), dtype=torch.float32, device=dev)
        hh = torch.empty((B, F), dtype=torch.bfloat16, device=dev)
        y = torch.empty((B, H), dtype=torch.bfloat16, device=dev)
        ws1 = gpu.gemm_fp8_workspace(B, 2 * F, H) if B >= 2 else None
        ws2 = gpu.gemm_fp8_workspace(B, H, F) if B >= 2 else None

        def mlp(i):
            (q1, s1), (q2, s2) = mats[i % 2]
            gpu.gemm_fp8(x, q1, s1, gu, B, 2 * F, H, hb.SCALE_128X128, ws1)
            gpu.silu_mul_rows(gu, hh, B, F)
            gpu.gemm_fp8(hh, q2, s2, y, B, H, F, hb.SCALE_128X128, ws2)

        for i in range(4):
            mlp(i)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for i in range(steps):
                mlp(i)
        g.replay()
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        best = float("inf")
        for _ in range(3):
            with torch.cuda.stream(s):
                ev0.record(s)
                g.replay()
                ev1.record(s)
            ev1.synchronize()
            best = min(best, ev0.elapsed_time(ev1) / steps)
        us = best * 1e3
        nbytes = wbytes + B * (H * 2 + 2 * F * 4 * 2 + F * 2 * 2 + H * 2)
        out[f"B{B}"] = {"us_per_mlp": us, "tokens_per_s": B / (us * 1e-6), "gbs": nbytes / (us * 1e-6) / 1e9,
                        "path": "tcgen05" if B >= 2 else "cuda-core stream"}
        del g
    return out


def measure_experts_config5(gpu, dev, s, batches=(32, 128, 1024), steps=6, experts=256,
                            forms=("tcgen05_grouped", "cuda_core"), warm=3):
    """BASELINE config 5's routed experts on one GPU: hidden 4096, 256 experts, top-8,
    intermediate 2048, 128x128 scales (6.44 GB of records, beyond L2 many times).
    Per batch, one seeded routing (grouped by expert as Moe::finish_routed does) and
    two step forms over it: the CUDA-core expert kernels (oomb_moe_gate_up_fp8 +
    oomb_moe_down_fp8) and the tensor-core grouped GEMM (oomb_moe_tiled_fp8 for gate,
    up and down + oomb_moe_swiglu_range, the order of Moe::run_group's tiled branch)."""
    import numpy as np
    import torch

    import homelab_b200 as hb
    from homelab_b200.records import ExpertBank
    H, I, E, K = 4096, 2048, experts, 8
    bank = ExpertBank(E, H, I, hb.SCALE_128X128, dev)
    bank.fill_random(gpu, seed=29)
    torch.cuda.synchronize()
    g = bank.geo
    rec_bytes = 3 * H * I + 3 * (H // 128) * (I // 128) * 4
    rng = np.random.default_rng(31)
    gen = torch.Generator(device=dev)
    gen.manual_seed(37)
    out = {}
    for B in batches:
        ids = np.argsort(rng.standard_normal((B, E)), axis=1)[:, :K].astype(np.int32)
        flat = ids.reshape(-1)
        order = np.argsort(flat, kind="stable")
        active, counts = np.unique(flat, return_counts=True)
        off = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
        tok = (order // K).astype(np.int32)
        A, n_e, maxn = B * K, len(active), int(counts.max())
        recs = bank.addrs[torch.from_numpy(active).long().to(dev)].contiguous()
        offd = torch.from_numpy(off).to(dev)
        tokd = torch.from_numpy(tok).to(dev)
        x = torch.randn((B, H), generator=gen, device=dev).to(torch.bfloat16)
        gg = torch.empty((A, I), dtype=torch.float32, device=dev)
        uu = torch.empty_like(gg)
        hh = torch.empty_like(gg)
        y = torch.empty((A, H), dtype=torch.float32, device=dev)

        def tiled():
            gpu.moe_tiled(recs, offd, tokd, n_e, maxn, x, gg, I, H, (g.gate_weight, g.gate_scale), g.layout)
            gpu.moe_tiled(recs, offd, tokd, n_e, maxn, x, uu, I, H, (g.up_weight, g.up_scale), g.layout)
            gpu.moe_swiglu_range(gg, uu, hh, 0, A * I)
            gpu.moe_tiled(recs, offd, None, n_e, maxn, hh, y, H, I, (g.down_weight, g.down_scale), g.layout)

        def cuda_cores():
            gpu.moe_gate_up(recs, offd, tokd, n_e, x, hh, g, maxn)
            gpu.moe_down(recs, offd, n_e, hh, y, g, maxn)

        res = {"assignments": A, "distinct_experts": n_e, "max_per_expert": maxn}
        for name, fn in (("tcgen05_grouped", tiled), ("cuda_core", cuda_cores)):
            if name not in forms:
                continue
            with torch.cuda.stream(s):
                for _ in range(warm):
                    fn()
                s.synchronize()
                ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                ev0.record(s)
                for _ in range(steps):
                    fn()
                ev1.record(s)
            ev1.synchronize()
            us = ev0.elapsed_time(ev1) / steps * 1e3
            res[name] = {"us_per_step": us, "tokens_per_s": B / (us * 1e-6),
                         "weight_gbs": n_e * rec_bytes / (us * 1e-6) / 1e9,
                         "tflops": 2.0 * A * 3 * H * I / (us * 1e-6) / 1e12}
        out[f"B{B}"] = res
        del gg, uu, hh, y
    del bank
    torch.cuda.empty_cache()
    return out


def measure_staging(dev, records=8, reps=5):
    """BASELINE config 5 offload: cold expert records (hidden 4096, intermediate
    2048, FP8 128x128: 25.2 MB each) staged from a pinned host arena into device
    slots on a copy queue (homelab_b200.stage), one copy per record; device-timed
    on the queue.  Returns the host-to-device GB/s (PCIe)."""
    import torch

    import homelab_b200 as hb
    from homelab_b200.records import record_layout
    from homelab_b200.stage import HostArena, Transfer, stage_records
    geo, stride = record_layout(4096, 2048, hb.SCALE_128X128)
    arena = HostArena(records, stride)
    arena.buf.fill_(1)
    slots = torch.empty(records * stride, dtype=torch.uint8, device=dev)
    addrs = [slots.data_ptr() + j * stride for j in range(records)]
    tr = Transfer(dev)
    q = torch.cuda.ExternalStream(tr.queue, device=dev)
    stage_records(tr, arena, range(records), addrs)
    tr.copies_sync()
    best = float("inf")
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(q)
        stage_records(tr, arena, range(records), addrs)
        e1.record(q)
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1))
    tr.copies_sync()
    tr.close()
    return {"record_bytes": stride, "records": records, "h2d_gbs": records * stride / (best * 1e-3) / 1e9,
            "ms_per_batch": best}


def measure_gemv_config1(gpu, dev, s, copies=16, launches=320):
    """y = W x, W 4096 x 4096 e4m3 with 128x128 block scales,
    x bf16 [1, 4096], bf16 out; back-to-back launches over `copies` weight
    copies (268 MB, beyond L2).  Returns GB/s of algorithmic bytes."""
    import torch

    import homelab_b200 as hb
    n = k = 4096
    gen = torch.Generator(device=dev)
    gen.manual_seed(11)
    qs, ss = [], []
    for c in range(copies):
        w = (torch.randn((n, k), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
        q, sc = gpu.quantize_fp8(w.view(torch.int16), n, k, hb.SCALE_128X128)
        qs.append(q)
        ss.append(sc)
    x = torch.randn((1, k), generator=gen, device=dev).to(torch.bfloat16)
    y = torch.empty((1, n), dtype=torch.bfloat16, device=dev)
    for i in range(8):
        gpu.gemm_fp8(x, qs[i % copies], ss[i % copies], y, 1, n, k, hb.SCALE_128X128)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(launches):
            gpu.gemm_fp8(x, qs[i % copies], ss[i % copies], y, 1, n, k, hb.SCALE_128X128)
    g.replay()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    best = float("inf")
    for _ in range(3):
        with torch.cuda.stream(s):
            ev0.record(s)
            g.replay()
            ev1.record(s)
        ev1.synchronize()
        best = min(best, ev0.elapsed_time(ev1) / launches)
    nbytes = n * k + (n // 128) * (k // 128) * 4 + k * 2 + n * 2
    us = best * 1e3
    return {"gbs": nbytes / (us * 1e-6) / 1e9, "bytes": nbytes, "us": us}


def measure_fp8_peak(dev, s, n=8192, launches=20):
    """The dense FP8 tensor-core peak of this GPU as a library reaches it: cuBLASLt's
    e4m3 x e4m3 GEMM (torch._scaled_mm, unit scales, bf16 out) at n^3, the
    denominator for the tensor-core kernels' TFLOP/s (MEASURED_PEAKS holds bf16
    only).  None if the library call is unavailable."""
    import torch
    try:
        gen = torch.Generator(device=dev)
        gen.manual_seed(17)
        a = torch.randn((n, n), generator=gen, device=dev).to(torch.float8_e4m3fn)
        b = torch.randn((n, n), generator=gen, device=dev).to(torch.float8_e4m3fn).t()  # column-major
        one = torch.ones((), dtype=torch.float32, device=dev)
        out = torch.empty((n, n), dtype=torch.bfloat16, device=dev)

        def mm(i):
            torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16, out=out)

        mm(0)
        torch.cuda.synchronize()
        us = _graph_time(s, mm, launches)
        return {"tflops": 2.0 * n ** 3 / (us * 1e-6) / 1e12, "us": us,
                "how": f"torch._scaled_mm (cuBLASLt) e4m3 x e4m3, {n}^3, unit scales, bf16 out"}
    except Exception as e:  # a measurement aid only
        return {"error": str(e)[:200]}


def _graph_time(s, fn, launches, reps=3):
    """Best per-call time (us) of `launches` calls of fn captured in one CUDA graph."""
    import torch
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(launches):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    best = float("inf")
    for _ in range(reps):
        with torch.cuda.stream(s):
            ev0.record(s)
            g.replay()
            ev1.record(s)
        ev1.synchronize()
        best = min(best, ev0.elapsed_time(ev1) / launches)
    del g
    return best * 1e3


def measure_attention_config4(gpu, dev, s, batches=(1, 8, 32), ctx=4096, peak=6541.5):
    """BASELINE config 4's attention: 32 query heads over 8 kv heads, head_dim 128,
    bf16 KV cache, context 4096, one query token per sequence.  Enough cache copies
    rotate that every launch reads from HBM (>= 256 MB a rotation)."""
    import torch
    H, Hkv, D = 32, 8, 128
    out = {}
    for B in batches:
        per = B * ctx * Hkv * D * 2 * 2
        copies = max(1, -(-256 * 2 ** 20 // per))
        gen = torch.Generator(device=dev)
        gen.manual_seed(17 + B)
        caches = [(torch.randn((B, ctx, Hkv, D), generator=gen, device=dev).to(torch.bfloat16),
                   torch.randn((B, ctx, Hkv, D), generator=gen, device=dev).to(torch.bfloat16)) for _ in range(copies)]
        q = torch.randn((B, H, D), generator=gen, device=dev).to(torch.bfloat16)
        o = torch.empty((B, H, D), dtype=torch.bfloat16, device=dev)
        ws = gpu.attention_workspace(B, H, Hkv, D, ctx)

        def one(i):
            k, v = caches[i % copies]
            gpu.attention_decode(q, k, v, o, ctx, 1.0 / D ** 0.5, ws, Hkv)

        for i in range(4):
            one(i)
        us = _graph_time(s, one, max(40, 4 * copies))
        nbytes = per + 2 * B * H * D * 2
        out[f"B{B}"] = {"us": us, "gbs": nbytes / (us * 1e-6) / 1e9, "frac": nbytes / (us * 1e-6) / 1e9 / peak,
                        "algorithmic_bytes": nbytes}
        del caches
        torch.cuda.empty_cache()
    return out


def measure_layers_config4(gpu, dev, s, batches=(1, 8, 32), layers=32, ctx=4096, steps=3, peak=6541.5):
    """BASELINE config 4 as a decode step over `layers` layers: per layer the q and
    kv projections (FP8 4096 x 4096 and 2048 x 4096, the projection shapes assumed:
    BASELINE gives none), the KV append of the new token, GQA attention (32 / 8
    heads, head_dim 128, bf16 cache at context 4096), the output projection (FP8
    4096 x 4096) and the MoE layer (router, 64 experts top-6, intermediate 1408, 2
    shared experts with a sigmoid gate).  Norms, rotary embedding and residual adds
    are not part of the path and are left out.  Weights random-init; every layer
    has its own allocations (one random bank is quantized, then copied)."""
    import torch

    import homelab_b200 as hb
    from homelab_b200.records import ExpertBank, SharedExpertBank
    Hd, E, K, I, SI, NH, NKV, D = 4096, 64, 6, 1408, 2816, 32, 8, 128
    Bmax = max(batches)
    gen = torch.Generator(device=dev)
    gen.manual_seed(23)
    src = ExpertBank(E, Hd, I, hb.SCALE_128X128, dev)
    src.fill_random(gpu, seed=24)
    sh_src = SharedExpertBank(Hd, SI, hb.SCALE_128X128, dev)
    sh_src.fill_random(gpu, seed=25)
    proj = []
    for (n, k) in ((Hd, Hd), (2 * NKV * D, Hd), (Hd, Hd)):
        w = (torch.randn((n, k), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
        proj.append(gpu.quantize_fp8(w.view(torch.int16), n, k, hb.SCALE_128X128))
    kc0 = torch.randn((Bmax, ctx, NKV, D), generator=gen, device=dev).to(torch.bfloat16)
    vc0 = torch.randn((Bmax, ctx, NKV, D), generator=gen, device=dev).to(torch.bfloat16)
    L = []
    for li in range(layers):
        bank = ExpertBank(E, Hd, I, hb.SCALE_128X128, dev)
        bank.buf.copy_(src.buf)
        sh = SharedExpertBank(Hd, SI, hb.SCALE_128X128, dev)
        for a, b in ((sh.gate_up_q, sh_src.gate_up_q), (sh.gate_up_s, sh_src.gate_up_s), (sh.down_q, sh_src.down_q),
                     (sh.down_s, sh_src.down_s), (sh.gate_w, sh_src.gate_w)):
            a.copy_(b)
        router = (torch.randn((E, Hd), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
        ml = hb.MoeLayer(hidden=Hd, experts=E, top_k=K, router_w=router.data_ptr(), recs=bank.addrs.data_ptr())
        ml.geo = bank.geo
        w = [(q.clone(), sc.clone()) for q, sc in proj]
        L.append(dict(bank=bank, sh=sh, S=sh.view(), router=router, ml=ml, w=w, kc=kc0.clone(), vc=vc0.clone()))
    del src, sh_src, kc0, vc0
    torch.cuda.empty_cache()
    out = {}
    for B in batches:
        xs = [torch.randn((B, Hd), generator=gen, device=dev).to(torch.bfloat16) for _ in range(2)]
        q = torch.empty((B, Hd), dtype=torch.float32, device=dev)
        kv = torch.empty((B, 2 * NKV * D), dtype=torch.float32, device=dev)
        att = torch.empty((B, NH, D), dtype=torch.bfloat16, device=dev)
        o = torch.empty((B, Hd), dtype=torch.bfloat16, device=dev)
        nxt = [torch.empty((B, Hd), dtype=torch.bfloat16, device=dev) for _ in range(2)]
        wsq = gpu.gemm_fp8_workspace(B, Hd, Hd) if B >= 2 else None
        wskv = gpu.gemm_fp8_workspace(B, 2 * NKV * D, Hd) if B >= 2 else None
        wso = gpu.gemm_fp8_workspace(B, Hd, Hd) if B >= 2 else None
        wsa = gpu.attention_workspace(B, NH, NKV, D, ctx)
        wsl = gpu.moe_layer_workspace(L[0]["ml"], L[0]["S"], B)

        def step(i):
            x = xs[i % 2]
            for li, ly in enumerate(L):
                (wq, sq), (wkv, skv), (wo, so) = ly["w"]
                kc, vc = ly["kc"][:B], ly["vc"][:B]
                gpu.gemm_fp8(x, wq, sq, q, B, Hd, Hd, hb.SCALE_128X128, wsq)
                gpu.gemm_fp8(x, wkv, skv, kv, B, 2 * NKV * D, Hd, hb.SCALE_128X128, wskv)
                gpu.kv_append(kv[:, :NKV * D], kc, ctx - 1)
                gpu.kv_append(kv[:, NKV * D:], vc, ctx - 1)
                gpu.attention_decode(q.view(B, NH, D), kc, vc, att, ctx, 1.0 / D ** 0.5, wsa, NKV)
                gpu.gemm_fp8(att.view(B, Hd), wo, so, o, B, Hd, Hd, hb.SCALE_128X128, wso)
                y = nxt[li % 2]
                gpu.moe_layer_decode(ly["ml"], ly["S"], o, B, y, wsl)
                x = y

        for i in range(2):
            step(i)
        torch.cuda.synchronize()
        us = _graph_time(s, step, steps, reps=2)
        distinct = E * (1.0 - ((E - K) / E) ** B)  # expected distinct routed experts a layer
        wb = L[0]["bank"].stride  # upper bound of an expert's bytes (record stride)
        from homelab_b200.records import weight_bytes
        eb = weight_bytes(L[0]["bank"].geo)
        per_layer = (2 * Hd * Hd + 2 * NKV * D * Hd + B * ctx * NKV * D * 2 * 2 + E * Hd * 2 +
                     (2 * SI * Hd + Hd * SI) + distinct * eb)
        nbytes = layers * per_layer
        out[f"B{B}"] = {"us_per_step": us, "tokens_per_s": B / (us * 1e-6), "gbs": nbytes / (us * 1e-6) / 1e9,
                        "frac": nbytes / (us * 1e-6) / 1e9 / peak, "expected_distinct_experts": distinct,
                        "algorithmic_bytes_per_step": nbytes, "record_stride": wb}
    del L
    torch.cuda.empty_cache()
    return out


def measure_offload_config5(gpu, dev, s, batch=8, experts=64, cold=(0, 2, 4, 8), reps=3):
    """BASELINE config 5's offload: expert records of hidden 4096 / intermediate 2048
    (25.2 MB each) in a pinned host arena served by the expert tier
    (homelab_b200.stage.ExpertTier: the two-phase fetch).  A step routes `batch`
    tokens over `experts` experts (top-8), fetches them with `c` of them cold (their
    records copy in on the copy queue while the resident ones compute), then runs
    the cold ones and the slot combine.  Reported per c: the whole step on the
    compute stream, the same step with every record resident, and the c records'
    copies alone."""
    import numpy as np
    import torch

    import homelab_b200 as hb
    from homelab_b200.records import ExpertBank
    from homelab_b200.stage import ExpertTier, HostArena, Transfer, stage_records
    Hd, I, K = 4096, 2048, 8
    bank = ExpertBank(experts, Hd, I, hb.SCALE_128X128, dev)
    bank.fill_random(gpu, seed=41)
    arena = HostArena(experts, bank.stride)
    arena.buf.copy_(bank.buf.cpu())
    gen = torch.Generator(device=dev)
    gen.manual_seed(42)
    router = (torch.randn((experts, Hd), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
    x = torch.randn((batch, Hd), generator=gen, device=dev).to(torch.bfloat16)
    logits = torch.empty((batch, experts), dtype=torch.float32, device=dev)
    ids = torch.empty((batch, K), dtype=torch.int32, device=dev)
    w = torch.empty((batch, K), dtype=torch.float32, device=dev)
    gpu.router_logits(x, router, logits, batch, experts, Hd)
    gpu.router_topk(logits, ids, w, batch, experts, K)
    ids_h = ids.cpu().numpy()
    active = np.unique(ids_h)
    geo = bank.geo
    # exactly the step's experts fit: fetching c others evicts c of them (LRU)
    tier = ExpertTier(arena, 1, experts, slots=len(active), device=dev)
    out = {"batch": batch, "distinct_experts": int(len(active)), "record_bytes": bank.stride}
    flat = ids_h.reshape(-1)
    pos = np.searchsorted(active, flat)  # expert index of every slot

    def tables(addrs, ready):
        """Resident groups first, then the loading ones (Moe::begin_routed's order); numpy, O(A)."""
        ready = np.asarray(ready, dtype=bool)
        rank_of = np.empty(len(active), dtype=np.int64)
        order = np.concatenate([np.flatnonzero(ready), np.flatnonzero(~ready)])
        rank_of[order] = np.arange(len(order))
        a_order = np.argsort(rank_of[pos], kind="stable")  # assignments grouped, slots in slot order
        slot = np.empty(batch * K, dtype=np.int32)
        slot[a_order] = np.arange(batch * K, dtype=np.int32)
        counts = np.bincount(rank_of[pos], minlength=len(active))
        off = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
        tok = (a_order // K).astype(np.int32)
        recs = np.asarray(addrs, dtype=np.int64)[order]
        return (torch.from_numpy(recs).to(dev), torch.from_numpy(off).to(dev), torch.from_numpy(tok).to(dev),
                torch.from_numpy(slot).to(dev), int(ready.sum()))

    A = batch * K
    h = torch.empty((A, I), dtype=torch.float32, device=dev)
    y = torch.empty((A, Hd), dtype=torch.float32, device=dev)
    o = torch.empty((batch, Hd), dtype=torch.float32, device=dev)

    def run(recs, offd, tokd, slotd, nr):
        n = len(active)
        if nr:
            gpu.moe_gate_up(recs[:nr], offd[:nr + 1], tokd, nr, x, h, geo)
            gpu.moe_down(recs[:nr], offd[:nr + 1], nr, h, y, geo)
        tier.finish_fetch()
        if nr < n:
            gpu.moe_gate_up(recs[nr:], offd[nr:], tokd, n - nr, x, h, geo)
            gpu.moe_down(recs[nr:], offd[nr:], n - nr, h, y, geo)
        gpu.moe_combine_slots(y, slotd, w, o, batch, Hd, K)

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    tr = Transfer(dev)
    q = torch.cuda.ExternalStream(tr.queue, device=dev)
    for c in cold:
        best, best_h2d = float("inf"), float("inf")
        for r in range(reps + 1):
            # make every active record resident, then evict c of them by fetching others
            tier.begin_fetch(0, active)
            tier.finish_fetch()
            others = [e for e in range(experts) if e not in set(active.tolist())][:c]
            if c:
                tier.begin_fetch(0, list(active[c:]) + others)
                tier.finish_fetch()
            torch.cuda.synchronize()
            with torch.cuda.stream(torch.cuda.current_stream(dev)):
                ev0.record()
                addrs, ready = tier.begin_fetch(0, active)
                run(*tables(addrs, ready))
                ev1.record()
            ev1.synchronize()
            if r:
                best = min(best, ev0.elapsed_time(ev1) * 1e3)
            if c and r:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                slots = torch.empty(c * bank.stride, dtype=torch.uint8, device=dev)
                e0.record(q)
                stage_records(tr, arena, list(range(c)), [slots.data_ptr() + j * bank.stride for j in range(c)])
                e1.record(q)
                e1.synchronize()
                best_h2d = min(best_h2d, e0.elapsed_time(e1) * 1e3)
                del slots
        out[f"cold{c}"] = {"us_per_step": best, "h2d_only_us": best_h2d if c else 0.0,
                           "ready": int(len(active) - c)}
    tier.close()
    tr.close()
    del bank
    torch.cuda.empty_cache()
    return out


def measure_ep_config5(gpu, dev, s, rank, world, batches=(32, 128), steps=8):
    """BASELINE config 5 sharded over the ranks (expert parallelism): hidden 4096,
    256 experts top-8, intermediate 2048, 128x128 block scales, experts e on rank
    e / (256 / world) (32 per GPU at 8 GPUs); each rank decodes `batch` tokens per
    step with the chain of kernels whose dispatch and return are stores into the
    peers' mailboxes over NVLink (homelab_b200.ep.EpPeerMoeLayer).  Device-timed,
    max over ranks; tokens/s over all ranks."""
    import torch
    import torch.distributed as dist

    import homelab_b200 as hb
    from homelab_b200.ep import EpGpuOps, EpPeerMailboxes, EpPeerMoeLayer
    from homelab_b200.records import ExpertBank
    Hd, I, E, K = 4096, 2048, 256, 8
    epr = E // world
    bank = ExpertBank(epr, Hd, I, hb.SCALE_128X128, dev)
    bank.fill_random(gpu, seed=100 + rank)
    gen = torch.Generator(device=dev)
    gen.manual_seed(7)
    router = (torch.randn((E, Hd), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
    out = {"experts_per_gpu": epr, "transport": "peer mailboxes over NVLink, chain of kernels"}
    for B in batches:
        mb = EpPeerMailboxes(dist.group.WORLD, Hd, K, B, torch.bfloat16, dev)
        layer = EpPeerMoeLayer(EpGpuOps(dev), mb, rank, Hd, E, K, I, router, bank.addrs, bank.geo, B)
        gen.manual_seed(50 + rank)
        xs = [torch.randn((B, Hd), generator=gen, device=dev).to(torch.bfloat16) for _ in range(4)]
        o = torch.empty((B, Hd), dtype=torch.float32, device=dev)
        with torch.cuda.stream(s):
            for i in range(3):
                layer.forward(xs[i % 4], B, o)
        torch.cuda.synchronize()
        dist.barrier()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s):
            ev0.record(s)
            for i in range(steps):
                layer.forward(xs[i % 4], B, o)
            ev1.record(s)
        ev1.synchronize()
        ms = torch.tensor([ev0.elapsed_time(ev1) / steps], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        us = float(ms.item()) * 1e3
        out[f"B{B}"] = {"batch_per_gpu": B, "us_per_step": us, "tokens_per_s": world * B / (us * 1e-6)}
        torch.cuda.synchronize()
        mb.close()
    del bank
    torch.cuda.empty_cache()
    return out


def measure_reference_gemv_config1(gpu, dev, s, copies=16, launches=320):
    """The reference's own FP8 GEMV kernel (gemv_fp8_t1, crates/oominf-cuda/kernels/
    ops.cu:338-440, built from the reference sources by oracle/ref/Makefile and
    launched with the plan of Gpu::gemv_at, linear.rs:259-350) beside ours, on
    config 1 with the reference's 1x128 scales and fp32 x / y (its types),
    back-to-back launches over `copies` weight copies.  None if the reference
    build is absent."""
    import ctypes as C

    import torch

    import homelab_b200 as hb
    import oracle.refk as refk
    if not refk.available():
        return None
    ref = refk.RefKernels(dev)
    n = k = 4096
    gen = torch.Generator(device=dev)
    gen.manual_seed(12)
    qs, ss = [], []
    for c in range(copies):
        wt = (torch.randn((n, k), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
        q, sc = gpu.quantize_fp8(wt.view(torch.int16), n, k, hb.SCALE_1X128)
        qs.append(q)
        ss.append(sc)
    x = torch.randn((1, k), generator=gen, device=dev)
    y = torch.empty((1, n), dtype=torch.float32, device=dev)
    splits, _, tiles = ref.gemv_plan(1, n, k)
    partial = torch.empty(max(splits * n, 1), dtype=torch.float32, device=dev)
    tickets = torch.zeros(max(tiles, 1), dtype=torch.int32, device=dev)

    def theirs(i):
        rc = ref.L.orl_gemv_fp8(x.data_ptr(), qs[i % copies].data_ptr(), ss[i % copies].data_ptr(), y.data_ptr(),
                                partial.data_ptr(), tickets.data_ptr(), 1, n, k,
                                C.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
        if rc != 0:
            raise RuntimeError(f"reference gemv failed ({rc})")

    def ours(i):
        gpu.gemm_fp8(x, qs[i % copies], ss[i % copies], y, 1, n, k, hb.SCALE_1X128)

    for i in range(8):
        theirs(i)
        ours(i)
    nbytes = n * k + n * (k // 128) * 4 + k * 4 + n * 4
    res = {}
    for name, fn in (("reference_gemv_fp8_t1", theirs), ("ours", ours)):
        us = _graph_time(s, fn, launches)
        res[name] = {"us": us, "gbs": nbytes / (us * 1e-6) / 1e9}
    res["workload"] = "config1 4096x4096 e4m3 with 1x128 scales, x fp32 batch 1, fp32 out"
    res["algorithmic_bytes"] = nbytes
    return res


def measure_reference_mlp_config3(gpu, dev, s, B=64, launches=40):
    """The reference's own path above 16 tokens (Linear::gemm_fp8, crates/oominf-cuda/
    src/linear.rs:35-81, 140-205) on config 3's MLP at batch B: its fp8_dequantize_blocks
    kernel (ops.cu:583-590) makes bf16 weights, its f32_to_bf16 rounds the activations,
    cuBLAS multiplies in bf16 with fp32 output (gemm_ex, here torch.mm), and its
    silu_mul_rows joins the two GEMMs; 1x128 scales (its format).  Two forms: the bf16
    weights already dequantized (the reference keeps up to 512 MB of them, one layer of
    this model) and dequantized on every call (a model of many layers cycles that
    cache).  Reference kernels built from its sources by oracle/ref/Makefile; None if
    that build is absent."""
    import torch

    import homelab_b200 as hb
    import oracle.refk as refk
    if not refk.available():
        return None
    ref = refk.RefKernels(dev)
    H, I2 = 4096, 28672
    I = I2 // 2
    gen = torch.Generator(device=dev)
    gen.manual_seed(31)
    w_gu = (torch.randn((I2, H), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
    q_gu, s_gu = gpu.quantize_fp8(w_gu.view(torch.int16), I2, H, hb.SCALE_1X128)
    del w_gu
    w_d = (torch.randn((H, I), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
    q_d, s_d = gpu.quantize_fp8(w_d.view(torch.int16), H, I, hb.SCALE_1X128)
    del w_d
    bf_gu = torch.empty((I2, H), dtype=torch.bfloat16, device=dev)
    bf_d = torch.empty((H, I), dtype=torch.bfloat16, device=dev)
    ref.dequant_fp8(q_gu, s_gu, bf_gu, I2, H)
    ref.dequant_fp8(q_d, s_d, bf_d, H, I)
    x = torch.randn((B, H), generator=gen, device=dev)
    xb = torch.empty((B, H), dtype=torch.bfloat16, device=dev)
    gu = torch.empty((B, I2), dtype=torch.float32, device=dev)
    h = torch.empty((B, I), dtype=torch.float32, device=dev)
    hb16 = torch.empty((B, I), dtype=torch.bfloat16, device=dev)
    y = torch.empty((B, H), dtype=torch.float32, device=dev)

    def mlp(dequant):
        if dequant:
            ref.dequant_fp8(q_gu, s_gu, bf_gu, I2, H)
        ref.f32_to_bf16(x, xb, B * H)
        torch.mm(xb, bf_gu.t(), out_dtype=torch.float32, out=gu)
        ref.silu_mul_rows(gu, h, B, I)
        if dequant:
            ref.dequant_fp8(q_d, s_d, bf_d, H, I)
        ref.f32_to_bf16(h, hb16, B * I)
        torch.mm(hb16, bf_d.t(), out_dtype=torch.float32, out=y)

    mlp(True)
    torch.cuda.synchronize()
    res = {"workload": f"config3 MLP batch {B}: fused gate/up [28672, 4096] + SwiGLU + down [4096, 14336], "
                       "FP8 e4m3 1x128 scales, x fp32",
           "weight_bytes_fp8": I2 * H + H * I, "weight_bytes_bf16": 2 * (I2 * H + H * I)}
    for name, dq in (("bf16_weights_cached", False), ("dequantized_each_call", True)):
        us = _graph_time(s, lambda i, dq=dq: mlp(dq), launches)
        res[name] = {"us_per_mlp": us, "tokens_per_s": B / (us * 1e-6)}
    del bf_gu, bf_d
    torch.cuda.empty_cache()
    return res


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    result, _ = run_ours(args, rank, world, local_rank)
    if args.profile:
        print(f"ran {args.profile} eager decode steps", flush=True)
        return
    if rank == 0 and world == 1 and not args.no_cpu:
        per, threads, sample, _ = time_cpu(args.batch, args.cpu_seconds)
        per1, _, sample1, _ = time_cpu(args.batch, args.cpu_seconds / 3, threads=1)
        try:
            import torch
            from homelab_b200.backend import Gpu
            result["reference_gpu_gemv_config1"] = measure_reference_gemv_config1(
                Gpu(0), torch.device("cuda", 0), torch.cuda.Stream(torch.device("cuda", 0)))
        except Exception as e:  # the reference's kernels are a baseline: report, do not fail the run
            result["reference_gpu_gemv_config1"] = {"error": str(e)[:200]}
        try:
            result["reference_gpu_mlp_config3"] = measure_reference_mlp_config3(
                Gpu(0), torch.device("cuda", 0), torch.cuda.Stream(torch.device("cuda", 0)))
        except Exception as e:
            result["reference_gpu_mlp_config3"] = {"error": str(e)[:200]}
        result["cpu_baseline"] = {"value": args.batch / per, "unit": "tokens/s", "cores": threads,
                                  "kind": "port", "cpu_model": cpu_model(), "value_1_thread": args.batch / per1,
                                  "sample": sample + "; oominf-cpu host expert path restated in C++/AVX-512; "
                                            "one thread: " + sample1}
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
