"""Device timeline of the decode step and of the stand-alone GEMV.

    python -m homelab_b200.build --timeline      # liboomb_timeline.so (-DOOMB_TIMELINE)
    python -m homelab_b200.timeline [decode|gemv|all]

The tracing build stamps %globaltimer at fixed points of every kernel into a
slot per (kind, event, CTA); each launch overwrites its kind's slots, so after
a CUDA-graph replay of back-to-back launches the table holds the last launch.
This tool replays the config-2 decode step (batch 1, 16 steps over 4 layer
replicas) and the config-1 GEMV (64 launches over 16 weight copies), then prints
each event's time from the launch's first CTA entry as min / median / max over
CTAs.  The stamps cost a store each: step times of the tracing build run about
1 us longer than the plain library's.
"""
from __future__ import annotations

import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
TRACE_LIB = os.path.join(HERE, "liboomb_timeline.so")
KINDS, EVENTS, CTAS = 8, 16, 1024
KIND = {1: "route", 2: "gate_up", 3: "down", 4: "combine", 5: "gemv"}
EVENT = {0: "entry", 1: "waited", 2: "end", 3: "first_copy", 4: "first_stage", 5: "logits_done", 6: "last_cta",
         7: "x_staged", 8: "topk_done", 9: "first_meta", 10: "last_copy"}


def _table(raw) -> np.ndarray:
    import torch
    buf = np.zeros((KINDS, EVENTS, CTAS), dtype=np.uint64)
    torch.cuda.synchronize()
    if raw.oomb_timeline_read(buf.ctypes.data_as(C.c_void_p), C.c_size_t(buf.nbytes)) != 0:
        raise RuntimeError("oomb_timeline_read failed")
    return buf


def report(buf: np.ndarray, kinds, title: str) -> str:
    starts = [buf[k, 0][buf[k, 0] > 0] for k in kinds]
    t0 = min(int(v.min()) for v in starts if len(v))
    lines = [f"== {title} (us from the first CTA entry; min / median / max over CTAs)"]
    for k in kinds:
        for e in range(EVENTS):
            v = buf[k, e][buf[k, e] > 0].astype(np.int64)
            if len(v) == 0:
                continue
            d = (v - t0) / 1e3
            lines.append(f"  {KIND[k]:8s} {EVENT.get(e, str(e)):12s} n={len(v):4d} "
                         f"{d.min():7.2f} {np.median(d):7.2f} {d.max():7.2f}")
    return "\n".join(lines)


def _timed_replay(g, s, n):
    import torch
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        e0.record(s)
        g.replay()
        e1.record(s)
    e1.synchronize()
    return e0.elapsed_time(e1) * 1e3 / n


def run_gemv(gpu, raw, dev, s) -> str:
    import torch

    import homelab_b200 as hb
    n = k = 4096
    gen = torch.Generator(device=dev)
    gen.manual_seed(11)
    mats = []
    for _ in range(16):
        w = (torch.randn((n, k), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
        mats.append(gpu.quantize_fp8(w.view(torch.int16), n, k, hb.SCALE_128X128))
    x = torch.randn((1, k), generator=gen, device=dev).to(torch.bfloat16)
    y = torch.empty((1, n), dtype=torch.bfloat16, device=dev)
    for i in range(8):
        gpu.gemm_fp8(x, mats[i % 16][0], mats[i % 16][1], y, 1, n, k, hb.SCALE_128X128)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(64):
            gpu.gemm_fp8(x, mats[i % 16][0], mats[i % 16][1], y, 1, n, k, hb.SCALE_128X128)
    us = _timed_replay(g, s, 64)
    del g
    return report(_table(raw), [5], f"config-1 GEMV, last of 64 back-to-back launches ({us:.2f} us per launch)")


def run_decode(gpu, raw, dev, s) -> str:
    import torch

    import homelab_b200 as hb
    from homelab_b200.records import ExpertBank
    H, E, K, I = 2048, 128, 8, 768
    gen = torch.Generator(device=dev)
    gen.manual_seed(7)
    layers = []
    for li in range(4):
        bank = ExpertBank(E, H, I, hb.SCALE_128X128, dev)
        bank.fill_random(gpu, seed=5 + li)
        router = (torch.randn((E, H), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
        L = hb.MoeLayer(hidden=H, experts=E, top_k=K, router_w=router.data_ptr(), recs=bank.addrs.data_ptr())
        L.geo = bank.geo
        layers.append((bank, router, L))
    ws = gpu.moe_decode_workspace(layers[0][2], 1)
    xs = [torch.randn((1, H), generator=gen, device=dev).to(torch.bfloat16) for _ in range(4)]
    out = torch.empty((1, H), dtype=torch.bfloat16, device=dev)
    for i in range(4):
        gpu.moe_decode(layers[i % 4][2], xs[i % 4], 1, out, ws)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(16):
            gpu.moe_decode(layers[i % 4][2], xs[i % 4], 1, out, ws)
    us = _timed_replay(g, s, 16)
    del g
    if gpu.device_error() != 0:
        raise RuntimeError("a bounded device wait ran out")
    return report(_table(raw), [1, 2, 3, 4], f"config-2 decode_kernel, last of 16 graph steps ({us:.2f} us per step)")


def main(argv) -> int:
    import torch

    from homelab_b200 import _lib
    from homelab_b200.backend import Gpu
    if not os.path.exists(TRACE_LIB):
        raise SystemExit(f"{TRACE_LIB} is missing: python -m homelab_b200.build --timeline")
    if _lib._LIB is not None:
        raise SystemExit("the plain library is already loaded in this process")
    _lib.LIB_PATH = TRACE_LIB  # the same C ABI, with the device timeline compiled in
    _lib.lib()
    raw = C.CDLL(TRACE_LIB)
    what = argv[1] if len(argv) > 1 else "all"
    dev = torch.device("cuda", 0)
    gpu = Gpu(0)
    s = torch.cuda.Stream(dev)
    if what in ("all", "gemv"):
        print(run_gemv(gpu, raw, dev, s))
        torch.cuda.empty_cache()
    if what in ("all", "decode"):
        print(run_decode(gpu, raw, dev, s))
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
