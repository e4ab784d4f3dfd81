"""FP8 expert records: the byte layout the expert kernels read in place.

One record per expert, as the .oom format keeps them (projects/oom-inference/
docs/dev/format.md:40-76): parts at PART_ALIGN = 256-byte offsets, the record
stride rounded up to ALIGN = 4096.  Layout tag "fp8-e4m3-b128x128" (or
"-b1x128"): gate and up e4m3 [inter, hidden], down e4m3 [hidden, inter], each
followed by its fp32 block scales.
"""
from __future__ import annotations

import torch

from ._lib import SCALE_128X128, SCALE_1X128, Fp8Record

PART_ALIGN = 256
ALIGN = 4096


def _up(v: int, a: int) -> int:
    return (v + a - 1) // a * a


def scale_rows(n: int, layout: int) -> int:
    return (n + 127) // 128 if layout == SCALE_128X128 else n


def scale_bytes(n: int, k: int, layout: int) -> int:
    return scale_rows(n, layout) * ((k + 127) // 128) * 4


def record_layout(hidden: int, inter: int, layout: int = SCALE_128X128):
    """(geometry, stride) of an FP8 expert record: gate, up, down, then their
    scales, each part at a PART_ALIGN offset, the stride rounded up to ALIGN
    (the library's oomb_fp8_record_layout)."""
    import ctypes as C

    from . import _lib
    g = Fp8Record()
    stride = C.c_size_t()
    _lib.check(_lib.lib().oomb_fp8_record_layout(hidden, inter, layout, C.byref(g), C.byref(stride)),
               "record_layout")
    return g, int(stride.value)


def weight_bytes(g: Fp8Record) -> int:
    """Bytes of weights and scales one expert's FFN reads (the roofline unit)."""
    return (3 * g.hidden * g.inter + 2 * scale_bytes(g.inter, g.hidden, g.layout)
            + scale_bytes(g.hidden, g.inter, g.layout))


class ExpertBank:
    """`experts` FP8 records in one device allocation, plus their address table."""

    def __init__(self, experts: int, hidden: int, inter: int, layout: int = SCALE_128X128,
                 device: torch.device | str = "cuda"):
        self.geo, self.stride = record_layout(hidden, inter, layout)
        self.experts = experts
        self.buf = torch.zeros(experts * self.stride, dtype=torch.uint8, device=device)
        base = self.buf.data_ptr()
        self.addrs = torch.tensor([base + e * self.stride for e in range(experts)], dtype=torch.int64,
                                  device=device)

    def part(self, e: int, off: int, nbytes: int) -> torch.Tensor:
        s = e * self.stride + off
        return self.buf[s:s + nbytes]

    def views(self, e: int):
        """(gate_q, gate_s, up_q, up_s, down_q, down_s) tensors aliasing record e."""
        g = self.geo
        H, I, L = g.hidden, g.inter, g.layout
        nb_h, nb_i = (H + 127) // 128, (I + 127) // 128
        gq = self.part(e, g.gate_weight, I * H).view(I, H)
        uq = self.part(e, g.up_weight, I * H).view(I, H)
        dq = self.part(e, g.down_weight, H * I).view(H, I)
        gs = self.part(e, g.gate_scale, scale_bytes(I, H, L)).view(torch.float32).view(scale_rows(I, L), nb_h)
        us = self.part(e, g.up_scale, scale_bytes(I, H, L)).view(torch.float32).view(scale_rows(I, L), nb_h)
        ds = self.part(e, g.down_scale, scale_bytes(H, I, L)).view(torch.float32).view(scale_rows(H, L), nb_i)
        return gq, gs, uq, us, dq, ds

    def fill_random(self, gpu, seed: int, sigma: float = 0.02):
        """Quantize N(0, sigma) bf16 weights of every expert into the records on the device."""
        g = self.geo
        H, I, L = g.hidden, g.inter, g.layout
        gen = torch.Generator(device=self.buf.device)
        gen.manual_seed(seed)
        for e in range(self.experts):
            gq, gs, uq, us, dq, ds = self.views(e)
            for (q, s, n, k) in ((gq, gs, I, H), (uq, us, I, H), (dq, ds, H, I)):
                w = (torch.randn((n, k), generator=gen, device=self.buf.device) * sigma).to(torch.bfloat16)
                gpu.quantize_fp8(w.view(torch.int16), n, k, L, q, s)

    def host_records(self):
        """A host copy of every record as numpy uint8 arrays (for the CPU oracle)."""
        host = self.buf.cpu().numpy()
        return [host[e * self.stride:(e + 1) * self.stride] for e in range(self.experts)]


class SharedExpertBank:
    """A layer's shared expert(s) on the device: one FP8 SwiGLU MLP of width `inter`
    (all shared experts side by side; gate rows then up rows of gate_up [2 * inter,
    hidden], down [hidden, inter]) and a bf16 gate-logit row [hidden] (or none),
    with the oomb_shared_expert view the layer entry point takes."""

    def __init__(self, hidden: int, inter: int, layout: int = SCALE_128X128, device: torch.device | str = "cuda",
                 gated: bool = True):
        self.hidden, self.inter, self.layout = hidden, inter, layout
        dev = torch.device(device)
        nb_h, nb_i = (hidden + 127) // 128, (inter + 127) // 128
        self.gate_up_q = torch.zeros((2 * inter, hidden), dtype=torch.uint8, device=dev)
        self.gate_up_s = torch.zeros((scale_rows(2 * inter, layout), nb_h), dtype=torch.float32, device=dev)
        self.down_q = torch.zeros((hidden, inter), dtype=torch.uint8, device=dev)
        self.down_s = torch.zeros((scale_rows(hidden, layout), nb_i), dtype=torch.float32, device=dev)
        self.gate_w = torch.zeros(hidden, dtype=torch.bfloat16, device=dev) if gated else None

    def fill_random(self, gpu, seed: int, sigma: float = 0.02):
        """Quantize N(0, sigma) bf16 weights on the device; the gate row N(0, sigma) in bf16."""
        gen = torch.Generator(device=self.gate_up_q.device)
        gen.manual_seed(seed)
        for (q, s, n, k) in ((self.gate_up_q, self.gate_up_s, 2 * self.inter, self.hidden),
                             (self.down_q, self.down_s, self.hidden, self.inter)):
            w = (torch.randn((n, k), generator=gen, device=q.device) * sigma).to(torch.bfloat16)
            gpu.quantize_fp8(w.view(torch.int16), n, k, self.layout, q, s)
        if self.gate_w is not None:
            self.gate_w.copy_((torch.randn(self.hidden, generator=gen, device=q.device) * sigma).to(torch.bfloat16))

    def view(self):
        from ._lib import SharedExpert
        return SharedExpert(hidden=self.hidden, inter=self.inter, scale_layout=self.layout,
                            gate_up_q=self.gate_up_q.data_ptr(), gate_up_scale=self.gate_up_s.data_ptr(),
                            down_q=self.down_q.data_ptr(), down_scale=self.down_s.data_ptr(),
                            gate_w=self.gate_w.data_ptr() if self.gate_w is not None else None)
