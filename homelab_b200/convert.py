"""FP8 expert records in the engine's weight format (an `.oom` directory).

The routed experts of a model become one record per (layer, expert) in
experts.bin, grouped by layer, each group described in index.json by its
record schema (projects/oom-inference/docs/dev/format.md:37-106): this module
adds the layout tags "fp8-e4m3-b128x128" and "fp8-e4m3-b1x128", whose parts are

    gate.weight        F8_E4M3 [inter, hidden]
    up.weight          F8_E4M3 [inter, hidden]
    down.weight        F8_E4M3 [hidden, inter]
    gate.weight_scale  F32     [ceil(inter/128), ceil(hidden/128)]   (1x128: [inter, ...])
    up.weight_scale    F32     same
    down.weight_scale  F32     [ceil(hidden/128), ceil(inter/128)]   (1x128: [hidden, ...])

at PART_ALIGN (256-byte) offsets, the record stride rounded up to ALIGN (4096):
the byte layout the expert kernels read in place (oomb_fp8_record_layout), so a
record copied verbatim into a device slot is ready to run.  Conversion
quantizes on the device (oomb_quantize_fp8_record, byte-identical to the
engine's fp8::quantize_blocks and its 128x128 generalisation).

Record checksums: the format keeps an xxh3-64 per record; this writer leaves
the "xxh3" list empty (no xxh3 implementation here), which the engine's own
writer fills from the same bytes when its converter adapter calls the
per-expert quantizer.  The loader here checks the layout tag
and the schema instead, and refuses anything else.
"""
from __future__ import annotations

import ctypes as C
import json
import os

import numpy as np
import torch

from . import _lib
from ._lib import SCALE_128X128, SCALE_1X128, Fp8Record, check

LAYOUT_TAGS = {SCALE_128X128: "fp8-e4m3-b128x128", SCALE_1X128: "fp8-e4m3-b1x128"}


def record_layout(hidden: int, inter: int, layout: int = SCALE_128X128):
    """(geometry, stride) of an FP8 expert record, from the library's C layout function."""
    g = Fp8Record()
    stride = C.c_size_t()
    check(_lib.lib().oomb_fp8_record_layout(hidden, inter, layout, C.byref(g), C.byref(stride)), "record_layout")
    return g, int(stride.value)


def record_schema(hidden: int, inter: int, layout: int = SCALE_128X128):
    """The index.json parts list of an FP8 record, and its stride."""
    g, stride = record_layout(hidden, inter, layout)
    nb_h, nb_i = (hidden + 127) // 128, (inter + 127) // 128
    r_i = (inter + 127) // 128 if layout == SCALE_128X128 else inter
    r_h = (hidden + 127) // 128 if layout == SCALE_128X128 else hidden
    parts = [
        ("gate.weight", "F8_E4M3", [inter, hidden], g.gate_weight, inter * hidden),
        ("up.weight", "F8_E4M3", [inter, hidden], g.up_weight, inter * hidden),
        ("down.weight", "F8_E4M3", [hidden, inter], g.down_weight, hidden * inter),
        ("gate.weight_scale", "F32", [r_i, nb_h], g.gate_scale, r_i * nb_h * 4),
        ("up.weight_scale", "F32", [r_i, nb_h], g.up_scale, r_i * nb_h * 4),
        ("down.weight_scale", "F32", [r_h, nb_i], g.down_scale, r_h * nb_i * 4),
    ]
    return [dict(name=n, dtype=d, shape=s, offset=int(o), nbytes=int(b)) for n, d, s, o, b in parts], stride


def convert_experts(out_dir: str, layers, hidden: int, inter: int, layout: int = SCALE_128X128,
                    device="cuda", source: dict | None = None) -> dict:
    """Writes experts.bin and index.json under out_dir.  `layers` yields, per
    layer, (gate [E, inter, hidden], up [E, inter, hidden], down [E, hidden,
    inter]) bf16 tensors (host or device); each expert is quantized on the
    device into a zeroed record and appended.  Returns the index."""
    os.makedirs(out_dir, exist_ok=True)
    dev = torch.device(device)
    L = _lib.lib()
    parts, stride = record_schema(hidden, inter, layout)
    geo, _ = record_layout(hidden, inter, layout)
    rec = torch.zeros(stride, dtype=torch.uint8, device=dev)
    groups, offset = [], 0
    with open(os.path.join(out_dir, "experts.bin"), "wb") as f:
        for li, (gate, up, down) in enumerate(layers):
            n_e = int(gate.shape[0])
            if tuple(gate.shape) != (n_e, inter, hidden) or tuple(up.shape) != (n_e, inter, hidden) or \
                    tuple(down.shape) != (n_e, hidden, inter):
                raise ValueError(f"layer {li}: expert shapes do not match hidden {hidden}, inter {inter}")
            for e in range(n_e):
                gq, uq, dq = (t[e].to(dev).to(torch.bfloat16).contiguous() for t in (gate, up, down))
                rec.zero_()
                check(L.oomb_quantize_fp8_record(gq.data_ptr(), uq.data_ptr(), dq.data_ptr(), C.byref(geo),
                                                 rec.data_ptr(), torch.cuda.current_stream(dev).cuda_stream),
                      "quantize_fp8_record")
                f.write(rec.cpu().numpy().tobytes())
            groups.append(dict(layer=li, num_experts=n_e, offset=offset, stride=stride, layout=LAYOUT_TAGS[layout],
                               parts=parts, xxh3=[]))
            offset += n_e * stride
    index = {"format": "oominf", "version": 0, "source": source or {},
             "files": {"experts": {"bytes": offset}}, "tensors": [], "expert_groups": groups}
    with open(os.path.join(out_dir, "index.json"), "w") as f:
        json.dump(index, f, indent=1)
    return index


def load_expert_group(model_dir: str, layer: int, device="cuda"):
    """Reads one layer's FP8 records from a converted directory into device memory:
    returns (records uint8 tensor [E * stride], record address tensor [E], geometry,
    stride).  Refuses groups whose layout tag or schema is not this module's."""
    with open(os.path.join(model_dir, "index.json")) as f:
        index = json.load(f)
    group = next((g for g in index["expert_groups"] if g["layer"] == layer), None)
    if group is None:
        raise KeyError(f"no expert group for layer {layer}")
    tag = group["layout"]
    layout = next((k for k, v in LAYOUT_TAGS.items() if v == tag), None)
    if layout is None:
        raise ValueError(f"layout {tag!r} is not an FP8 record layout this loader implements")
    shape = {p["name"]: p["shape"] for p in group["parts"]}
    inter, hidden = shape["gate.weight"]
    parts, stride = record_schema(hidden, inter, layout)
    if parts != group["parts"] or stride != group["stride"]:
        raise ValueError("record schema does not match the FP8 record layout")
    n_e = group["num_experts"]
    raw = np.fromfile(os.path.join(model_dir, "experts.bin"), dtype=np.uint8, count=n_e * stride,
                      offset=group["offset"])
    dev = torch.device(device)
    buf = torch.from_numpy(raw).to(dev)
    addrs = torch.tensor([buf.data_ptr() + e * stride for e in range(n_e)], dtype=torch.int64, device=dev)
    geo, _ = record_layout(hidden, inter, layout)
    return buf, addrs, geo, stride
