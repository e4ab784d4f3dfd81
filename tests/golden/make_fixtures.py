"""Writes tests/golden/ref_kernels.npz: outputs of the reference's own CUDA kernels.

Runs on a machine with an sm_100 GPU and the reference kernels built into
oracle/_ref (oracle/ref/Makefile).  Every input is regenerated from a seed by
the *_inputs() functions below (numpy and the oracle's seeded generators), so
the fixture holds only the reference kernels' outputs; tests/test_golden.py
rebuilds the same inputs on the CPU and checks the oracle against them.

    python tests/golden/make_fixtures.py [out.npz]
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle as O  # noqa: E402

# (t, n, k) of the reference gemv_fp8_t{t} cases (x fp32, 1x128 scales)
GEMV_CASES = [(1, 128, 1024), (3, 96, 768), (2, 40, 2560), (4, 64, 4096)]
# (t, e, k) of the router cases; logits ~ N(0, 1)
ROUTER_CASES = [(8, 128, 8), (4, 256, 8), (3, 64, 6), (2, 40, 32)]
# routed experts: bf16 records holding exactly the dequantised FP8 weights
EXPERTS = dict(E=6, H=256, I=128, t=3, k=4)


def gemv_inputs(t, n, k):
    w = O.normal_bf16(1000 + n + k, n * k, 0.0, 0.02)
    q, s = O.quantize_blocks(w, n, k, O.SCALE_1X128)
    x = O.normal_f32(2000 + t + k, t * k).reshape(t, k)
    return x, q, s


def router_inputs(t, e, k):
    logits = O.normal_f32(3000 + e + k, t * e).reshape(t, e)
    if t >= 2:
        logits[1, :4] = logits[1, 4]  # a tie on the row's fifth value
    return logits


def pow2(s):
    """Block scales rounded to powers of two (so e4m3 x scale is exact in bf16)."""
    return np.exp2(np.round(np.log2(s))).astype(np.float32)


def expert_inputs():
    """FP8 expert parts (q, scale) per expert with 128x128 power-of-two scales,
    their dequantised fp32 weights, the routing and the activations."""
    E, H, I, t, k = (EXPERTS[c] for c in ("E", "H", "I", "t", "k"))
    parts = []
    for e in range(E):
        pe = []
        for j, (n, kk) in enumerate(((I, H), (I, H), (H, I))):
            w = O.normal_bf16(4000 + 10 * e + j, n * kk, 0.0, 0.02)
            q, s = O.quantize_blocks(w, n, kk, O.SCALE_128X128)
            s = pow2(s)
            pe.append((q.reshape(n, kk), s, O.dequantize(q, s, O.SCALE_128X128).reshape(n, kk)))
        parts.append(pe)
    rng = np.random.default_rng(4100)
    ids = np.stack([rng.choice(E, k, replace=False) for _ in range(t)]).astype(np.int32)
    w = rng.random((t, k)).astype(np.float32)
    w /= w.sum(1, keepdims=True)
    x = O.normal_f32(4200, t * H).reshape(t, H)
    return parts, ids, w, x


def main(out_path):
    import torch

    from oracle import refk
    dev = torch.device("cuda", 0)
    ref = refk.RefKernels(dev)

    def up(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(dev)

    res = {}
    for (t, n, k) in GEMV_CASES:
        x, q, s = gemv_inputs(t, n, k)
        res[f"gemv_{t}_{n}_{k}"] = ref.gemv_fp8(up(x), up(q), up(s), t, n, k).cpu().numpy()
    for (t, e, k) in ROUTER_CASES:
        ids, w = ref.router_topk(up(router_inputs(t, e, k)), t, e, k)
        res[f"router_ids_{t}_{e}_{k}"] = ids.cpu().numpy()
        res[f"router_w_{t}_{e}_{k}"] = w.cpu().numpy()

    E, H, I, t, k = (EXPERTS[c] for c in ("E", "H", "I", "t", "k"))
    parts, ids, w, x = expert_inputs()
    active, off, tok, slot = O.group_assignments(ids, E)
    stride = 3 * I * H * 2
    recs = np.zeros((E, stride), dtype=np.uint8)
    for e in range(E):
        blob = np.concatenate([O.bf16_from_f32(p[2].reshape(-1)).view(np.uint8) for p in parts[e]])
        recs[e, :blob.size] = blob
    recs_d = up(recs.reshape(-1))
    addrs = up(np.array([recs_d.data_ptr() + int(e) * stride for e in active], dtype=np.int64))
    A = t * k
    h = torch.empty((A, I), dtype=torch.float32, device=dev)
    y = torch.empty((A, H), dtype=torch.float32, device=dev)
    out = torch.empty((t, H), dtype=torch.float32, device=dev)
    offd, tokd, slotd = up(off), up(tok), up(slot)
    ref.moe_gate_up_bf16(addrs, offd, tokd, len(active), up(x), h, H, I, 0, I * H * 2)
    ref.moe_down_bf16(addrs, offd, len(active), h, y, H, I, 2 * I * H * 2)
    ref.moe_combine_slots(y, slotd, up(w), out, t, H, k)
    torch.cuda.synchronize()
    res["experts_h"] = h.cpu().numpy()
    res["experts_y"] = y.cpu().numpy()
    res["experts_out"] = out.cpu().numpy()
    np.savez_compressed(out_path, **res)
    print(f"wrote {out_path}: {len(res)} arrays")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(os.path.dirname(os.path.abspath(__file__)),
                                                           "ref_kernels.npz"))
