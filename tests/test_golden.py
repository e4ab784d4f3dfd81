"""The CPU oracle against outputs recorded from the reference's own CUDA kernels.

tests/golden/ref_kernels.npz holds what projects/oom-inference's ops.cu and
moe.cu kernels (built from the reference sources, launched with the reference
host code's geometry) returned on a B200 for inputs that
tests/golden/make_fixtures.py regenerates from seeds.  Here, without a GPU:
  - gemv_fp8_t{1..4}: the oracle's restatement of the kernel's fp32 order is
    bit-exact, and within the fp32 bound of the float64 truth;
  - router_topk: the oracle picks the same ids; weights agree to 4 ulps (the
    reference calls CUDA expf, the oracle a Cody-Waite/Taylor exp);
  - experts: the oracle's float64 expert FFN agrees with the reference's fp32
    kernels, and its slot combine equals the reference's bit for bit.
"""
import os
import sys

import numpy as np
import pytest

import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_fixtures as M  # noqa: E402

FIX = os.path.join(HERE, "golden", "ref_kernels.npz")
if not os.path.exists(FIX):
    pytest.skip("tests/golden/ref_kernels.npz not generated", allow_module_level=True)
REF = np.load(FIX)


@pytest.mark.parametrize("t,n,k", M.GEMV_CASES)
def test_gemv_order_matches_reference_kernel(t, n, k):
    x, q, s = M.gemv_inputs(t, n, k)
    want = REF[f"gemv_{t}_{n}_{k}"]
    got = O.gemv_fp8_reforder(x, q, s)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    truth, mag = O.gemv_fp8_f64(x, q, s, O.SCALE_1X128)
    assert (np.abs(want - truth) <= 4e-6 * mag + 1e-30).all()


@pytest.mark.parametrize("t,e,k", M.ROUTER_CASES)
def test_router_topk_matches_reference_kernel(t, e, k):
    logits = M.router_inputs(t, e, k)
    ids, w = O.router_topk(logits, k)
    assert np.array_equal(ids, REF[f"router_ids_{t}_{e}_{k}"])
    want_w = REF[f"router_w_{t}_{e}_{k}"]
    ulps = np.abs(w.view(np.int32).astype(np.int64) - want_w.view(np.int32).astype(np.int64))
    assert ulps.max() <= 4


def _fp8_records(parts, E, H, I):
    """FP8 records (oracle layout: gate, up, down, then their scales) of the experts."""
    g = O.Fp8Record()
    g.hidden, g.inter, g.layout = H, I, O.SCALE_128X128
    sizes = [I * H, I * H, H * I]
    offs, o = [], 0
    for sz in sizes:
        offs.append(o)
        o += sz
    g.gate_weight, g.up_weight, g.down_weight = offs
    soffs = []
    for (q, s, _) in parts[0]:
        soffs.append(o)
        o += s.size * 4
    g.gate_scale, g.up_scale, g.down_scale = soffs
    recs = []
    for e in range(E):
        r = np.zeros(o, dtype=np.uint8)
        for j, (q, s, _) in enumerate(parts[e]):
            r[offs[j]:offs[j] + q.size] = q.reshape(-1)
            r[soffs[j]:soffs[j] + s.size * 4] = s.astype(np.float32).view(np.uint8)
        recs.append(r)
    return recs, g


def test_experts_match_reference_kernels():
    E, H, I, t, k = (M.EXPERTS[c] for c in ("E", "H", "I", "t", "k"))
    parts, ids, w, x = M.expert_inputs()
    active, off, tok, slot = O.group_assignments(ids, E)
    recs, geo = _fp8_records(parts, E, H, I)
    y64 = O.moe_experts_f64([recs[e] for e in active], geo, off, tok, x)
    y_ref = REF["experts_y"]
    assert np.abs(y_ref - y64).max() / np.abs(y64).max() <= 1e-5
    # the oracle's slot combine over the reference's y is the reference's out, bit for bit
    out = O.combine_slots(y_ref, slot, w, t, H, k)
    assert np.array_equal(out.view(np.uint32), REF["experts_out"].view(np.uint32))
