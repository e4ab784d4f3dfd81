"""The CPU oracle pinned against the reference's own known-answer tests.

Golden vectors are the constants of projects/oom-inference's Rust tests:
crates/oominf-core/src/fp8.rs:90-139 (codec, rounding, saturation, block
scales) and crates/oominf-cpu/src/kernel.rs:531-539 (decode KATs).  The
arithmetic checks mirror crates/oominf-cuda/tests/gemv.rs:129-186 (quantizer
relative RMS < 0.05) and kernel.rs:444-510 (fp32 result within sum|w*x| * 1e-6
of a float64 evaluation).
"""
import math

import numpy as np
import pytest

import oracle as O


def f32(v):
    return float(np.float32(v))


# ---- crates/oominf-core/src/fp8.rs:94-108 every_code_round_trips ------------------------

def test_every_code_round_trips():
    for b in range(256):
        if b & 0x7F == 0x7F:
            continue
        v = O.e4m3_to_f32(b)
        back = O.e4m3_from_f32(v)
        assert back == b or (v == 0.0 and back & 0x7F == 0), (hex(b), v, hex(back))


# ---- fp8.rs:110-121 rounds_to_nearest_even_and_saturates --------------------------------

def test_rounds_to_nearest_even_and_saturates():
    assert O.e4m3_from_f32(1.0625) == 0x38
    assert O.e4m3_from_f32(1.07) == 0x39
    assert O.e4m3_from_f32(1000.0) == 0x7E
    assert O.e4m3_from_f32(-1000.0) == 0xFE
    assert O.e4m3_from_f32(2.0 ** -9) == 0x01
    assert O.e4m3_from_f32(2.0 ** -10) == 0x00
    assert O.e4m3_from_f32(f32(2.0 ** -6 * 0.99)) == 0x08


# ---- fp8.rs:123-138 blocks_scale_to_448 (1x128, partial second block) -----------------

def test_blocks_scale_to_448():
    k = 128 + 2
    vals = np.zeros(2 * k, dtype=np.float32)
    vals[0], vals[1], vals[128] = 1.0, -2.0, 0.5
    w = (vals.view(np.uint32) >> 16).astype(np.uint16)
    q, s = O.quantize_blocks(w, 2, k, O.SCALE_1X128)
    assert s.tolist() == [f32(2.0 / 448.0), f32(0.5 / 448.0), 1.0, 1.0]
    q = q.reshape(-1)
    assert f32(O.e4m3_to_f32(q[1]) * s[0]) == -2.0
    assert f32(O.e4m3_to_f32(q[128]) * s[1]) == 0.5
    assert (q[k:] == 0).all()


# ---- crates/oominf-cpu/src/kernel.rs:531-539 e4m3_decodes_known_values ---------------

def test_e4m3_decodes_known_values():
    assert O.e4m3_to_f32_nan(0x00) == 0.0
    assert O.e4m3_to_f32_nan(0x38) == 1.0
    assert O.e4m3_to_f32_nan(0x7E) == 448.0
    assert O.e4m3_to_f32_nan(0x01) == 2.0 ** -9
    assert O.e4m3_to_f32_nan(0xB8) == -1.0
    assert math.isnan(O.e4m3_to_f32_nan(0x7F))
    # fp8.rs:29 reads the never-produced NaN codes as 448.
    assert O.e4m3_to_f32(0x7F) == 448.0 and O.e4m3_to_f32(0xFF) == -448.0


def test_e4m3_matches_torch_float8():
    torch = pytest.importorskip("torch")
    codes = torch.arange(256, dtype=torch.uint8)
    ref = codes.view(torch.float8_e4m3fn).float().numpy()
    ours = np.array([O.e4m3_to_f32_nan(b) for b in range(256)], dtype=np.float32)
    nan = np.isnan(ref)
    assert (np.isnan(ours) == nan).all()
    assert (ours[~nan] == ref[~nan]).all()


def test_encoder_matches_torch_rne():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(5)
    x = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s for s in (1e-3, 0.1, 3, 100)])
    x = np.concatenate([x, np.float32([447.9, 448.0, 464.0, 465.0, 1e-4, 2 ** -9 * 1.5, 2 ** -10])])
    ours = np.array([O.e4m3_from_f32(v) for v in x], dtype=np.uint8)
    # torch saturates nothing: clamp to the finite range first, as fp8.rs does.
    ref = torch.from_numpy(np.clip(x, -448, 448)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert (ours == ref).all()


# ---- quantizer accuracy (crates/oominf-cuda/tests/gemv.rs:141-154) ---------------------

@pytest.mark.parametrize("layout", [O.SCALE_1X128, O.SCALE_128X128])
def test_quantizer_relative_rms(layout):
    n, k = 300, 640
    w = O.normal_bf16(9, n * k, 0.0, 0.02)
    q, s = O.quantize_blocks(w, n, k, layout)
    deq = O.dequantize(q, s, layout)
    ref = O.bf16_to_f32(w).reshape(n, k).astype(np.float64)
    rel = math.sqrt(((deq - ref) ** 2).sum() / (ref ** 2).sum())
    assert rel < 0.05, rel
    # every block's largest weight maps to +-448 exactly (amax / 448 scaling)
    assert np.abs(O.e4m3_table()[q]).max() == 448.0


def test_quantizer_128x128_block_amax():
    n, k = 130, 260  # partial blocks in both dimensions
    vals = np.zeros((n, k), dtype=np.float32)
    vals[5, 3] = 7.0
    vals[129, 259] = -0.25
    w = O.bf16_from_f32(vals.reshape(-1))
    q, s = O.quantize_blocks(w, n, k, O.SCALE_128X128)
    assert s.shape == (2 * 3,)
    assert s[0] == f32(7.0 / 448.0) and s[5] == f32(0.25 / 448.0)
    assert (s[[1, 2, 3, 4]] == 1.0).all()
    assert q[5, 3] == 0x7E and q[129, 259] == 0xFE


# ---- shared exp -------------------------------------------------------------------------

def test_expf_within_two_ulp_of_libm():
    rng = np.random.default_rng(1)
    xs = np.concatenate([rng.uniform(-104, 0, 4000), rng.uniform(-10, 10, 4000), [0.0, -0.0, -87.5, -100.0, 88.0]])
    for x in xs.astype(np.float32):
        got = np.float32(O.expf(float(x)))
        want = np.float32(math.exp(float(x)))
        if want == 0:
            assert got == 0
            continue
        ulp = np.spacing(want)
        assert abs(float(got) - float(want)) <= 2 * float(ulp), (x, got, want)
    assert O.expf(-1e9) == 0.0 and O.expf(float("-inf")) == 0.0


# ---- GEMV truth vs the reference-order emulation (kernel.rs:444-510 style bound) ------

@pytest.mark.parametrize("t,n,k", [(1, 64, 2560), (2, 37, 640), (4, 9, 10240), (3, 300, 512)])
def test_gemv_reforder_within_fp32_accumulation(t, n, k):
    w = O.normal_bf16(7, n * k, 0.0, 0.02)
    q, s = O.quantize_blocks(w, n, k, O.SCALE_1X128)
    x = O.bf16_to_f32(O.normal_bf16(3 + t, t * k))
    y = O.gemv_fp8_reforder(x.reshape(t, k), q, s)
    truth, mag = O.gemv_fp8_f64(x.reshape(t, k), q, s, O.SCALE_1X128)
    assert (np.abs(y - truth) <= mag * 1e-6 + 1e-12).all()


def test_gemv_ref_plan_matches_linear_rs():
    # (n, k) = (4096, 4096), t = 1: 1024 row groups -> want 2 splits of 2048.
    assert O.gemv_ref_plan(1, 4096, 4096) == (2, 2048)
    # Few rows: want saturates at kchunks.
    assert O.gemv_ref_plan(1, 128, 2048) == (4, 512)
    # Many rows: one split, klen = k.
    assert O.gemv_ref_plan(1, 28672, 4096) == (1, 4096)


# ---- router -----------------------------------------------------------------------------

def test_router_topk_properties():
    rng = np.random.default_rng(2)
    t, e, k = 16, 128, 8
    logits = rng.standard_normal((t, e)).astype(np.float32)
    ids, w = O.router_topk(logits, k)
    for i in range(t):
        order = sorted(range(e), key=lambda j: (-logits[i, j], j))
        assert ids[i].tolist() == order[:k]
        assert abs(float(w[i].sum()) - 1.0) < 1e-6
        assert (np.diff(w[i]) <= 0).all()


def test_router_topk_ties_go_to_lower_id():
    logits = np.zeros((1, 64), dtype=np.float32)
    logits[0, [5, 9, 40]] = 2.0
    ids, w = O.router_topk(logits, 5)
    assert ids[0].tolist() == [5, 9, 40, 0, 1]
    assert w[0, 0] == w[0, 1] == w[0, 2]


def test_router_logits_close_to_truth():
    t, e, h = 3, 128, 2048
    x = O.bf16_to_f32(O.normal_bf16(11, t * h)).reshape(t, h)
    w = O.normal_bf16(12, e * h, 0.0, 0.02).reshape(e, h)
    got = O.router_logits(x, w)
    truth = np.empty((t, e))
    O.lib().oo_gemv_bf16_f64(x.ctypes.data, t, w.ctypes.data, e, h, truth.ctypes.data)
    mag = np.abs(x).astype(np.float64) @ np.abs(O.bf16_to_f32(w.reshape(-1)).reshape(e, h)).T
    assert (np.abs(got - truth) <= mag * 1e-6).all()


# ---- grouping (moe.rs:532-582, 638-649) ------------------------------------------------

def test_group_assignments_expert_order_then_slot_order():
    ids = np.array([[3, 1], [1, 7], [3, 0]], dtype=np.int32)
    active, off, tok, slot = O.group_assignments(ids, 8)
    assert active.tolist() == [0, 1, 3, 7]
    assert off.tolist() == [0, 1, 3, 5, 6]
    # expert 0: slot 5 (token 2); expert 1: slots 1, 2; expert 3: slots 0, 4; expert 7: slot 3
    assert tok.tolist() == [2, 0, 1, 0, 2, 1]
    assert slot.tolist() == [3, 1, 2, 5, 4, 0]
    with pytest.raises(ValueError):
        O.group_assignments(np.array([[8]], dtype=np.int32), 8)


def test_combine_slots_is_slot_ordered_fma():
    rng = np.random.default_rng(4)
    t, h, k = 3, 40, 4
    y = rng.standard_normal((t * k, h)).astype(np.float32)
    slot = rng.permutation(t * k).astype(np.int32)
    w = rng.random((t, k)).astype(np.float32)
    out = O.combine_slots(y, slot, w, t, h, k)
    truth = O.combine_slots_f64(y.astype(np.float64), slot, w, t, h, k)
    assert np.abs(out - truth).max() < 1e-5


def test_split_terms_exactness():
    """The tensor-core activation split: two e4m3 terms reproduce bf16 activations
    exactly; six terms keep fp32 activations to within 2^-24 of their 128-column
    block's largest magnitude, including values far below it (2^-20), which four
    terms (16 bits) leave with a few bits only."""
    xb = O.bf16_to_f32(O.normal_bf16(1300, 4 * 256)).reshape(4, 256)
    assert np.array_equal(O.split_terms(xb, 2), xb.astype(np.float64))
    rng = np.random.default_rng(1301)
    x = rng.standard_normal((3, 256)).astype(np.float32)
    x[1] = (2.0 ** -20 * (1.0 + rng.random(256))).astype(np.float32)
    x[1, ::128] = (1.0 + rng.random(2)).astype(np.float32)
    bm = np.abs(x.reshape(3, 2, 128)).max(2).repeat(128, 1).astype(np.float64)
    err6 = np.abs(O.split_terms(x, 6) - x) / bm
    assert err6.max() <= 2.0 ** -24
    small = np.ones(256, dtype=bool)
    small[::128] = False
    rel4 = np.abs(O.split_terms(x[1:2], 4)[0] - x[1]) / np.abs(x[1])
    rel6 = np.abs(O.split_terms(x[1:2], 6)[0] - x[1]) / np.abs(x[1])
    assert rel4[small].max() > 2.0 ** -13  # four terms: about 12 bits of the small values
    assert rel6[small].max() < 2.0 ** -20  # six terms: the bits down to 2^-24 of the block's largest


def test_fast_expert_truth_matches_c_loop():
    """The numpy float64 expert truth (large shapes) agrees with the C loop."""
    from homelab_b200.records import record_layout
    H, I = 256, 128
    geo, stride = record_layout(H, I, O.SCALE_128X128)
    g = O.Fp8Record()
    for f, _ in O.Fp8Record._fields_:
        setattr(g, f, getattr(geo, f))
    recs = []
    for e in range(3):
        r = np.zeros(stride, np.uint8)
        for part, (n, k) in (("gate", (I, H)), ("up", (I, H)), ("down", (H, I))):
            q, sc = O.quantize_blocks(O.normal_bf16(1400 + 3 * e + len(part), n * k, 0.0, 0.02), n, k,
                                      O.SCALE_128X128)
            wo, so = getattr(g, part + "_weight"), getattr(g, part + "_scale")
            r[wo:wo + n * k] = q.reshape(-1)
            r[so:so + 4 * sc.size] = sc.view(np.uint8)
        recs.append(r)
    x = O.normal_f32(1410, 2 * H).reshape(2, H)
    off = np.array([0, 2, 3, 4], np.int32)
    tok = np.array([0, 1, 1, 0], np.int32)
    a = O.moe_experts_f64(recs, g, off, tok, x)
    b = O.moe_experts_f64_fast(recs, g, off, tok, x)
    assert np.abs(a - b).max() <= 1e-12 * np.abs(a).max()
