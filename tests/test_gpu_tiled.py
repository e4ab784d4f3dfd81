"""The grouped tensor-core expert GEMM (oomb_moe_tiled_fp8, the moe_tiled path of
Moe::run_group, crates/oominf-models-qwen/src/moe.rs:746-758) against the CPU
oracle, through the C ABI.

Bars, as for the dense tensor-core GEMM: every projection output within the
fp32-accumulation bound of a float64 evaluation over the exactly decoded weights,
|y - y64| <= 4e-6 * sum|x*w| (fp32 activations keep 24 bits of each 128-column
block, the reference Exact precision's bar), and the BASELINE max relative error 1e-3; the
tiled gate -> up -> swiglu -> down chain within 1e-4 of the oracle's float64
experts (the bar of the CUDA-core expert kernels); repeated calls give
identical bits; an assignment's output does not depend on the chunk size.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import oracle as O  # noqa: E402
from homelab_b200 import SCALE_128X128, SCALE_1X128  # noqa: E402
from homelab_b200.backend import Gpu  # noqa: E402
from homelab_b200.records import ExpertBank  # noqa: E402

if not torch.cuda.is_available():
    pytest.skip("needs a GPU", allow_module_level=True)

DEV = torch.device("cuda", 0)
FP32_BOUND = 4e-6
MAX_REL = 1e-3


@pytest.fixture(scope="module")
def gpu():
    g = Gpu(0)
    yield g
    torch.cuda.synchronize()
    assert g.device_error() == 0, "a bounded device wait ran out"


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


@pytest.fixture(scope="module")
def banks(gpu):
    out = {}
    for layout, (E, H, I) in ((SCALE_128X128, (16, 2048, 768)), (SCALE_1X128, (8, 1024, 384))):
        b = ExpertBank(E, H, I, layout, DEV)
        b.fill_random(gpu, seed=11 + layout)
        out[layout] = b
    torch.cuda.synchronize()
    return out


def routing(seed, t, k, E):
    """A seeded top-k routing of t tokens, grouped by expert as Moe::finish_routed does."""
    rng = np.random.default_rng(seed)
    ids = np.stack([rng.choice(E, k, replace=False) for _ in range(t)]).astype(np.int32)
    w = rng.random((t, k)).astype(np.float32)
    w /= w.sum(1, keepdims=True)
    active, off, tok, slot = O.group_assignments(ids, E)
    return active, off, tok, slot, w


def activations(seed, t, h, xbf16):
    if xbf16:
        xb = O.normal_bf16(seed, t * h)
        return O.bf16_to_f32(xb).reshape(t, h), dev(xb.view(np.int16)).view(torch.bfloat16).view(t, h)
    x32 = O.normal_f32(seed, t * h).reshape(t, h)
    return x32, dev(x32)


def projection_truth(host, active, off, rows, x32, w_off, s_off, n, k, layout):
    """float64 y[a] = x[row(a)] . W_e^T and sum|x*w| per output, group by group."""
    A = int(off[-1])
    y = np.zeros((A, n))
    mag = np.zeros((A, n))
    sc = O.scale_count(n, k, layout)
    for i, e in enumerate(active):
        a0, a1 = int(off[i]), int(off[i + 1])
        if a1 == a0:
            continue
        rec = host[e]
        q = rec[w_off:w_off + n * k].reshape(n, k)
        s = rec[s_off:s_off + 4 * sc].view(np.float32)
        xr = x32[rows[a0:a1]] if rows is not None else x32[a0:a1]
        y[a0:a1], mag[a0:a1] = O.gemv_fp8_f64_fast(xr, q, s, layout)
    return y, mag


def check_bound(got, truth, mag, what):
    err = np.abs(np.asarray(got, dtype=np.float64) - truth)
    worst = float((err / (mag * FP32_BOUND + 1e-30)).max())
    assert worst <= 1.0, f"{what}: error {worst:.3g}x the fp32 accumulation bound"
    rel = float(err.max() / max(np.abs(truth).max(), 1e-30))
    assert rel <= MAX_REL, f"{what}: max relative error {rel:.3g}"


# (tokens, top-k): groups of ~1, ~4, ~30 and ~250 assignments (the last cut into several chunks)
STEPS = [(1, 8), (8, 8), (60, 8), (500, 8)]


@pytest.mark.parametrize("t,k", STEPS)
@pytest.mark.parametrize("layout", [SCALE_128X128, SCALE_1X128])
@pytest.mark.parametrize("xbf16", [True, False])
def test_tiled_projections_match_oracle(gpu, banks, t, k, layout, xbf16):
    bank = banks[layout]
    g = bank.geo
    H, I, E = g.hidden, g.inter, bank.experts
    k = min(k, E)
    active, off, tok, slot, _ = routing(1000 + t * 7 + layout, t, k, E)
    x32, xd = activations(1100 + t, t, H, xbf16)
    A = int(off[-1])
    recs = bank.addrs[torch.from_numpy(active).long().to(DEV)].contiguous()
    offd, tokd = dev(off), dev(tok)
    maxn = int(np.diff(off).max())
    host = bank.host_records()
    # gate with rows (the layer input, row(a) = tok(a)), then down without rows (x = h)
    yg = torch.empty((A, I), dtype=torch.float32, device=DEV)
    gpu.moe_tiled(recs, offd, tokd, len(active), maxn, xd, yg, I, H, (g.gate_weight, g.gate_scale), layout)
    yg2 = torch.empty_like(yg)
    gpu.moe_tiled(recs, offd, tokd, len(active), maxn, xd, yg2, I, H, (g.gate_weight, g.gate_scale), layout)
    h32 = O.normal_f32(1200 + t, A * I).reshape(A, I)
    yd = torch.empty((A, H), dtype=torch.float32, device=DEV)
    gpu.moe_tiled(recs, offd, None, len(active), maxn, dev(h32), yd, H, I, (g.down_weight, g.down_scale), layout)
    torch.cuda.synchronize()
    truth, mag = projection_truth(host, active, off, tok, x32, g.gate_weight, g.gate_scale, I, H, layout)
    check_bound(yg.cpu().numpy(), truth, mag, "gate")
    assert torch.equal(yg, yg2), "repeated calls differ"
    truth, mag = projection_truth(host, active, off, None, h32, g.down_weight, g.down_scale, H, I, layout)
    check_bound(yd.cpu().numpy(), truth, mag, "down")


@pytest.mark.parametrize("t,k", [(8, 8), (60, 8), (300, 6)])
def test_tiled_chain_matches_oracle_experts(gpu, banks, t, k):
    """gate, up, swiglu, down and the slot combine: the reference's tiled step order."""
    bank = banks[SCALE_128X128]
    g = bank.geo
    H, I, E = g.hidden, g.inter, bank.experts
    active, off, tok, slot, w = routing(1300 + t, t, k, E)
    x32, xd = activations(1400 + t, t, H, True)
    A = int(off[-1])
    recs = bank.addrs[torch.from_numpy(active).long().to(DEV)].contiguous()
    offd, tokd = dev(off), dev(tok)
    maxn = int(np.diff(off).max())
    n_e = len(active)
    gg = torch.empty((A, I), dtype=torch.float32, device=DEV)
    uu = torch.empty_like(gg)
    h = torch.empty_like(gg)
    y = torch.empty((A, H), dtype=torch.float32, device=DEV)
    out = torch.empty((t, H), dtype=torch.float32, device=DEV)
    gpu.moe_tiled(recs, offd, tokd, n_e, maxn, xd, gg, I, H, (g.gate_weight, g.gate_scale), g.layout)
    gpu.moe_tiled(recs, offd, tokd, n_e, maxn, xd, uu, I, H, (g.up_weight, g.up_scale), g.layout)
    gpu.moe_swiglu_range(gg, uu, h, 0, A * I)
    gpu.moe_tiled(recs, offd, None, n_e, maxn, h, y, H, I, (g.down_weight, g.down_scale), g.layout)
    gpu.moe_combine_slots(y, dev(slot), dev(w), out, t, H, k)
    # the CUDA-core expert kernels on the same grouping
    h_cc = torch.empty_like(gg)
    y_cc = torch.empty_like(y)
    gpu.moe_gate_up(recs, offd, tokd, n_e, xd, h_cc, g, 0)
    gpu.moe_down(recs, offd, n_e, h_cc, y_cc, g, 0)
    torch.cuda.synchronize()
    host = bank.host_records()
    y_truth = O.moe_experts_f64([host[e] for e in active], g, off, tok, x32)
    yg = y.cpu().numpy()
    rel = np.abs(yg - y_truth).max() / np.abs(y_truth).max()
    assert rel <= 1e-4, rel
    rel_cc = np.abs(yg - y_cc.cpu().numpy()).max() / np.abs(y_truth).max()
    assert rel_cc <= 1e-4, rel_cc
    out_truth = O.combine_slots_f64(y_truth, slot, w, t, H, k)
    assert np.abs(out.cpu().numpy() - out_truth).max() / np.abs(out_truth).max() <= MAX_REL


def test_tiled_output_independent_of_chunk_size(gpu, banks):
    """max_per_expert only picks the chunk; an assignment's bits do not depend on it."""
    bank = banks[SCALE_128X128]
    g = bank.geo
    H, I, E = g.hidden, g.inter, bank.experts
    t, k = 120, 8
    active, off, tok, slot, _ = routing(1500, t, k, E)
    _, xd = activations(1501, t, H, True)
    A = int(off[-1])
    recs = bank.addrs[torch.from_numpy(active).long().to(DEV)].contiguous()
    offd, tokd = dev(off), dev(tok)
    outs = []
    for maxn in (1, 9, 20, 0):
        y = torch.empty((A, I), dtype=torch.float32, device=DEV)
        gpu.moe_tiled(recs, offd, tokd, len(active), maxn, xd, y, I, H, (g.up_weight, g.up_scale), g.layout)
        outs.append(y)
    torch.cuda.synchronize()
    for y in outs[1:]:
        assert torch.equal(y, outs[0])


def test_tiled_groups_with_empty_experts_and_offset_start(gpu, banks):
    """Groups may be empty, and off need not start at 0 (a slice of a larger grouping, as
    Moe::run_group passes): only the assignments in [off[0], off[-1]) are written."""
    bank = banks[SCALE_128X128]
    g = bank.geo
    H, I = g.hidden, g.inter
    counts = np.array([0, 3, 0, 70, 1, 0], dtype=np.int32)
    base = 5
    off = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32) + base
    A = int(off[-1])
    rows = np.random.default_rng(1600).integers(0, 7, size=A).astype(np.int32)
    x32, xd = activations(1601, 7, H, False)
    active = np.array([2, 4, 9, 1, 0, 15])
    recs = bank.addrs[torch.from_numpy(active).long().to(DEV)].contiguous()
    sentinel = -1234.5
    y = torch.full((A, I), sentinel, dtype=torch.float32, device=DEV)
    gpu.moe_tiled(recs, dev(off), dev(rows), len(active), 0, xd, y, I, H, (g.gate_weight, g.gate_scale), g.layout)
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    assert np.all(got[:base] == sentinel)
    host = bank.host_records()
    truth, mag = projection_truth(host, active, off, rows, x32, g.gate_weight, g.gate_scale, I, H, g.layout)
    check_bound(got[base:], truth[base:], mag[base:], "gate")


def test_tiled_fp32_split_keeps_24_bits(gpu):
    """The down projection with fp32 h whose values lie 2^-20..2^-19 below their
    block's largest (bits a 16-bit split loses), over weights that are zero in
    the block-maximum column: within the fp32 bound of float64."""
    from test_gpu_tc import small_value_case
    H, I, E = 1024, 128, 3
    bank = ExpertBank(E, H, I, SCALE_128X128, DEV)
    bank.fill_random(gpu, seed=90)
    counts = [5, 0, 17]
    off = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    A = int(off[-1])
    h32 = None
    for e in range(E):
        wb, xe = small_value_case(900 + e, max(counts[e], 1), H, I)
        dq, ds = bank.views(e)[4], bank.views(e)[5]
        gpu.quantize_fp8(torch.from_numpy(wb.view(np.int16)).to(DEV), H, I, SCALE_128X128, dq, ds)
        if counts[e]:
            h32 = xe if h32 is None else np.concatenate([h32, xe])
    torch.cuda.synchronize()
    g = bank.geo
    recs = bank.addrs.contiguous()
    y = torch.empty((A, H), dtype=torch.float32, device=DEV)
    gpu.moe_tiled(recs, dev(off), None, E, max(counts), dev(h32), y, H, I, (g.down_weight, g.down_scale),
                  SCALE_128X128)
    torch.cuda.synchronize()
    truth, mag = projection_truth(bank.host_records(), np.arange(E), off, None, h32, g.down_weight, g.down_scale,
                                  H, I, SCALE_128X128)
    check_bound(y.cpu().numpy(), truth, mag, "down, fp32 h with small values")


def test_tiled_rejects_bad_arguments(gpu, banks):
    from homelab_b200 import _lib
    L = _lib.lib()
    g = banks[SCALE_128X128].geo
    x = torch.zeros((4, 2048), dtype=torch.bfloat16, device=DEV)
    y = torch.zeros((4, 768), dtype=torch.float32, device=DEV)
    off = torch.zeros(2, dtype=torch.int32, device=DEV)
    recs = banks[SCALE_128X128].addrs[:1].contiguous()
    args = dict(n=768, k=2048)
    nws = L.oomb_moe_tiled_fp8_workspace_bytes(4, 2048, _lib.BF16)
    ws = torch.empty(nws, dtype=torch.uint8, device=DEV)
    call = lambda n, k, w_off=g.gate_weight, wsb=nws, amax=4: L.oomb_moe_tiled_fp8(  # noqa: E731
        recs.data_ptr(), off.data_ptr(), None, 1, 0, amax, x.data_ptr(), _lib.BF16, y.data_ptr(), n, k, w_off,
        g.gate_scale, g.layout, ws.data_ptr(), wsb, None)
    assert call(**args) == 0
    assert call(700, 2048) == _lib.E_SHAPE
    assert call(768, 2000) == _lib.E_SHAPE
    assert call(768, 2048, g.gate_weight + 8) == _lib.E_ALIGN
    assert call(768, 2048, wsb=nws - 1) == _lib.E_WORKSPACE
    assert call(768, 2048, amax=0) == _lib.E_SHAPE
    torch.cuda.synchronize()


def test_swiglu_range_matches_float64(gpu):
    n = 3 * 1408
    gv = O.normal_f32(1700, n) * 3.0
    uv = O.normal_f32(1701, n)
    h = torch.full((n,), 7.0, dtype=torch.float32, device=DEV)
    gpu.moe_swiglu_range(dev(gv), dev(uv), h, 100, n - 50)
    torch.cuda.synchronize()
    got = h.cpu().numpy()
    g64, u64 = gv.astype(np.float64), uv.astype(np.float64)
    want = g64 / (1.0 + np.exp(-g64)) * u64
    assert np.all(got[:100] == 7.0) and np.all(got[n - 50:] == 7.0)
    sl = slice(100, n - 50)
    assert np.abs(got[sl] - want[sl]).max() / np.abs(want[sl]).max() <= 1e-6
