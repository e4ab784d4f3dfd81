"""Parity of the sm_100a kernels (through the C ABI) with the CPU oracle.

Bars (BASELINE north star and the reference's own tests):
  - integer work is bit-exact: quantizer bytes, top-k ids, grouping tables;
  - the router logits, softmax weights and the slot combine are bit-exact with
    the oracle's restatement of the same fp32 order;
  - fp32 results stay within the fp32-accumulation bound of a float64
    evaluation over the exactly decoded weights, |y - y64| <= 4e-6 * sum|x*w|
    (the style of crates/oominf-cpu/src/kernel.rs:444-510 and
    crates/oominf-cuda/tests/moe_tiled.rs:190-211), and within the BASELINE
    max relative error 1e-3 (max |y - y64| / max |y64|);
  - bf16 outputs are the round-to-nearest-even of the same call's fp32
    accumulator (fp32 accumulate, bf16 out).
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


def bf16_tensor(bits):
    return dev(bits.view(np.int16)).view(torch.bfloat16)


def check_close(got, truth, mag, what):
    got = np.asarray(got, dtype=np.float64)
    err = np.abs(got - truth)
    bound = mag * FP32_BOUND + 1e-30
    worst = float((err / bound).max())
    assert worst <= 1.0, f"{what}: error {worst:.3g}x the fp32 accumulation bound"
    rel = float(err.max() / max(np.abs(truth).max(), 1e-30))
    assert rel <= MAX_REL, f"{what}: max relative error {rel:.3g}"


# ---- quantizer ------------------------------------------------------------------------------

@pytest.mark.parametrize("n,k", [(300, 640), (130, 260), (1024, 4096)])
@pytest.mark.parametrize("layout", [SCALE_1X128, SCALE_128X128])
def test_device_quantizer_matches_fp8_rs(gpu, n, k, layout):
    w = O.normal_bf16(41 + n, n * k, 0.0, 0.02)
    w[::97] = O.bf16_from_f32(np.float32([0.0]))[0]
    q_ref, s_ref = O.quantize_blocks(w, n, k, layout)
    q, s = gpu.quantize_fp8(bf16_tensor(w).view(torch.int16).view(n, k), n, k, layout)
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(s.cpu().numpy().reshape(-1).view(np.uint32), s_ref.view(np.uint32))


# ---- dense GEMV -----------------------------------------------------------------------------

GEMV_CASES = [
    # (t, n, k, layout)   config 1, reference dense shapes, odd and multi-stage K
    (1, 4096, 4096, SCALE_128X128),
    (1, 4096, 4096, SCALE_1X128),
    (2, 640, 2560, SCALE_1X128),
    (4, 2560, 640, SCALE_1X128),
    (3, 300, 10240, SCALE_128X128),
    (1, 300, 10240, SCALE_1X128),
    (4, 1024, 14336, SCALE_128X128),
    (5, 96, 768, SCALE_128X128),
    (8, 17, 1408, SCALE_1X128),
    (1, 28672, 4096, SCALE_128X128),
    (16, 64, 512, SCALE_128X128),
]


@pytest.mark.parametrize("t,n,k,layout", GEMV_CASES)
@pytest.mark.parametrize("xbf16", [True, False])
def test_gemm_fp8_matches_oracle(gpu, t, n, k, layout, xbf16):
    w = O.normal_bf16(7 + n + k, n * k, 0.0, 0.02)
    q, s = O.quantize_blocks(w, n, k, layout)
    xb = O.normal_bf16(5 + t, t * k)
    x32 = O.bf16_to_f32(xb).reshape(t, k) if xbf16 else O.normal_f32(6 + t, t * k).reshape(t, k)
    truth, mag = O.gemv_fp8_f64(x32, q, s, layout)
    xd = bf16_tensor(xb).view(t, k) if xbf16 else dev(x32)
    qd, sd = dev(q), dev(s)
    y32 = torch.empty((t, n), dtype=torch.float32, device=DEV)
    y16 = torch.empty((t, n), dtype=torch.bfloat16, device=DEV)
    gpu.gemm_fp8(xd, qd, sd, y32, t, n, k, layout)
    gpu.gemm_fp8(xd, qd, sd, y16, t, n, k, layout)
    torch.cuda.synchronize()
    got = y32.cpu().numpy()
    check_close(got, truth, mag, f"gemm_fp8 t={t} {n}x{k}")
    # bf16 out is the correctly rounded fp32 accumulator of the same call
    assert torch.equal(y16.cpu(), y32.cpu().to(torch.bfloat16))


def test_gemm_fp8_back_to_back_launches_agree(gpu):
    # Consecutive launches overlap (programmatic dependent launch); results
    # must not depend on it.
    n, k = 4096, 4096
    w = O.normal_bf16(3, n * k, 0.0, 0.02)
    q, s = O.quantize_blocks(w, n, k, SCALE_128X128)
    qd, sd = dev(q), dev(s)
    x = bf16_tensor(O.normal_bf16(4, k)).view(1, k)
    ys = [torch.empty((1, n), dtype=torch.bfloat16, device=DEV) for _ in range(8)]
    for y in ys:
        gpu.gemm_fp8(x, qd, sd, y, 1, n, k, SCALE_128X128)
    torch.cuda.synchronize()
    for y in ys[1:]:
        assert torch.equal(y, ys[0])


# ---- router ---------------------------------------------------------------------------------

@pytest.mark.parametrize("t,e,h", [(1, 128, 2048), (3, 64, 4096), (16, 256, 4096), (5, 100, 520)])
@pytest.mark.parametrize("xbf16", [True, False])
def test_router_logits_bit_exact(gpu, t, e, h, xbf16):
    w = O.normal_bf16(11 + e, e * h, 0.0, 0.02).reshape(e, h)
    xb = O.normal_bf16(12 + t, t * h)
    x32 = O.bf16_to_f32(xb).reshape(t, h) if xbf16 else O.normal_f32(13, t * h).reshape(t, h)
    want = O.router_logits(x32, w)
    xd = bf16_tensor(xb).view(t, h) if xbf16 else dev(x32)
    got = torch.empty((t, e), dtype=torch.float32, device=DEV)
    gpu.router_logits(xd, bf16_tensor(w.reshape(-1)), got, t, e, h)
    torch.cuda.synchronize()
    assert np.array_equal(got.cpu().numpy().view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("t,e,k", [(1, 128, 8), (128, 256, 8), (7, 64, 6), (3, 8192, 32), (2, 40, 32)])
def test_router_topk_bit_exact(gpu, t, e, k):
    logits = O.normal_f32(100 + e, t * e).reshape(t, e)
    logits[0, 3] = logits[0, 5] = logits[0].max() + 0.5  # a tie: lower id first
    want_ids, want_w = O.router_topk(logits, k)
    ids = torch.empty((t, k), dtype=torch.int32, device=DEV)
    wts = torch.empty((t, k), dtype=torch.float32, device=DEV)
    gpu.router_topk(dev(logits), ids, wts, t, e, k)
    torch.cuda.synchronize()
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    assert np.array_equal(wts.cpu().numpy().view(np.uint32), want_w.view(np.uint32))
    assert want_ids[0, 0] == 3 and want_ids[0, 1] == 5


# ---- routed experts, reference-style calls ---------------------------------------------------

@pytest.fixture(scope="module")
def bank(gpu):
    b = ExpertBank(16, 2048, 768, SCALE_128X128, DEV)
    b.fill_random(gpu, seed=5)
    torch.cuda.synchronize()
    return b


@pytest.mark.parametrize("t,k", [(1, 8), (2, 5), (4, 4), (9, 6)])
@pytest.mark.parametrize("xbf16", [True, False])
@pytest.mark.parametrize("hint", [True, False])
def test_gate_up_down_combine_match_oracle(gpu, bank, t, k, xbf16, hint):
    H, I, E = 2048, 768, bank.experts
    rng = np.random.default_rng(t * 10 + k)
    ids = np.stack([rng.choice(E, k, replace=False) for _ in range(t)]).astype(np.int32)
    w = rng.random((t, k)).astype(np.float32)
    w /= w.sum(1, keepdims=True)
    active, off, tok, slot = O.group_assignments(ids, E)
    xb = O.normal_bf16(70 + t, t * H)
    x32 = O.bf16_to_f32(xb).reshape(t, H) if xbf16 else O.normal_f32(71, t * H).reshape(t, H)
    xd = bf16_tensor(xb).view(t, H) if xbf16 else dev(x32)
    A = t * k
    recs = bank.addrs[torch.from_numpy(active).long().to(DEV)].contiguous()
    h = torch.empty((A, I), dtype=torch.float32, device=DEV)
    y = torch.empty((A, H), dtype=torch.float32, device=DEV)
    out = torch.empty((t, H), dtype=torch.float32, device=DEV)
    offd, tokd, slotd = dev(off), dev(tok), dev(slot)
    # with the hint the kernels keep every group's activations in registers;
    # without it they take the general path (any number of assignments)
    maxn = int(np.diff(off).max()) if hint else 0
    gpu.moe_gate_up(recs, offd, tokd, len(active), xd, h, bank.geo, maxn, tables_ready=hint)
    gpu.moe_down(recs, offd, len(active), h, y, bank.geo, maxn, tables_ready=hint)
    gpu.moe_combine_slots(y, slotd, dev(w), out, t, H, k)
    torch.cuda.synchronize()
    host = bank.host_records()
    y_truth = O.moe_experts_f64([host[e] for e in active], bank.geo, off, tok, x32)
    yg = y.cpu().numpy()
    rel = np.abs(yg - y_truth).max() / np.abs(y_truth).max()
    assert rel <= 1e-4, rel
    # the combine is bit-exact with the oracle's slot-order fma over the same y
    assert np.array_equal(out.cpu().numpy().view(np.uint32),
                          O.combine_slots(yg, slot, w, t, H, k).view(np.uint32))
    out_truth = O.combine_slots_f64(y_truth, slot, w, t, H, k)
    assert np.abs(out.cpu().numpy() - out_truth).max() / np.abs(out_truth).max() <= MAX_REL


# ---- fused decode step (config 2 shapes) ------------------------------------------------------

@pytest.fixture(scope="module")
def layer2(gpu):
    """hidden 2048, 128 experts, top-8, intermediate 768."""
    import homelab_b200 as hb
    H, E, K, I = 2048, 128, 8, 768
    b = ExpertBank(E, H, I, SCALE_128X128, DEV)
    b.fill_random(gpu, seed=2)
    router = O.normal_bf16(21, E * H, 0.0, 0.02).reshape(E, H)
    router_d = bf16_tensor(router.reshape(-1))
    L = hb.MoeLayer(hidden=H, experts=E, top_k=K, router_w=router_d.data_ptr(), recs=b.addrs.data_ptr())
    L.geo = b.geo
    torch.cuda.synchronize()
    return dict(bank=b, router=router, router_d=router_d, layer=L, host=b.host_records())


@pytest.mark.parametrize("t", [1, 3, 16])
@pytest.mark.parametrize("out_bf16", [True, False])
def test_moe_decode_matches_oracle(gpu, layer2, t, out_bf16):
    H, E, K = 2048, 128, 8
    L = layer2["layer"]
    xb = O.normal_bf16(300 + t, t * H)
    x32 = O.bf16_to_f32(xb).reshape(t, H)
    want_ids, want_w = O.router_topk(O.router_logits(x32, layer2["router"]), K)
    ws = gpu.moe_decode_workspace(L, t)
    ids = torch.empty((t, K), dtype=torch.int32, device=DEV)
    wts = torch.empty((t, K), dtype=torch.float32, device=DEV)
    out = torch.empty((t, H), dtype=torch.bfloat16 if out_bf16 else torch.float32, device=DEV)
    for _ in range(2):  # the workspace is reused: the arrival ticket must self-reset
        gpu.moe_decode(L, bf16_tensor(xb).view(t, H), t, out, ws, ids, wts)
    torch.cuda.synchronize()
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    assert np.array_equal(wts.cpu().numpy().view(np.uint32), want_w.view(np.uint32))
    active, off, tok, slot = O.group_assignments(want_ids, E)
    y = O.moe_experts_f64([layer2["host"][e] for e in active], L.geo, off, tok, x32)
    truth = O.combine_slots_f64(y, slot, want_w, t, H, K)
    got = out.float().cpu().numpy()
    rel = np.abs(got - truth).max() / np.abs(truth).max()
    assert rel <= (2 ** -8 + 1e-4 if out_bf16 else 1e-4), rel


def test_moe_decode_equals_separate_calls(gpu, layer2):
    """The fused step gives the same bits as the reference-style sequence of calls
    (up to 16 tokens; larger batches take the grouped tensor-core path)."""
    H, E, K, I = 2048, 128, 8, 768
    t = 3
    L, b = layer2["layer"], layer2["bank"]
    xd = bf16_tensor(O.normal_bf16(77, t * H)).view(t, H)
    ws = gpu.moe_decode_workspace(L, t)
    out_fused = torch.empty((t, H), dtype=torch.float32, device=DEV)
    ids = torch.empty((t, K), dtype=torch.int32, device=DEV)
    wts = torch.empty((t, K), dtype=torch.float32, device=DEV)
    gpu.moe_decode(L, xd, t, out_fused, ws, ids, wts)
    logits = torch.empty((t, E), dtype=torch.float32, device=DEV)
    gpu.router_logits(xd, layer2["router_d"], logits, t, E, H)
    ids2 = torch.empty_like(ids)
    w2 = torch.empty_like(wts)
    gpu.router_topk(logits, ids2, w2, t, E, K)
    torch.cuda.synchronize()
    assert torch.equal(ids, ids2) and torch.equal(wts, w2)
    active, off, tok, slot = O.group_assignments(ids2.cpu().numpy(), E)
    recs = b.addrs[torch.from_numpy(active).long().to(DEV)].contiguous()
    h = torch.empty((t * K, I), dtype=torch.float32, device=DEV)
    y = torch.empty((t * K, H), dtype=torch.float32, device=DEV)
    out = torch.empty((t, H), dtype=torch.float32, device=DEV)
    gpu.moe_gate_up(recs, dev(off), dev(tok), len(active), xd, h, L.geo, t)
    gpu.moe_down(recs, dev(off), len(active), h, y, L.geo, t)
    gpu.moe_combine_slots(y, dev(slot), w2, out, t, H, K)
    torch.cuda.synchronize()
    assert torch.equal(out, out_fused)
