"""Pins the CPU oracle and the sm_100a path to the reference's own CUDA kernels.

The reference's decode kernels (projects/oom-inference/crates/oominf-cuda/
kernels/ops.cu and moe.cu) are built from the reference sources into
oracle/_ref and launched with the reference host code's geometry
(oracle/ref/launch.cpp).  On identical seeded device inputs:
  - ops.cu gemv_fp8_t{1..4} (fp32 x, 1x128 scales) equals the oracle's
    restatement of its arithmetic order bit for bit, and the sm_100a GEMV is
    within the fp32-accumulation bound and max relative error 1e-3 of it;
  - router_topk picks the same expert ids in the same order as the sm_100a
    router, and its renormalised weights agree to a few ulps (the reference
    calls CUDA expf, the sm_100a router a Cody-Waite/Taylor exp that the CPU
    oracle restates bit for bit);
  - the reference's expert kernels run on bf16 records that hold exactly the
    dequantised FP8 weights (power-of-two block scales make e4m3 x scale exact
    in bf16); the sm_100a FP8 kernels and the oracle agree with them, and the
    slot combine is bit-exact with the oracle's slot-order fma.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import oracle as O  # noqa: E402
from oracle import refk  # noqa: E402
from homelab_b200 import SCALE_128X128, SCALE_1X128  # noqa: E402
from homelab_b200.backend import Gpu  # noqa: E402
from homelab_b200.records import ExpertBank  # noqa: E402

if not torch.cuda.is_available():
    pytest.skip("needs a GPU", allow_module_level=True)
if not refk.available():
    pytest.skip("the reference kernels are not built (oracle/ref/Makefile needs the reference sources)",
                allow_module_level=True)

DEV = torch.device("cuda", 0)
FP32_BOUND = 4e-6
MAX_REL = 1e-3


@pytest.fixture(scope="module")
def gpu():
    g = Gpu(0)
    yield g
    torch.cuda.synchronize()
    assert g.device_error() == 0, "a bounded device wait ran out"


@pytest.fixture(scope="module")
def ref():
    return refk.RefKernels(DEV)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


# ---- dense FP8 GEMV ---------------------------------------------------------------------------

@pytest.mark.parametrize("t,n,k", [(1, 4096, 4096), (4, 640, 2560), (2, 300, 10240), (3, 96, 768),
                                   (1, 2048, 14336)])
@pytest.mark.parametrize("x_from_bf16", [True, False])
def test_reference_gemv_equals_oracle_order(gpu, ref, t, n, k, x_from_bf16):
    w = O.normal_bf16(500 + n, n * k, 0.0, 0.02)
    q, s = O.quantize_blocks(w, n, k, SCALE_1X128)
    x = (O.bf16_to_f32(O.normal_bf16(501 + t, t * k)) if x_from_bf16 else O.normal_f32(502 + t, t * k))
    x = x.reshape(t, k)
    y_ref = ref.gemv_fp8(dev(x), dev(q), dev(s), t, n, k)
    torch.cuda.synchronize()
    y_ref = y_ref.cpu().numpy()
    # the oracle restates the reference kernel's order exactly
    assert np.array_equal(y_ref.view(np.uint32), O.gemv_fp8_reforder(x, q, s).view(np.uint32))
    # the sm_100a GEMV agrees with the reference within the fp32 bound
    y = torch.empty((t, n), dtype=torch.float32, device=DEV)
    gpu.gemm_fp8(dev(x), dev(q), dev(s), y, t, n, k, SCALE_1X128)
    torch.cuda.synchronize()
    truth, mag = O.gemv_fp8_f64(x, q, s, SCALE_1X128)
    err = np.abs(y.cpu().numpy().astype(np.float64) - y_ref)
    assert (err <= 2 * FP32_BOUND * mag + 1e-30).all()
    assert err.max() / np.abs(y_ref).max() <= MAX_REL
    assert (np.abs(y_ref - truth) <= FP32_BOUND * mag + 1e-30).all()


# ---- router top-k -----------------------------------------------------------------------------

def _ulps(a, b):
    ia = a.view(np.int32).astype(np.int64)
    ib = b.view(np.int32).astype(np.int64)
    return np.abs(ia - ib)


@pytest.mark.parametrize("t,e,k", [(32, 256, 8), (32, 128, 8), (16, 64, 6), (5, 40, 32)])
def test_router_topk_ids_match_reference(gpu, ref, t, e, k):
    logits = O.normal_f32(600 + e, t * e).reshape(t, e)
    ld = dev(logits)
    ids_ref, w_ref = ref.router_topk(ld, t, e, k)
    ids = torch.empty((t, k), dtype=torch.int32, device=DEV)
    w = torch.empty((t, k), dtype=torch.float32, device=DEV)
    gpu.router_topk(ld, ids, w, t, e, k)
    torch.cuda.synchronize()
    assert np.array_equal(ids.cpu().numpy(), ids_ref.cpu().numpy())
    assert _ulps(w.cpu().numpy(), w_ref.cpu().numpy()).max() <= 4


def test_router_topk_ties_match_reference(gpu, ref):
    """Equal logits: both pick the lower id first (ops.cu:230-233)."""
    t, e, k = 2, 16, 4
    logits = np.zeros((t, e), dtype=np.float32)
    logits[0, [3, 5, 9]] = 1.0
    logits[1, :] = -0.5
    ld = dev(logits)
    ids_ref, w_ref = ref.router_topk(ld, t, e, k)
    ids = torch.empty((t, k), dtype=torch.int32, device=DEV)
    w = torch.empty((t, k), dtype=torch.float32, device=DEV)
    gpu.router_topk(ld, ids, w, t, e, k)
    torch.cuda.synchronize()
    assert np.array_equal(ids.cpu().numpy(), ids_ref.cpu().numpy())
    assert ids_ref.cpu().numpy()[0, :3].tolist() == [3, 5, 9]
    assert _ulps(w.cpu().numpy(), w_ref.cpu().numpy()).max() <= 4


def test_router_on_config2_logits_matches_reference(gpu, ref):
    """Config 2 router: bf16 W [128, 2048] ~ N(0, 0.02), x ~ N(0, 1), top-8."""
    t, e, h, k = 16, 128, 2048, 8
    wr = O.normal_bf16(610, e * h, 0.0, 0.02).reshape(e, h)
    x = O.bf16_to_f32(O.normal_bf16(611, t * h)).reshape(t, h)
    logits = torch.empty((t, e), dtype=torch.float32, device=DEV)
    gpu.router_logits(dev(x), dev(wr.view(np.int16)).view(torch.bfloat16), logits, t, e, h)
    ids_ref, _ = ref.router_topk(logits, t, e, k)
    ids = torch.empty((t, k), dtype=torch.int32, device=DEV)
    w = torch.empty((t, k), dtype=torch.float32, device=DEV)
    gpu.router_topk(logits, ids, w, t, e, k)
    torch.cuda.synchronize()
    assert np.array_equal(ids.cpu().numpy(), ids_ref.cpu().numpy())


# ---- routed experts ---------------------------------------------------------------------------

@pytest.fixture(scope="module")
def pow2_bank(gpu):
    """FP8 records whose 128x128 block scales are powers of two, plus bf16
    records (the reference's Bf16Record layout: gate [I, H], up [I, H],
    down [H, I]) holding exactly the same dequantised weights."""
    E, H, I = 12, 2048, 768
    b = ExpertBank(E, H, I, SCALE_128X128, DEV)
    b.fill_random(gpu, seed=9)
    gw_off, uw_off, dw_off = 0, I * H * 2, 2 * I * H * 2
    stride = 3 * I * H * 2
    bf = torch.empty(E * stride, dtype=torch.uint8, device=DEV)
    for e in range(E):
        parts = b.views(e)
        for (q, s), off, (n, k) in zip(((parts[0], parts[1]), (parts[2], parts[3]), (parts[4], parts[5])),
                                       (gw_off, uw_off, dw_off), ((I, H), (I, H), (H, I))):
            s.copy_(torch.exp2(torch.round(torch.log2(s))))
            full = s.repeat_interleave(128, 0)[:n].repeat_interleave(128, 1)[:, :k]
            wdq = q.view(torch.float8_e4m3fn).float() * full
            wb = wdq.to(torch.bfloat16)
            assert torch.equal(wb.float(), wdq), "dequantised weight not exact in bf16"
            bf[e * stride + off:e * stride + off + n * k * 2].copy_(wb.view(torch.uint8).reshape(-1))
    addrs = torch.tensor([bf.data_ptr() + e * stride for e in range(E)], dtype=torch.int64, device=DEV)
    torch.cuda.synchronize()
    return dict(bank=b, bf=bf, addrs=addrs, offs=(gw_off, uw_off, dw_off), H=H, I=I, E=E,
                host=b.host_records())


@pytest.mark.parametrize("t,k", [(1, 8), (3, 6), (8, 4)])
def test_experts_match_reference_kernels(gpu, ref, pow2_bank, t, k):
    P = pow2_bank
    H, I, E = P["H"], P["I"], P["E"]
    rng = np.random.default_rng(700 + t)
    ids = np.stack([rng.choice(E, k, replace=False) for _ in range(t)]).astype(np.int32)
    wts = rng.random((t, k)).astype(np.float32)
    wts /= wts.sum(1, keepdims=True)
    active, off, tok, slot = O.group_assignments(ids, E)
    x = O.normal_f32(701 + t, t * H).reshape(t, H)
    A, n_e = t * k, len(active)
    sel = torch.from_numpy(active).long().to(DEV)
    offd, tokd, slotd, wd, xd = dev(off), dev(tok), dev(slot), dev(wts), dev(x)

    # reference kernels on the bf16 records
    h_ref = torch.empty((A, I), dtype=torch.float32, device=DEV)
    y_ref = torch.empty((A, H), dtype=torch.float32, device=DEV)
    out_ref = torch.empty((t, H), dtype=torch.float32, device=DEV)
    gw, uw, dw = P["offs"]
    recs_bf = P["addrs"][sel].contiguous()
    ref.moe_gate_up_bf16(recs_bf, offd, tokd, n_e, xd, h_ref, H, I, gw, uw)
    ref.moe_down_bf16(recs_bf, offd, n_e, h_ref, y_ref, H, I, dw)
    ref.moe_combine_slots(y_ref, slotd, wd, out_ref, t, H, k)

    # the sm_100a FP8 kernels on the FP8 records
    recs = P["bank"].addrs[sel].contiguous()
    h = torch.empty_like(h_ref)
    y = torch.empty_like(y_ref)
    out = torch.empty_like(out_ref)
    gpu.moe_gate_up(recs, offd, tokd, n_e, xd, h, P["bank"].geo)
    gpu.moe_down(recs, offd, n_e, h, y, P["bank"].geo)
    gpu.moe_combine_slots(y, slotd, wd, out, t, H, k)
    torch.cuda.synchronize()

    def rel(a, b):
        a, b = a.cpu().numpy().astype(np.float64), b.cpu().numpy().astype(np.float64)
        return np.abs(a - b).max() / np.abs(b).max()

    assert rel(h, h_ref) <= 1e-4
    assert rel(y, y_ref) <= 1e-4
    assert rel(out, out_ref) <= MAX_REL
    # the slot combine is the oracle's slot-order fma, bit for bit, on the reference's y
    assert np.array_equal(out_ref.cpu().numpy().view(np.uint32),
                          O.combine_slots(y_ref.cpu().numpy(), slot, wts, t, H, k).view(np.uint32))
    # the oracle's float64 experts agree with the reference's
    y64 = O.moe_experts_f64([P["host"][e] for e in active], P["bank"].geo, off, tok, x)
    assert np.abs(y_ref.cpu().numpy() - y64).max() / np.abs(y64).max() <= 1e-4
