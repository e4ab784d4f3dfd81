"""A whole MoE layer at BASELINE config 4 (oomb_moe_layer_decode_fp8): hidden
4096, 64 routed experts top-6, intermediate 1408, plus 2 shared experts (one
SwiGLU MLP of width 2816) with a sigmoid gate, FP8 128x128 block scales.

Bars: the layer equals, bit for bit, the separate entry points in the
reference's order (shared gate/up GEMV, SwiGLU, down GEMV, gate logit, the
routed decode, moe_combine), for one token (CUDA-core GEMVs) and for batches
that take the tensor cores; and it is within 1e-4 (relative to the largest
output) of the float64 layer over the exactly decoded weights, BASELINE's max
relative error 1e-3 with it.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import oracle as O  # noqa: E402
import homelab_b200 as hb  # noqa: E402
from homelab_b200.backend import Gpu  # noqa: E402
from homelab_b200.records import ExpertBank, SharedExpertBank  # noqa: E402

if not torch.cuda.is_available():
    pytest.skip("needs a GPU", allow_module_level=True)

DEV = torch.device("cuda", 0)
H, E, K, I, SI = 4096, 64, 6, 1408, 2816


@pytest.fixture(scope="module")
def gpu():
    g = Gpu(0)
    yield g
    torch.cuda.synchronize()
    assert g.device_error() == 0, "a bounded device wait ran out"


@pytest.fixture(scope="module")
def layer(gpu):
    bank = ExpertBank(E, H, I, hb.SCALE_128X128, DEV)
    bank.fill_random(gpu, seed=61)
    shared = SharedExpertBank(H, SI, hb.SCALE_128X128, DEV)
    shared.fill_random(gpu, seed=62)
    router = O.normal_bf16(63, E * H, 0.0, 0.02).reshape(E, H)
    router_d = torch.from_numpy(router.reshape(-1).view(np.int16)).to(DEV).view(torch.bfloat16).view(E, H)
    L = hb.MoeLayer(hidden=H, experts=E, top_k=K, router_w=router_d.data_ptr(), recs=bank.addrs.data_ptr())
    L.geo = bank.geo
    torch.cuda.synchronize()
    return dict(bank=bank, shared=shared, S=shared.view(), router=router, router_d=router_d, L=L)


def xin(seed, t):
    xb = O.normal_bf16(seed, t * H)
    return O.bf16_to_f32(xb).reshape(t, H), torch.from_numpy(xb.view(np.int16)).to(DEV).view(torch.bfloat16).view(t, H)


@pytest.mark.parametrize("t", [1, 4, 16])
def test_layer_equals_separate_calls(gpu, layer, t):
    L, S, sh = layer["L"], layer["S"], layer["shared"]
    _, xd = xin(900 + t, t)
    ws = gpu.moe_layer_workspace(L, S, t)
    out = torch.full((t, H), float("nan"), dtype=torch.float32, device=DEV)
    for _ in range(2):
        gpu.moe_layer_decode(L, S, xd, t, out, ws)
    # the separate calls
    tcw1 = gpu.gemm_fp8_workspace(t, 2 * SI, H) if t >= 2 else None
    tcw2 = gpu.gemm_fp8_workspace(t, H, SI, torch.float32) if t >= 2 else None
    gu = torch.empty((t, 2 * SI), dtype=torch.float32, device=DEV)
    sact = torch.empty((t, SI), dtype=torch.float32, device=DEV)
    shared = torch.empty((t, H), dtype=torch.float32, device=DEV)
    gate = torch.empty((t, 1), dtype=torch.float32, device=DEV)
    routed = torch.empty((t, H), dtype=torch.float32, device=DEV)
    want = torch.empty((t, H), dtype=torch.float32, device=DEV)
    gpu.gemm_fp8(xd, sh.gate_up_q, sh.gate_up_s, gu, t, 2 * SI, H, hb.SCALE_128X128, tcw1)
    gpu.silu_mul_rows(gu, sact, t, SI)
    gpu.gemm_fp8(sact, sh.down_q, sh.down_s, shared, t, H, SI, hb.SCALE_128X128, tcw2)
    gpu.router_logits(xd, sh.gate_w.view(1, H), gate, t, 1, H)
    gpu.moe_decode(L, xd, t, routed, gpu.moe_decode_workspace(L, t))
    gpu.moe_combine(routed, shared, gate, want, t, H)
    torch.cuda.synchronize()
    assert torch.equal(out, want)


@pytest.mark.parametrize("t", [1, 3])
@pytest.mark.parametrize("out_bf16", [False, True])
def test_layer_matches_float64(gpu, layer, t, out_bf16):
    L, S, sh, bank = layer["L"], layer["S"], layer["shared"], layer["bank"]
    x32, xd = xin(950 + t, t)
    ws = gpu.moe_layer_workspace(L, S, t)
    ids = torch.empty((t, K), dtype=torch.int32, device=DEV)
    wts = torch.empty((t, K), dtype=torch.float32, device=DEV)
    out = torch.empty((t, H), dtype=torch.bfloat16 if out_bf16 else torch.float32, device=DEV)
    gpu.moe_layer_decode(L, S, xd, t, out, ws, ids, wts)
    torch.cuda.synchronize()
    want_ids, want_w = O.router_topk(O.router_logits(x32, layer["router"]), K)
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    assert np.array_equal(wts.cpu().numpy().view(np.uint32), want_w.view(np.uint32))
    active, off, tok, slot = O.group_assignments(want_ids, E)
    recs = [bank.buf[int(e) * bank.stride:(int(e) + 1) * bank.stride].cpu().numpy() for e in active]
    y = O.moe_experts_f64_fast(recs, L.geo, off, tok, x32)
    routed = O.combine_slots_f64(y, slot, want_w, t, H, K)
    x64 = x32.astype(np.float64)
    wgu = O.dequantize(sh.gate_up_q.cpu().numpy(), sh.gate_up_s.cpu().numpy().reshape(-1), hb.SCALE_128X128)
    wd = O.dequantize(sh.down_q.cpu().numpy(), sh.down_s.cpu().numpy().reshape(-1), hb.SCALE_128X128)
    gu = x64 @ wgu.T
    g, u = gu[:, :SI], gu[:, SI:]
    shared = (g / (1.0 + np.exp(-g)) * u) @ wd.T
    gw = O.bf16_to_f32(sh.gate_w.view(torch.int16).cpu().numpy().view(np.uint16)).astype(np.float64)
    gate = x64 @ gw
    truth = routed + (1.0 / (1.0 + np.exp(-gate)))[:, None] * shared
    got = out.float().cpu().numpy()
    rel = np.abs(got - truth).max() / np.abs(truth).max()
    assert rel <= (2 ** -8 + 1e-4 if out_bf16 else 1e-4), rel
