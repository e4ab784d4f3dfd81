"""The tensor-core FP8 GEMV/GEMM (tcgen05) against the CPU oracle, through the C ABI.

Bars: within the fp32-accumulation bound of a float64 evaluation over the
exactly decoded weights, |y - y64| <= 4e-6 * sum|x*w| (the activation split
into e4m3 terms is exact for bf16 inputs and keeps 24 bits of each 128-column
block for fp32 inputs), and the
BASELINE max relative error 1e-3; bf16 outputs equal RN of the fp32 result;
repeated calls on one workspace give identical bits (self-resetting split-K
counters, fixed summation order).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import oracle as O  # noqa: E402
from homelab_b200 import SCALE_128X128, SCALE_1X128  # noqa: E402
from homelab_b200.backend import Gpu  # noqa: E402

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


CASES = [
    # (t, n, k, layout)
    (1, 4096, 4096, SCALE_128X128),
    (1, 4096, 4096, SCALE_1X128),
    (1, 256, 1024, SCALE_128X128),
    (2, 384, 2048, SCALE_1X128),
    (3, 1536, 2048, SCALE_128X128),
    (4, 2048, 768, SCALE_128X128),
    (5, 640, 2560, SCALE_1X128),
    (8, 1024, 1408, SCALE_128X128),
    (16, 512, 4096, SCALE_128X128),
    (16, 128, 128, SCALE_1X128),
    (32, 256, 2048, SCALE_128X128),
    (64, 384, 1024, SCALE_1X128),
    (64, 4096, 4096, SCALE_128X128),
]


@pytest.mark.parametrize("t,n,k,layout", CASES)
@pytest.mark.parametrize("xbf16", [True, False])
@pytest.mark.parametrize("tiles", [False, True])
def test_tc_gemm_matches_oracle(gpu, t, n, k, layout, xbf16, tiles):
    w = O.normal_bf16(800 + n + k, n * k, 0.0, 0.02)
    q, s = O.quantize_blocks(w, n, k, layout)
    if xbf16:
        xb = O.normal_bf16(801 + t, t * k)
        x32 = O.bf16_to_f32(xb).reshape(t, k)
        xd = dev(xb.view(np.int16)).view(torch.bfloat16).view(t, k)
    else:
        x32 = O.normal_f32(802 + t, t * k).reshape(t, k)
        xd = dev(x32)
    from homelab_b200 import _lib
    if not _lib.lib().oomb_gemm_fp8_workspace_bytes(t, n, k, _lib.BF16 if xbf16 else _lib.F32):
        pytest.skip("batch too large for the tensor-core path with fp32 activations")
    ws = gpu.gemm_fp8_workspace(t, n, k, xd.dtype)
    y = torch.empty((t, n), dtype=torch.float32, device=DEV)
    yb = torch.empty((t, n), dtype=torch.bfloat16, device=DEV)
    qd, sd = dev(q), dev(s)
    if tiles:
        qd = gpu.pack_fp8_tiles(qd, n, k)
    gpu.gemm_fp8_tc(xd, qd, sd, y, t, n, k, layout, ws, tiles)
    gpu.gemm_fp8_tc(xd, qd, sd, yb, t, n, k, layout, ws, tiles)
    y2 = torch.empty_like(y)
    gpu.gemm_fp8_tc(xd, qd, sd, y2, t, n, k, layout, ws, tiles)
    torch.cuda.synchronize()
    truth, mag = O.gemv_fp8_f64(x32, q, s, layout)
    got = y.cpu().numpy().astype(np.float64)
    err = np.abs(got - truth)
    worst = float((err / (mag * FP32_BOUND + 1e-30)).max())
    assert worst <= 1.0, f"error {worst:.3g}x the fp32 bound"
    assert err.max() / np.abs(truth).max() <= MAX_REL
    assert torch.equal(y, y2), "repeated calls differ"
    assert torch.equal(yb, y.to(torch.bfloat16))


def small_value_case(seed, t, n, k):
    """Weights whose first column of every 128-column block is zero, and fp32
    activations whose block maximum (a full-mantissa value in [1, 2)) sits in
    that column while every other value lies in [2^-20, 2^-19): sum|x*w| comes
    from values below 2^-16 of their block's largest, which a split keeping 16
    bits of each block (four e4m3 terms) represents with a few bits only (it
    misses the fp32 bound several times over), while six terms (24 bits) meet it."""
    w = O.bf16_to_f32(O.normal_bf16(seed, n * k, 0.0, 0.02)).reshape(n, k)
    w[:, ::128] = 0.0
    wb = O.bf16_from_f32(w.reshape(-1))
    rng = np.random.default_rng(seed + 1)
    x = (2.0 ** -20 * (1.0 + rng.random((t, k))) * rng.choice([-1.0, 1.0], (t, k))).astype(np.float32)
    x[:, ::128] = (1.0 + rng.random((t, k // 128))).astype(np.float32)
    return wb, x


@pytest.mark.parametrize("t", [1, 5, 32])
def test_tc_fp32_split_keeps_24_bits(gpu, t):
    n, k = 256, 128
    wb, x32 = small_value_case(870 + t, t, n, k)
    q, s = O.quantize_blocks(wb, n, k, SCALE_128X128)
    ws = gpu.gemm_fp8_workspace(t, n, k, torch.float32)
    y = torch.empty((t, n), dtype=torch.float32, device=DEV)
    gpu.gemm_fp8_tc(dev(x32), dev(q), dev(s), y, t, n, k, SCALE_128X128, ws)
    torch.cuda.synchronize()
    truth, mag = O.gemv_fp8_f64(x32, q, s, SCALE_128X128)
    bound = mag * FP32_BOUND + 1e-30
    worst = float((np.abs(y.cpu().numpy().astype(np.float64) - truth) / bound).max())
    assert worst <= 1.0, f"error {worst:.3g}x the fp32 bound"
    # the case discriminates: the same split with four terms (16 bits) misses the bound
    wq = O.dequantize(q, s, SCALE_128X128).astype(np.float64)
    y4 = O.split_terms(x32, 4) @ wq.T
    assert float((np.abs(y4 - truth) / bound).max()) > 2.0


def test_tc_rejects_unsupported_shapes(gpu):
    from homelab_b200 import _lib
    L = _lib.lib()
    assert L.oomb_gemm_fp8_workspace_bytes(1, 100, 1024, _lib.BF16) == 0
    assert L.oomb_gemm_fp8_workspace_bytes(65, 128, 1024, _lib.BF16) == 0
    assert L.oomb_gemm_fp8_workspace_bytes(33, 128, 1024, _lib.F32) == 0
    assert L.oomb_gemm_fp8_workspace_bytes(32, 128, 1024, _lib.F32) > 0
    assert L.oomb_gemm_fp8_workspace_bytes(1, 128, 1000, _lib.BF16) == 0


@pytest.mark.parametrize("t", [2, 16])
def test_gemm_fp8_dispatches_to_tensor_cores_with_a_workspace(gpu, t):
    """oomb_gemm_fp8 with a workspace gives the tensor-core path's bits for t >= 2."""
    n, k = 512, 1024
    w = O.normal_bf16(850, n * k, 0.0, 0.02)
    q, s = O.quantize_blocks(w, n, k, SCALE_128X128)
    xd = dev(O.normal_bf16(851, t * k).view(np.int16)).view(torch.bfloat16).view(t, k)
    qd, sd = dev(q), dev(s)
    ws = gpu.gemm_fp8_workspace(t, n, k)
    y1 = torch.empty((t, n), dtype=torch.float32, device=DEV)
    y2 = torch.empty_like(y1)
    gpu.gemm_fp8(xd, qd, sd, y1, t, n, k, SCALE_128X128, ws)
    gpu.gemm_fp8_tc(xd, qd, sd, y2, t, n, k, SCALE_128X128, ws)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)


@pytest.mark.parametrize("out_bf16", [False, True])
def test_silu_mul_rows_matches_float64(gpu, out_bf16):
    rows, n = 5, 1408
    gu = O.normal_f32(860, rows * 2 * n).reshape(rows, 2 * n) * 3.0
    y = torch.empty((rows, n), dtype=torch.bfloat16 if out_bf16 else torch.float32, device=DEV)
    gpu.silu_mul_rows(dev(gu), y, rows, n)
    torch.cuda.synchronize()
    g, u = gu[:, :n].astype(np.float64), gu[:, n:].astype(np.float64)
    want = g / (1.0 + np.exp(-g)) * u
    got = y.float().cpu().numpy()
    rel = np.abs(got - want).max() / np.abs(want).max()
    assert rel <= (2 ** -8 if out_bf16 else 1e-6), rel


def test_gemm_fp8_entry_reaches_the_tensor_cores_with_a_workspace(gpu):
    """The drop-in oomb_gemm_fp8 (Linear::gemm_fp8's counterpart, through ctypes)
    at 4 tokens: given a workspace it launches the activation split and the
    tcgen05 GEMM, without one the CUDA-core stream kernel (kernel names from the
    CUDA activity trace), and both give the same y within the fp32 bound."""
    from torch.profiler import ProfilerActivity, profile
    t, n, k = 4, 1024, 2048
    w = O.normal_bf16(71, n * k, 0.0, 0.02)
    q, s = gpu.quantize_fp8(dev(w.view(np.int16)), n, k, SCALE_128X128)
    x = dev(O.normal_bf16(72, t * k).view(np.int16)).view(torch.bfloat16).view(t, k)
    ws = gpu.gemm_fp8_workspace(t, n, k)
    y_tc = torch.empty((t, n), dtype=torch.float32, device=DEV)
    y_cc = torch.empty_like(y_tc)
    gpu.gemm_fp8(x, q, s, y_tc, t, n, k, SCALE_128X128, ws)  # first call outside the trace
    torch.cuda.synchronize()

    def kernels(fn):
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            fn()
            torch.cuda.synchronize()
        return [e.key for e in prof.key_averages()]

    with_ws = kernels(lambda: gpu.gemm_fp8(x, q, s, y_tc, t, n, k, SCALE_128X128, ws))
    without = kernels(lambda: gpu.gemm_fp8(x, q, s, y_cc, t, n, k, SCALE_128X128))
    assert any("tc_gemm_kernel" in nm for nm in with_ws), with_ws
    assert any("xsplit_kernel" in nm for nm in with_ws), with_ws
    assert not any("tc_gemm_kernel" in nm for nm in without), without
    assert any("stream_kernel" in nm for nm in without), without
    bound = FP32_BOUND * (x.float().abs() @ (torch.from_numpy(O.bf16_to_f32(w)).to(DEV).view(n, k).abs().t())).max()
    assert (y_tc - y_cc).abs().max().item() <= 2 * bound.item()
