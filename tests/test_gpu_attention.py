"""GQA decode attention over a bf16 KV cache (oomb_attention_decode) against float64.

BASELINE config 4's attention: 32 query heads over 8 kv heads, head_dim 128,
bf16 cache, context 4096, batch 1-32.  Bars: outputs within 1e-5 of the
float64 softmax-weighted sum over the exact cache values, relative to the
largest output (fp32 softmax and accumulation), and BASELINE's max relative
error 1e-3; bf16 outputs equal RN of the fp32 result to within one bf16 ulp;
repeated calls on one workspace give identical bits (self-resetting arrival
counters, fixed merge order); ragged and empty sequences; every supported
head grouping.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import oracle as O  # noqa: E402
from homelab_b200.backend import Gpu  # noqa: E402

if not torch.cuda.is_available():
    pytest.skip("needs a GPU", allow_module_level=True)

DEV = torch.device("cuda", 0)
D = 128


@pytest.fixture(scope="module")
def gpu():
    g = Gpu(0)
    yield g
    torch.cuda.synchronize()
    assert g.device_error() == 0, "a bounded device wait ran out or a length was out of range"


def cache(seed, B, kv_max, Hkv):
    """bf16 K and V caches [B, kv_max, Hkv, D] ~N(0, 1) and their exact fp32 values."""
    out = []
    for i in range(2):
        bits = O.normal_bf16(seed + i, B * kv_max * Hkv * D)
        out.append((torch.from_numpy(bits.view(np.int16)).to(DEV).view(torch.bfloat16).view(B, kv_max, Hkv, D),
                    O.bf16_to_f32(bits).reshape(B, kv_max, Hkv, D)))
    return out


def run(gpu, B, H, Hkv, kv_max, lens, q_bf16=False, out_bf16=False, seed=0, repeat=2):
    (kd, k32), (vd, v32) = cache(1000 + seed, B, kv_max, Hkv)
    if q_bf16:
        qb = O.normal_bf16(2000 + seed, B * H * D)
        q32 = O.bf16_to_f32(qb).reshape(B, H, D)
        qd = torch.from_numpy(qb.view(np.int16)).to(DEV).view(torch.bfloat16).view(B, H, D)
    else:
        q32 = O.normal_f32(2000 + seed, B * H * D).reshape(B, H, D)
        qd = torch.from_numpy(q32).to(DEV)
    scale = 1.0 / np.sqrt(D)
    ws = gpu.attention_workspace(B, H, Hkv, D, kv_max)
    lens_arg = lens if isinstance(lens, int) else torch.tensor(lens, dtype=torch.int32, device=DEV)
    outs = []
    for _ in range(repeat):
        out = torch.full((B, H, D), float("nan"), dtype=torch.bfloat16 if out_bf16 else torch.float32, device=DEV)
        gpu.attention_decode(qd, kd, vd, out, lens_arg, scale, ws, Hkv)
        outs.append(out)
    torch.cuda.synchronize()
    for o in outs[1:]:
        assert torch.equal(o, outs[0]), "repeated calls differ"
    truth = O.attention_decode_f64(q32, k32, v32, lens, scale)
    return outs[0].float().cpu().numpy(), truth


def check(got, truth, out_bf16=False):
    err = np.abs(got.astype(np.float64) - truth)
    top = max(np.abs(truth).max(), 1e-30)
    assert err.max() / top <= (2 ** -8 if out_bf16 else 1e-5), err.max() / top
    assert err.max() / top <= 1e-3 or out_bf16


@pytest.mark.parametrize("B,kv", [(1, 4096), (4, 4096), (32, 512)])
def test_config4_attention_matches_float64(gpu, B, kv):
    got, truth = run(gpu, B, 32, 8, kv, kv, seed=B)
    check(got, truth)


@pytest.mark.parametrize("G", [1, 2, 4, 8])
@pytest.mark.parametrize("q_bf16,out_bf16", [(False, False), (True, True)])
def test_head_groups_and_dtypes(gpu, G, q_bf16, out_bf16):
    Hkv = 4
    got, truth = run(gpu, 2, G * Hkv, Hkv, 300, 300, q_bf16, out_bf16, seed=10 + G)
    check(got, truth, out_bf16)


def test_ragged_and_empty_sequences(gpu):
    lens = [4096, 1, 0, 1000, 33]
    got, truth = run(gpu, len(lens), 32, 8, 4096, lens, seed=50)
    assert not got[2].any(), "a sequence with no visible position gives zeros"
    check(got, truth)


def test_rejects_bad_arguments(gpu):
    from homelab_b200 import _lib
    L = _lib.lib()
    assert L.oomb_attention_decode_workspace_bytes(1, 32, 8, 64, 128) == 0   # head_dim 128 only
    assert L.oomb_attention_decode_workspace_bytes(1, 30, 8, 128, 128) == 0  # heads % kv_heads
    assert L.oomb_attention_decode_workspace_bytes(1, 48, 4, 128, 128) == 0  # G = 12 unsupported
    assert L.oomb_attention_decode_workspace_bytes(1, 32, 8, 128, 128) > 0


@pytest.mark.parametrize("src_bf16", [False, True])
def test_kv_append_then_attend(gpu, src_bf16):
    """Keys and values of a new token appended (from a fused projection's output,
    rows strided) at ragged positions; the cache holds bf16(src) there, nothing
    else changes, and attention over the grown sequences matches float64."""
    B, Hkv, H, kv_max = 3, 8, 32, 64
    (kd, k32), (vd, v32) = cache(3000, B, kv_max, Hkv)
    lens = [10, 0, 63]
    kv = torch.from_numpy(O.normal_f32(3100, B * 3 * Hkv * D).reshape(B, 3 * Hkv * D)).to(DEV)
    if src_bf16:
        kv = kv.to(torch.bfloat16)
    start = torch.tensor(lens, dtype=torch.int32, device=DEV)
    k_before = kd.clone()
    gpu.kv_append(kv[:, Hkv * D:2 * Hkv * D], kd, start)
    gpu.kv_append(kv[:, 2 * Hkv * D:], vd, start)
    torch.cuda.synchronize()
    kvf = kv.float().cpu().numpy()
    kb16 = torch.from_numpy(kvf).to(torch.bfloat16).float().numpy()
    for b, L in enumerate(lens):
        assert np.array_equal(kd[b, L].float().cpu().numpy().reshape(-1), kb16[b, Hkv * D:2 * Hkv * D])
        assert np.array_equal(vd[b, L].float().cpu().numpy().reshape(-1), kb16[b, 2 * Hkv * D:])
        others = [j for j in range(kv_max) if j != L]
        assert torch.equal(kd[b, others], k_before[b, others])
    q32 = O.normal_f32(3200, B * H * D).reshape(B, H, D)
    ws = gpu.attention_workspace(B, H, Hkv, D, kv_max)
    out = torch.empty((B, H, D), dtype=torch.float32, device=DEV)
    newlen = torch.tensor([L + 1 for L in lens], dtype=torch.int32, device=DEV)
    gpu.attention_decode(torch.from_numpy(q32).to(DEV), kd, vd, out, newlen, 1.0 / np.sqrt(D), ws, Hkv)
    torch.cuda.synchronize()
    truth = O.attention_decode_f64(q32, kd.float().cpu().numpy(), vd.float().cpu().numpy(),
                                   [L + 1 for L in lens], 1.0 / np.sqrt(D))
    check(out.cpu().numpy(), truth)
