"""oomb_moe_decode_fp8_noalloc against oomb_moe_decode_fp8, through the C ABI.

The no-alloc entry point runs the fused decode step with its scratch in one
fixed device array inside liboomb.so instead of a caller workspace.  Two calls
in a row must each give the workspace entry point's results on the same
inputs (the same kernels run: ids and weights bit-exact, outputs within the
fused-decode tolerance), and a call that needs more than the array holds is
refused before any launch.  This file is collected last so the set-up of the
array also runs after every other test has used the library.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import oracle as O  # noqa: E402
from homelab_b200 import _lib  # noqa: E402
from homelab_b200 import MoeLayer, SCALE_128X128  # noqa: E402
from homelab_b200.backend import Gpu  # noqa: E402
from homelab_b200.records import ExpertBank  # noqa: E402

if not torch.cuda.is_available():
    pytest.skip("needs a GPU", allow_module_level=True)

DEV = torch.device("cuda", 0)
H, E, K, I = 2048, 128, 8, 768


@pytest.fixture(scope="module")
def layer():
    gpu = Gpu(0)
    bank = ExpertBank(E, H, I, SCALE_128X128, DEV)
    bank.fill_random(gpu, seed=12)
    router = O.normal_bf16(13, E * H, 0.0, 0.02)
    router_d = torch.from_numpy(router.view(np.int16)).to(DEV)
    L = MoeLayer(hidden=H, experts=E, top_k=K, router_w=router_d.data_ptr(), recs=bank.addrs.data_ptr())
    L.geo = bank.geo
    torch.cuda.synchronize()
    yield dict(gpu=gpu, bank=bank, router_d=router_d, L=L)
    torch.cuda.synchronize()
    assert gpu.device_error() == 0, "a bounded device wait ran out"


def noalloc(L, x, t, out, ids, wts):
    return _lib.lib().oomb_moe_decode_fp8_noalloc(
        C.byref(L), x.data_ptr(), _lib.BF16, t, out.data_ptr(),
        _lib.BF16 if out.dtype == torch.bfloat16 else _lib.F32, ids.data_ptr(), wts.data_ptr(),
        torch.cuda.current_stream(DEV).cuda_stream)


@pytest.mark.parametrize("t", [1, 16])
def test_noalloc_matches_workspace_entry_two_calls_in_a_row(layer, t):
    gpu, L = layer["gpu"], layer["L"]
    x = torch.from_numpy(O.normal_bf16(900 + t, t * H).view(np.int16)).to(DEV).view(torch.bfloat16).view(t, H)
    ws = gpu.moe_decode_workspace(L, t)
    out_ws = torch.empty((t, H), dtype=torch.float32, device=DEV)
    ids_ws = torch.empty((t, K), dtype=torch.int32, device=DEV)
    w_ws = torch.empty((t, K), dtype=torch.float32, device=DEV)
    gpu.moe_decode(L, x, t, out_ws, ws, ids_ws, w_ws)
    for _ in range(2):
        out = torch.full((t, H), float("nan"), dtype=torch.float32, device=DEV)
        ids = torch.full((t, K), -1, dtype=torch.int32, device=DEV)
        wts = torch.full((t, K), float("nan"), dtype=torch.float32, device=DEV)
        assert noalloc(L, x, t, out, ids, wts) == _lib.OK
        torch.cuda.synchronize()
        assert torch.equal(ids, ids_ws)
        assert torch.equal(wts, w_ws)
        rel = ((out - out_ws).abs().max() / out_ws.abs().max()).item()
        assert rel <= 1e-4, rel


def test_noalloc_refuses_calls_larger_than_its_scratch(layer):
    L = layer["L"]
    t_fit = 92
    t_big = t_fit + 1
    need = _lib.lib().oomb_moe_decode_workspace_bytes(t_big, C.byref(L))
    assert need > _lib.NOALLOC_SCRATCH_BYTES >= _lib.lib().oomb_moe_decode_workspace_bytes(t_fit, C.byref(L))
    x = torch.zeros((t_big, H), dtype=torch.bfloat16, device=DEV)
    out = torch.zeros((t_big, H), dtype=torch.float32, device=DEV)
    ids = torch.zeros((t_big, K), dtype=torch.int32, device=DEV)
    wts = torch.zeros((t_big, K), dtype=torch.float32, device=DEV)
    assert noalloc(L, x, t_big, out, ids, wts) == _lib.E_WORKSPACE
    torch.cuda.synchronize()
    assert not out.any(), "a refused call must launch nothing"
