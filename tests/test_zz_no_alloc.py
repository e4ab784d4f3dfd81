"""oomb_moe_decode_fp8_noalloc against oomb_moe_decode_fp8, through the C ABI.

The no-alloc entry point serves callers that cannot allocate device memory
where they run the decode step (an allocation may synchronise the device, and
some hosts have no device allocator at the call site): it runs the fused
decode step with its scratch in one fixed device array inside liboomb.so
instead of a caller workspace.  The same kernels run on the same inputs, so
two calls in a row must each reproduce the workspace entry point's ids,
weights and outputs bit for bit, for one-launch batches (t <= 16) and for the
grouped tensor-core path (t >= 17, whose self-resetting route ticket and split
activations live in the shared array).  A call that needs more than the array holds is refused before
any launch, and after a bounded device wait has run out, clearing the error
zeroes the array's sync words so the next calls are again exact.  This file is
collected last so the set-up of the array also runs after every other test
has used the library.
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


@pytest.mark.parametrize("t", [1, 16, 32])
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
        assert torch.equal(out, out_ws)


def test_noalloc_refuses_calls_larger_than_its_scratch(layer):
    L = layer["L"]
    sizes = {t: _lib.lib().oomb_moe_decode_workspace_bytes(t, C.byref(L)) for t in range(1, 200)}
    t_fit = max(t for t, n in sizes.items() if n <= _lib.NOALLOC_SCRATCH_BYTES)
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


def test_noalloc_exact_after_a_device_error_is_cleared(layer):
    """A bounded wait runs out (two virtual expert-parallel ranks, one of which
    never returns its rows, with a 1 ms wait limit); clearing the error also
    zeroes the no-alloc array's sync words, and the next two no-alloc calls
    equal the workspace entry point bit for bit."""
    from homelab_b200.ep import EpGpuOps, EpPeerMailboxes, EpPeerMoeLayer
    gpu, L, bank = layer["gpu"], layer["L"], layer["bank"]
    router = layer["router_d"].view(torch.bfloat16).view(E, H)
    G, t1 = 2, 1
    epr = E // G
    mb = EpPeerMailboxes(None, H, K, t1, torch.bfloat16, DEV, ranks=G)
    ranks = [EpPeerMoeLayer(EpGpuOps(DEV), mb, g, H, E, K, I, router, bank.addrs[g * epr:(g + 1) * epr].contiguous(),
                            bank.geo, t1) for g in range(G)]
    try:
        gpu.set_wait_limit(1_000_000)
        xe = torch.from_numpy(O.normal_bf16(950, G * H).view(np.int16)).to(DEV).view(torch.bfloat16).view(G, H)
        for g, r in enumerate(ranks):
            r.phase_route(xe[g:g + 1], t1)
        ranks[0].phase_experts(t1)
        ranks[0].phase_combine(t1, torch.empty((t1, H), dtype=torch.float32, device=DEV))
        torch.cuda.synchronize()
        gpu.set_wait_limit(0)
        assert gpu.device_error(clear=False) != 0, "the wait should have run out"
        assert _lib.lib().oomb_device_error(None, 1) == _lib.E_TIMEOUT
        assert gpu.device_error() == 0
    finally:
        gpu.set_wait_limit(0)
        mb.close()
    for t in (1, 32):
        x = torch.from_numpy(O.normal_bf16(960 + t, t * H).view(np.int16)).to(DEV).view(torch.bfloat16).view(t, H)
        ws = gpu.moe_decode_workspace(L, t)
        out_ws = torch.empty((t, H), dtype=torch.float32, device=DEV)
        gpu.moe_decode(L, x, t, out_ws, ws)
        for _ in range(2):
            out = torch.full((t, H), float("nan"), dtype=torch.float32, device=DEV)
            ids = torch.full((t, K), -1, dtype=torch.int32, device=DEV)
            wts = torch.full((t, K), float("nan"), dtype=torch.float32, device=DEV)
            assert noalloc(L, x, t, out, ids, wts) == _lib.OK
            torch.cuda.synchronize()
            assert torch.equal(out, out_ws)
    assert gpu.device_error() == 0
