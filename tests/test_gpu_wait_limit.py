"""A bounded device wait that nothing will satisfy runs out, reports its code,
and leaves the context usable.

The peer-memory expert-parallel step over two virtual ranks on one GPU: rank 0
runs every phase, rank 1 never returns its expert outputs, so rank 0's combine
waits for a return flag that no kernel raises.  With the wait limit shortened
to a millisecond (oomb_set_wait_limit) the wait gives up: the combine writes
nothing, the device error word reads ERR_EP_RETURN_WAIT (0x710), and after
the error is cleared and the mailboxes are zeroed the next steps are again
bit-identical to the single-GPU decode.  No GPU fault is involved: the kernel
polls a flag with a time limit and returns.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import oracle as O  # noqa: E402
import homelab_b200 as hb  # noqa: E402
from homelab_b200 import _lib  # noqa: E402
from homelab_b200.backend import Gpu  # noqa: E402
from homelab_b200.ep import EpGpuOps, EpPeerMailboxes, EpPeerMoeLayer  # noqa: E402
from homelab_b200.records import ExpertBank  # noqa: E402

if not torch.cuda.is_available():
    pytest.skip("needs a GPU", allow_module_level=True)

DEV = torch.device("cuda", 0)
H, E, K, I = 2048, 64, 8, 768
ERR_EP_RETURN_WAIT = 0x710


@pytest.fixture(scope="module")
def layer():
    gpu = Gpu(0)
    bank = ExpertBank(E, H, I, hb.SCALE_128X128, DEV)
    bank.fill_random(gpu, seed=77)
    router = torch.from_numpy(O.normal_bf16(78, E * H, 0.0, 0.02).view(np.int16)).to(DEV).view(torch.bfloat16)
    router = router.view(E, H)
    L = hb.MoeLayer(hidden=H, experts=E, top_k=K, router_w=router.data_ptr(), recs=bank.addrs.data_ptr())
    L.geo = bank.geo
    torch.cuda.synchronize()
    yield dict(gpu=gpu, bank=bank, router=router, L=L)
    gpu.set_wait_limit(0)
    torch.cuda.synchronize()
    assert gpu.device_error() == 0


def _x(seed, T):
    return torch.from_numpy(O.normal_bf16(seed, T * H).view(np.int16)).to(DEV).view(torch.bfloat16).view(T, H)


def test_return_wait_runs_out_then_recovers(layer):
    gpu, L, bank, router = layer["gpu"], layer["L"], layer["bank"], layer["router"]
    G, t = 2, 1
    T = G * t
    epr = E // G
    ops = EpGpuOps(DEV)
    mb = EpPeerMailboxes(None, H, K, t, torch.bfloat16, DEV, ranks=G)
    ranks = [EpPeerMoeLayer(ops, mb, g, H, E, K, I, router, bank.addrs[g * epr:(g + 1) * epr].contiguous(),
                            bank.geo, t) for g in range(G)]
    ws = gpu.moe_decode_workspace(L, T)
    try:
        assert gpu.device_error() == 0

        # rank 1 dispatches (so rank 0's grouping finds every dispatch flag) but
        # never runs its experts: it never raises its return flag on rank 0
        gpu.set_wait_limit(1_000_000)  # 1 ms
        x = _x(500, T)
        for g, r in enumerate(ranks):
            r.phase_route(x[g * t:(g + 1) * t], t)
        ranks[0].phase_experts(t)
        out = torch.full((t, H), float("nan"), dtype=torch.float32, device=DEV)
        ranks[0].phase_combine(t, out)
        torch.cuda.synchronize()  # the combine returned: the wait ran out instead of hanging
        code = gpu.device_error(clear=False)
        assert code == ERR_EP_RETURN_WAIT, hex(code)
        assert torch.isnan(out).all(), "a step whose wait ran out must write no output"
        status = _lib.lib().oomb_device_error(None, 1)
        assert status == _lib.E_TIMEOUT
        assert gpu.device_error() == 0
        gpu.set_wait_limit(0)

        # recovery: zero the mailboxes (step counters, flags, tickets), then run
        # whole steps on both ranks; each must equal the single-GPU decode
        for base in mb.bases:
            _lib.check(_lib.lib().oomb_workspace_clear(base, mb.nbytes, torch.cuda.current_stream(DEV).cuda_stream))
        for step in range(2):
            x = _x(510 + step, T)
            outs = [torch.full((t, H), float("nan"), dtype=torch.float32, device=DEV) for _ in range(G)]
            for g, r in enumerate(ranks):
                r.phase_route(x[g * t:(g + 1) * t], t)
            for r in ranks:
                r.phase_experts(t)
            for g, r in enumerate(ranks):
                r.phase_combine(t, outs[g])
            want = torch.empty((T, H), dtype=torch.float32, device=DEV)
            gpu.moe_decode(L, x, T, want, ws)
            torch.cuda.synchronize()
            assert gpu.device_error() == 0
            for g in range(G):
                assert torch.equal(outs[g], want[g * t:(g + 1) * t]), f"step {step} rank {g}"
    finally:
        gpu.set_wait_limit(0)
        mb.close()
