"""Offload staging inside a decode step: the expert tier's two-phase fetch
(oomb_tier: ExpertSource::begin_fetch / finish_fetch over device slots and a
pinned host arena, with the LRU / LRFU policies).

A step routes on the device, reads the routing on the host (as Moe::begin_routed
does), fetches its experts, runs the experts that were resident while the others'
records copy in (resident groups first, as begin_routed orders them), waits for
the copies (finish_fetch), runs the rest, and combines in slot order.  Every
step's output must equal, bit for bit, the all-resident fused decode of the same
layer: a staged record is read in place like a resident one, and an expert's
output does not depend on which launch computes it.  Steps revisit experts so
fetches see hits, misses and evictions.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import oracle as O  # noqa: E402
import homelab_b200 as hb  # noqa: E402
from homelab_b200.backend import Gpu  # noqa: E402
from homelab_b200.records import ExpertBank  # noqa: E402
from homelab_b200.stage import ExpertTier, HostArena  # noqa: E402

if not torch.cuda.is_available():
    pytest.skip("needs a GPU", allow_module_level=True)

DEV = torch.device("cuda", 0)
H, E, K, I, LAYERS = 2048, 16, 8, 768, 2


@pytest.fixture(scope="module")
def setup():
    gpu = Gpu(0)
    bank = ExpertBank(LAYERS * E, H, I, hb.SCALE_128X128, DEV)
    bank.fill_random(gpu, seed=81)
    arena = HostArena(LAYERS * E, bank.stride)
    arena.buf.copy_(bank.buf.cpu())
    routers = [O.normal_bf16(82 + l, E * H, 0.0, 0.02).reshape(E, H) for l in range(LAYERS)]
    routers_d = [torch.from_numpy(r.reshape(-1).view(np.int16)).to(DEV).view(torch.bfloat16).view(E, H)
                 for r in routers]
    layers = []
    for l in range(LAYERS):
        addrs = bank.addrs[l * E:(l + 1) * E].contiguous()
        L = hb.MoeLayer(hidden=H, experts=E, top_k=K, router_w=routers_d[l].data_ptr(), recs=addrs.data_ptr())
        L.geo = bank.geo
        layers.append((L, addrs))
    torch.cuda.synchronize()
    yield dict(gpu=gpu, bank=bank, arena=arena, routers_d=routers_d, layers=layers)
    torch.cuda.synchronize()
    assert gpu.device_error() == 0


def staged_step(gpu, tier, layer, router_d, geo, xd, t):
    """One decode step of `layer` through the tier; returns (out, ready flags)."""
    logits = torch.empty((t, E), dtype=torch.float32, device=DEV)
    ids = torch.empty((t, K), dtype=torch.int32, device=DEV)
    w = torch.empty((t, K), dtype=torch.float32, device=DEV)
    gpu.router_logits(xd, router_d, logits, t, E, H)
    gpu.router_topk(logits, ids, w, t, E, K)
    ids_h = ids.cpu().numpy()  # the routing download (Moe::begin_routed)
    active = np.unique(ids_h)
    addrs, ready = tier.begin_fetch(layer, active)
    # resident groups first, then the loading ones; each in expert order
    order = [i for i in range(len(active)) if ready[i]] + [i for i in range(len(active)) if not ready[i]]
    off, tok, slot = [0], [], np.empty(t * K, dtype=np.int32)
    for i in order:
        e = active[i]
        for tt in range(t):
            for s in range(K):
                if ids_h[tt, s] == e:
                    slot[tt * K + s] = len(tok)
                    tok.append(tt)
        off.append(len(tok))
    A = len(tok)
    recs = torch.tensor([addrs[i] for i in order], dtype=torch.int64, device=DEV)
    offd = torch.tensor(off, dtype=torch.int32, device=DEV)
    tokd = torch.tensor(tok, dtype=torch.int32, device=DEV)
    h = torch.empty((A, I), dtype=torch.float32, device=DEV)
    y = torch.empty((A, H), dtype=torch.float32, device=DEV)
    nr = sum(ready)
    if nr:  # the resident experts compute while the copies run
        gpu.moe_gate_up(recs[:nr], offd[:nr + 1], tokd, nr, xd, h, geo)
        gpu.moe_down(recs[:nr], offd[:nr + 1], nr, h, y, geo)
    tier.finish_fetch()
    if nr < len(order):
        gpu.moe_gate_up(recs[nr:], offd[nr:], tokd, len(order) - nr, xd, h, geo)
        gpu.moe_down(recs[nr:], offd[nr:], len(order) - nr, h, y, geo)
    out = torch.empty((t, H), dtype=torch.float32, device=DEV)
    gpu.moe_combine_slots(y, torch.from_numpy(slot).to(DEV), w, out, t, H, K)
    return out, ready


@pytest.mark.parametrize("policy", ["lru", "lrfu:4"])
def test_staged_steps_equal_resident_decode(setup, policy):
    gpu, layers, bank = setup["gpu"], setup["layers"], setup["bank"]
    tier = ExpertTier(setup["arena"], LAYERS, E, slots=12, device=DEV, policy=policy)
    t = 1  # top-8 of 16 experts: 8 distinct records a step, 12 slots for 32 records
    seen_ready = seen_cold = 0
    try:
        for step in range(6):
            layer = step % LAYERS
            L, _ = layers[layer]
            xd = torch.from_numpy(O.normal_bf16(1000 + step, t * H).view(np.int16)).to(DEV).view(torch.bfloat16)
            xd = xd.view(t, H)
            out, ready = staged_step(gpu, tier, layer, setup["routers_d"][layer], bank.geo, xd, t)
            want = torch.empty((t, H), dtype=torch.float32, device=DEV)
            gpu.moe_decode(L, xd, t, want, gpu.moe_decode_workspace(L, t))
            torch.cuda.synchronize()
            assert torch.equal(out, want), f"step {step}"
            seen_ready += sum(ready)
            seen_cold += len(ready) - sum(ready)
        st = tier.stats()
        assert st["misses"] == seen_cold and st["hits"] == seen_ready
        assert st["evictions"] > 0 and seen_ready > 0, st
        assert st["bytes_copied"] == st["misses"] * bank.stride
    finally:
        tier.close()


def test_fetch_larger_than_the_slots_is_refused(setup):
    from homelab_b200._lib import OombError
    tier = ExpertTier(setup["arena"], LAYERS, E, slots=4, device=DEV)
    try:
        with pytest.raises(OombError):
            tier.begin_fetch(0, list(range(5)))
        addrs, ready = tier.begin_fetch(0, [3, 3, 1])
        assert addrs[0] == addrs[1] and ready == [False, False, False]
        tier.finish_fetch()
        addrs2, ready2 = tier.begin_fetch(0, [1, 3])
        assert ready2 == [True, True] and addrs2 == [addrs[2], addrs[0]]
        tier.finish_fetch()
        torch.cuda.synchronize()
    finally:
        tier.close()
