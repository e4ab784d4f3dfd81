"""The fused decode, the kernel chain and expert parallelism at BASELINE configs 4 and 5.

Config 4: hidden 4096, 64 experts, top-6, intermediate 1408.  Config 5: hidden
4096, 256 experts, top-8, intermediate 2048 (32 experts per GPU at 8 GPUs).
128x128 block scales, bf16 activations ~N(0, 1), router ~N(0, 0.02).  Bars:
top-k ids and weights bit-exact with the oracle; outputs within 1e-4 of the
float64 experts (relative to the largest) and within BASELINE's max relative
error 1e-3; up to 16 tokens the one-launch step and the chain of kernels give
the same bits, from 17 tokens the grouped tensor-core path agrees with the chain
to 1e-5; every expert-parallel rank (virtual ranks on one GPU, G = 2, 4, 8)
gives the bits of the single-GPU decode on the same CUDA-core kernels.
"""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import oracle as O  # noqa: E402
import homelab_b200 as hb  # noqa: E402
from homelab_b200.backend import Gpu  # noqa: E402
from homelab_b200.records import ExpertBank  # noqa: E402

if not torch.cuda.is_available():
    pytest.skip("needs a GPU", allow_module_level=True)

DEV = torch.device("cuda", 0)
CONFIGS = {4: (4096, 64, 6, 1408), 5: (4096, 256, 8, 2048)}


@pytest.fixture(scope="module")
def gpu():
    g = Gpu(0)
    yield g
    torch.cuda.synchronize()
    assert g.device_error() == 0, "a bounded device wait ran out"


def bf16_dev(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).to(DEV).view(torch.bfloat16)


@pytest.fixture(scope="module")
def layers(gpu):
    out = {}
    for c, (H, E, K, I) in CONFIGS.items():
        bank = ExpertBank(E, H, I, hb.SCALE_128X128, DEV)
        bank.fill_random(gpu, seed=40 + c)
        router = O.normal_bf16(50 + c, E * H, 0.0, 0.02).reshape(E, H)
        router_d = bf16_dev(router.reshape(-1)).view(E, H)
        L = hb.MoeLayer(hidden=H, experts=E, top_k=K, router_w=router_d.data_ptr(), recs=bank.addrs.data_ptr())
        L.geo = bank.geo
        out[c] = dict(bank=bank, router=router, router_d=router_d, L=L, shape=(H, E, K, I))
    torch.cuda.synchronize()
    yield out


def host_record(bank, e):
    e = int(e)
    return bank.buf[e * bank.stride:(e + 1) * bank.stride].cpu().numpy()


def decode(gpu, lay, xd, t, chain=False, out_dtype=torch.float32):
    H, E, K, I = lay["shape"]
    ws = gpu.moe_decode_workspace(lay["L"], t)
    ids = torch.empty((t, K), dtype=torch.int32, device=DEV)
    wts = torch.empty((t, K), dtype=torch.float32, device=DEV)
    out = torch.full((t, H), float("nan"), dtype=out_dtype, device=DEV)
    old = os.environ.get("OOMB_DECODE_CHAIN")
    os.environ["OOMB_DECODE_CHAIN"] = "1" if chain else "0"
    try:
        for _ in range(2):  # the workspace is reused: its sync words must stay consistent
            gpu.moe_decode(lay["L"], xd, t, out, ws, ids, wts)
        torch.cuda.synchronize()
    finally:
        if old is None:
            del os.environ["OOMB_DECODE_CHAIN"]
        else:
            os.environ["OOMB_DECODE_CHAIN"] = old
    return out, ids, wts


@pytest.mark.parametrize("config", [4, 5])
@pytest.mark.parametrize("t", [1, 4, 16, 32])
def test_decode_matches_oracle(gpu, layers, config, t):
    lay = layers[config]
    H, E, K, I = lay["shape"]
    xb = O.normal_bf16(600 + 10 * config + t, t * H)
    x32 = O.bf16_to_f32(xb).reshape(t, H)
    xd = bf16_dev(xb).view(t, H)
    out, ids, wts = decode(gpu, lay, xd, t)
    out_c, ids_c, wts_c = decode(gpu, lay, xd, t, chain=True)
    want_ids, want_w = O.router_topk(O.router_logits(x32, lay["router"]), K)
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    assert np.array_equal(wts.cpu().numpy().view(np.uint32), want_w.view(np.uint32))
    assert torch.equal(ids, ids_c) and torch.equal(wts, wts_c)
    if t <= 16:
        assert torch.equal(out, out_c), "one launch and the kernel chain differ"
    else:  # the grouped tensor-core path sums in another order
        rel_c = ((out - out_c).abs().max() / out_c.abs().max()).item()
        assert rel_c <= 1e-5, rel_c
    if t <= 4:
        active, off, tok, slot = O.group_assignments(want_ids, E)
        recs = [host_record(lay["bank"], e) for e in active]
        y = O.moe_experts_f64_fast(recs, lay["L"].geo, off, tok, x32)
        truth = O.combine_slots_f64(y, slot, want_w, t, H, K)
        rel = np.abs(out.cpu().numpy() - truth).max() / np.abs(truth).max()
        assert rel <= 1e-4, rel


def run_virtual(lay, x, G, t, transport):
    """The expert-parallel step over G virtual ranks on this GPU, t tokens each:
    the NCCL layout with tensor copies as the all-to-alls, or the chain over peer
    mailboxes (each phase for every rank before the next)."""
    from homelab_b200.ep import EpGpuOps, EpMoeLayer, EpPeerMailboxes, EpPeerMoeLayer, exchange_local
    H, E, K, I = lay["shape"]
    bank, router = lay["bank"], lay["router_d"]
    ops = EpGpuOps(DEV)
    epr = E // G
    outs = [torch.full((t, H), float("nan"), dtype=torch.float32, device=DEV) for _ in range(G)]
    if transport == "copy":
        ranks = [EpMoeLayer(ops, None, H, E, K, I, router, bank.addrs[g * epr:(g + 1) * epr].contiguous(), bank.geo,
                            t, ranks=G, rank=g) for g in range(G)]
        ex = [r.phase_route(x[g * t:(g + 1) * t], t) for g, r in enumerate(ranks)]
        for j in range(len(ex[0])):
            exchange_local([e[j][0] for e in ex], [e[j][1] for e in ex])
        rb = [r.phase_experts(t) for r in ranks]
        exchange_local([b[0] for b in rb], [b[1] for b in rb])
        for g, r in enumerate(ranks):
            r.phase_combine(t, outs[g])
        torch.cuda.synchronize()
        return outs
    mb = EpPeerMailboxes(None, H, K, t, torch.bfloat16, DEV, ranks=G)
    ranks = [EpPeerMoeLayer(ops, mb, g, H, E, K, I, router, bank.addrs[g * epr:(g + 1) * epr].contiguous(), bank.geo,
                            t) for g in range(G)]
    for g, r in enumerate(ranks):
        r.phase_route(x[g * t:(g + 1) * t], t)
    for r in ranks:
        r.phase_experts(t)
    for g, r in enumerate(ranks):
        r.phase_combine(t, outs[g])
    torch.cuda.synchronize()
    mb.close()
    return outs


@pytest.mark.parametrize("G,t", [(2, 2), (4, 1), (8, 2)])
@pytest.mark.parametrize("transport", ["copy", "peer"])
def test_expert_parallel_config5_equals_single_gpu(gpu, layers, G, t, transport):
    lay = layers[5]
    H, E, K, I = lay["shape"]
    T = G * t
    xd = bf16_dev(O.normal_bf16(700 + 10 * G + t, T * H)).view(T, H)
    want, _, _ = decode(gpu, lay, xd, T, chain=True)  # the CUDA-core expert kernels the ranks use
    outs = run_virtual(lay, xd, G, t, transport)
    for g in range(G):
        assert torch.equal(outs[g], want[g * t:(g + 1) * t]), f"rank {g} of {G} differs from one GPU"


def test_one_launch_expert_parallel_config5_single_rank(gpu, layers):
    """The expert-parallel one-launch kernel at config 5 with one rank (256 local
    experts): its output equals the single-GPU decode."""
    from homelab_b200.ep import EpDecodeLayer, EpPeerMailboxes
    lay = layers[5]
    H, E, K, I = lay["shape"]
    t = 2
    mb = EpPeerMailboxes(None, H, K, t, torch.bfloat16, DEV, ranks=1)
    ep = EpDecodeLayer(mb, 0, H, E, K, lay["router_d"], lay["bank"].addrs, lay["bank"].geo, t)
    for step in range(2):
        xd = bf16_dev(O.normal_bf16(800 + step, t * H)).view(t, H)
        out = torch.full((t, H), float("nan"), dtype=torch.float32, device=DEV)
        ep.forward(xd, t, out)
        want, _, _ = decode(gpu, lay, xd, t)
        assert torch.equal(out, want), f"step {step}"
    mb.close()
