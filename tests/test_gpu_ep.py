"""Expert parallelism on one GPU with virtual ranks, against the single-GPU decode.

The virtual ranks share the device; their all-to-alls are tensor copies
(exchange_local).  Every rank's output must equal, bit for bit, the rows of the
single-GPU decode (oomb_moe_decode_fp8) of the whole batch on the same CUDA-core
expert kernels (OOMB_DECODE_CHAIN=1: batches of 17 and more otherwise take the
grouped tensor-core path, whose summation order differs), and an expert's
output for an assignment must not depend on which other assignments share its
launch.
"""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import oracle as O  # noqa: E402
import homelab_b200 as hb  # noqa: E402
from homelab_b200.backend import Gpu  # noqa: E402
from homelab_b200.ep import EpGpuOps, EpMoeLayer, exchange_local  # noqa: E402
from homelab_b200.records import ExpertBank  # noqa: E402

if not torch.cuda.is_available():
    pytest.skip("needs a GPU", allow_module_level=True)

DEV = torch.device("cuda", 0)
H, E, K, I = 2048, 64, 8, 768


@pytest.fixture(scope="module")
def layer():
    gpu = Gpu(0)
    bank = ExpertBank(E, H, I, hb.SCALE_128X128, DEV)
    bank.fill_random(gpu, seed=31)
    router = torch.from_numpy(O.normal_bf16(32, E * H, 0.0, 0.02).view(np.int16)).to(DEV).view(torch.bfloat16)
    router = router.view(E, H)
    L = hb.MoeLayer(hidden=H, experts=E, top_k=K, router_w=router.data_ptr(), recs=bank.addrs.data_ptr())
    L.geo = bank.geo
    torch.cuda.synchronize()
    yield dict(gpu=gpu, bank=bank, router=router, L=L)
    torch.cuda.synchronize()
    assert gpu.device_error() == 0


def cuda_core_decode(gpu, L, x, T, out, ws, ids=None, wts=None):
    """The single-GPU decode on the CUDA-core expert kernels (the arithmetic the ranks use)."""
    os.environ["OOMB_DECODE_CHAIN"] = "1"
    try:
        gpu.moe_decode(L, x, T, out, ws, ids, wts)
    finally:
        os.environ.pop("OOMB_DECODE_CHAIN", None)


def run_virtual(layer, x, G, t):
    """The expert-parallel step over G virtual ranks, t tokens each."""
    bank, router = layer["bank"], layer["router"]
    ops = EpGpuOps(DEV)
    epr = E // G
    ranks = [EpMoeLayer(ops, None, H, E, K, I, router, bank.addrs[g * epr:(g + 1) * epr].contiguous(), bank.geo, t,
                        ranks=G, rank=g) for g in range(G)]
    outs = [torch.empty((t, H), dtype=torch.float32, device=DEV) for _ in range(G)]
    ex = [r.phase_route(x[g * t:(g + 1) * t], t) for g, r in enumerate(ranks)]
    for j in range(len(ex[0])):
        exchange_local([e[j][0] for e in ex], [e[j][1] for e in ex])
    rb = [r.phase_experts(t) for r in ranks]
    exchange_local([b[0] for b in rb], [b[1] for b in rb])
    routing = [r.phase_combine(t, outs[g]) for g, r in enumerate(ranks)]
    return outs, routing


@pytest.mark.parametrize("G,t", [(2, 1), (2, 3), (4, 2), (8, 1)])
def test_expert_parallel_equals_single_gpu(layer, G, t):
    gpu, L = layer["gpu"], layer["L"]
    T = G * t
    x = torch.from_numpy(O.normal_bf16(40 + G * 10 + t, T * H).view(np.int16)).to(DEV).view(torch.bfloat16).view(T, H)
    ws = gpu.moe_decode_workspace(L, T)
    want = torch.empty((T, H), dtype=torch.float32, device=DEV)
    ids = torch.empty((T, K), dtype=torch.int32, device=DEV)
    wts = torch.empty((T, K), dtype=torch.float32, device=DEV)
    cuda_core_decode(gpu, L, x, T, want, ws, ids, wts)
    outs, routing = run_virtual(layer, x, G, t)
    torch.cuda.synchronize()
    for g in range(G):
        assert torch.equal(routing[g][0], ids[g * t:(g + 1) * t])
        assert torch.equal(routing[g][1], wts[g * t:(g + 1) * t])
        assert torch.equal(outs[g], want[g * t:(g + 1) * t]), f"rank {g} differs from one GPU"


def test_expert_outputs_do_not_depend_on_grouping(layer):
    """The same (expert, token) assignment gives the same bits alone or in a larger launch."""
    gpu, bank = layer["gpu"], layer["bank"]
    t = 3
    x = torch.from_numpy(O.normal_bf16(77, t * H).view(np.int16)).to(DEV).view(torch.bfloat16).view(t, H)

    def run(experts, toks):
        recs = bank.addrs[torch.tensor(experts, device=DEV)].contiguous()
        off = torch.tensor(np.concatenate([[0], np.cumsum([len(tk) for tk in toks])]), dtype=torch.int32, device=DEV)
        tok = torch.tensor([v for tk in toks for v in tk], dtype=torch.int32, device=DEV)
        A = int(off[-1])
        h = torch.empty((A, I), dtype=torch.float32, device=DEV)
        y = torch.empty((A, H), dtype=torch.float32, device=DEV)
        gpu.moe_gate_up(recs, off, tok, len(experts), x, h, bank.geo)
        gpu.moe_down(recs, off, len(experts), h, y, bank.geo)
        torch.cuda.synchronize()
        return y

    big = run([3, 9, 20, 41], [[0, 2], [1], [0, 1, 2], [2]])
    alone = run([20], [[1]])
    assert torch.equal(big[4], alone[0])  # expert 20, token 1
    pair = run([9, 41], [[1], [2]])
    assert torch.equal(big[2], pair[0]) and torch.equal(big[6], pair[1])


def run_virtual_peer(layer, xs, G, t):
    """Steps of the peer-memory expert-parallel path over G virtual ranks (one
    mailbox each, in this process); every phase runs for all ranks before the
    next, so each wait finds its flags already raised by finished kernels."""
    from homelab_b200.ep import EpPeerMailboxes, EpPeerMoeLayer
    bank, router = layer["bank"], layer["router"]
    ops = EpGpuOps(DEV)
    epr = E // G
    mb = EpPeerMailboxes(None, H, K, t, torch.bfloat16, DEV, ranks=G)
    ranks = [EpPeerMoeLayer(ops, mb, g, H, E, K, I, router, bank.addrs[g * epr:(g + 1) * epr].contiguous(), bank.geo, t)
             for g in range(G)]
    results = []
    for x in xs:
        outs = [torch.full((t, H), float("nan"), dtype=torch.float32, device=DEV) for _ in range(G)]
        for g, r in enumerate(ranks):
            r.phase_route(x[g * t:(g + 1) * t], t)
        for r in ranks:
            r.phase_experts(t)
        routing = [r.phase_combine(t, outs[g]) for g, r in enumerate(ranks)]
        torch.cuda.synchronize()
        results.append((outs, [(i.clone(), w.clone()) for i, w in routing]))
    mb.close()
    return results


@pytest.mark.parametrize("G,t", [(2, 1), (4, 2), (8, 1)])
def test_peer_expert_parallel_equals_single_gpu(layer, G, t):
    """Three consecutive steps (the mailbox epochs advance) equal the single-GPU decode."""
    gpu, L = layer["gpu"], layer["L"]
    T = G * t
    xs = [torch.from_numpy(O.normal_bf16(60 + 7 * G + t + i, T * H).view(np.int16)).to(DEV).view(torch.bfloat16)
          .view(T, H) for i in range(3)]
    ws = gpu.moe_decode_workspace(L, T)
    results = run_virtual_peer(layer, xs, G, t)
    for x, (outs, routing) in zip(xs, results):
        want = torch.empty((T, H), dtype=torch.float32, device=DEV)
        ids = torch.empty((T, K), dtype=torch.int32, device=DEV)
        wts = torch.empty((T, K), dtype=torch.float32, device=DEV)
        cuda_core_decode(gpu, L, x, T, want, ws, ids, wts)
        torch.cuda.synchronize()
        for g in range(G):
            assert torch.equal(routing[g][0], ids[g * t:(g + 1) * t])
            assert torch.equal(outs[g], want[g * t:(g + 1) * t]), f"rank {g} differs from one GPU"


def test_one_launch_expert_parallel_single_rank_equals_single_gpu(layer):
    """The expert-parallel one-launch kernel with one rank: it dispatches to and
    returns into its own mailbox (the waits are on flags that CTAs of the same,
    fully resident launch raise), and its output equals the single-GPU decode."""
    from homelab_b200.ep import EpDecodeLayer, EpPeerMailboxes
    gpu, L, bank, router = layer["gpu"], layer["L"], layer["bank"], layer["router"]
    for t in (1, 3):
        mb = EpPeerMailboxes(None, H, K, t, torch.bfloat16, DEV, ranks=1)
        ep = EpDecodeLayer(mb, 0, H, E, K, router, bank.addrs, bank.geo, t)
        ws = gpu.moe_decode_workspace(L, t)
        for step in range(3):
            x = torch.from_numpy(O.normal_bf16(400 + 10 * t + step, t * H).view(np.int16)).to(DEV).view(torch.bfloat16)
            x = x.view(t, H)
            out = torch.full((t, H), float("nan"), dtype=torch.float32, device=DEV)
            ep.forward(x, t, out)
            want = torch.empty((t, H), dtype=torch.float32, device=DEV)
            gpu.moe_decode(L, x, t, want, ws)
            torch.cuda.synchronize()
            assert torch.equal(out, want), f"t={t} step {step}"
        mb.close()


def test_one_launch_expert_parallel_takes_pinned_host_buffers(layer):
    """x and out in pinned host memory: the step stages x itself and stores out
    straight to the host, with the same bits as on device buffers."""
    from homelab_b200.ep import EpDecodeLayer, EpPeerMailboxes
    bank, router = layer["bank"], layer["router"]
    t = 2
    mb = EpPeerMailboxes(None, H, K, t, torch.bfloat16, DEV, ranks=1)
    ep = EpDecodeLayer(mb, 0, H, E, K, router, bank.addrs, bank.geo, t)
    for step in range(3):
        x = torch.from_numpy(O.normal_bf16(700 + step, t * H).view(np.int16)).to(DEV).view(torch.bfloat16).view(t, H)
        want = torch.full((t, H), float("nan"), dtype=torch.float32, device=DEV)
        ep.forward(x, t, want)
        xh = x.cpu().pin_memory()
        oh = torch.full((t, H), float("nan"), dtype=torch.float32).pin_memory()
        ep.forward(xh, t, oh)
        torch.cuda.synchronize()
        assert torch.equal(oh, want.cpu()), f"step {step}"
    mb.close()


@pytest.mark.parametrize("G,t", [(2, 16), (4, 8)])
def test_peer_expert_parallel_on_tensor_cores_matches_single_gpu(layer, G, t):
    """From 17 tokens over the ranks the chain over peer memory runs its local
    experts on the tensor cores (oomb_moe_experts_tiled_fp8); the single-GPU decode
    of the whole batch takes its tensor-core path too.  Routing and outputs
    bit-exact: an output's bits depend neither on the chunking of its expert's
    assignments nor on which other assignments share the launch."""
    from homelab_b200.ep import EP_TILED_MIN_TOKENS
    assert G * t >= EP_TILED_MIN_TOKENS
    gpu, L = layer["gpu"], layer["L"]
    T = G * t
    xs = [torch.from_numpy(O.normal_bf16(900 + 7 * G + t + i, T * H).view(np.int16)).to(DEV).view(torch.bfloat16)
          .view(T, H) for i in range(2)]
    ws = gpu.moe_decode_workspace(L, T)
    results = run_virtual_peer(layer, xs, G, t)
    for x, (outs, routing) in zip(xs, results):
        want = torch.empty((T, H), dtype=torch.float32, device=DEV)
        ids = torch.empty((T, K), dtype=torch.int32, device=DEV)
        wts = torch.empty((T, K), dtype=torch.float32, device=DEV)
        gpu.moe_decode(L, x, T, want, ws, ids, wts)
        torch.cuda.synchronize()
        got = torch.cat(outs)
        for g in range(G):
            assert torch.equal(routing[g][0], ids[g * t:(g + 1) * t])
        assert torch.equal(got, want), "expert-parallel tensor-core step differs from one GPU"
