"""The one-launch decode step (decode_kernel) against the chain of kernels.

oomb_moe_decode_fp8 runs the whole routed step of a resident layer in one
persistent launch for up to 16 tokens and routers of at most 256 experts;
OOMB_DECODE_CHAIN=1 makes it run the chain route -> gate/up -> down -> combine
instead (each of those kernels is checked against the oracle in
test_gpu_parity.py).  The two must agree bit for bit on every output (ids,
weights, out) across activation dtypes, scale layouts, output dtypes, batch
sizes (one token, two, and the chunked path) and layer shapes; repeated
launches on one workspace (grid-barrier and row-group counters reset
themselves), launches of different batch sizes on one workspace and CUDA graph
replays must keep giving the same bits; the one-launch result must meet the
float64 bound on its own; and activations and outputs in pinned host memory
(read and written by the step's kernels over the bus) must give the same bits
as device buffers, in graphs too, while pageable host memory is refused.
"""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import oracle as O  # noqa: E402
import homelab_b200 as hb  # noqa: E402
from homelab_b200 import SCALE_128X128, SCALE_1X128  # noqa: E402
from homelab_b200.backend import Gpu  # noqa: E402
from homelab_b200.records import ExpertBank  # noqa: E402

if not torch.cuda.is_available():
    pytest.skip("needs a GPU", allow_module_level=True)

DEV = torch.device("cuda", 0)

# hidden, experts, top_k, inter, scale layout
LAYERS = {
    "config2": (2048, 128, 8, 768, SCALE_128X128),
    "small": (1024, 64, 6, 512, SCALE_1X128),
    "wide": (4096, 256, 8, 256, SCALE_128X128),
    "odd": (528, 40, 5, 272, SCALE_1X128),
}


@pytest.fixture(scope="module")
def gpu():
    g = Gpu(0)
    yield g
    torch.cuda.synchronize()
    assert g.device_error() == 0, "a bounded device wait ran out"


_layers = {}


def get_layer(gpu, name):
    if name not in _layers:
        H, E, K, I, layout = LAYERS[name]
        b = ExpertBank(E, H, I, layout, DEV)
        b.fill_random(gpu, seed=sum(map(ord, name)))
        router = O.normal_bf16(7 + E, E * H, 0.0, 0.02)
        router_d = torch.from_numpy(router.view(np.int16)).to(DEV).view(torch.bfloat16)
        L = hb.MoeLayer(hidden=H, experts=E, top_k=K, router_w=router_d.data_ptr(), recs=b.addrs.data_ptr())
        L.geo = b.geo
        torch.cuda.synchronize()
        _layers[name] = dict(bank=b, router=router, router_d=router_d, L=L)
    return _layers[name]


def make_x(H, t, xbf16, seed):
    xb = O.normal_bf16(seed, t * H)
    x = torch.from_numpy(xb.view(np.int16)).to(DEV).view(torch.bfloat16).view(t, H)
    return x if xbf16 else x.float()


def run(gpu, lay, x, t, out_dtype, chain, ws=None):
    H, K = lay["L"].hidden, lay["L"].top_k
    if ws is None:
        ws = gpu.moe_decode_workspace(lay["L"], t)
    out = torch.full((t, H), float("nan"), dtype=out_dtype, device=DEV)
    ids = torch.full((t, K), -1, dtype=torch.int32, device=DEV)
    wts = torch.full((t, K), float("nan"), dtype=torch.float32, device=DEV)
    if chain:
        os.environ["OOMB_DECODE_CHAIN"] = "1"
    try:
        gpu.moe_decode(lay["L"], x, t, out, ws, ids, wts)
    finally:
        os.environ.pop("OOMB_DECODE_CHAIN", None)
    return out, ids, wts


def same(a, b):
    return a.shape == b.shape and torch.equal(a.view(torch.int32) if a.dtype == torch.float32 else a,
                                              b.view(torch.int32) if b.dtype == torch.float32 else b)


@pytest.mark.parametrize("name", list(LAYERS))
@pytest.mark.parametrize("xbf16", [True, False])
@pytest.mark.parametrize("t", [1, 2, 5, 11])
def test_one_launch_equals_chain(gpu, name, xbf16, t):
    lay = get_layer(gpu, name)
    H = lay["L"].hidden
    out_dtype = torch.bfloat16 if (t % 2 == 1) else torch.float32
    x = make_x(H, t, xbf16, 500 + t)
    got = run(gpu, lay, x, t, out_dtype, chain=False)
    want = run(gpu, lay, x, t, out_dtype, chain=True)
    torch.cuda.synchronize()
    for g, w, what in zip(got, want, ("out", "ids", "weights")):
        assert same(g, w), f"{what} differs from the chain of kernels"


def test_repeated_launches_and_batch_sizes_share_a_workspace(gpu):
    lay = get_layer(gpu, "config2")
    H = lay["L"].hidden
    ws = gpu.moe_decode_workspace(lay["L"], 16)
    xs = {t: make_x(H, t, True, 900 + t) for t in (1, 3, 16)}
    # each path on a fresh workspace (t = 16 takes the tensor-core path unless chained)
    want = {t: run(gpu, lay, xs[t], t, torch.float32, chain=False) for t in xs}
    want_chain = {t: run(gpu, lay, xs[t], t, torch.float32, chain=True) for t in xs}
    for i, t in enumerate((1, 1, 16, 3, 1, 16, 16, 3)):
        got = run(gpu, lay, xs[t], t, torch.float32, chain=False, ws=ws)
        got_chain = None
        if i % 3 == 2:  # the chain of kernels on the same workspace in between
            got_chain = run(gpu, lay, xs[t], t, torch.float32, chain=True, ws=ws)
        torch.cuda.synchronize()
        for g, w in zip(got, want[t]):
            assert same(g, w)
        if got_chain is not None:
            for g, w in zip(got_chain, want_chain[t]):
                assert same(g, w)


def test_graph_replays_give_the_same_bits(gpu):
    lay = get_layer(gpu, "config2")
    L, H, K = lay["L"], lay["L"].hidden, lay["L"].top_k
    t = 1
    ws = gpu.moe_decode_workspace(L, t)
    xs = [make_x(H, t, True, 1000 + i) for i in range(3)]
    outs = [torch.empty((t, H), dtype=torch.bfloat16, device=DEV) for _ in xs]
    ids = torch.empty((t, K), dtype=torch.int32, device=DEV)
    wts = torch.empty((t, K), dtype=torch.float32, device=DEV)
    want = [run(gpu, lay, x, t, torch.bfloat16, chain=True)[0] for x in xs]
    s = torch.cuda.Stream(DEV)
    s.wait_stream(torch.cuda.current_stream(DEV))
    with torch.cuda.stream(s):
        gpu.moe_decode(L, xs[0], t, outs[0], ws, ids, wts)  # warm-up outside the capture
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for x, o in zip(xs, outs):
                gpu.moe_decode(L, x, t, o, ws, ids, wts)
    torch.cuda.current_stream(DEV).wait_stream(s)
    for _ in range(3):
        for o in outs:
            o.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        for o, w in zip(outs, want):
            assert torch.equal(o, w)
    del g


@pytest.mark.parametrize("name,xbf16,t", [("small", False, 3), ("odd", True, 7), ("wide", True, 2)])
def test_one_launch_meets_the_float64_bound(gpu, name, xbf16, t):
    lay = get_layer(gpu, name)
    L = lay["L"]
    H, E, K = L.hidden, L.experts, L.top_k
    x = make_x(H, t, xbf16, 1200 + t)
    out, ids, wts = run(gpu, lay, x, t, torch.float32, chain=False)
    torch.cuda.synchronize()
    x32 = x.float().cpu().numpy()
    want_ids, want_w = O.router_topk(O.router_logits(x32, lay["router"].reshape(E, H)), K)
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    assert np.array_equal(wts.cpu().numpy().view(np.uint32), want_w.view(np.uint32))
    active, off, tok, slot = O.group_assignments(want_ids, E)
    host = lay["bank"].host_records()
    y = O.moe_experts_f64([host[e] for e in active], L.geo, off, tok, x32)
    truth = O.combine_slots_f64(y, slot, want_w, t, H, K)
    got = out.cpu().numpy()
    assert np.abs(got - truth).max() / np.abs(truth).max() <= 1e-4


def _same_bits(a, b):
    if a.dtype == torch.float32:
        return torch.equal(a.view(torch.int32), b.view(torch.int32))
    return torch.equal(a.view(torch.int16), b.view(torch.int16))


@pytest.mark.parametrize("chain", [False, True])
@pytest.mark.parametrize("xbf16,out_dtype,t", [(True, torch.bfloat16, 1), (False, torch.float32, 3),
                                               (True, torch.float32, 16), (False, torch.bfloat16, 24)])
def test_pinned_host_activations_and_outputs(gpu, chain, xbf16, out_dtype, t):
    """x and out in pinned host memory: the same bits as device buffers (the step
    reads x over the bus into its workspace and stores out into host memory)."""
    lay = get_layer(gpu, "config2")
    L, H, K = lay["L"], lay["L"].hidden, lay["L"].top_k
    x = make_x(H, t, xbf16, 1300 + t)
    want = run(gpu, lay, x, t, out_dtype, chain=chain)
    xh = x.cpu().pin_memory()
    oh = torch.full((t, H), float("nan"), dtype=out_dtype).pin_memory()
    ids = torch.full((t, K), -1, dtype=torch.int32, device=DEV)
    wts = torch.full((t, K), float("nan"), dtype=torch.float32, device=DEV)
    ws = gpu.moe_decode_workspace(L, t)
    if chain:
        os.environ["OOMB_DECODE_CHAIN"] = "1"
    try:
        for _ in range(2):  # the second call reuses the workspace's staged copy region
            gpu.moe_decode(L, xh, t, oh, ws, ids, wts)
    finally:
        os.environ.pop("OOMB_DECODE_CHAIN", None)
    torch.cuda.synchronize()
    assert _same_bits(oh, want[0].cpu())
    assert torch.equal(ids, want[1]) and _same_bits(wts, want[2])


def test_pinned_host_buffers_in_a_graph(gpu):
    """Graph replays of steps whose x and out are pinned host buffers, new host
    contents before every replay."""
    lay = get_layer(gpu, "config2")
    L, H = lay["L"], lay["L"].hidden
    t = 1
    xs = [make_x(H, t, True, 1400 + i) for i in range(4)]
    want = [run(gpu, lay, x, t, torch.bfloat16, chain=True)[0].cpu() for x in xs]
    xh = [torch.empty((t, H), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    oh = [torch.empty((t, H), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    ws = gpu.moe_decode_workspace(L, t)
    s = torch.cuda.Stream(DEV)
    s.wait_stream(torch.cuda.current_stream(DEV))
    with torch.cuda.stream(s):
        xh[0].copy_(xs[0].cpu())
        gpu.moe_decode(L, xh[0], t, oh[0], ws)  # warm-up outside the capture
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for j in range(2):
                gpu.moe_decode(L, xh[j], t, oh[j], ws)
    torch.cuda.current_stream(DEV).wait_stream(s)
    torch.cuda.synchronize()
    for r in range(2):
        for j in range(2):
            xh[j].copy_(xs[2 * r + j].cpu())
            oh[j].fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        for j in range(2):
            assert _same_bits(oh[j], want[2 * r + j])
    del g


def test_pageable_host_memory_is_refused(gpu):
    lay = get_layer(gpu, "small")
    L, H = lay["L"], lay["L"].hidden
    ws = gpu.moe_decode_workspace(L, 1)
    x = torch.zeros((1, H), dtype=torch.bfloat16)  # pageable
    out = torch.empty((1, H), dtype=torch.bfloat16, device=DEV)
    with pytest.raises(hb.OombError):
        gpu.moe_decode(L, x, 1, out, ws)
    with pytest.raises(hb.OombError):
        gpu.moe_decode(L, x.to(DEV), 1, torch.empty((1, H), dtype=torch.bfloat16), ws)
    torch.cuda.synchronize()


@pytest.mark.parametrize("name,xbf16,t", [("small", True, 12), ("small", False, 16), ("wide", True, 12)])
def test_tiled_decode_equals_tiled_calls_and_float64(gpu, name, xbf16, t):
    """From 17 tokens (here from 12, forced with OOMB_DECODE_TILED_MIN_T) the decode
    step runs the grouped tensor-core path: route, x split once for gate and up,
    SwiGLU, down, combine.  Its bits equal the public calls in that order
    (oomb_moe_tiled_fp8 for gate, up and down, oomb_moe_swiglu_range,
    oomb_moe_combine_slots on the same routing), and it is within 1e-4 of the
    float64 step."""
    lay = get_layer(gpu, name)
    L = lay["L"]
    H, E, K, I = L.hidden, L.experts, L.top_k, L.geo.inter
    if H % 128 or I % 128 or H < 2 * I:
        pytest.skip("layer shape outside the grouped tensor-core path")
    x = make_x(H, t, xbf16, 1500 + t)
    os.environ["OOMB_DECODE_TILED_MIN_T"] = "12"
    try:
        out, ids, wts = run(gpu, lay, x, t, torch.float32, chain=False)
    finally:
        os.environ.pop("OOMB_DECODE_TILED_MIN_T", None)
    torch.cuda.synchronize()
    x32 = x.float().cpu().numpy()
    want_ids, want_w = O.router_topk(O.router_logits(x32, lay["router"].reshape(E, H)), K)
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    active, off, tok, slot = O.group_assignments(want_ids, E)
    A = t * K
    b, g = lay["bank"], L.geo
    recs = b.addrs[torch.from_numpy(active).long().to(DEV)].contiguous()
    offd, tokd = torch.from_numpy(off).to(DEV), torch.from_numpy(tok).to(DEV)
    gg = torch.empty((A, I), dtype=torch.float32, device=DEV)
    uu, hh = torch.empty_like(gg), torch.empty_like(gg)
    y = torch.empty((A, H), dtype=torch.float32, device=DEV)
    gpu.moe_tiled(recs, offd, tokd, len(active), t, x, gg, I, H, (g.gate_weight, g.gate_scale), g.layout)
    gpu.moe_tiled(recs, offd, tokd, len(active), t, x, uu, I, H, (g.up_weight, g.up_scale), g.layout)
    gpu.moe_swiglu_range(gg, uu, hh, 0, A * I)
    gpu.moe_tiled(recs, offd, None, len(active), t, hh, y, H, I, (g.down_weight, g.down_scale), g.layout)
    want = torch.empty((t, H), dtype=torch.float32, device=DEV)
    gpu.moe_combine_slots(y, torch.from_numpy(slot).to(DEV), wts, want, t, H, K)
    torch.cuda.synchronize()
    assert torch.equal(out, want), "the decode step's tensor-core path differs from the public calls"
    host = lay["bank"].host_records()
    yv = O.moe_experts_f64([host[e] for e in active], L.geo, off, tok, x32)
    truth = O.combine_slots_f64(yv, slot, want_w, t, H, K)
    assert np.abs(out.cpu().numpy() - truth).max() / np.abs(truth).max() <= 1e-4
