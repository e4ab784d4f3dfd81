"""Expert-parallel orchestration on CPU ranks (gloo), with the oracle as the device.

homelab_b200.ep.EpMoeLayer drives the step; here its device ops are the CPU
oracle (test infrastructure) and its exchanges gloo all-to-alls between two
spawned processes.  Checked:
  - two ranks give, bit for bit, the single-rank result of the whole batch
    (the exchange layout, grouping order and slot-order combine are right);
  - a rank that fails before the exchange makes the other rank's step end
    with an error within the process group's timeout instead of hanging.
"""
import datetime
import os
import socket
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

H, E, K, I = 256, 8, 4, 128


class CpuOps:
    """The EpMoeLayer device steps restated on the CPU with the oracle."""

    def __init__(self, records, geo):
        self.records, self.geo = records, geo

    def route(self, x, router_w, logits, ids, weights, t, e, k, hidden):
        import oracle as O
        lg = O.router_logits(x[:t].float().numpy(), router_w.view(torch.int16).numpy().view(np.uint16))
        i, w = O.router_topk(lg, k)
        ids.view(-1)[: t * k] = torch.from_numpy(i.reshape(-1))
        weights.view(-1)[: t * k] = torch.from_numpy(w.reshape(-1))

    def meta(self, ids, t, k, epr, ranks, meta):
        idv = ids.view(-1)[: t * k].numpy().reshape(1, t, k)
        g = np.arange(ranks).reshape(ranks, 1, 1)
        m = np.where(idv // epr == g, idv % epr, -1).astype(np.int32)
        meta.view(-1)[: ranks * t * k] = torch.from_numpy(m.reshape(-1))

    def group(self, recv_meta, ranks, t, k, epr, recs_local, n_active, off, assign_row, assign_ret, recs_active):
        rm = recv_meta.reshape(-1).numpy()
        rows, rets, offs, active = [], [], [0], []
        for e in range(epr):
            hit = np.nonzero(rm == e)[0]  # (g, t, s) order: flat index order
            if len(hit) == 0:
                continue
            active.append(int(recs_local[e]))
            for i in hit:
                g, ts = divmod(int(i), t * k)
                rows.append(g * t + ts // k)
                rets.append(int(i))
            offs.append(len(rows))
        n_active[0] = len(active)
        off[: len(offs)] = torch.tensor(offs, dtype=torch.int32)
        assign_row[: len(rows)] = torch.tensor(rows, dtype=torch.int32)
        assign_ret[: len(rets)] = torch.tensor(rets, dtype=torch.int32)
        recs_active[: len(active)] = torch.tensor(active, dtype=torch.int64)

    def experts(self, recs_active, off, assign_row, n_active, max_active, x, h, y, geo, max_per_expert):
        import oracle as O
        n = int(n_active[0])
        if n == 0:
            return
        offs = off[: n + 1].numpy().copy()
        A = int(offs[-1])
        recs = [self.records[int(r)] for r in recs_active[:n]]
        y64 = O.moe_experts_f64(recs, self.geo, offs, assign_row[:A].numpy().copy(), x.float().numpy())
        y[:A] = torch.from_numpy(y64.astype(np.float32))

    def scatter(self, y, n_active, off, assign_ret, hidden, max_rows, ret):
        n = int(n_active[0])
        A = int(off[n]) if n else 0
        flat = ret.view(-1, hidden)
        flat[assign_ret[:A].long()] = y[:A]

    def combine(self, back, ids, weights, t, k, hidden, epr, ranks, out):
        import oracle as O
        idv = ids.view(-1)[: t * k].numpy().reshape(t, k)
        slot = ((idv // epr) * (t * k) + np.arange(t).reshape(t, 1) * k + np.arange(k).reshape(1, k)).astype(np.int32)
        res = O.combine_slots(back.reshape(-1, hidden).numpy(), slot, weights.view(-1)[: t * k].numpy().reshape(t, k),
                              t, hidden, k)
        out[:t] = torch.from_numpy(res)


def make_layer():
    """The synthetic layer (deterministic): records, geometry, router, activations."""
    sys.path.insert(0, ROOT)
    import oracle as O
    geo = O.Fp8Record()
    geo.hidden, geo.inter, geo.layout = H, I, O.SCALE_128X128
    geo.gate_weight, geo.up_weight, geo.down_weight = 0, I * H, 2 * I * H
    sc = [O.scale_count(I, H, 1), O.scale_count(I, H, 1), O.scale_count(H, I, 1)]
    geo.gate_scale = 3 * I * H
    geo.up_scale = geo.gate_scale + 4 * sc[0]
    geo.down_scale = geo.up_scale + 4 * sc[1]
    size = geo.down_scale + 4 * sc[2]
    records = []
    for e in range(E):
        r = np.zeros(size, dtype=np.uint8)
        for j, (n, k, wo, so) in enumerate(((I, H, geo.gate_weight, geo.gate_scale), (I, H, geo.up_weight, geo.up_scale),
                                            (H, I, geo.down_weight, geo.down_scale))):
            w = O.normal_bf16(100 + 3 * e + j, n * k, 0.0, 0.02)
            q, s = O.quantize_blocks(w, n, k, O.SCALE_128X128)
            r[wo:wo + n * k] = q.reshape(-1)
            r[so:so + s.size * 4] = s.view(np.uint8)
        records.append(r)
    router = torch.from_numpy(O.normal_bf16(200, E * H, 0.0, 0.02).view(np.int16)).view(torch.bfloat16).view(E, H)
    return records, geo, router


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def single_rank_result(x, records, geo, router, T):
    from homelab_b200.ep import EpMoeLayer, exchange_local
    ops = CpuOps(records, geo)
    layer = EpMoeLayer(ops, None, H, E, K, I, router, torch.arange(E, dtype=torch.int64), geo, T, ranks=1, rank=0)
    out = torch.empty((T, H), dtype=torch.float32)
    ex = layer.phase_route(x, T)
    for send, recv in ex:
        exchange_local([send], [recv])
    ret, back = layer.phase_experts(T)
    exchange_local([ret], [back])
    layer.phase_combine(T, out)
    return out


def _worker(rank, world, port, t, result_dir, fail_rank):
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        import oracle as O
        from homelab_b200.ep import EpMoeLayer
        records, geo, router = make_layer()
        epr = E // world
        ops = CpuOps(records, geo)
        layer = EpMoeLayer(ops, dist.group.WORLD, H, E, K, I, router,
                           torch.arange(rank * epr, (rank + 1) * epr, dtype=torch.int64), geo, t)
        x = torch.from_numpy(O.normal_bf16(300, world * t * H).view(np.int16)).view(torch.bfloat16).view(world * t, H)
        out = torch.empty((t, H), dtype=torch.float32)
        if rank == fail_rank:
            raise SystemExit(3)  # this rank dies before its first exchange
        try:
            layer.forward(x[rank * t:(rank + 1) * t], t, out)
            np.save(os.path.join(result_dir, f"out{rank}.npy"), out.numpy())
        except Exception as exc:  # the peer vanished: the collective must fail, not hang
            with open(os.path.join(result_dir, f"err{rank}.txt"), "w") as f:
                f.write(type(exc).__name__)
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_two_cpu_ranks_equal_one(tmp_path):
    sys.path.insert(0, ROOT)
    import oracle as O
    world, t = 2, 2
    mp.spawn(_worker, args=(world, free_port(), t, str(tmp_path), -1), nprocs=world, join=True)
    records, geo, router = make_layer()
    x = torch.from_numpy(O.normal_bf16(300, world * t * H).view(np.int16)).view(torch.bfloat16).view(world * t, H)
    want = single_rank_result(x, records, geo, router, world * t).numpy()
    for r in range(world):
        got = np.load(os.path.join(tmp_path, f"out{r}.npy"))
        assert np.array_equal(got.view(np.uint32), want[r * t:(r + 1) * t].view(np.uint32)), f"rank {r}"


def test_a_failed_rank_ends_the_peers_step_with_an_error(tmp_path):
    ctx = mp.get_context("spawn")
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, 1, str(tmp_path), 1)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung after its peer died"
    assert procs[1].exitcode == 3
    assert os.path.exists(os.path.join(tmp_path, "err0.txt")), "rank 0's exchange did not report the failure"
