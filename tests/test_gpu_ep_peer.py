"""Expert parallelism over two GPUs with the all-to-alls done by the kernels
through peer memory (CUDA IPC mailboxes, NVLink stores and epoch flags).

Two spawned processes, one per GPU, shard a 64-expert layer; each runs several
steps of the chain of kernels (EpPeerMoeLayer) or of the one-launch step
(EpDecodeLayer, whose kernels on the two GPUs wait on each other) and compares
its tokens' outputs, bit for bit, with the single-GPU fused decode of the whole
batch on its own GPU (which holds the full layer too).  Skipped on a box with
fewer than two GPUs.
"""
import datetime
import os
import socket
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
    pytest.skip("needs two GPUs", allow_module_level=True)

import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
H, E, K, I = 2048, 64, 8, 768
STEPS = 4


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, t, result_dir, fused):
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    ok = False
    try:
        import oracle as O
        import homelab_b200 as hb
        from homelab_b200.backend import Gpu
        from homelab_b200.ep import EpDecodeLayer, EpGpuOps, EpPeerMailboxes, EpPeerMoeLayer
        from homelab_b200.records import ExpertBank
        gpu = Gpu(rank)
        bank = ExpertBank(E, H, I, hb.SCALE_128X128, dev)
        bank.fill_random(gpu, seed=91)  # the same full layer on every rank
        router = torch.from_numpy(O.normal_bf16(92, E * H, 0.0, 0.02).view(np.int16)).to(dev).view(torch.bfloat16)
        router = router.view(E, H)
        full = hb.MoeLayer(hidden=H, experts=E, top_k=K, router_w=router.data_ptr(), recs=bank.addrs.data_ptr())
        full.geo = bank.geo
        epr = E // world
        mb = EpPeerMailboxes(dist.group.WORLD, H, K, t, torch.bfloat16, dev)
        recs_local = bank.addrs[rank * epr:(rank + 1) * epr].contiguous()
        if fused:
            layer = EpDecodeLayer(mb, rank, H, E, K, router, recs_local, bank.geo, t)
        else:
            layer = EpPeerMoeLayer(EpGpuOps(dev), mb, rank, H, E, K, I, router, recs_local, bank.geo, t)
        ws = gpu.moe_decode_workspace(full, world * t)
        same = True
        for step in range(STEPS):
            xall = torch.from_numpy(O.normal_bf16(200 + step, world * t * H).view(np.int16)).to(dev)
            xall = xall.view(torch.bfloat16).view(world * t, H)
            out = torch.full((t, H), float("nan"), dtype=torch.float32, device=dev)
            layer.forward(xall[rank * t:(rank + 1) * t].contiguous(), t, out)
            want = torch.empty((world * t, H), dtype=torch.float32, device=dev)
            os.environ["OOMB_DECODE_CHAIN"] = "1"  # the CUDA-core expert kernels the ranks use
            try:
                gpu.moe_decode(full, xall, world * t, want, ws)
            finally:
                os.environ.pop("OOMB_DECODE_CHAIN", None)
            torch.cuda.synchronize()
            same &= bool(torch.equal(out, want[rank * t:(rank + 1) * t]))
        ok = same and gpu.device_error() == 0
        dist.barrier()
        mb.close()
    finally:
        with open(os.path.join(result_dir, f"rank{rank}.txt"), "w") as f:
            f.write("ok" if ok else "mismatch")
        try:
            dist.destroy_process_group()
        except Exception:
            pass


@pytest.mark.parametrize("fused", [False, True])
@pytest.mark.parametrize("t", [1, 3])
def test_two_gpu_peer_expert_parallel_equals_one_gpu(tmp_path, t, fused):
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), t, str(tmp_path), fused), nprocs=world, join=True)
    for r in range(world):
        assert open(os.path.join(tmp_path, f"rank{r}.txt")).read() == "ok", f"rank {r}"
