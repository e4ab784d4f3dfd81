"""Offload staging (Transfer) on the GPU.

Cold expert records staged from pinned host memory into device slots on a copy
queue give the same expert outputs, bit for bit, as the same records resident
on the device; the events order copies after the compute that last read a slot
and compute after the copies it reads.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import oracle as O  # noqa: E402
import homelab_b200 as hb  # noqa: E402
from homelab_b200.backend import Gpu  # noqa: E402
from homelab_b200.records import ExpertBank  # noqa: E402
from homelab_b200.stage import HostArena, Transfer, stage_records  # noqa: E402

if not torch.cuda.is_available():
    pytest.skip("needs a GPU", allow_module_level=True)

DEV = torch.device("cuda", 0)
H, I = 2048, 768


@pytest.fixture(scope="module")
def gpu():
    g = Gpu(0)
    yield g
    torch.cuda.synchronize()
    assert g.device_error() == 0


def run_experts(gpu, addrs, geo, x, t):
    n = len(addrs)
    recs = torch.tensor(addrs, dtype=torch.int64, device=DEV)
    off = torch.arange(0, n + 1, dtype=torch.int32, device=DEV) * t
    tok = torch.arange(t, dtype=torch.int32, device=DEV).repeat(n)
    h = torch.empty((n * t, I), dtype=torch.float32, device=DEV)
    y = torch.empty((n * t, H), dtype=torch.float32, device=DEV)
    gpu.moe_gate_up(recs, off, tok, n, x, h, geo)
    gpu.moe_down(recs, off, n, h, y, geo)
    return y


def test_staged_records_compute_like_resident_ones(gpu):
    bank = ExpertBank(6, H, I, hb.SCALE_128X128, DEV)
    bank.fill_random(gpu, seed=51)
    torch.cuda.synchronize()
    arena = HostArena(6, bank.stride)
    arena.buf.copy_(bank.buf.cpu())
    slots = torch.zeros(3 * bank.stride, dtype=torch.uint8, device=DEV)
    slot_addrs = [slots.data_ptr() + j * bank.stride for j in range(3)]
    tr = Transfer(0)
    t = 2
    x = torch.from_numpy(O.normal_bf16(52, t * H).view(np.int16)).to(DEV).view(torch.bfloat16).view(t, H)
    which = [4, 1, 5]
    ready = stage_records(tr, arena, which, slot_addrs)
    tr.compute_wait(ready)
    y_staged = run_experts(gpu, slot_addrs, bank.geo, x, t)
    y_resident = run_experts(gpu, [int(bank.addrs[i]) for i in which], bank.geo, x, t)
    torch.cuda.synchronize()
    assert torch.equal(y_staged, y_resident)
    # restage other records into the same slots once the compute that read them is done
    done_reading = tr.record_compute()
    ready2 = stage_records(tr, arena, [0, 2, 3], slot_addrs, after=done_reading)
    tr.compute_wait(ready2)
    y2 = run_experts(gpu, slot_addrs, bank.geo, x, t)
    y2_resident = run_experts(gpu, [int(bank.addrs[i]) for i in (0, 2, 3)], bank.geo, x, t)
    torch.cuda.synchronize()
    assert torch.equal(y2, y2_resident)
    assert tr.event_done(ready2)
    tr.close()


def test_copies_wait_for_compute_and_compute_for_copies(gpu):
    tr = Transfer(0)
    n = 1 << 22
    a = torch.zeros(n, dtype=torch.float32, device=DEV)
    b = torch.empty_like(a)
    # compute writes a (after a long fill), the copy queue copies a -> b only after it
    big = torch.empty(1 << 26, dtype=torch.float32, device=DEV)
    big.fill_(1.0)
    a.fill_(3.0)
    ev = tr.record_compute()
    tr.copies_wait(ev)
    tr.copy_on_device(b.data_ptr(), a.data_ptr(), n * 4)
    done = tr.record_copies()
    tr.compute_wait(done)
    c = b * 2.0  # compute after the copy
    tr.event_wait(done)
    torch.cuda.synchronize()
    assert bool((b == 3.0).all()) and bool((c == 6.0).all())
    tr.copies_sync()
    tr.close()


def test_pin_host_registers_and_copies(gpu):
    tr = Transfer(0)
    host = np.arange(1 << 20, dtype=np.uint8)
    ptr = host.ctypes.data
    tr.pin_host(ptr, host.nbytes)
    dst = torch.empty(host.nbytes, dtype=torch.uint8, device=DEV)
    tr.copy_to_device(dst.data_ptr(), ptr, host.nbytes)
    tr.copies_sync()
    assert np.array_equal(dst.cpu().numpy(), host)
    tr.unpin_host(ptr)
    tr.close()
