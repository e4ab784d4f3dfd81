"""FP8 expert records written in the engine's weight format and read back
(homelab_b200.convert): every record part byte-identical to the device
quantizer's output for the same bf16 weights, padding zero, and a decode step
over the loaded records equal to one over records quantized in place."""
import json
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import homelab_b200 as hb  # noqa: E402
from homelab_b200.backend import Gpu  # noqa: E402
from homelab_b200.convert import convert_experts, load_expert_group  # noqa: E402
from homelab_b200.records import ExpertBank  # noqa: E402

if not torch.cuda.is_available():
    pytest.skip("needs a GPU", allow_module_level=True)

DEV = torch.device("cuda", 0)
H, I, E, K = 2048, 768, 8, 4


def test_convert_round_trip(tmp_path):
    gpu = Gpu(0)
    gen = torch.Generator(device=DEV)
    gen.manual_seed(5)
    mk = lambda *s: (torch.randn(s, generator=gen, device=DEV) * 0.02).to(torch.bfloat16)  # noqa: E731
    layers = [(mk(E, I, H), mk(E, I, H), mk(E, H, I)) for _ in range(2)]
    index = convert_experts(str(tmp_path), layers, H, I, hb.SCALE_128X128, device=DEV)
    assert [g["layout"] for g in index["expert_groups"]] == ["fp8-e4m3-b128x128"] * 2
    assert json.load(open(os.path.join(tmp_path, "index.json")))["expert_groups"][1]["offset"] == \
        E * index["expert_groups"][0]["stride"]
    for li, (gate, up, down) in enumerate(layers):
        buf, addrs, geo, stride = load_expert_group(str(tmp_path), li, DEV)
        bank = ExpertBank(E, H, I, hb.SCALE_128X128, DEV)
        assert bank.stride == stride
        for e in range(E):
            gq, gs, uq, us, dq, ds = bank.views(e)
            for (w, q, s, n, k) in ((gate[e], gq, gs, I, H), (up[e], uq, us, I, H), (down[e], dq, ds, H, I)):
                gpu.quantize_fp8(w.contiguous().view(torch.int16), n, k, hb.SCALE_128X128, q, s)
        torch.cuda.synchronize()
        assert torch.equal(buf, bank.buf), f"layer {li}: records differ from the device quantizer's bytes"
        # a decode step over the loaded records
        router = (torch.randn((E, H), generator=gen, device=DEV) * 0.02).to(torch.bfloat16)
        x = torch.randn((2, H), generator=gen, device=DEV).to(torch.bfloat16)
        outs = []
        for a in (addrs, bank.addrs):
            L = hb.MoeLayer(hidden=H, experts=E, top_k=K, router_w=router.data_ptr(), recs=a.data_ptr())
            L.geo = geo
            out = torch.empty((2, H), dtype=torch.float32, device=DEV)
            gpu.moe_decode(L, x, 2, out, gpu.moe_decode_workspace(L, 2))
            outs.append(out)
        torch.cuda.synchronize()
        assert torch.equal(outs[0], outs[1])


def test_loader_refuses_other_layouts(tmp_path):
    index = {"format": "oominf", "version": 0, "files": {}, "tensors": [],
             "expert_groups": [{"layer": 0, "num_experts": 1, "offset": 0, "stride": 4096,
                                "layout": "nvfp4-modelopt-g16", "parts": [], "xxh3": []}]}
    (tmp_path / "index.json").write_text(json.dumps(index))
    (tmp_path / "experts.bin").write_bytes(bytes(4096))
    with pytest.raises(ValueError):
        load_expert_group(str(tmp_path), 0, DEV)
