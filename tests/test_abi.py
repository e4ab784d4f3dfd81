"""The C-ABI library without a GPU: it loads, exports every symbol include/oomb.h
declares, and its host-side checks reject bad arguments before any launch (the
`ensure!` checks of Gpu::check, crates/oominf-cuda/src/lib.rs:157-160)."""
import ctypes as C
import os
import re

import pytest

import homelab_b200 as hb
from homelab_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            src = open(os.path.join(ROOT, "include", fn)).read()
            names |= set(re.findall(r"\b(oomb_[a-z0-9_]+)\s*\(", src))
    return names


def test_library_exports_every_declared_symbol():
    L = hb.lib()
    names = declared_symbols()
    assert len(names) >= 14
    for n in sorted(names):
        assert hasattr(L, n), n


def test_python_signatures_cover_header():
    assert {n for n, _, _ in _lib.SIGNATURES} == declared_symbols()


def test_no_oracle_dependency():
    # The product never links, loads or imports the CPU oracle.
    import subprocess
    out = subprocess.run(["ldd", _lib.LIB_PATH], capture_output=True, text=True).stdout
    assert "oracle" not in out and "cpubase" not in out
    pkg = os.path.join(ROOT, "homelab_b200")
    for f in os.listdir(pkg):
        if f.endswith(".py"):
            src = open(os.path.join(pkg, f)).read()
            assert not re.search(r"^\s*(import|from)\s+oracle", src, re.M), f
            assert "liboomb_oracle" not in src and "liboomb_cpubase" not in src, f


def test_status_strings():
    L = hb.lib()
    assert L.oomb_status_string(0) == b"ok"
    assert b"shape" in L.oomb_status_string(_lib.E_SHAPE)
    assert L.oomb_version().startswith(b"oomb")


def test_checks_run_before_launch():
    L = hb.lib()
    fake = 0x10000  # never dereferenced: every call below fails its checks first
    # k not a multiple of 16
    assert L.oomb_gemm_fp8(fake, 0, fake, fake, 1, fake, 0, 1, 64, 17, None, 0, None) == _lib.E_SHAPE
    # null inputs
    assert L.oomb_gemm_fp8(0, 0, fake, fake, 1, fake, 0, 1, 64, 32, None, 0, None) == _lib.E_ARG
    # bad dtype / layout enums
    assert L.oomb_gemm_fp8(fake, 7, fake, fake, 1, fake, 0, 1, 64, 32, None, 0, None) == _lib.E_ARG
    assert L.oomb_gemm_fp8(fake, 0, fake, fake, 9, fake, 0, 1, 64, 32, None, 0, None) == _lib.E_ARG
    # misaligned pointer
    assert L.oomb_gemm_fp8(fake + 4, 0, fake, fake, 1, fake, 0, 1, 64, 32, None, 0, None) == _lib.E_ALIGN
    # top-k limits of experts.rs:19 (k <= 32, e <= 8192), and k <= e
    assert L.oomb_router_topk(fake, fake, fake, 1, 8193, 8, None) == _lib.E_SHAPE
    assert L.oomb_router_topk(fake, fake, fake, 1, 64, 33, None) == _lib.E_SHAPE
    assert L.oomb_router_topk(fake, fake, fake, 1, 4, 8, None) == _lib.E_SHAPE
    # expert widths must be multiples of 16 (experts.rs:55-58), hidden <= 4096
    g = hb.Fp8Record(hidden=2048, inter=770, layout=1)
    assert L.oomb_moe_gate_up_fp8(fake, fake, fake, 1, fake, 0, fake, C.byref(g), 0, 0, None) == _lib.E_SHAPE
    g = hb.Fp8Record(hidden=8192, inter=768, layout=1)
    assert L.oomb_moe_gate_up_fp8(fake, fake, fake, 1, fake, 0, fake, C.byref(g), 0, 0, None) == _lib.E_SHAPE
    g = hb.Fp8Record(hidden=2048, inter=768, layout=1)
    assert L.oomb_moe_down_fp8(fake, fake, 1, fake, fake, C.byref(g), 0, 4, None) == _lib.E_ARG  # unknown flag
    g = hb.Fp8Record(hidden=2048, inter=768, layout=1, down_weight=8)
    assert L.oomb_moe_down_fp8(fake, fake, 1, fake, fake, C.byref(g), 0, 0, None) == _lib.E_ALIGN


def test_decode_workspace_size_and_checks():
    L = hb.lib()
    layer = hb.MoeLayer(hidden=2048, experts=128, top_k=8, router_w=0x10000, recs=0x10000)
    from homelab_b200.records import record_layout
    layer.geo, _ = record_layout(2048, 768)
    n1 = L.oomb_moe_decode_workspace_bytes(1, C.byref(layer))
    n16 = L.oomb_moe_decode_workspace_bytes(16, C.byref(layer))
    assert n1 > 0 and n16 > n1
    # A = t * k assignments of h [A, inter] and y [A, hidden] fp32 dominate
    assert n16 >= 16 * 8 * (768 + 2048) * 4
    bad = hb.MoeLayer(hidden=2048, experts=128, top_k=200, router_w=0x10000, recs=0x10000)
    bad.geo = layer.geo
    assert L.oomb_moe_decode_workspace_bytes(1, C.byref(bad)) == 0
    ws = 0x10000
    assert L.oomb_moe_decode_fp8(C.byref(layer), 0x10000, 1, 1, 0x10000, 1, None, None, ws, 16, None) == _lib.E_WORKSPACE


def test_no_gpu_fails_loudly():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    L = hb.lib()
    fake = 0x10000
    assert L.oomb_gemm_fp8(fake, 0, fake, fake, 1, fake, 0, 1, 64, 32, None, 0, None) == _lib.E_DEVICE


def test_expert_parallel_peer_entry_points_check_arguments():
    L = hb.lib()
    fake = 0x10000  # never dereferenced: every call below fails its checks first
    assert L.oomb_ep_mailbox_bytes(2, 1, 8, 2048, _lib.BF16) > 0
    assert L.oomb_ep_mailbox_bytes(0, 1, 8, 2048, _lib.BF16) == 0
    assert L.oomb_ep_mailbox_bytes(2, 1, 8, 2048, 9) == 0  # unknown activation type
    assert L.oomb_ep_mailbox_x_offset(2, 1, 8, 2048, _lib.BF16) % 256 == 0
    # the x region grows with the ranks, and the later regions after it
    assert L.oomb_ep_mailbox_bytes(4, 2, 8, 2048, _lib.BF16) > L.oomb_ep_mailbox_bytes(2, 2, 8, 2048, _lib.BF16)
    q = _lib.EpPeer(fake, fake, 2, 0, 4, 8, 2048, _lib.BF16)
    assert L.oomb_ep_dispatch_peer(None, fake, 1, 32, fake, None) == _lib.E_ARG
    assert L.oomb_ep_dispatch_peer(C.byref(q), fake, 5, 32, fake, None) == _lib.E_SHAPE  # t > t_max
    assert L.oomb_ep_dispatch_peer(C.byref(q), fake, 1, 32, fake + 4, None) == _lib.E_ALIGN
    bad = _lib.EpPeer(fake, fake, 2, 2, 4, 8, 2048, _lib.BF16)  # rank out of range
    assert L.oomb_ep_dispatch_peer(C.byref(bad), fake, 1, 32, fake, None) == _lib.E_ARG
    assert L.oomb_ep_group_peer(C.byref(q), 0, 32, fake, fake, fake, fake, fake, fake, None) == _lib.E_SHAPE
    assert L.oomb_ep_return_peer(C.byref(q), fake, fake, fake, fake, 1, 0, None) == _lib.E_SHAPE
    assert L.oomb_ep_combine_peer(C.byref(q), fake, fake, 1, 32, fake, 7, None) == _lib.E_ARG  # out dtype
    layer = hb.MoeLayer(hidden=2048, experts=64, top_k=8, router_w=fake, recs=fake)
    layer.geo = hb.Fp8Record(hidden=2048, inter=768, layout=1, gate_weight=0, up_weight=768 * 2048,
                             down_weight=2 * 768 * 2048, gate_scale=3 * 768 * 2048, up_scale=3 * 768 * 2048 + 512,
                             down_scale=3 * 768 * 2048 + 1024)
    assert L.oomb_moe_decode_ep_workspace_bytes(1, 2, C.byref(layer)) > L.oomb_moe_decode_workspace_bytes(1, C.byref(layer))
    # activation dtype must match the mailboxes'; hidden must match the layer's
    assert L.oomb_moe_decode_ep_fp8(C.byref(layer), C.byref(q), fake, _lib.F32, 1, fake, 0, None, None, fake, 1 << 30,
                                    None) == _lib.E_ARG
    q2 = _lib.EpPeer(fake, fake, 2, 0, 4, 8, 1024, _lib.BF16)
    assert L.oomb_moe_decode_ep_fp8(C.byref(layer), C.byref(q2), fake, _lib.BF16, 1, fake, 0, None, None, fake,
                                    1 << 30, None) == _lib.E_SHAPE


def test_integration_rust_block_names_every_entry_point():
    """The Rust FFI block a maintainer adds declares every entry
    point of include/oomb.h, and nothing else."""
    doc = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    blocks = re.findall(r"```rust\n(.*?)```", doc, re.S)
    ffi = next(b for b in blocks if 'extern "C"' in b and "#[link" in b)
    rust = set(re.findall(r"pub fn (oomb_[a-z0-9_]+)\s*\(", ffi))
    assert rust == declared_symbols(), sorted(rust ^ declared_symbols())


def test_new_entry_points_check_arguments():
    L = hb.lib()
    fake = 0x10000
    # attention: head_dim 128 only, G in {1, 2, 4, 8}, uniform length within kv_max
    assert L.oomb_attention_decode(fake, 0, fake, fake, 0, None, 5, fake, 0, 1, 32, 8, 128, 4, 1.0, fake, 1 << 20,
                                   None) == _lib.E_SHAPE
    assert L.oomb_attention_decode(fake, 3, fake, fake, 0, None, 1, fake, 0, 1, 32, 8, 128, 4, 1.0, fake, 1 << 20,
                                   None) == _lib.E_ARG
    assert L.oomb_attention_decode(fake + 4, 0, fake, fake, 0, None, 1, fake, 0, 1, 32, 8, 128, 4, 1.0, fake,
                                   1 << 20, None) == _lib.E_ALIGN
    # kv append: positions past the cache, odd strides
    assert L.oomb_kv_append(fake, 0, 1024, fake, 0, None, 4, 1, 1, 8, 128, 4, None) == _lib.E_SHAPE
    assert L.oomb_kv_append(fake, 0, 1028, fake, 0, None, 0, 1, 1, 8, 128, 4, None) == _lib.E_ALIGN
    # grouped tensor-core GEMM: a workspace is required
    assert L.oomb_moe_tiled_fp8(fake, fake, None, 1, 0, 4, fake, 1, fake, 768, 2048, 0, 0, 1, None, 0,
                                None) == _lib.E_ARG
    assert L.oomb_moe_tiled_fp8_workspace_bytes(4, 2048, _lib.BF16) >= 4 * 2 * 2048
    assert L.oomb_moe_tiled_fp8_workspace_bytes(4, 2048, _lib.F32) >= 4 * 6 * 2048
    # the MoE layer entry: a shared expert of another width is refused
    layer = hb.MoeLayer(hidden=2048, experts=64, top_k=8, router_w=fake, recs=fake)
    from homelab_b200.records import record_layout
    layer.geo, _ = record_layout(2048, 768)
    sh = hb.SharedExpert(hidden=1024, inter=1536, scale_layout=1, gate_up_q=fake, gate_up_scale=fake, down_q=fake,
                         down_scale=fake, gate_w=fake)
    assert L.oomb_moe_layer_workspace_bytes(1, C.byref(layer), C.byref(sh), _lib.BF16) == 0
    assert L.oomb_moe_layer_decode_fp8(C.byref(layer), C.byref(sh), fake, 1, 1, fake, 1, None, None, fake, 1 << 30,
                                       None) == _lib.E_SHAPE


def test_tensor_core_expert_entry_checks_arguments():
    L = hb.lib()
    fake = 0x10000
    from homelab_b200.records import record_layout
    geo, _ = record_layout(2048, 768)
    assert L.oomb_moe_experts_tiled_fp8_workspace_bytes(64, C.byref(geo), _lib.BF16) > 0
    narrow, _ = record_layout(1024, 768)  # hidden < 2 * intermediate: g and u do not fit in y
    assert L.oomb_moe_experts_tiled_fp8_workspace_bytes(64, C.byref(narrow), _lib.BF16) == 0
    odd, _ = record_layout(2048, 720)  # intermediate not a multiple of 128
    assert L.oomb_moe_experts_tiled_fp8_workspace_bytes(64, C.byref(odd), _lib.BF16) == 0
    # a workspace is required, and must be large enough
    assert L.oomb_moe_experts_tiled_fp8(fake, fake, fake, fake, 8, 64, fake, _lib.BF16, fake, fake, C.byref(geo), 8,
                                        None, 0, None) == _lib.E_ARG
    assert L.oomb_moe_experts_tiled_fp8(fake, fake, fake, fake, 8, 64, fake, _lib.BF16, fake, fake, C.byref(geo), 8,
                                        fake, 16, None) == _lib.E_WORKSPACE
    assert L.oomb_moe_experts_tiled_fp8(fake, fake, fake, fake, 8, 64, fake, _lib.BF16, fake, fake, C.byref(narrow),
                                        8, fake, 1 << 30, None) == _lib.E_SHAPE
