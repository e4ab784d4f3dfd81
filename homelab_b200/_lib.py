"""Loads liboomb.so (the sm_100a kernels behind include/oomb.h) and declares its C ABI.

The library is required: there is no CPU fallback.  Importing the package
without a built library raises, and every entry point fails with
OOMB_E_DEVICE when no sm_100 GPU is present.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboomb.so")

OK = 0
E_SHAPE = -1
E_ALIGN = -2
E_LAUNCH = -3
E_TIMEOUT = -4
E_ARG = -5
E_DEVICE = -6
E_WORKSPACE = -7

F32 = 0
BF16 = 1
SCALE_1X128 = 0
SCALE_128X128 = 1
TABLES_READY = 1
NOALLOC_SCRATCH_BYTES = 8 * 1024 * 1024
PART_ALIGN = 256
RECORD_ALIGN = 4096
Q_ROWS = 0
Q_TILES = 1


class Fp8Record(C.Structure):
    """oomb_fp8_record: byte offsets of the parts of an FP8 expert record."""

    _fields_ = [
        ("hidden", C.c_int64), ("inter", C.c_int64),
        ("gate_weight", C.c_int64), ("gate_scale", C.c_int64),
        ("up_weight", C.c_int64), ("up_scale", C.c_int64),
        ("down_weight", C.c_int64), ("down_scale", C.c_int64),
        ("layout", C.c_int32), ("pad_", C.c_int32),
    ]


class MoeLayer(C.Structure):
    """oomb_moe_layer: a resident MoE layer for the fused decode path."""

    _fields_ = [
        ("hidden", C.c_int32), ("experts", C.c_int32), ("top_k", C.c_int32), ("pad_", C.c_int32),
        ("router_w", C.c_void_p), ("recs", C.c_void_p),
        ("geo", Fp8Record),
    ]


class EpPeer(C.Structure):
    """oomb_ep_peer: a rank's view of the expert-parallel mailboxes."""

    _fields_ = [
        ("peers", C.c_void_p), ("mailbox", C.c_void_p),
        ("ranks", C.c_int32), ("rank", C.c_int32), ("t_max", C.c_int32),
        ("top_k", C.c_int32), ("hidden", C.c_int32), ("x_dtype", C.c_int32),
    ]


class SharedExpert(C.Structure):
    """oomb_shared_expert: a layer's shared expert(s) as one FP8 SwiGLU MLP plus a bf16 gate row."""

    _fields_ = [
        ("hidden", C.c_int32), ("inter", C.c_int32), ("scale_layout", C.c_int32), ("pad_", C.c_int32),
        ("gate_up_q", C.c_void_p), ("gate_up_scale", C.c_void_p),
        ("down_q", C.c_void_p), ("down_scale", C.c_void_p), ("gate_w", C.c_void_p),
    ]


IPC_HANDLE_BYTES = 64

# (name, restype, argtypes) of every entry point in include/oomb.h
P, I, Z, S = C.c_void_p, C.c_int, C.c_size_t, C.c_void_p
SIGNATURES = [
    ("oomb_version", C.c_char_p, []),
    ("oomb_status_string", C.c_char_p, [I]),
    ("oomb_device_error", I, [C.POINTER(C.c_int), I]),
    ("oomb_set_wait_limit", I, [C.c_uint64]),
    ("oomb_gemm_fp8", I, [P, I, P, P, I, P, I, I, I, I, P, Z, S]),
    ("oomb_gemm_fp8_workspace_bytes", Z, [I, I, I, I]),
    ("oomb_gemm_fp8_tc", I, [P, I, P, I, P, I, P, I, I, I, I, P, Z, S]),
    ("oomb_pack_fp8_tiles", I, [P, I, I, P, S]),
    ("oomb_silu_mul_rows", I, [P, P, I, I, I, S]),
    ("oomb_moe_experts_fp8", I, [P, P, P, P, I, P, I, P, P, C.POINTER(Fp8Record), I, S]),
    ("oomb_moe_experts_tiled_fp8_workspace_bytes", Z, [I, C.POINTER(Fp8Record), I]),
    ("oomb_moe_experts_tiled_fp8", I, [P, P, P, P, I, I, P, I, P, P, C.POINTER(Fp8Record), I, P, Z, S]),
    ("oomb_ep_meta", I, [P, I, I, I, I, P, S]),
    ("oomb_ep_group", I, [P, I, I, I, I, P, P, P, P, P, P, S]),
    ("oomb_ep_scatter", I, [P, P, P, P, I, I, P, S]),
    ("oomb_ep_combine", I, [P, P, P, I, I, I, I, I, P, I, S]),
    ("oomb_moe_decode_ep_workspace_bytes", Z, [I, I, C.POINTER(MoeLayer)]),
    ("oomb_moe_decode_ep_fp8", I, [C.POINTER(MoeLayer), C.POINTER(EpPeer), P, I, I, P, I, P, P, P, Z, S]),
    ("oomb_ep_mailbox_bytes", Z, [I, I, I, I, I]),
    ("oomb_ep_mailbox_x_offset", Z, [I, I, I, I, I]),
    ("oomb_ep_mailbox_alloc", I, [Z, C.POINTER(C.c_void_p)]),
    ("oomb_ep_mailbox_free", I, [P]),
    ("oomb_ipc_handle", I, [P, P]),
    ("oomb_ipc_open", I, [P, C.POINTER(C.c_void_p)]),
    ("oomb_ipc_close", I, [P]),
    ("oomb_ep_dispatch_peer", I, [C.POINTER(EpPeer), P, I, I, P, S]),
    ("oomb_ep_group_peer", I, [C.POINTER(EpPeer), I, I, P, P, P, P, P, P, S]),
    ("oomb_ep_return_peer", I, [C.POINTER(EpPeer), P, P, P, P, I, I, S]),
    ("oomb_ep_combine_peer", I, [C.POINTER(EpPeer), P, P, I, I, P, I, S]),
    ("oomb_copy_queue_create", I, [C.POINTER(C.c_void_p)]),
    ("oomb_copy_queue_destroy", I, [P]),
    ("oomb_pin_host", I, [P, Z]),
    ("oomb_unpin_host", I, [P]),
    ("oomb_copy_to_device", I, [P, P, P, Z]),
    ("oomb_copy_on_device", I, [P, P, P, Z]),
    ("oomb_record_compute", I, [S, C.POINTER(C.c_void_p)]),
    ("oomb_record_copies", I, [P, C.POINTER(C.c_void_p)]),
    ("oomb_copies_wait", I, [P, P]),
    ("oomb_compute_wait", I, [S, P]),
    ("oomb_event_done", I, [P]),
    ("oomb_event_wait", I, [P]),
    ("oomb_event_destroy", I, [P]),
    ("oomb_copies_sync", I, [P]),
    ("oomb_router_logits", I, [P, I, P, P, I, I, I, S]),
    ("oomb_router_topk", I, [P, P, P, I, I, I, S]),
    ("oomb_moe_gate_up_fp8", I, [P, P, P, I, P, I, P, C.POINTER(Fp8Record), I, I, S]),
    ("oomb_moe_down_fp8", I, [P, P, I, P, P, C.POINTER(Fp8Record), I, I, S]),
    ("oomb_moe_combine_slots", I, [P, P, P, P, I, I, I, I, S]),
    ("oomb_moe_combine", I, [P, P, P, P, I, I, S]),
    ("oomb_moe_tiled_fp8_workspace_bytes", Z, [I, I, I]),
    ("oomb_moe_tiled_fp8", I, [P, P, P, I, I, I, P, I, P, I, I, C.c_int64, C.c_int64, I, P, Z, S]),
    ("oomb_moe_swiglu_range", I, [P, P, P, C.c_int64, C.c_int64, S]),
    ("oomb_moe_decode_workspace_bytes", Z, [I, C.POINTER(MoeLayer)]),
    ("oomb_moe_decode_fp8", I, [C.POINTER(MoeLayer), P, I, I, P, I, P, P, P, Z, S]),
    ("oomb_workspace_clear", I, [P, Z, S]),
    ("oomb_moe_decode_fp8_noalloc", I, [C.POINTER(MoeLayer), P, I, I, P, I, P, P, S]),
    ("oomb_quantize_fp8", I, [P, I, I, I, P, P, S]),
    ("oomb_attention_decode_workspace_bytes", Z, [I, I, I, I, I]),
    ("oomb_kv_append", I, [P, I, C.c_int64, P, C.c_int64, P, I, I, I, I, I, I, S]),
    ("oomb_fp8_record_layout", I, [C.c_int64, C.c_int64, I, C.POINTER(Fp8Record), C.POINTER(C.c_size_t)]),
    ("oomb_quantize_fp8_record", I, [P, P, P, C.POINTER(Fp8Record), P, S]),
    ("oomb_policy_create", I, [C.c_char_p, C.POINTER(C.c_void_p)]),
    ("oomb_policy_destroy", I, [P]),
    ("oomb_policy_touch", I, [P, C.c_uint32, C.c_uint64]),
    ("oomb_policy_remove", I, [P, C.c_uint32]),
    ("oomb_policy_victim", C.c_int64, [P, P, I]),
    ("oomb_tier_create", I, [P, Z, I, I, P, I, C.c_char_p, C.POINTER(C.c_void_p)]),
    ("oomb_tier_destroy", I, [P]),
    ("oomb_tier_begin_fetch", I, [P, S, I, P, I, P, P]),
    ("oomb_tier_finish_fetch", I, [P, S]),
    ("oomb_tier_stats", I, [P, P]),
    ("oomb_moe_layer_workspace_bytes", Z, [I, C.POINTER(MoeLayer), C.POINTER(SharedExpert), I]),
    ("oomb_moe_layer_decode_fp8", I, [C.POINTER(MoeLayer), C.POINTER(SharedExpert), P, I, I, P, I, P, P, P, Z,
                                      S]),
    ("oomb_attention_decode", I, [P, I, P, P, C.c_int64, P, I, P, I, I, I, I, I, I, C.c_float, P, Z, S]),
]

_LIB = None


def lib() -> C.CDLL:
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m homelab_b200.build` "
                "(the FP8 path has no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        for name, res, args in SIGNATURES:
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _LIB = L
    return _LIB


class OombError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = status
        msg = lib().oomb_status_string(status).decode()
        super().__init__(f"{what}: {msg} (status {status})" if what else msg)


def check(status: int, what: str = "") -> None:
    if status != OK:
        raise OombError(status, what)
