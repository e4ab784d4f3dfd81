"""The reference's own CUDA kernels, launched on torch device buffers.

TEST INFRASTRUCTURE ONLY: the tests run these beside the sm_100a path to pin
the CPU oracle (and the product) to the reference's actual outputs.  The
kernels come from projects/oom-inference/crates/oominf-cuda/kernels/{ops,moe}.cu,
built into oracle/_ref by oracle/ref/Makefile; oracle/ref/launch.cpp launches
them with the reference host code's geometry.
"""
from __future__ import annotations

import ctypes as C
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
LIB_PATH = os.path.join(REF_DIR, "libref.so")


def available() -> bool:
    return all(os.path.exists(os.path.join(REF_DIR, f)) for f in ("libref.so", "ops.cubin", "moe.cubin"))


class RefKernels:
    """Handles to the reference kernels in the current CUDA context."""

    def __init__(self, device: torch.device):
        if not available():
            raise FileNotFoundError(f"{REF_DIR} holds no built reference kernels")
        self.device = device
        torch.cuda.init()
        torch.empty(1, device=device)  # make the primary context current on this thread
        L = C.CDLL(LIB_PATH)
        P, I, LL = C.c_void_p, C.c_int, C.c_longlong
        L.orl_open.argtypes = [C.c_char_p]
        L.orl_gemv_plan.argtypes = [I, I, I, C.POINTER(I), C.POINTER(I), C.POINTER(I)]
        L.orl_gemv_plan.restype = None
        L.orl_gemv_fp8.argtypes = [P, P, P, P, P, P, I, I, I, P]
        L.orl_router_topk.argtypes = [P, P, P, I, I, I, P]
        L.orl_moe_gate_up_bf16.argtypes = [P, P, P, I, P, P, I, I, LL, LL, P]
        L.orl_moe_down_bf16.argtypes = [P, P, I, P, P, I, I, LL, P]
        L.orl_moe_combine_slots.argtypes = [P, P, P, P, I, I, I, P]
        L.orl_dequant_fp8.argtypes = [P, P, P, I, I, P]
        L.orl_f32_to_bf16.argtypes = [P, P, I, P]
        L.orl_silu_mul_rows.argtypes = [P, P, I, I, P]
        rc = L.orl_open(REF_DIR.encode())
        if rc != 0:
            raise RuntimeError(f"loading the reference kernels failed ({rc})")
        self.L = L

    def _s(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    @staticmethod
    def _check(rc: int, what: str) -> None:
        if rc != 0:
            raise RuntimeError(f"reference {what} failed ({rc})")

    def gemv_plan(self, t: int, n: int, k: int):
        s, kl, tl = C.c_int(), C.c_int(), C.c_int()
        self.L.orl_gemv_plan(t, n, k, C.byref(s), C.byref(kl), C.byref(tl))
        return s.value, kl.value, tl.value

    def gemv_fp8(self, x: torch.Tensor, q: torch.Tensor, scale: torch.Tensor, t: int, n: int, k: int):
        """y = x . dequant(q)^T, x fp32 [t, k], q e4m3 [n, k], scale fp32 [n, ceil(k/128)]."""
        splits, _, tiles = self.gemv_plan(t, n, k)
        y = torch.empty((t, n), dtype=torch.float32, device=self.device)
        partial = torch.empty(max(splits * t * n, 1), dtype=torch.float32, device=self.device)
        tickets = torch.zeros(max(tiles, 1), dtype=torch.int32, device=self.device)
        self._check(self.L.orl_gemv_fp8(x.data_ptr(), q.data_ptr(), scale.data_ptr(), y.data_ptr(),
                                        partial.data_ptr(), tickets.data_ptr(), t, n, k, self._s()), "gemv_fp8")
        return y

    def router_topk(self, logits: torch.Tensor, t: int, e: int, k: int):
        ids = torch.empty((t, k), dtype=torch.int32, device=self.device)
        w = torch.empty((t, k), dtype=torch.float32, device=self.device)
        self._check(self.L.orl_router_topk(logits.data_ptr(), ids.data_ptr(), w.data_ptr(), t, e, k, self._s()),
                    "router_topk")
        return ids, w

    def moe_gate_up_bf16(self, recs, off, assign_tok, n_experts, x, h, hidden, inter, gw_off, uw_off):
        self._check(self.L.orl_moe_gate_up_bf16(recs.data_ptr(), off.data_ptr(), assign_tok.data_ptr(), n_experts,
                                                x.data_ptr(), h.data_ptr(), hidden, inter, gw_off, uw_off,
                                                self._s()), "moe_gate_up_bf16")

    def moe_down_bf16(self, recs, off, n_experts, h, y, hidden, inter, dw_off):
        self._check(self.L.orl_moe_down_bf16(recs.data_ptr(), off.data_ptr(), n_experts, h.data_ptr(), y.data_ptr(),
                                             hidden, inter, dw_off, self._s()), "moe_down_bf16")

    def moe_combine_slots(self, y, slot_assign, w, out, t, hidden, k):
        self._check(self.L.orl_moe_combine_slots(y.data_ptr(), slot_assign.data_ptr(), w.data_ptr(), out.data_ptr(),
                                                 t, hidden, k, self._s()), "moe_combine_slots")

    def dequant_fp8(self, q: torch.Tensor, scale: torch.Tensor, w: torch.Tensor, n: int, k: int):
        """w[n, k] bf16 = e4m3 q * scale (1x128 blocks), the reference's fp8_dequantize_blocks."""
        self._check(self.L.orl_dequant_fp8(q.data_ptr(), scale.data_ptr(), w.data_ptr(), n, k, self._s()), "dequant")

    def f32_to_bf16(self, x: torch.Tensor, y: torch.Tensor, n: int):
        self._check(self.L.orl_f32_to_bf16(x.data_ptr(), y.data_ptr(), n, self._s()), "f32_to_bf16")

    def silu_mul_rows(self, gu: torch.Tensor, y: torch.Tensor, rows: int, n: int):
        self._check(self.L.orl_silu_mul_rows(gu.data_ptr(), y.data_ptr(), rows, n, self._s()), "silu_mul_rows")
