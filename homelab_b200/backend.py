"""The B200 backend's Linear / Experts methods, named and shaped as the engine's traits.

Mirrors crates/oominf-core/src/backend.rs (projects/oom-inference): each method
takes device buffers (torch CUDA tensors here, plain device addresses at the C
ABI) and the same dimensions, and raises where the Rust method returns an
`Err` (shape or alignment checks before launch, `Gpu::check`,
crates/oominf-cuda/src/lib.rs:157-160).  All work is stream-ordered on the
current torch stream; nothing synchronises the host.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from ._lib import BF16, F32, SCALE_128X128, SCALE_1X128, Fp8Record, MoeLayer, check

__all__ = ["Gpu", "Fp8Record", "MoeLayer", "SCALE_1X128", "SCALE_128X128", "F32", "BF16"]


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return F32
    if t.dtype == torch.bfloat16:
        return BF16
    raise TypeError(f"activations must be float32 or bfloat16, got {t.dtype}")


def _dtype_code_of(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return F32
    if dt == torch.bfloat16:
        return BF16
    raise TypeError(f"activations must be float32 or bfloat16, got {dt}")


def _ptr(t) -> int:
    if t is None:
        return 0
    if isinstance(t, int):
        return t
    if not t.is_cuda:
        raise ValueError("buffers must live on the GPU")
    return t.data_ptr()


def _ptr_or_host(t) -> int:
    """A device tensor's address, or a host tensor's (the library takes pinned
    host memory where its entry points say so and refuses pageable memory)."""
    if t is None:
        return 0
    if isinstance(t, int):
        return t
    return t.data_ptr()


class Gpu:
    """One device's backend (the counterpart of `oominf_cuda::Gpu`)."""

    def __init__(self, device: int = 0):
        self.device = torch.device("cuda", device)
        self.L = _lib.lib()
        self._tiled_ws = None  # grown on demand by moe_tiled calls without a workspace

    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    # ---- Linear -------------------------------------------------------------------------
    def gemm_fp8(self, x, q, scale, y, t: int, n: int, k: int, layout: int = SCALE_128X128, workspace=None):
        """y[t, n] = x[t, k] @ w[n, k]^T for FP8 w (Linear::gemm_fp8, backend.rs:199-209).
        With a workspace (gemm_fp8_workspace), batches of 2+ tokens run on the tensor cores."""
        check(self.L.oomb_gemm_fp8(_ptr(x), _dtype_code(x), _ptr(q), _ptr(scale), layout, _ptr(y),
                                   _dtype_code(y), t, n, k, _ptr(workspace) if workspace is not None else None,
                                   workspace.numel() if workspace is not None else 0, self._stream()), "gemm_fp8")

    def silu_mul_rows(self, gu, y, rows: int, n: int):
        """y[r, i] = silu(gu[r, i]) * gu[r, n + i] (silu_mul_rows, ops.cu:302-309)."""
        check(self.L.oomb_silu_mul_rows(_ptr(gu), _ptr(y), _dtype_code(y), rows, n, self._stream()),
              "silu_mul_rows")

    def gemm_fp8_workspace(self, t: int, n: int, k: int, x_dtype=torch.bfloat16) -> torch.Tensor:
        """A zeroed workspace for gemm_fp8_tc (split-K partial sums and counters)."""
        n_bytes = int(self.L.oomb_gemm_fp8_workspace_bytes(t, n, k, BF16 if x_dtype == torch.bfloat16 else F32))
        if n_bytes == 0:
            raise ValueError("shape not supported by the tensor-core path")
        ws = torch.empty(n_bytes, dtype=torch.uint8, device=self.device)
        check(self.L.oomb_workspace_clear(_ptr(ws), n_bytes, self._stream()), "workspace_clear")
        return ws

    def gemm_fp8_tc(self, x, q, scale, y, t: int, n: int, k: int, layout: int, workspace, tiles: bool = False):
        """y = x . w^T on the tensor cores (tcgen05); n % 128 == k % 128 == 0, t <= 64.
        tiles: q is in the packed tile layout of pack_fp8_tiles."""
        check(self.L.oomb_gemm_fp8_tc(_ptr(x), _dtype_code(x), _ptr(q), _lib.Q_TILES if tiles else _lib.Q_ROWS,
                                      _ptr(scale), layout, _ptr(y), _dtype_code(y), t, n, k, _ptr(workspace),
                                      workspace.numel(), self._stream()), "gemm_fp8_tc")

    def pack_fp8_tiles(self, q, n: int, k: int, tiles=None):
        """The packed 128 x 128 tile layout of a row-major e4m3 matrix (load time)."""
        if tiles is None:
            tiles = torch.empty(n * k, dtype=torch.uint8, device=self.device)
        check(self.L.oomb_pack_fp8_tiles(_ptr(q), n, k, _ptr(tiles), self._stream()), "pack_fp8_tiles")
        return tiles

    def router_logits(self, x, w_bf16, logits, t: int, e: int, hidden: int):
        """logits = x . W^T for the bf16 router (moe.rs:289-298), canonical order."""
        check(self.L.oomb_router_logits(_ptr(x), _dtype_code(x), _ptr(w_bf16), _ptr(logits), t, e,
                                        hidden, self._stream()), "router_logits")

    # ---- Experts ------------------------------------------------------------------------
    def router_topk(self, logits, ids, weights, t: int, e: int, k: int):
        """Softmax top-k with renormalised weights (Experts::router_topk, backend.rs:816-824)."""
        check(self.L.oomb_router_topk(_ptr(logits), _ptr(ids), _ptr(weights), t, e, k,
                                      self._stream()), "router_topk")

    def moe_gate_up(self, recs, off, assign_tok, n_experts: int, x, h, geo: Fp8Record, max_per_expert: int = 0,
                    tables_ready: bool = False):
        """h[a] = silu(x[tok(a)] . Wg) * (x[tok(a)] . Wu) (Experts::moe_gate_up, backend.rs:827-836)."""
        check(self.L.oomb_moe_gate_up_fp8(_ptr(recs), _ptr(off), _ptr(assign_tok), n_experts, _ptr(x),
                                          _dtype_code(x), _ptr(h), C.byref(geo), max_per_expert,
                                          _lib.TABLES_READY if tables_ready else 0, self._stream()), "moe_gate_up")

    def moe_down(self, recs, off, n_experts: int, h, y, geo: Fp8Record, max_per_expert: int = 0,
                 tables_ready: bool = False):
        """y[a] = h[a] . Wd^T (Experts::moe_down, backend.rs:860-868)."""
        check(self.L.oomb_moe_down_fp8(_ptr(recs), _ptr(off), n_experts, _ptr(h), _ptr(y), C.byref(geo),
                                       max_per_expert, _lib.TABLES_READY if tables_ready else 0, self._stream()),
              "moe_down")

    def moe_tiled_workspace(self, max_assignments: int, k: int, x_dtype=torch.bfloat16) -> torch.Tensor:
        """A workspace for moe_tiled calls of up to max_assignments assignments over k columns."""
        n = int(self.L.oomb_moe_tiled_fp8_workspace_bytes(max_assignments, k, _dtype_code_of(x_dtype)))
        if n == 0:
            raise ValueError("unsupported moe_tiled shape")
        return torch.empty(n, dtype=torch.uint8, device=self.device)

    def moe_tiled(self, recs, off, rows, n_experts: int, max_per_expert: int, x, y, n: int, k: int,
                  proj: tuple, layout: int, workspace=None, max_assignments: int = 0):
        """y[a] = x[row(a)] . W_e^T for one projection (w_off, s_off) of every group, on the tensor
        cores (Experts::moe_tiled, backend.rs:873-886); rows None means row(a) = a.  The assignment
        count is bounded by y's rows unless max_assignments says otherwise; without a workspace one
        is kept per Gpu object and grown as needed (allocate it once up front before graph capture)."""
        w_off, s_off = proj
        A = int(max_assignments) if max_assignments else int(y.shape[0])
        if workspace is None:
            need = int(self.L.oomb_moe_tiled_fp8_workspace_bytes(A, k, _dtype_code(x)))
            if need == 0:
                raise ValueError("unsupported moe_tiled shape")
            if self._tiled_ws is None or self._tiled_ws.numel() < need:
                self._tiled_ws = torch.empty(need, dtype=torch.uint8, device=self.device)
            workspace = self._tiled_ws
        check(self.L.oomb_moe_tiled_fp8(_ptr(recs), _ptr(off), None if rows is None else _ptr(rows), n_experts,
                                        max_per_expert, A, _ptr(x), _dtype_code(x), _ptr(y), n, k, w_off, s_off,
                                        layout, _ptr(workspace), workspace.numel(), self._stream()), "moe_tiled")

    def moe_swiglu_range(self, g, u, h, start: int, end: int):
        """h[i] = silu(g[i]) * u[i] for i in [start, end) (Experts::moe_swiglu_range, backend.rs:888)."""
        if not (0 <= start <= end <= min(g.numel(), u.numel(), h.numel())):
            raise ValueError("moe_swiglu_range bounds")
        check(self.L.oomb_moe_swiglu_range(_ptr(g), _ptr(u), _ptr(h), start, end, self._stream()),
              "moe_swiglu_range")

    def moe_combine_slots(self, y, slot_assign, w, out, t: int, h: int, k: int):
        """out[t] = sum_s w[t, s] * y[slot_assign[t, s]] in slot order (backend.rs:898-907)."""
        check(self.L.oomb_moe_combine_slots(_ptr(y), _ptr(slot_assign), _ptr(w), _ptr(out), _dtype_code(out),
                                            t, h, k, self._stream()), "moe_combine_slots")

    def moe_combine(self, routed, shared, gate_logit, out, t: int, h: int):
        """out = routed + sigmoid(gate_logit[t]) * shared (backend.rs:909-917)."""
        check(self.L.oomb_moe_combine(_ptr(routed), _ptr(shared), _ptr(gate_logit), _ptr(out), t, h,
                                      self._stream()), "moe_combine")

    # ---- fused decode step --------------------------------------------------------------
    def moe_decode_workspace(self, layer: MoeLayer, t: int) -> torch.Tensor:
        n = int(self.L.oomb_moe_decode_workspace_bytes(t, C.byref(layer)))
        if n == 0:
            raise ValueError("unsupported MoE layer shape")
        ws = torch.empty(n, dtype=torch.uint8, device=self.device)
        check(self.L.oomb_workspace_clear(_ptr(ws), n, self._stream()), "workspace_clear")
        return ws

    def moe_decode(self, layer: MoeLayer, x, t: int, out, workspace, ids=None, weights=None):
        """One resident MoE layer step: route, group, gate/up, down, combine.
        x and out may be pinned host tensors (read and written by the kernels over the bus)."""
        check(self.L.oomb_moe_decode_fp8(C.byref(layer), _ptr_or_host(x), _dtype_code(x), t, _ptr_or_host(out),
                                         _dtype_code(out), _ptr(ids), _ptr(weights), _ptr(workspace),
                                         workspace.numel(), self._stream()), "moe_decode")

    # ---- weights ------------------------------------------------------------------------
    def quantize_fp8(self, w_bf16, n: int, k: int, layout: int, q=None, scale=None):
        """FP8 block quantization on the device (fp8::quantize_blocks, fp8.rs:52-88)."""
        if q is None:
            q = torch.empty((n, k), dtype=torch.uint8, device=self.device)
        if scale is None:
            rows = (n + 127) // 128 if layout == SCALE_128X128 else n
            scale = torch.empty((rows, (k + 127) // 128), dtype=torch.float32, device=self.device)
        check(self.L.oomb_quantize_fp8(_ptr(w_bf16), n, k, layout, _ptr(q), _ptr(scale), self._stream()),
              "quantize_fp8")
        return q, scale

    def moe_layer_workspace(self, layer: MoeLayer, shared, t: int, x_dtype=torch.bfloat16) -> torch.Tensor:
        """A zeroed workspace for moe_layer_decode of up to t tokens."""
        n = int(self.L.oomb_moe_layer_workspace_bytes(t, C.byref(layer), C.byref(shared), _dtype_code_of(x_dtype)))
        if n == 0:
            raise ValueError("unsupported MoE layer shape")
        return torch.zeros(n, dtype=torch.uint8, device=self.device)

    def moe_layer_decode(self, layer: MoeLayer, shared, x, t: int, out, workspace, ids=None, weights=None):
        """One MoE layer (Moe::forward, moe.rs:479-495): shared expert, routed experts and the gated combine."""
        check(self.L.oomb_moe_layer_decode_fp8(C.byref(layer), C.byref(shared), _ptr(x), _dtype_code(x), t, _ptr(out),
                                               _dtype_code(out), _ptr(ids), _ptr(weights), _ptr(workspace),
                                               workspace.numel(), self._stream()), "moe_layer_decode")

    # ---- Attention ----------------------------------------------------------------------

    def attention_workspace(self, batch: int, heads: int, kv_heads: int, head_dim: int, kv_max: int) -> torch.Tensor:
        n = int(self.L.oomb_attention_decode_workspace_bytes(batch, heads, kv_heads, head_dim, kv_max))
        if n == 0:
            raise ValueError("unsupported attention shape")
        return torch.zeros(n, dtype=torch.uint8, device=self.device)

    def attention_decode(self, q, k_cache, v_cache, out, kv_len, scale: float, workspace, kv_heads: int):
        """out[b, h] = softmax(scale * q[b, h] . K[b, :, h / G]) V[b, :, h / G] over each sequence's
        first kv_len positions (Attention::attention for one token per sequence, backend.rs:551-568).
        q, out [B, H, D]; k_cache, v_cache bf16 [B, kv_max, kv_heads, D]; kv_len an int (all
        sequences) or a device int32 tensor [B]."""
        B, H, D = q.shape
        kv_max = k_cache.shape[1]
        if k_cache.shape != v_cache.shape or k_cache.dtype != torch.bfloat16 or k_cache.shape[2] != kv_heads:
            raise ValueError("k_cache and v_cache must be bf16 [B, kv_max, kv_heads, D]")
        lens, all_len = (None, int(kv_len)) if isinstance(kv_len, int) else (_ptr(kv_len), 0)
        check(self.L.oomb_attention_decode(_ptr(q), _dtype_code(q), _ptr(k_cache), _ptr(v_cache),
                                           k_cache.stride(0), lens, all_len, _ptr(out), _dtype_code(out), B, H,
                                           kv_heads, D, kv_max, float(scale), _ptr(workspace), workspace.numel(),
                                           self._stream()), "attention_decode")

    def kv_append(self, src, cache, start, t: int = 1):
        """cache[b, start(b) + i] = bf16(src rows of sequence b) (Attention::kv_append, backend.rs:518-531).
        src: [B * t, kv_heads * D] rows (any row stride, fp32 or bf16); cache bf16 [B, kv_max, kv_heads, D];
        start: an int for every sequence, or a device int32 tensor [B]."""
        B, kv_max, Hkv, D = cache.shape
        starts, all_start = (None, int(start)) if isinstance(start, int) else (_ptr(start), 0)
        check(self.L.oomb_kv_append(_ptr(src), _dtype_code(src), src.stride(0), _ptr(cache), cache.stride(0), starts,
                                    all_start, B, t, Hkv, D, kv_max, self._stream()), "kv_append")

    def device_error(self, clear: bool = True) -> int:
        code = C.c_int(0)
        self.L.oomb_device_error(C.byref(code), int(clear))
        return code.value

    def set_wait_limit(self, ns: int = 0) -> None:
        """How long a bounded device wait polls before it gives up (0: the default 2 s)."""
        check(self.L.oomb_set_wait_limit(int(ns)), "set_wait_limit")
