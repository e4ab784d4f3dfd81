"""ctypes/numpy front end of the CPU oracle and the CPU baseline.

TEST INFRASTRUCTURE ONLY.  Imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg, never by the homelab_b200 package.  The libraries
are built by oracle/Makefile (``make -C oracle``).

The C sources cite the reference (projects/oom-inference in jomcgi-org/homelab)
function by function; this module only moves numpy arrays across.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SCALE_1X128 = 0
SCALE_128X128 = 1

_LIB = None
_CPU = None


def build() -> None:
    """Compile liboomb_oracle.so and liboomb_cpubase.so in place."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def _load(name: str) -> C.CDLL:
    path = os.path.join(HERE, name)
    if not os.path.exists(path):
        build()
    return C.CDLL(path)


def lib() -> C.CDLL:
    global _LIB
    if _LIB is None:
        L = _load("liboomb_oracle.so")
        P, I64, F = C.c_void_p, C.c_int64, C.c_float
        L.oo_e4m3_from_f32.argtypes = [F]
        L.oo_e4m3_from_f32.restype = C.c_uint8
        L.oo_e4m3_to_f32.argtypes = [C.c_uint8]
        L.oo_e4m3_to_f32.restype = F
        L.oo_e4m3_to_f32_nan.argtypes = [C.c_uint8]
        L.oo_e4m3_to_f32_nan.restype = F
        L.oo_bf16_from_f32.argtypes = [F]
        L.oo_bf16_from_f32.restype = C.c_uint16
        L.oo_expf.argtypes = [F]
        L.oo_expf.restype = F
        L.oo_quantize_blocks.argtypes = [P, I64, I64, C.c_int, P, P]
        L.oo_scale_count.argtypes = [I64, I64, C.c_int]
        L.oo_scale_count.restype = I64
        L.oo_gemv_fp8_f64.argtypes = [P, I64, P, P, C.c_int, I64, I64, P, P]
        L.oo_gemv_fp8_reforder.argtypes = [P, I64, P, P, I64, I64, P]
        L.oo_gemv_ref_plan.argtypes = [I64, I64, I64, C.POINTER(I64)]
        L.oo_gemv_ref_plan.restype = I64
        L.oo_gemv_bf16_f64.argtypes = [P, I64, P, I64, I64, P]
        L.oo_router_logits.argtypes = [P, I64, P, I64, I64, P]
        L.oo_router_topk.argtypes = [P, I64, I64, I64, P, P]
        L.oo_group_assignments.argtypes = [P, I64, I64, I64, P, P, P, P]
        L.oo_group_assignments.restype = I64
        L.oo_moe_experts_f64.argtypes = [P, P, P, P, I64, P, P]
        L.oo_combine_slots.argtypes = [P, P, P, I64, I64, I64, P]
        L.oo_combine_slots_f64.argtypes = [P, P, P, I64, I64, I64, P]
        L.oo_fill_normal_bf16.argtypes = [C.c_uint64, F, F, P, I64]
        L.oo_fill_normal_f32.argtypes = [C.c_uint64, F, F, P, I64]
        _LIB = L
    return _LIB


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"], "arrays passed to the oracle must be contiguous"
    return a.ctypes.data


# ---- codecs -----------------------------------------------------------------

def e4m3_from_f32(x: float) -> int:
    return int(lib().oo_e4m3_from_f32(float(x)))


def e4m3_to_f32(b: int) -> float:
    return float(lib().oo_e4m3_to_f32(int(b)))


def e4m3_to_f32_nan(b: int) -> float:
    return float(lib().oo_e4m3_to_f32_nan(int(b)))


def e4m3_table() -> np.ndarray:
    """Exact value of every e4m3 code (NaN codes read as 448, fp8.rs:29-43)."""
    return np.array([e4m3_to_f32(b) for b in range(256)], dtype=np.float32)


def split_terms(x: np.ndarray, terms: int) -> np.ndarray:
    """The tensor-core paths' activation split, restated (xsplit_kernel in
    homelab_b200/csrc/tc.cuh): each 128-column block of every row of fp32 x as
    `terms` e4m3 terms q_i with power-of-two scales s_i, s_i = 2^(floor(log2 m)
    - 7) for m the block's largest residual magnitude, q_i = e4m3(residual /
    s_i) (round to nearest even, saturating), residual -= q_i * s_i in fp32.
    Returns the represented values sum_i s_i * q_i in float64."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    t, k = x.shape
    tab = e4m3_table().astype(np.float64)
    enc = np.vectorize(e4m3_from_f32, otypes=[np.int64])
    out = np.zeros((t, k))
    for r in range(t):
        for b in range(0, k, 128):
            v = x[r, b:b + 128].copy()
            acc = np.zeros(v.shape)
            for _ in range(terms):
                m = np.float32(np.abs(v).max())
                e = 0 if m == 0 else max(-100, min(100, int((m.view(np.uint32) >> 23) & 0xff) - 127 - 7))
                sc = np.float32(2.0 ** e)
                qv = tab[enc(v * np.float32(2.0 ** -e))]
                acc += qv * float(sc)
                v = (v - (qv.astype(np.float32) * sc)).astype(np.float32)
            out[r, b:b + 128] = acc
    return out


def bf16_from_f32(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even bf16 bits of fp32 values (vectorised)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    return r


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def expf(x: float) -> float:
    return float(lib().oo_expf(float(x)))


# ---- generators -------------------------------------------------------------

def normal_bf16(seed: int, n: int, mu: float = 0.0, sigma: float = 1.0) -> np.ndarray:
    out = np.empty(n, dtype=np.uint16)
    lib().oo_fill_normal_bf16(seed, mu, sigma, _p(out), n)
    return out


def normal_f32(seed: int, n: int, mu: float = 0.0, sigma: float = 1.0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().oo_fill_normal_f32(seed, mu, sigma, _p(out), n)
    return out


# ---- quantizer and GEMV -----------------------------------------------------

def scale_count(n: int, k: int, layout: int) -> int:
    return int(lib().oo_scale_count(n, k, layout))


def quantize_blocks(w_bf16: np.ndarray, n: int, k: int, layout: int = SCALE_1X128):
    """fp8.rs:52-88 (1x128) or its 128x128 generalisation -> (q uint8 [n,k], scale f32)."""
    w = np.ascontiguousarray(w_bf16, dtype=np.uint16).reshape(-1)
    assert w.size == n * k
    q = np.empty(n * k, dtype=np.uint8)
    s = np.empty(scale_count(n, k, layout), dtype=np.float32)
    lib().oo_quantize_blocks(_p(w), n, k, layout, _p(q), _p(s))
    return q.reshape(n, k), s


def dequantize(q: np.ndarray, scale: np.ndarray, layout: int) -> np.ndarray:
    """e4m3(q) * scale in float64 (exact), shape [n, k]."""
    n, k = q.shape
    tab = e4m3_table().astype(np.float64)
    nb = (k + 127) // 128
    rows = np.arange(n) // 128 if layout == SCALE_128X128 else np.arange(n)
    s = scale.reshape(-1, nb).astype(np.float64)[rows]            # [n, nb]
    s = np.repeat(s, 128, axis=1)[:, :k]
    return tab[q] * s


def gemv_fp8_f64(x: np.ndarray, q: np.ndarray, scale: np.ndarray, layout: int):
    """Truth (double) and error scale sum|x*w| for y = x . W^T; x fp32 [t, k]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    t, k = x.shape
    n = q.shape[0]
    y = np.empty((t, n), dtype=np.float64)
    mag = np.empty((t, n), dtype=np.float64)
    lib().oo_gemv_fp8_f64(_p(x), t, _p(np.ascontiguousarray(q)), _p(scale), layout, n, k, _p(y), _p(mag))
    return y, mag


def gemv_fp8_f64_fast(x: np.ndarray, q: np.ndarray, scale: np.ndarray, layout: int):
    """Same truth through numpy float64 matmuls (for sizes the C loop is slow on)."""
    w = dequantize(q, scale, layout)
    xd = np.asarray(x, dtype=np.float64)
    return xd @ w.T, np.abs(xd) @ np.abs(w).T


def gemv_ref_plan(t: int, n: int, k: int):
    kl = C.c_int64(0)
    s = lib().oo_gemv_ref_plan(t, n, k, C.byref(kl))
    return int(s), int(kl.value)


def gemv_fp8_reforder(x: np.ndarray, q: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """The reference GEMV's exact fp32 result (1x128 scales, t <= 4)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    t, k = x.shape
    n = q.shape[0]
    y = np.empty((t, n), dtype=np.float32)
    lib().oo_gemv_fp8_reforder(_p(x), t, _p(np.ascontiguousarray(q)), _p(scale), n, k, _p(y))
    return y


# ---- router -----------------------------------------------------------------

def router_logits(x: np.ndarray, w_bf16: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    t, h = x.shape
    e = w_bf16.shape[0]
    out = np.empty((t, e), dtype=np.float32)
    lib().oo_router_logits(_p(x), t, _p(np.ascontiguousarray(w_bf16, dtype=np.uint16)), e, h, _p(out))
    return out


def router_topk(logits: np.ndarray, k: int):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    t, e = logits.shape
    ids = np.empty((t, k), dtype=np.int32)
    w = np.empty((t, k), dtype=np.float32)
    lib().oo_router_topk(_p(logits), t, e, k, _p(ids), _p(w))
    return ids, w


# ---- routed experts ---------------------------------------------------------

class Fp8Record(C.Structure):
    """Byte offsets of the parts of an FP8 expert record (see include/oomb.h)."""
    _fields_ = [
        ("hidden", C.c_int64), ("inter", C.c_int64),
        ("gate_weight", C.c_int64), ("gate_scale", C.c_int64),
        ("up_weight", C.c_int64), ("up_scale", C.c_int64),
        ("down_weight", C.c_int64), ("down_scale", C.c_int64),
        ("layout", C.c_int32), ("pad_", C.c_int32),
    ]


def group_assignments(ids: np.ndarray, e: int):
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    t, k = ids.shape
    a = t * k
    active = np.empty(max(a, 1), dtype=np.int32)
    off = np.empty(a + 1, dtype=np.int32)
    tok = np.empty(max(a, 1), dtype=np.int32)
    slot = np.empty(max(a, 1), dtype=np.int32)
    n_e = lib().oo_group_assignments(_p(ids), t, k, e, _p(active), _p(off), _p(tok), _p(slot))
    if n_e < 0:
        raise ValueError("router picked an expert out of range")
    return active[:n_e].copy(), off[: n_e + 1].copy(), tok[:a].copy(), slot[:a].copy()


def moe_experts_f64(recs: list, geo: Fp8Record, off: np.ndarray, assign_tok: np.ndarray,
                    x: np.ndarray) -> np.ndarray:
    """Expert outputs y [A, hidden] in double; recs[i] is a uint8 record array."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n_e = len(recs)
    ptrs = (C.c_void_p * max(n_e, 1))(*[r.ctypes.data for r in recs])
    a = int(off[-1])
    y = np.zeros((max(a, 1), geo.hidden), dtype=np.float64)
    lib().oo_moe_experts_f64(C.cast(ptrs, C.c_void_p), C.addressof(geo), _p(off), _p(assign_tok),
                             n_e, _p(x), _p(y))
    return y[:a]


def record_matrix(rec: np.ndarray, geo: Fp8Record, part: str) -> np.ndarray:
    """The exactly decoded float64 matrix of one part ("gate", "up" or "down") of an FP8 record."""
    H, I = int(geo.hidden), int(geo.inter)
    n, k = (H, I) if part == "down" else (I, H)
    w_off, s_off = int(getattr(geo, part + "_weight")), int(getattr(geo, part + "_scale"))
    q = rec[w_off:w_off + n * k].reshape(n, k)
    sc = rec[s_off:s_off + 4 * scale_count(n, k, int(geo.layout))].view(np.float32)
    return dequantize(q, sc, int(geo.layout))


def moe_experts_f64_fast(recs: list, geo: Fp8Record, off: np.ndarray, assign_tok: np.ndarray,
                         x: np.ndarray) -> np.ndarray:
    """moe_experts_f64 through numpy float64 matmuls, expert by expert (large shapes):
    h = silu(x Wg^T) * (x Wu^T), y = h Wd^T, silu(v) = v / (1 + exp(-v))."""
    xd = np.asarray(x, dtype=np.float64)
    a = int(off[-1])
    y = np.zeros((max(a, 1), int(geo.hidden)), dtype=np.float64)
    for i, rec in enumerate(recs):
        a0, a1 = int(off[i]), int(off[i + 1])
        if a1 == a0:
            continue
        xr = xd[np.asarray(assign_tok[a0:a1])]
        g = xr @ record_matrix(rec, geo, "gate").T
        u = xr @ record_matrix(rec, geo, "up").T
        h = g / (1.0 + np.exp(-g)) * u
        y[a0:a1] = h @ record_matrix(rec, geo, "down").T
    return y[:a]


def attention_decode_f64(q: np.ndarray, k: np.ndarray, v: np.ndarray, kv_len, scale: float) -> np.ndarray:
    """Decode attention in float64: q [B, H, D]; k, v [B, kv_max, Hkv, D] (exact values);
    out[b, h] = softmax_j(scale * q[b, h] . k[b, j, h // G]) v[b, j, h // G] over j < kv_len[b]."""
    B, H, D = q.shape
    Hkv = k.shape[2]
    G = H // Hkv
    lens = np.full(B, int(kv_len)) if np.isscalar(kv_len) else np.asarray(kv_len)
    out = np.zeros((B, H, D))
    for b in range(B):
        L = int(lens[b])
        if L == 0:
            continue
        for h in range(H):
            kk = k[b, :L, h // G].astype(np.float64)
            s = kk @ q[b, h].astype(np.float64) * scale
            p = np.exp(s - s.max())
            out[b, h] = (p / p.sum()) @ v[b, :L, h // G].astype(np.float64)
    return out


def combine_slots(y: np.ndarray, slot_assign: np.ndarray, w: np.ndarray, t: int, h: int, k: int):
    y = np.ascontiguousarray(y, dtype=np.float32)
    out = np.empty((t, h), dtype=np.float32)
    lib().oo_combine_slots(_p(y), _p(np.ascontiguousarray(slot_assign, dtype=np.int32)),
                           _p(np.ascontiguousarray(w, dtype=np.float32)), t, h, k, _p(out))
    return out


def combine_slots_f64(y: np.ndarray, slot_assign: np.ndarray, w: np.ndarray, t: int, h: int, k: int):
    y = np.ascontiguousarray(y, dtype=np.float64)
    out = np.empty((t, h), dtype=np.float64)
    lib().oo_combine_slots_f64(_p(y), _p(np.ascontiguousarray(slot_assign, dtype=np.int32)),
                               _p(np.ascontiguousarray(w, dtype=np.float32)), t, h, k, _p(out))
    return out


# ---- CPU baseline (reference host expert path, AVX-512 port) -----------------

def cpu() -> C.CDLL:
    global _CPU
    if _CPU is None:
        L = _load("liboomb_cpubase.so")
        P, I64 = C.c_void_p, C.c_int64
        L.ocb_pool_create.argtypes = [C.c_int]
        L.ocb_pool_create.restype = P
        L.ocb_pool_destroy.argtypes = [P]
        L.ocb_pool_threads.argtypes = [P]
        L.ocb_pool_threads.restype = C.c_int
        L.ocb_has_avx512.restype = C.c_int
        L.ocb_gemv_fp8.argtypes = [P, P, I64, P, P, C.c_int, I64, I64, P]
        L.ocb_moe_layer.argtypes = [P, P, I64, P, I64, I64, P, P, P]
        L.ocb_moe_layer.restype = C.c_int
        _CPU = L
    return _CPU


class CpuPool:
    """Worker pool of the CPU baseline (stand-in for oominf-cpu's rayon pool)."""

    def __init__(self, threads: int):
        self.h = cpu().ocb_pool_create(int(threads))
        self.threads = int(cpu().ocb_pool_threads(self.h))

    def close(self):
        if self.h:
            cpu().ocb_pool_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def gemv_fp8(self, x, q, scale, layout):
        x = np.ascontiguousarray(x, dtype=np.float32)
        t, k = x.shape
        n = q.shape[0]
        y = np.empty((t, n), dtype=np.float32)
        cpu().ocb_gemv_fp8(self.h, _p(x), t, _p(np.ascontiguousarray(q)), _p(scale), layout, n, k, _p(y))
        return y

    def moe_layer(self, x, router_w, k, rec_ptrs, geo):
        """rec_ptrs: ctypes array of host record addresses for all E experts."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        t, h = x.shape
        e = router_w.shape[0]
        out = np.empty((t, h), dtype=np.float32)
        rc = cpu().ocb_moe_layer(self.h, _p(x), t, _p(router_w), e, k, C.cast(rec_ptrs, C.c_void_p),
                                 C.addressof(geo), _p(out))
        if rc != 0:
            raise ValueError("cpu baseline: unsupported shape")
        return out
