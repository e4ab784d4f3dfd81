"""B200-native (sm_100a) FP8 decode path of oom-inference.

The kernels live in liboomb.so (C ABI: include/oomb.h).  `Gpu` exposes them
under the names of the engine's backend traits; `records` lays out FP8 expert
records.  There is no CPU fallback: without the built library or an sm_100
GPU every call raises.
"""
from ._lib import BF16, F32, SCALE_128X128, SCALE_1X128, Fp8Record, MoeLayer, OombError, SharedExpert, lib  # noqa: F401

__version__ = "0.1.0"
