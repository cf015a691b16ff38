"""rumik_fast_b200 - B200 (sm_100a) implementation of rumik-fast's weight-only quantised linear path.

Drop-in modules with the reference's signatures:
    rumik_fast_b200.cuda_gemv  gemv_int4_cuda, gemv_int8_cuda, quantize_int8_rows, SHAPE
    rumik_fast_b200.mm_int4    mm_int4, warmup, G
    rumik_fast_b200.int4_gemv  quantize, gemv_int4, G
Beyond them: Int4GemvSet (a list of GEMVs in one launch), fused (the decode-layer glue in the GEMV launches),
attention (decode attention), sample (the sampling tail), scales8 (8-bit double-quantised scales).
All compute runs in librumik_b200.so (hand-written CUDA for sm_100a behind the C ABI in
include/rumik_b200.h), loaded with ctypes from this directory.
"""
from . import config  # noqa: F401
from ._lib import RumikKernelError, device_error, lib  # noqa: F401
from .config import set_weight_prefetch, weight_prefetch  # noqa: F401
from .cuda_gemv import SHAPE, gemv_int4_cuda, gemv_int8_cuda, quantize_int8_rows  # noqa: F401
from .gemv_set import Int4GemvSet  # noqa: F401
from .int4_gemv import quantize  # noqa: F401
from . import mm_int4  # noqa: F401  (module: mm_int4.mm_int4, mm_int4.warmup, as in the reference)
from . import scales8  # noqa: F401

__all__ = ["Int4GemvSet", "gemv_int4_cuda", "gemv_int8_cuda", "quantize_int8_rows", "quantize", "SHAPE",
           "set_weight_prefetch", "weight_prefetch", "device_error", "RumikKernelError"]
