"""ctypes binding of the C ABI in include/rumik_b200.h (librumik_b200.so, built in-tree for sm_100a).

There is no fallback: if the library is missing or the device is not an sm_100 GPU, calls raise.
"""
import ctypes
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "librumik_b200.so")

# status codes (enum rb_status)
OK, ERR_NULL, ERR_SHAPE, ERR_DTYPE, ERR_ALIGN, ERR_LAUNCH, ERR_DEVICE, ERR_TIMEOUT = range(8)
# dtype codes (enum rb_dtype)
F16, BF16, F32 = 0, 1, 2
# launch flags (enum rb_flags)
FLAG_PDL, FLAG_PREFETCH_WEIGHTS, FLAG_KERNEL_TC, FLAG_KERNEL_MMA, FLAG_ATTN_TICKET = 1, 2, 4, 8, 16
KERNEL_FLAGS = {None: 0, "tc": FLAG_KERNEL_TC, "mma": FLAG_KERNEL_MMA}

_DTYPE_CODE = {torch.float16: F16, torch.bfloat16: BF16, torch.float32: F32}

_c = ctypes
_vp, _i64, _int = _c.c_void_p, _c.c_int64, _c.c_int


class MmDesc(ctypes.Structure):
    """struct rb_mm_desc (include/rumik_b200.h)."""
    _fields_ = [("X", _vp), ("ldx", _i64), ("q", _vp), ("s", _vp), ("m", _vp), ("Y", _vp), ("ldy", _i64),
                ("N", _i64), ("K", _i64)]


class GemvDesc(ctypes.Structure):
    """struct rb_gemv_desc (include/rumik_b200.h)."""
    _fields_ = [("x", _vp), ("y", _vp), ("q", _vp), ("s", _vp), ("m", _vp), ("N", _i64), ("K", _i64),
                ("s_row", _vp), ("w8", _int)]


W8_NONE, W8_SIGNED, W8_OFFSET = 0, 1, 2

class AddLn(ctypes.Structure):
    """struct rb_add_ln (include/rumik_b200.h)."""
    _fields_ = [("x", _vp), ("a", _vp), ("b", _vp), ("w", _vp), ("x_out", _vp), ("h_out", _vp), ("H", _i64),
                ("eps", _c.c_float), ("emb_q", _vp), ("emb_s", _vp), ("tok", _vp), ("vocab", _i64),
                ("emb_s_dtype", _int)]


class GemvEpi(ctypes.Structure):
    """struct rb_gemv_epi (include/rumik_b200.h)."""
    _fields_ = [("kind", _int), ("rope", _int), ("n_q_heads", _int), ("n_kv_heads", _int), ("head_dim", _int),
                ("cache_len", _i64), ("pos", _vp), ("cos", _vp), ("sin", _vp), ("q_out", _vp), ("k_cache", _vp),
                ("v_cache", _vp), ("act_out", _vp)]


class AttnSrc(ctypes.Structure):
    """struct rb_attn_src (include/rumik_b200.h)."""
    _fields_ = [("q", _vp), ("k_cache", _vp), ("v_cache", _vp), ("pos", _vp), ("out", _vp), ("n_q_heads", _int),
                ("n_kv_heads", _int), ("head_dim", _int), ("cache_len", _i64), ("scale", _c.c_float), ("ws", _vp),
                ("ws_bytes", _i64)]


class Sampler(ctypes.Structure):
    """struct rb_sampler (include/rumik_b200.h)."""
    _fields_ = [("logits", _vp), ("logits_dtype", _int), ("n_vocab", _i64), ("end_idx", _i64), ("ids", _vp),
                ("top_k", _int), ("inv_temp", _c.c_float), ("u", _vp), ("h", _vp), ("h_dtype", _int), ("H", _i64),
                ("ln_w", _vp), ("ln_b", _vp), ("w1", _vp), ("w1_dtype", _int), ("nz", _int), ("b1", _vp),
                ("w2", _vp), ("b2", _vp), ("end_id", _i64), ("min_new", _i64), ("step", _vp), ("tok", _vp),
                ("out", _vp), ("out_len", _i64), ("ws", _vp)]


EPI_STORE, EPI_ROPE_KV, EPI_SWIGLU = 0, 1, 2
# device error word bits (rb_get_device_error): a wait that ran out, or an out-of-range device-side argument
DEVERR_TC_WAIT, DEVERR_TP_WAIT, DEVERR_ARG, DEVERR_ATT_WAIT, DEVERR_STEP_WAIT = 1 << 7, 1 << 8, 1 << 9, 1 << 10, 1 << 11

SIGNATURES = {
    "rb_gemv_int4": (_int, [_vp, _int, _i64, _vp, _vp, _vp, _vp, _int, _i64, _i64, _i64, _i64, _int, _vp]),
    "rb_gemv_int8": (_int, [_vp, _int, _i64, _vp, _int, _vp, _int, _vp, _int, _i64, _i64, _i64, _i64, _int, _vp]),
    "rb_mm_int4": (_int, [_vp, _int, _i64, _vp, _vp, _vp, _vp, _int, _i64, _i64, _i64, _i64, _int, _vp]),
    "rb_mm_int4_workspace": (_i64, [_i64, _i64, _i64]),
    "rb_mm_int4_static": (_int, [_vp, _int, _i64, _vp, _vp, _vp, _vp, _int, _i64, _i64, _i64, _i64, _int, _vp]),
    "rb_mm_int4_list": (_int, [_vp, _int, _i64, _int, _int, _int, _vp]),
    "rb_mm_int4_ws": (_int, [_vp, _int, _i64, _vp, _vp, _vp, _vp, _int, _i64, _i64, _i64, _i64, _vp, _i64, _int, _vp]),
    "rb_gemv_int4_multi": (_int, [_c.POINTER(GemvDesc), _int, _int, _int, _int, _vp]),
    "rb_gemv_int4_fused": (_int, [_c.POINTER(GemvDesc), _c.POINTER(GemvEpi), _int, _c.POINTER(AddLn),
                                  _c.POINTER(AttnSrc), _vp, _i64, _int, _int, _int, _vp]),
    "rb_gemv_int4_workspace": (_i64, [_c.POINTER(GemvDesc), _int, _int]),
    "rb_gemv_int4_multi_ws": (_int, [_c.POINTER(GemvDesc), _int, _vp, _i64, _int, _int, _int, _vp]),
    "rb_add_layernorm": (_int, [_c.POINTER(AddLn), _int, _int, _vp]),
    "rb_attn_decode_workspace": (_i64, [_int, _int, _int]),
    "rb_sample": (_int, [_c.POINTER(Sampler), _int, _vp]),
    "rb_sample_workspace": (_i64, [_int]),
    "rb_attn_decode": (_int, [_vp, _vp, _vp, _vp, _vp, _int, _int, _int, _i64, _c.c_float, _vp, _i64, _int, _int,
                              _vp]),
    "rb_status_string": (_c.c_char_p, [_int]),
    "rb_version": (_int, []),
    "rb_get_device_error": (_int, [_c.POINTER(_c.c_uint), _vp]),
    "rb_set_wait_limit": (_int, [_c.c_uint64, _vp]),
    "rb_decode_layers_workspace": (_i64, [_vp]),
    "rb_decode_layers": (_int, [_vp, _int, _int, _vp]),
    "rb_ipc_alloc": (_int, [_c.c_uint64, _c.POINTER(_vp), _vp]),
    "rb_ipc_free": (_int, [_vp]),
    "rb_ipc_open": (_int, [_vp, _c.c_uint64, _c.POINTER(_vp), _c.POINTER(_vp)]),
    "rb_ipc_close": (_int, [_vp]),
    "rb_tp_allreduce_f16": (_int, [_vp, _vp, _vp, _i64, _c.POINTER(_vp), _int, _int, _c.c_uint32, _c.c_uint32, _int,
                                   _vp]),
}

_lib = None


class RumikKernelError(RuntimeError):
    """A native entry point returned a non-zero rb_status (the reference raises RuntimeError too)."""

    def __init__(self, fn, status):
        self.status = status
        super().__init__(f"{fn}: {lib().rb_status_string(status).decode()} (status {status})")


def lib():
    """Load librumik_b200.so (once). Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m rumik_fast_b200.build` "
                              "(there is no non-CUDA fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        _lib = L
    return _lib


def dtype_code(dt):
    try:
        return _DTYPE_CODE[dt]
    except KeyError:
        raise TypeError(f"unsupported dtype {dt}") from None


def stream_ptr(device):
    return torch.cuda.current_stream(device).cuda_stream


def check(fn, status):
    if status != OK:
        raise RumikKernelError(fn, status)


def device_error(device=None):
    """Read and clear the device-side error word (non-zero: a kernel gave up a bounded wait)."""
    out = ctypes.c_uint(0)
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        check("rb_get_device_error", lib().rb_get_device_error(ctypes.byref(out), stream_ptr(dev)))
    return out.value


def set_wait_limit(ns=0, device=None):
    """Longest wait of a kernel on `device` before it gives up and sets its error bit (0: the default 4 s)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        check("rb_set_wait_limit", lib().rb_set_wait_limit(int(ns), stream_ptr(dev)))
