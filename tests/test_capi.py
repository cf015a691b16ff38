"""The C ABI without a GPU: the library loads, exports every function include/rumik_b200.h declares, and
rejects bad arguments with the documented status codes before making any CUDA call."""
import ctypes
import os
import re

import pytest

from rumik_fast_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "rumik_b200.h")


def declared_functions():
    with open(HEADER) as f:
        txt = f.read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(rb_[a-z0-9_]+)\s*\(", txt)))


def test_header_declares_expected_api():
    names = declared_functions()
    for want in ("rb_gemv_int4", "rb_gemv_int8", "rb_mm_int4", "rb_status_string", "rb_version",
                 "rb_get_device_error"):
        assert want in names


def test_library_exports_every_declared_symbol(native_lib):
    for name in declared_functions():
        assert hasattr(native_lib, name), f"{name} declared in rumik_b200.h but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature in _lib.py"


def test_version_and_status_strings(native_lib):
    assert native_lib.rb_version() >= 100
    for st in range(8):
        assert native_lib.rb_status_string(st)
    assert native_lib.rb_status_string(0) == b"ok"
    assert b"unknown" in native_lib.rb_status_string(99)


A = 0x1000  # a 16-byte-aligned dummy address; validation rejects the call before it is dereferenced


def gemv4(L, x=A, xd=_lib.F16, ldx=0, q=A, s=A, m=A, y=A, yd=_lib.F16, ldy=0, N=64, K=256, B=1):
    return L.rb_gemv_int4(x, xd, ldx, q, s, m, y, yd, ldy, N, K, B, 0, None)


def test_gemv_int4_validation(native_lib):
    L = native_lib
    assert gemv4(L, K=200) == _lib.ERR_SHAPE           # K % 128
    assert gemv4(L, K=0) == _lib.ERR_SHAPE
    assert gemv4(L, K=16384 + 128) == _lib.ERR_SHAPE   # above the supported K
    assert gemv4(L, N=-1) == _lib.ERR_SHAPE
    assert gemv4(L, N=0) == _lib.OK                    # empty: no-op, no launch
    assert gemv4(L, B=0) == _lib.OK
    assert gemv4(L, q=None) == _lib.ERR_NULL
    assert gemv4(L, x=None) == _lib.ERR_NULL
    assert gemv4(L, xd=_lib.F32) == _lib.ERR_DTYPE
    assert gemv4(L, yd=7) == _lib.ERR_DTYPE
    assert gemv4(L, x=A + 2) == _lib.ERR_ALIGN
    assert gemv4(L, s=A + 8) == _lib.ERR_ALIGN
    assert gemv4(L, B=2, ldx=256 + 4, ldy=64) == _lib.ERR_ALIGN   # row stride not a multiple of 8
    assert gemv4(L, B=2, ldx=128, ldy=64) == _lib.ERR_SHAPE       # row stride shorter than K


def test_gemv_int8_validation(native_lib):
    L = native_lib

    def g8(q=A, s=A, sd=_lib.F32, N=64, K=256, x=A):
        return L.rb_gemv_int8(x, _lib.F16, 0, q, 0, s, sd, A, _lib.F16, 0, N, K, 1, 0, None)

    assert g8(K=96) == _lib.ERR_SHAPE
    assert g8(N=0) == _lib.OK
    assert g8(s=None) == _lib.ERR_NULL
    assert g8(sd=_lib.BF16) == _lib.ERR_DTYPE
    assert g8(q=A + 1) == _lib.ERR_ALIGN


def test_mm_int4_validation(native_lib):
    L = native_lib

    def mm(M=8, N=64, K=256, ldx=256, ldy=64, X=A, Y=A):
        return L.rb_mm_int4(X, _lib.F16, ldx, A, A, A, Y, _lib.F16, ldy, M, N, K, 0, None)

    assert mm(K=100) == _lib.ERR_SHAPE
    assert mm(M=0) == _lib.OK
    assert mm(ldx=128) == _lib.ERR_SHAPE
    assert mm(ldy=60) == _lib.ERR_SHAPE
    assert mm(ldx=260) == _lib.ERR_ALIGN
    assert mm(X=None) == _lib.ERR_NULL


def test_gemv_list_int8_entry_validation(native_lib):
    """int8 entries of a GEMV list (rb_gemv_desc::w8) are checked before any CUDA call: the kind, the row-scale
    pointer and alignments, and that no forced warp-MMA launch, fused epilogue or whole-step layer takes one."""
    L = native_lib

    def multi(flags=0, **kw):
        d = _lib.GemvDesc(A, A, A, A, None, 64, 256)
        d.w8 = _lib.W8_SIGNED
        for k, v in kw.items():
            setattr(d, k, v)
        arr = (_lib.GemvDesc * 1)(d)
        return L.rb_gemv_int4_multi(arr, 1, _lib.F16, _lib.F16, flags, None)

    assert multi(w8=3) == _lib.ERR_SHAPE
    assert multi(w8=-1) == _lib.ERR_SHAPE
    assert multi(K=200) == _lib.ERR_SHAPE
    assert multi(s=None) == _lib.ERR_NULL             # no row scales at all
    assert multi(q=None) == _lib.ERR_NULL
    assert multi(q=A + 8) == _lib.ERR_ALIGN
    assert multi(s=A + 1) == _lib.ERR_ALIGN           # fp16 row scales: 2-byte aligned
    assert multi(s=None, s_row=A + 2) == _lib.ERR_ALIGN  # fp32 row scales: 4-byte aligned
    assert multi(flags=_lib.FLAG_KERNEL_MMA) == _lib.ERR_SHAPE
    d = _lib.GemvDesc(A, A, A, A, None, 64, 256)
    d.w8 = _lib.W8_OFFSET
    assert L.rb_gemv_int4_fused((_lib.GemvDesc * 1)(d), None, 1, None, None, None, 0, _lib.F16, _lib.F16, 0,
                                None) == _lib.ERR_SHAPE


def test_mm_int4_list_validation(native_lib):
    L = native_lib

    def lst(M=8, xd=_lib.F16, **kw):
        d = _lib.MmDesc(A, 256, A, A, A, A, 64, 64, 256)
        for k, v in kw.items():
            setattr(d, k, v)
        return L.rb_mm_int4_list((_lib.MmDesc * 1)(d), 1, M, xd, _lib.F16, 0, None)

    assert lst(M=0) == _lib.OK
    assert lst(M=-1) == _lib.ERR_SHAPE
    assert lst(K=200) == _lib.ERR_SHAPE
    assert lst(ldx=128) == _lib.ERR_SHAPE
    assert lst(X=None) == _lib.ERR_NULL
    assert lst(m=None) == _lib.ERR_NULL
    assert lst(xd=_lib.F32) == _lib.ERR_DTYPE
    assert lst(ldy=68) == _lib.ERR_ALIGN
    assert lst(q=A + 8) == _lib.ERR_ALIGN
    assert L.rb_mm_int4_list(None, 1, 8, _lib.F16, _lib.F16, 0, None) == _lib.ERR_NULL
