"""The fused decode-layer glue without a GPU: argument checks of rb_gemv_int4_fused / rb_add_layernorm (they
return before any CUDA call) and the host-side weight re-ordering against the oracle."""
import ctypes

import numpy as np
import torch

from oracle import oracle as O
from rumik_fast_b200 import _lib, fused

A = 0x10000      # 16-byte-aligned dummy addresses; validation rejects each call before any is dereferenced
B = 0x20000
C = 0x30000
POS = 0x40000


def desc(x=A, y=B, N=256, K=256):
    return _lib.GemvDesc(x, y, C, C, C, N, K)


def epi_rope(nq=1, nkv=1, hd=64, rope=1, pos=POS, cos=C, sin=C, q=B, k=B, v=B):
    return _lib.GemvEpi(_lib.EPI_ROPE_KV, rope, nq, nkv, hd, 32, pos, cos, sin, q, k, v, None)


def epi_swiglu(act=B):
    return _lib.GemvEpi(_lib.EPI_SWIGLU, 0, 0, 0, 0, 0, None, None, None, None, None, None, act)


def call(L, descs, epis=None, ln=None, xd=_lib.F16, yd=_lib.F16, count=None, ws=None, ws_bytes=0):
    n = len(descs)
    d = (_lib.GemvDesc * max(n, 1))(*descs)
    e = (_lib.GemvEpi * max(n, 1))(*epis) if epis is not None else None
    return L.rb_gemv_int4_fused(d, e, n if count is None else count, ctypes.byref(ln) if ln is not None else None,
                                None, ws, ws_bytes, xd, yd, 0, None)


def add_ln(x=0x50000, a=0x60000, b=0x70000, w=0x80000, x_out=0x90000, h_out=None, H=256, eps=1e-5):
    return _lib.AddLn(x, a, b, w, x_out, h_out, H, eps)


def test_fused_argument_checks(native_lib):
    L = native_lib
    assert call(L, [desc()], count=0) == _lib.OK                              # empty list: no launch
    assert call(L, [desc()], count=161) == _lib.ERR_SHAPE                      # one launch holds 160 entries
    assert call(L, [desc(x=None)]) == _lib.ERR_NULL                            # x from a prologue that is absent
    assert call(L, [desc(y=None)]) == _lib.ERR_NULL                            # a stored entry needs y
    assert call(L, [desc(K=200)]) == _lib.ERR_SHAPE
    assert call(L, [desc()], xd=_lib.F32) == _lib.ERR_DTYPE
    # rotary / KV epilogue
    assert call(L, [desc(N=200)], [epi_rope()]) == _lib.ERR_SHAPE             # N != (nq + 2 nkv) hd
    assert call(L, [desc(N=3 * 63)], [epi_rope(hd=63)]) == _lib.ERR_SHAPE     # odd head_dim
    assert call(L, [desc(N=192)], [epi_rope(pos=None)]) == _lib.ERR_NULL
    assert call(L, [desc(N=192)], [epi_rope(cos=None)]) == _lib.ERR_NULL      # rope needs the tables
    assert call(L, [desc(N=192)], [epi_rope(k=None)]) == _lib.ERR_NULL
    # SwiGLU epilogue
    assert call(L, [desc(N=191)], [epi_swiglu()]) == _lib.ERR_SHAPE           # N odd
    assert call(L, [desc(N=256)], [epi_swiglu(act=None)]) == _lib.ERR_NULL
    assert call(L, [desc(N=256)] * 5, [epi_swiglu()] * 5) == _lib.ERR_SHAPE   # at most 4 routed entries
    bad = epi_swiglu()
    bad.kind = 7
    assert call(L, [desc()], [bad]) == _lib.ERR_SHAPE
    assert call(L, [desc()], ws=0x50008, ws_bytes=1024) == _lib.ERR_ALIGN       # split-K workspace alignment
    d = (_lib.GemvDesc * 1)(desc())
    assert L.rb_gemv_int4_multi_ws(d, 1, 0x50008, 1024, _lib.F16, _lib.F16, 0, None) == _lib.ERR_ALIGN
    assert L.rb_gemv_int4_workspace(d, 0, 0) == 0
    assert L.rb_gemv_int4_workspace(None, 1, 0) == -_lib.ERR_NULL
    assert L.rb_gemv_int4_workspace(d, 1, 0) == 0                   # a small list: warp-MMA kernel, no workspace
    d[0].K = 200
    assert L.rb_gemv_int4_workspace(d, 1, 0) == -_lib.ERR_SHAPE


def test_prologue_argument_checks(native_lib):
    L = native_lib
    assert call(L, [desc(x=None)], ln=add_ln(H=384)) == _lib.ERR_SHAPE        # K of an x == NULL entry != H
    assert call(L, [desc(x=None)], ln=add_ln(H=200)) == _lib.ERR_SHAPE        # H % 128
    assert call(L, [desc(x=None)], ln=add_ln(H=12288 + 128)) == _lib.ERR_SHAPE
    assert call(L, [desc(x=None)], ln=add_ln(w=None)) == _lib.ERR_NULL
    assert call(L, [desc(x=None)], ln=add_ln(x_out=0x50000 + 128)) == _lib.ERR_SHAPE   # x_out overlaps x
    assert call(L, [desc(x=None)], ln=add_ln(h_out=0x60000 + 16)) == _lib.ERR_SHAPE    # h_out overlaps a
    assert call(L, [desc(x=None)], ln=add_ln(x_out=0x90008)) == _lib.ERR_ALIGN
    assert call(L, [desc(x=None)], ln=add_ln(eps=float("nan"))) == _lib.ERR_SHAPE
    assert L.rb_add_layernorm(None, _lib.F16, 0, None) == _lib.ERR_NULL
    ln = add_ln()
    assert L.rb_add_layernorm(ctypes.byref(ln), _lib.F32, 0, None) == _lib.ERR_DTYPE
    ln = add_ln(H=100)
    assert L.rb_add_layernorm(ctypes.byref(ln), _lib.F16, 0, None) == _lib.ERR_SHAPE
    ln = add_ln(x_out=0x70000)                                                 # x_out == b
    assert L.rb_add_layernorm(ctypes.byref(ln), _lib.F16, 0, None) == _lib.ERR_SHAPE


def test_gate_up_order_matches_oracle():
    for inter in (1, 64, 256, 8192):
        assert np.array_equal(fused.gate_up_order(inter).numpy(), O.gate_up_order(inter))


def test_interleave_and_split_w_in_on_host_tensors():
    nq, nkv, hd, inter, K = 2, 1, 64, 128, 256
    n = (nq + 2 * nkv) * hd + 2 * inter
    q = torch.arange(n, dtype=torch.int64).remainder(251).to(torch.uint8)[:, None].repeat(1, K // 2).contiguous()
    s = torch.arange(n, dtype=torch.float16)[:, None].repeat(1, K // 128).contiguous()
    m = -s
    (qq, qs, qm), (gq, gs, gm) = fused.split_w_in(q, s, m, nq, nkv, hd)
    nqkv = (nq + 2 * nkv) * hd
    assert torch.equal(qq, q[:nqkv]) and torch.equal(qs, s[:nqkv]) and torch.equal(qm, m[:nqkv])
    order = O.gate_up_order(inter) + nqkv
    assert torch.equal(gs[:, 0], s[order, 0]) and torch.equal(gm, m[order]) and torch.equal(gq, q[order])
    # row 2c = gate channel c, row 2c + 1 = up channel c
    assert gs[1, 0].item() == nqkv + inter and gs[2, 0].item() == nqkv + 1


def test_attention_argument_checks(native_lib):
    L = native_lib
    assert L.rb_attn_decode_workspace(24, 8, 128) > 24 * 128 * 4
    assert L.rb_attn_decode_workspace(24, 8, 64) == -1           # head_dim 128 only
    assert L.rb_attn_decode_workspace(18, 2, 128) == -1          # rep 9 > 8
    assert L.rb_attn_decode_workspace(10, 4, 128) == -1          # n_q_heads not a multiple of n_kv_heads
    need = L.rb_attn_decode_workspace(8, 2, 128)
    args = [A, B, C, POS, 0x50000, 8, 2, 128, 64, 0.088, 0x60000, need, _lib.F16, 0, None]

    def with_(**kw):
        a = list(args)
        names = ["q", "k", "v", "pos", "out", "nq", "nkv", "hd", "S", "scale", "ws", "ws_bytes", "dt"]
        for k, v in kw.items():
            a[names.index(k)] = v
        return L.rb_attn_decode(*a)

    assert with_(ws_bytes=need - 1) == _lib.ERR_SHAPE
    assert with_(S=0) == _lib.ERR_SHAPE
    assert with_(hd=64) == _lib.ERR_SHAPE
    assert with_(pos=None) == _lib.ERR_NULL
    assert with_(ws=None) == _lib.ERR_NULL
    assert with_(dt=_lib.F32) == _lib.ERR_DTYPE
    assert with_(out=0x50008) == _lib.ERR_ALIGN
    assert with_(scale=float("nan")) == _lib.ERR_SHAPE


def test_embedding_prologue_argument_checks(native_lib):
    L = native_lib

    def emb(**kw):
        ln = add_ln(x=None, a=None, b=None)
        ln.emb_q, ln.emb_s, ln.tok, ln.vocab, ln.emb_s_dtype = 0xA0000, 0xB0000, 0xC0000, 100, _lib.F32
        for k, v in kw.items():
            setattr(ln, k, v)
        return ln

    assert L.rb_add_layernorm(ctypes.byref(emb(x=0x50000)), _lib.F16, 0, None) == _lib.ERR_SHAPE   # x and emb
    assert L.rb_add_layernorm(ctypes.byref(emb(a=0x60000)), _lib.F16, 0, None) == _lib.ERR_SHAPE
    assert L.rb_add_layernorm(ctypes.byref(emb(tok=None)), _lib.F16, 0, None) == _lib.ERR_NULL
    assert L.rb_add_layernorm(ctypes.byref(emb(emb_s=None)), _lib.F16, 0, None) == _lib.ERR_NULL
    assert L.rb_add_layernorm(ctypes.byref(emb(vocab=0)), _lib.F16, 0, None) == _lib.ERR_SHAPE
    assert L.rb_add_layernorm(ctypes.byref(emb(emb_s_dtype=_lib.BF16)), _lib.F16, 0, None) == _lib.ERR_DTYPE
    assert L.rb_add_layernorm(ctypes.byref(emb(emb_q=0xA0008)), _lib.F16, 0, None) == _lib.ERR_ALIGN
    assert call(L, [desc(x=None)], ln=emb(tok=None)) == _lib.ERR_NULL


def test_sampler_argument_checks(native_lib):
    L = native_lib

    def smp(**kw):
        s = _lib.Sampler(A, _lib.F16, 16385, 16384, B, 30, 1.25, C, POS, _lib.BF16, 2048, A, B, C, _lib.BF16, 512,
                         A, B, C, 50152, 8, 0x50000, 0x60000, 0x70000, 64, 0x80000)
        for k, v in kw.items():
            setattr(s, k, v)
        return L.rb_sample(ctypes.byref(s), 0, None)

    assert L.rb_sample(None, 0, None) == _lib.ERR_NULL
    assert smp(n_vocab=0) == _lib.ERR_SHAPE
    assert smp(n_vocab=32769) == _lib.ERR_SHAPE          # the pick CTA takes at most 32768 logits
    assert smp(top_k=33) == _lib.ERR_SHAPE
    assert smp(top_k=0) == _lib.ERR_SHAPE
    assert smp(H=8193) == _lib.ERR_SHAPE
    assert smp(inv_temp=float("nan")) == _lib.ERR_SHAPE
    assert smp(u=None) == _lib.ERR_NULL
    assert smp(step=None) == _lib.ERR_NULL
    assert smp(out=None) == _lib.ERR_NULL                # out_len > 0 needs out
    assert smp(logits_dtype=7) == _lib.ERR_DTYPE
    assert smp(w1_dtype=9) == _lib.ERR_DTYPE


def test_fused_attention_argument_checks(native_lib):
    """rb_attn_src (attention inside the o_proj/down_proj launch) is validated before any CUDA call."""
    L = native_lib
    OUT = 0x90000
    need = L.rb_attn_decode_workspace(8, 2, 128)

    def run(descs, flags=0, **kw):
        src = _lib.AttnSrc(A, B, C, POS, OUT, 8, 2, 128, 64, 0.088, 0xA0000, need)
        for k, v in kw.items():
            setattr(src, k, v)
        d = (_lib.GemvDesc * len(descs))(*descs)
        return L.rb_gemv_int4_fused(d, None, len(descs), None, ctypes.byref(src), None, 0, _lib.F16, _lib.F16,
                                    flags, None)

    o_proj = desc(x=OUT, N=256, K=8 * 128)
    down = desc(x=A, N=256, K=256)
    assert run([down]) == _lib.ERR_SHAPE                                   # no entry reads the attention output
    assert run([down, desc(x=OUT, N=256, K=512)]) == _lib.ERR_SHAPE        # K != n_q_heads * head_dim
    assert run([down, o_proj], n_q_heads=10, n_kv_heads=2) == _lib.ERR_SHAPE   # 5 query heads per key-value head
    assert run([down, o_proj], q=None) == _lib.ERR_NULL
    assert run([down, o_proj], ws=None) == _lib.ERR_NULL
    assert run([down, o_proj], k_cache=0x30008) == _lib.ERR_ALIGN
    assert run([down, o_proj], ws_bytes=need - 1) == _lib.ERR_SHAPE
    assert run([down, o_proj], cache_len=0) == _lib.ERR_SHAPE
    assert run([down, o_proj], flags=_lib.FLAG_KERNEL_TC) == _lib.ERR_SHAPE    # runs on the warp-MMA kernel only


def test_scales8_descriptor_checks(native_lib):
    """rb_gemv_desc::s_row (8-bit scales) is validated before any CUDA call: m may then be NULL, s_row must be
    4-byte aligned, and such a list cannot be forced onto the warp-MMA kernel or run with fused attention."""
    L = native_lib

    def d8(s_row=0xB0000, m=None, **kw):
        d = desc(**kw)
        d.m = m
        d.s_row = s_row
        return d

    one = lambda d: (_lib.GemvDesc * 1)(d)  # noqa: E731
    plain = desc()
    plain.m = None
    assert L.rb_gemv_int4_multi(one(plain), 1, _lib.F16, _lib.F16, 0, None) == _lib.ERR_NULL  # fp16 needs m
    assert L.rb_gemv_int4_multi(one(d8(s_row=0xB0002)), 1, _lib.F16, _lib.F16, 0, None) == _lib.ERR_ALIGN
    assert L.rb_gemv_int4_multi(one(d8()), 1, _lib.F16, _lib.F16, _lib.FLAG_KERNEL_MMA, None) == _lib.ERR_SHAPE
    assert L.rb_gemv_int4_workspace(one(d8()), 1, _lib.FLAG_KERNEL_MMA) == -_lib.ERR_SHAPE
    assert L.rb_gemv_int4_fused(one(d8()), None, 1, None, None, None, 0, _lib.F16, _lib.F16,
                                _lib.FLAG_KERNEL_MMA, None) == _lib.ERR_SHAPE
    OUT = 0x90000
    need = L.rb_attn_decode_workspace(8, 2, 128)
    src = _lib.AttnSrc(A, B, C, POS, OUT, 8, 2, 128, 64, 0.088, 0xA0000, need)
    two = (_lib.GemvDesc * 2)(desc(x=A), d8(x=OUT, K=8 * 128))
    assert L.rb_gemv_int4_fused(two, None, 2, None, ctypes.byref(src), None, 0, _lib.F16, _lib.F16, 0,
                                None) == _lib.ERR_SHAPE                   # fused attention: warp-MMA kernel only
