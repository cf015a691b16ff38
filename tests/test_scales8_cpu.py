"""8-bit double-quantised scales (rumik_fast_b200.scales8) against the oracle's restatement of the format, on CPU.

The reference names the format as its next byte saving but has none (engine/README.md:192-193), so there is no
reference output to pin to: these tests pin the product's packer and decoder to the oracle bit for bit, check the
code table's definition, and bound what the format costs in accuracy against the reference's fp16 scales."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O
from rumik_fast_b200 import _lib, scales8
from rumik_fast_b200 import synthetic as syn


def _np(sc):
    return sc.sz.numpy().view(np.uint16), sc.s_row.numpy()


def test_code_table():
    t = O.sc8_table()
    assert t.dtype == np.float32 and np.all(np.diff(t) > 0)
    assert t[255] == O.SC8_MAX == np.float32(1.9375)
    b = np.arange(256)
    assert np.array_equal(t, (2.0 ** ((b >> 4) - 15) * (1 + (b & 15) / 16)).astype(np.float32))
    assert torch.equal(scales8._table("cpu"), torch.from_numpy(t))


def _cases():
    g = syn.generator(11, "cpu")
    yield "synthetic", *syn.int4_weights(512, 3072, g, "cpu")[1:]
    rng = np.random.default_rng(5)
    w = rng.standard_normal((300, 1024)).astype(np.float32) * rng.uniform(0.001, 0.1, (300, 1))
    _, s, m = O.quantize_int4(w)
    yield "quantised", torch.from_numpy(s), torch.from_numpy(m)
    # edges: an all-zero row, zero-scale groups (constant weights), mins that push the zero point out of range
    s = torch.from_numpy(rng.uniform(0.001, 0.02, (6, 16)).astype(np.float16))
    m = (-7.5 * s.float()).half()
    s[0] = 0
    m[0] = 0
    s[1, :4] = 0
    m[1, :4] = torch.tensor([0.5, -0.5, 0.0, 3.0]).half()
    m[2] = (5.0 * s[2].float()).half()          # z < 0: clamped to 0
    m[3] = (-30.0 * s[3].float()).half()        # z > 15.94: clamped to 255
    s[4, 0] = 65504.0                           # the fp16 maximum
    s[5] = torch.tensor([6e-8] * 16).half()     # subnormal scales
    yield "edges", s, m


@pytest.mark.parametrize("name,s,m", list(_cases()), ids=lambda v: v if isinstance(v, str) else "")
def test_pack_and_unpack_match_the_oracle(name, s, m):
    sc = scales8.pack(s, m)
    scales8.check(sc, s.shape[0], s.shape[1])
    sz_o, row_o = O.pack_scales8(s.numpy(), m.numpy())
    sz, row = _np(sc)
    assert np.array_equal(row, row_o)
    assert np.array_equal(sz, sz_o)
    s16, m16 = scales8.unpack(sc)
    s16_o, m16_o = O.unpack_scales8(sz_o, row_o)
    assert np.array_equal(s16.numpy().view(np.uint16), s16_o.view(np.uint16))
    assert np.array_equal(m16.numpy().view(np.uint16), m16_o.view(np.uint16))


def test_accuracy_bounds():
    """Where the zero point is in range: the decoded scale is within 1/32 (plus one fp16 rounding) of the fp16
    scale, and the dequantised weights stay within a small fraction of the int4 step of the fp16-scale ones."""
    g = syn.generator(12, "cpu")
    q, s, m = syn.int4_weights(256, 3072, g, "cpu")
    sz, row = O.pack_scales8(s.numpy(), m.numpy())
    s8, m8 = O.unpack_scales8(sz, row)
    s32 = s.float().numpy()
    assert np.max(np.abs(s8.astype(np.float32) - s32) / s32) <= 1 / 32 + 2 ** -11
    w16 = O.dequantize_int4(q.numpy(), s.numpy(), m.numpy())
    w8 = O.dequantize_int4(q.numpy(), s8, m8)
    step = np.repeat(s32, 128, axis=1)
    assert np.max(np.abs(w8 - w16) / step) < 0.5
    rng = np.random.default_rng(0)
    wt = rng.standard_normal((256, 3072)).astype(np.float32) * 0.02
    qq, ss, mm = O.quantize_int4(wt)
    s8, m8 = O.unpack_scales8(*O.pack_scales8(ss, mm))
    e16 = np.linalg.norm(O.dequantize_int4(qq, ss, mm) - wt) / np.linalg.norm(wt)
    e8 = np.linalg.norm(O.dequantize_int4(qq, s8, m8) - wt) / np.linalg.norm(wt)
    assert e8 < 1.05 * e16                  # measured: 0.1008 against 0.0998


def test_pack_rejects_bad_input():
    s = torch.ones(4, 3, dtype=torch.float16)
    with pytest.raises(RuntimeError):
        scales8.pack(s.float(), s)
    with pytest.raises(RuntimeError):
        scales8.pack(s, s[:, :2])
    with pytest.raises(RuntimeError):
        scales8.check(scales8.pack(s, s), 4, 4)


def test_descriptor_layout():
    """struct rb_gemv_desc: five pointers, N, K, s_row, then the int8-entry kind w8 (72 bytes with padding)."""
    assert ctypes.sizeof(_lib.GemvDesc) == 72
    assert _lib.GemvDesc.s_row.offset == 56
    assert _lib.GemvDesc.w8.offset == 64
    d = _lib.GemvDesc(1, 2, 3, 4, 5, 6, 7)
    assert d.s_row is None and d.w8 == _lib.W8_NONE == 0


try:
    from hypothesis import given, settings, strategies as st
    from hypothesis.extra import numpy as hnp
except ImportError:  # pragma: no cover
    given = None

if given is not None:
    _f16 = hnp.arrays(np.float16, st.tuples(st.integers(1, 6), st.integers(1, 9)),
                      elements=st.floats(min_value=0, max_value=65504, width=16, allow_nan=False))

    @settings(max_examples=60, deadline=None)
    @given(_f16, st.data())
    def test_pack_matches_oracle_on_arbitrary_grids(s, data):
        """Any finite non-negative fp16 scales (zeros, subnormals, the fp16 maximum) and any finite fp16 mins:
        the torch packer and decoder agree with the oracle bit for bit (overflowing products included)."""
        m = data.draw(hnp.arrays(np.float16, s.shape,
                                 elements=st.floats(min_value=-65504, max_value=65504, width=16, allow_nan=False)))
        sc = scales8.pack(torch.from_numpy(s), torch.from_numpy(m))
        sz_o, row_o = O.pack_scales8(s, m)
        sz, row = _np(sc)
        assert np.array_equal(row, row_o) and np.array_equal(sz, sz_o)
        s16, m16 = scales8.unpack(sc)
        s16_o, m16_o = O.unpack_scales8(sz_o, row_o)
        assert np.array_equal(s16.numpy().view(np.uint16), s16_o.view(np.uint16))
        assert np.array_equal(m16.numpy().view(np.uint16), m16_o.view(np.uint16))
