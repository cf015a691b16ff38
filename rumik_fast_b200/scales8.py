"""8-bit double-quantised scales for the int4 group-128 format.

rumik-fast stores one fp16 scale and one fp16 min per 128 weights (4 bytes next to the group's 64 code bytes,
kernels/int4_gemv.py:16-24) and names quantising them to 8 bits as its next byte saving (engine/README.md:192-193);
it has no implementation. This module defines one and packs it:

  * per group one 16-bit word: the low byte b is an unsigned E4M4 scale code, sc8(b) = 2^((b >> 4) - 15) *
    (1 + (b & 15) / 16) (the fp32 whose bits are (b << 19) + 0x38000000), the high byte z a zero point in 1/16 steps;
  * per row one fp32 factor s_row = max(scale) / 1.9375 (1.9375 = sc8(255));
  * decoding gives the fp16 scale and min of the reference format: s = fp16(sc8(b) * s_row),
    m = fp16(-(z / 16) * s), so that every kernel of the fp16 format computes on them unchanged.

The scale keeps 4 significant bits (relative error at most 1/32), the zero point is chosen so that the weights
match at the middle code 7.5. Groups read 2 bytes of scales instead of 4: 66 instead of 68 bytes per group.
The GEMV-list kernel on the tensor cores decodes them while streaming (Int4GemvSet, rb_gemv_int4_multi with
rb_gemv_desc::s_row); everything else takes the fp16 pair from unpack().
"""
from typing import NamedTuple

import torch

SC8_MAX = 1.9375


class Scales8(NamedTuple):
    """The 8-bit scales of one int4 matrix: sz int16 [N, K/128] (the 16-bit words, as bit patterns) and s_row
    float32 [N]. Pass it as an entry's `s` (with m None) where the GEMV list accepts it."""
    sz: torch.Tensor
    s_row: torch.Tensor


def _table(device):
    b = torch.arange(256, dtype=torch.int32, device=device)
    return ((b << 19) + 0x38000000).view(torch.float32)


def pack(s, m):
    """fp16 scale and min [N, G] -> Scales8, on their device. The scale code is the nearest sc8 value to
    s / s_row (ties to the lower code; 0 for a row whose scales are all 0); the zero point is
    rint(16 * (7.5 - (7.5 s + m) / s')) clamped to 0..255 with s' the decoded fp16 scale (0 where s' is 0).
    fp32 arithmetic, one rounding per operation."""
    if s.dtype != torch.float16 or m.dtype != torch.float16 or s.shape != m.shape or s.dim() != 2:
        raise RuntimeError("s and m must be fp16 [N, G] tensors of one shape")
    s32, m32 = s.float(), m.float()
    mx = s32.amax(dim=1)
    s_row = mx / torch.full_like(mx, SC8_MAX)  # a true division (CUDA divides by a scalar via its reciprocal)
    tab = _table(s.device)
    mid = (tab[:-1] + tab[1:]) * 0.5
    ok = (s_row > 0)[:, None]
    r = torch.where(ok, s32 / torch.where(ok, s_row[:, None], torch.ones_like(s_row[:, None])), 0.0)
    b = torch.where(ok, torch.searchsorted(mid, r.contiguous(), right=False), 0).to(torch.int32)
    sp = (tab[b.long()] * s_row[:, None]).half().float()
    has = sp > 0
    t = (s32 * 7.5) + m32
    u = t / torch.where(has, sp, torch.ones_like(sp))
    zf = (7.5 - u) * 16.0
    z = torch.where(has, torch.round(zf).clamp(0, 255), 0.0).to(torch.int32)
    word = b | (z << 8)
    sz = torch.where(word >= 32768, word - 65536, word).to(torch.int16)
    return Scales8(sz.contiguous(), s_row.contiguous())


def unpack(sc):
    """Scales8 -> the fp16 scale and min [N, G] it stands for (what the GEMV kernel decodes while streaming)."""
    w = sc.sz.to(torch.int32) & 0xFFFF
    tab = _table(sc.sz.device)
    s16 = (tab[(w & 0xFF).long()] * sc.s_row.float()[:, None]).half()
    m16 = (-((w >> 8).float() * 0.0625) * s16.float()).half()
    return s16, m16


def check(sc, N, G, device=None, where=""):
    """Raise RuntimeError (the reference's argument-error type) unless sc is a Scales8 for an [N, G] scale grid
    (on `device` when given)."""
    ok = (isinstance(sc, Scales8) and sc.sz.dtype == torch.int16 and tuple(sc.sz.shape) == (N, G)
          and sc.sz.is_contiguous() and sc.s_row.dtype == torch.float32 and tuple(sc.s_row.shape) == (N,)
          and sc.s_row.is_contiguous())
    if ok and device is not None:
        ok = sc.sz.device == device and sc.s_row.device == device
    if not ok:
        raise RuntimeError(f"{where}8-bit scales must be Scales8(sz int16 [{N}, {G}], s_row float32 [{N}]), "
                           "contiguous, on the GEMV's device")
