"""A fixed list of independent int4 GEMVs executed as ONE persistent kernel launch (rb_gemv_int4_multi).

A decode step issued as one launch per projection pays a fixed cost per launch that on B200 is comparable
to the whole step's weight-streaming time. When the GEMVs of a list are independent (all inputs ready at
launch, as in rumik-fast's projection-set benchmark, kernels/bench_gemv.py:83-113), Int4GemvSet streams all
of their weights through one persistent kernel instead:

    step = Int4GemvSet([(x_h, *w_qkv, y_qkv), (x_h, *w_o, y_o), ...])   # built once
    step()                                                             # every call: all GEMVs

Entries are (x, q, s, m, y) with the layout of gemv_int4_cuda (x [K] fp16/bf16, q uint8 [N, K/2], s and m
fp16 [N, K/128], y [N]); all x share one dtype and all y share one dtype. Calling is graph-capture safe.
An entry may carry 8-bit double-quantised scales instead (s = scales8.Scales8, m = None); a list with such an
entry runs on the tcgen05 kernel. An entry may also be int8 rows, y = s * (q @ x), the layout of gemv_int8_cuda
(the int8 head: q torch.int8 [N, K], or uint8 [N, K] = int8 + 128 as quantize_int8_rows stores it; s fp32 or
fp16 [N]; m None): its rows stream through the same tcgen05 launch as more work items.
"""
import ctypes

import torch

from . import _lib, config, scales8
from .cuda_gemv import _on_device, _require

G = 128


class Int4GemvSet:
    """kernel: None (by the list's size: a decode layer's projections on the warp-MMA kernel, a whole step's on
    the tcgen05 kernel), "tc" or "mma"."""

    def __init__(self, entries, kernel=None):
        _require(len(entries) > 0, "empty GEMV list")
        self.entries = list(entries)
        x0, y0 = self.entries[0][0], self.entries[0][4]
        self.device = x0.device
        self.x_dtype, self.y_dtype = x0.dtype, y0.dtype
        descs = (_lib.GemvDesc * len(self.entries))()
        for i, (x, q, s, m, y) in enumerate(self.entries):
            w8 = is_int8_entry(q, s, m)
            N, K = q.shape[0], q.shape[1] * (1 if w8 else 2)
            _require(x.is_cuda and x.device == self.device, "all tensors must be on one CUDA device")
            _require(x.dtype == self.x_dtype and y.dtype == self.y_dtype, "one x dtype and one y dtype per set")
            _require(x.dtype in (torch.float16, torch.bfloat16), f"x must be fp16 or bf16, got {x.dtype}")
            _require(y.dtype in (torch.float16, torch.bfloat16), f"y must be fp16 or bf16, got {y.dtype}")
            _require(x.numel() == K and x.is_contiguous(), f"entry {i}: x must be a contiguous [{K}] vector")
            _require(y.numel() == N and y.is_contiguous(), f"entry {i}: y must be a contiguous [{N}] vector")
            _require(q.dtype in ((torch.int8, torch.uint8) if w8 else (torch.uint8,)) and q.is_contiguous(),
                     f"entry {i}: q must be contiguous uint8 [N, K/2] (int4) or int8/uint8 [N, K] (int8 rows)")
            _require(K % G == 0, f"entry {i}: K={K} must be a multiple of {G}")
            _require(q.device == self.device, f"entry {i}: q must be on {self.device}")
            if w8:
                _require(s.dtype in (torch.float32, torch.float16) and s.is_contiguous() and s.numel() == N
                         and s.device == self.device, f"entry {i}: s must be a contiguous fp32/fp16 [{N}] tensor")
                descs[i] = _lib.GemvDesc(x.data_ptr(), y.data_ptr(), q.data_ptr(),
                                         s.data_ptr() if s.dtype == torch.float16 else None, None, N, K)
                if s.dtype == torch.float32:
                    descs[i].s_row = s.data_ptr()
                descs[i].w8 = _lib.W8_SIGNED if q.dtype == torch.int8 else _lib.W8_OFFSET
                continue
            sp, mp = _scale_ptrs(s, m, N, K, i, self.device)
            descs[i] = _lib.GemvDesc(x.data_ptr(), y.data_ptr(), q.data_ptr(), sp, mp, N, K)
            if isinstance(s, scales8.Scales8):
                descs[i].s_row = s.s_row.data_ptr()
        self._descs = descs
        self.bytes = sum(entry_bytes(q, s, x, y) for x, q, s, m, y in self.entries)
        self.kflags = _lib.KERNEL_FLAGS[kernel]
        self.ws = workspace(descs, len(self.entries), self.device, self.kflags)

    def __call__(self):
        L = _lib.lib()
        with _on_device(self.device):
            st = L.rb_gemv_int4_multi_ws(self._descs, len(self.entries), _ws_ptr(self.ws), _ws_len(self.ws),
                                         _lib.dtype_code(self.x_dtype), _lib.dtype_code(self.y_dtype),
                                         config.flags() | self.kflags, _lib.stream_ptr(self.device))
        _lib.check("rb_gemv_int4_multi_ws", st)


def is_int8_entry(q, s, m):
    """An entry of int8 rows: m is None and s is the one-dimensional tensor of per-row scales (an int4 entry has
    fp16 scales [N, K/128] or a scales8.Scales8)."""
    return m is None and isinstance(s, torch.Tensor) and s.dim() == 1 and q.dim() == 2


def _scale_ptrs(s, m, N, K, i, device):
    """(s, m) pointers of an entry: fp16 scale and min tensors, or a scales8.Scales8 as s with m None."""
    if isinstance(s, scales8.Scales8):
        _require(m is None, f"entry {i}: with 8-bit scales m must be None")
        scales8.check(s, N, K // G, device, where=f"entry {i}: ")
        return s.sz.data_ptr(), None
    for t, nm in ((s, "s"), (m, "m")):
        _require(isinstance(t, torch.Tensor) and t.dtype == torch.float16 and t.is_contiguous()
                 and tuple(t.shape) == (N, K // G), f"entry {i}: {nm} must be a contiguous fp16 [{N}, {K // G}] tensor")
    return s.data_ptr(), m.data_ptr()


def entry_bytes(q, s, x, y):
    """HBM bytes one GEMV must move: codes, scales (fp16 pair or 8-bit word per group, plus the row factors; the
    row scales of int8 rows), x and y."""
    if isinstance(s, scales8.Scales8):
        sb = 2 * s.sz.numel() + 4 * s.s_row.numel()
    elif s.dim() == 1:
        sb = s.element_size() * s.numel()
    else:
        sb = 4 * s.numel()
    return q.numel() + sb + x.element_size() * x.numel() + y.element_size() * y.numel()


def workspace(descs, count, device, kflags=0):
    """The zeroed split-K workspace of a GEMV list (None when its launches do not split K): on the tcgen05
    kernel a list with fewer 128-row blocks than 3 x the SM count spreads each block over several converter
    sets."""
    with _on_device(device):
        need = _lib.lib().rb_gemv_int4_workspace(descs, count, kflags)
    if need < 0:
        _lib.check("rb_gemv_int4_workspace", -need)
    return torch.zeros(need, dtype=torch.uint8, device=device) if need > 0 else None


def _ws_ptr(ws):
    return ws.data_ptr() if ws is not None else None


def _ws_len(ws):
    return ws.numel() if ws is not None else 0
