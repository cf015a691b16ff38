"""Drop-in for rumik-fast kernels/mm_int4.py on B200: the int4-weight prefill matmul on tcgen05 tensor cores.

    mm_int4(x, q, s, m, BM=None, BN=64, num_warps=4, num_stages=3) -> y     (kernels/mm_int4.py:59)
    warmup(shapes)                                                          (kernels/mm_int4.py:49)
    G = 128
Y[T, N] = X[T, K] @ W^T with W in the int4 group-128 layout. X may be fp16 or bf16 and strided in its
first dimension; y has X's dtype and is newly allocated, as in the reference. The tensor-core operands are
fp16 (both operands of a kind::f16 MMA must share a type, and fp16 keeps the dequantised weight's rounding
~8x smaller than bf16): the kernel converts a bf16 X to fp16 in shared memory, so a call launches the kernel
(and, when K is split over the SMs, its reduction) and no torch op. The split-K workspace is kept per (device,
stream) and only grows; calls on one stream are ordered, so they can share it. The Triton tile knobs are
accepted and ignored. (While a CUDA graph is being captured each call takes its own workspace from the
graph's pool instead, so that graphs replayed on different streams never share one.) The kernel is compiled
ahead of time, so warmup() only performs one tiny call per shape
(it makes the first call inside a CUDA-graph capture cheap).
"""
import torch

from . import _lib, config
from .cuda_gemv import _on_device, _require

G = 128


def mm_int4(x, q, s, m, BM=None, BN=64, num_warps=4, num_stages=3, out=None):
    N, K = q.shape[0], q.shape[1] * 2
    _require(x.is_cuda and x.dim() == 2 and x.shape[1] == K, f"x must be a CUDA [T, {K}] tensor")
    _require(x.dtype in (torch.float16, torch.bfloat16), f"x must be fp16 or bf16, got {x.dtype}")
    _require(q.dtype == torch.uint8 and q.is_contiguous(), "q must be a contiguous uint8 [N, K/2] tensor")
    _require(K % G == 0, f"K={K} must be a multiple of {G}")
    for t, nm in ((s, "s"), (m, "m")):
        _require(t.dtype == torch.float16 and t.is_contiguous() and tuple(t.shape) == (N, K // G),
                 f"{nm} must be a contiguous fp16 [{N}, {K // G}] tensor")
    out_dtype = x.dtype
    if x.stride(1) != 1 or x.stride(0) % 8 != 0 or x.data_ptr() % 16 != 0:
        x = x.contiguous()
    T = x.shape[0]
    y = torch.empty(T, N, device=x.device, dtype=out_dtype) if out is None else out
    _require(y.shape == (T, N) and y.stride(1) == 1, "out must be [T, N] with unit column stride")
    L = _lib.lib()
    with _on_device(x.device):
        # a call with few 128-row x token-chunk tiles splits K over the idle SMs through an fp32 workspace
        ws_bytes = L.rb_mm_int4_workspace(T, N, K)
        ws = _workspace(x.device, ws_bytes) if ws_bytes > 0 else None
        st = L.rb_mm_int4_ws(x.data_ptr(), _lib.dtype_code(x.dtype), x.stride(0), q.data_ptr(), s.data_ptr(),
                             m.data_ptr(), y.data_ptr(), _lib.dtype_code(y.dtype), y.stride(0), T, N, K,
                             None if ws is None else ws.data_ptr(), ws_bytes, config.flags(),
                             _lib.stream_ptr(x.device))
    _lib.check("rb_mm_int4", st)
    return y


class MmInt4Set:
    """A fixed list of independent prefill products with one token count, run as persistent launches of up to 52
    products each (rb_mm_int4_list): entries (x [M, K], q, s, m, y [M, N]) in mm_int4's layout, one x dtype and
    one y dtype. Built once; every call launches the list (graph-capture safe). The products' work items share
    one launch instead of one launch, fill and tail each, and no split-K workspace is needed."""

    def __init__(self, entries):
        _require(len(entries) > 0, "empty product list")
        self.entries = list(entries)
        x0, y0 = self.entries[0][0], self.entries[0][4]
        self.device, self.M = x0.device, x0.shape[0]
        self.x_dtype, self.y_dtype = x0.dtype, y0.dtype
        _require(self.x_dtype in (torch.float16, torch.bfloat16), f"x must be fp16 or bf16, got {self.x_dtype}")
        _require(self.y_dtype in (torch.float16, torch.bfloat16), f"y must be fp16 or bf16, got {self.y_dtype}")
        descs = (_lib.MmDesc * len(self.entries))()
        for i, (x, q, s, m, y) in enumerate(self.entries):
            N, K = q.shape[0], q.shape[1] * 2
            _require(x.is_cuda and x.device == self.device and x.dim() == 2 and x.shape == (self.M, K),
                     f"entry {i}: x must be a CUDA [{self.M}, {K}] tensor on {self.device}")
            _require(x.dtype == self.x_dtype and y.dtype == self.y_dtype, "one x dtype and one y dtype per list")
            _require(x.stride(1) == 1 and x.stride(0) % 8 == 0, f"entry {i}: x rows must be contiguous, pitch % 8 == 0")
            _require(q.dtype == torch.uint8 and q.is_contiguous(), f"entry {i}: q must be a contiguous uint8 [N, K/2]")
            _require(K % G == 0, f"entry {i}: K={K} must be a multiple of {G}")
            for t, nm in ((s, "s"), (m, "m")):
                _require(t.dtype == torch.float16 and t.is_contiguous() and tuple(t.shape) == (N, K // G),
                         f"entry {i}: {nm} must be a contiguous fp16 [{N}, {K // G}] tensor")
            _require(y.shape == (self.M, N) and y.stride(1) == 1 and y.stride(0) % 8 == 0,
                     f"entry {i}: y must be [{self.M}, {N}] with unit column stride and pitch % 8 == 0")
            descs[i] = _lib.MmDesc(x.data_ptr(), x.stride(0), q.data_ptr(), s.data_ptr(), m.data_ptr(),
                                   y.data_ptr(), y.stride(0), N, K)
        self._descs = descs

    def __call__(self):
        L = _lib.lib()
        with _on_device(self.device):
            st = L.rb_mm_int4_list(self._descs, len(self.entries), self.M, _lib.dtype_code(self.x_dtype),
                                   _lib.dtype_code(self.y_dtype), config.flags(), _lib.stream_ptr(self.device))
        _lib.check("rb_mm_int4_list", st)


_WS = {}
_RETIRED = []  # outgrown workspaces stay allocated: work already queued on the stream may still use them


def _workspace(device, nbytes):
    """The split-K workspace of the current stream on `device`, grown to at least nbytes."""
    if torch.cuda.is_current_stream_capturing():
        return torch.empty((nbytes + 3) // 4, device=device, dtype=torch.float32)
    key = (device.index, _lib.stream_ptr(device))
    ws = _WS.get(key)
    if ws is None or ws.numel() * 4 < nbytes:
        if ws is not None:
            _RETIRED.append(ws)
        ws = torch.empty((nbytes + 3) // 4, device=device, dtype=torch.float32)
        _WS[key] = ws
    return ws


def warmup(shapes):
    """One tiny call per (N, K) so nothing is initialised lazily later (kernels/mm_int4.py:49-56)."""
    for n, k in shapes:
        q = torch.zeros(n, k // 2, device="cuda", dtype=torch.uint8)
        s = torch.zeros(n, k // G, device="cuda", dtype=torch.float16)
        for T in (17, 33):
            mm_int4(torch.zeros(T, k, device="cuda", dtype=torch.bfloat16), q, s, s)
    torch.cuda.synchronize()
