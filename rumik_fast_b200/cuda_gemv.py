"""Drop-in for rumik-fast kernels/cuda_gemv.py on B200: the decode-step GEMVs.

Same public names and call signatures as the reference module (kernels/cuda_gemv.py:223-249):
    gemv_int4_cuda(x, q, s, m, out=None, warps=None, rows=None) -> y
    gemv_int8_cuda(x, q, s, out=None) -> y
    quantize_int8_rows(w, pad_to=16) -> (q, s)
    SHAPE  (block-shape table; accepted for compatibility, the native side picks its own launch shape)
The kernels are the hand-written sm_100a CUDA in csrc/ reached through the C ABI (include/rumik_b200.h);
there is no other code path. Differences from the reference, all widening its contract:
  * x may be fp16 or bf16, and [K] or [B, K] with B <= 16 per kernel launch (larger B is split); the output
    dtype is out.dtype when `out` is given, else x.dtype (the reference is bf16-only).
  * gemv_int8_cuda accepts signed int8 codes (torch.int8) as well as uint8 = int8 + 128, an fp16 or fp32
    row scale, and any N (no padding to a multiple of 16 required).
Errors (shape, dtype, device, alignment) raise RuntimeError like the reference's TORCH_CHECK
(kernels/cuda_gemv.py:121,135,190).
"""
import torch

from . import _lib, config

G = 128
SHAPE = {}   # kernels/cuda_gemv.py:223 - kept so code that fills it keeps working; not consulted


def _require(cond, msg):
    if not cond:
        raise RuntimeError(msg)


def _act(x, K, name="x"):
    _require(x.is_cuda, f"{name} must be a CUDA tensor")
    _require(x.dtype in (torch.float16, torch.bfloat16), f"{name} must be fp16 or bf16, got {x.dtype}")
    _require(x.dim() in (1, 2) and x.shape[-1] == K, f"{name} must be [K] or [B, K] with K={K}, got {tuple(x.shape)}")
    _require(x.stride(-1) == 1, f"{name} must have unit stride in its last dimension")
    batch = 1 if x.dim() == 1 else x.shape[0]
    ld = K if x.dim() == 1 else x.stride(0)
    return batch, ld


def _out(x, N, out):
    if out is None:
        return torch.empty(x.shape[:-1] + (N,), device=x.device, dtype=x.dtype)
    _require(out.is_cuda and out.device == x.device, "out must be on x's device")
    _require(out.dtype in (torch.float16, torch.bfloat16), f"out must be fp16 or bf16, got {out.dtype}")
    _require(out.shape[-1] == N and out.numel() == (N if x.dim() == 1 else x.shape[0] * N),
             f"out has shape {tuple(out.shape)}, expected {tuple(x.shape[:-1]) + (N,)}")
    _require(out.stride(-1) == 1, "out must have unit stride in its last dimension")
    return out


class _on_device:
    """Make `dev` current for the call only when it is not already (cheap common case)."""

    def __init__(self, dev):
        self.dev = dev
        self.ctx = None

    def __enter__(self):
        if self.dev.index != torch.cuda.current_device():
            self.ctx = torch.cuda.device(self.dev)
            self.ctx.__enter__()

    def __exit__(self, *a):
        if self.ctx is not None:
            self.ctx.__exit__(*a)


def gemv_int4_cuda(x, q, s, m, out=None, warps=None, rows=None):
    """y = W x for int4 group-128 weights (q uint8 [N, K/2], s/m fp16 [N, K/128]); x [K] or [B, K].

    `warps` and `rows` (the reference's block-shape knobs) are accepted and ignored."""
    N, K = q.shape[0], q.shape[1] * 2
    _require(q.dtype == torch.uint8 and q.is_contiguous(), "q must be a contiguous uint8 [N, K/2] tensor")
    _require(K % G == 0, f"K={K} must be a multiple of {G}")
    for t, nm in ((s, "s"), (m, "m")):
        _require(t.dtype == torch.float16 and t.is_contiguous() and tuple(t.shape) == (N, K // G),
                 f"{nm} must be a contiguous fp16 [{N}, {K // G}] tensor")
        _require(t.device == q.device, f"{nm} must be on q's device")
    _require(q.device == x.device, "x and q must be on the same device")
    batch, ldx = _act(x, K)
    y = _out(x, N, out)
    ldy = N if y.dim() == 1 else y.stride(0)
    L = _lib.lib()
    with _on_device(x.device):
        st = L.rb_gemv_int4(x.data_ptr(), _lib.dtype_code(x.dtype), ldx, q.data_ptr(), s.data_ptr(), m.data_ptr(),
                            y.data_ptr(), _lib.dtype_code(y.dtype), ldy, N, K, batch, config.flags(),
                            _lib.stream_ptr(x.device))
    _lib.check("rb_gemv_int4", st)
    return y


def quantize_int8_rows(w, pad_to=16):
    """bf16 [N, K] -> (uint8 [N', K] = int8 + 128, fp32 scale [N']), rows zero-padded to a multiple of pad_to.

    The reference's load-time quantiser (kernels/cuda_gemv.py:234-242), same arithmetic, run on w's device.
    pad_to=1 keeps N unpadded (gemv_int8_cuda handles any N)."""
    n = w.shape[0]
    pad = (-n) % pad_to
    w = torch.cat([w, w.new_zeros(pad, w.shape[1])]) if pad else w
    s = (w.float().abs().amax(1) / 127).clamp(min=1e-8)
    q = ((w.float() / s[:, None]).round().clamp(-127, 127) + 128).to(torch.uint8).contiguous()
    return q, s.contiguous()


def gemv_int8_cuda(x, q, s, out=None):
    """y = s * ((q - 128) @ x) for uint8 q (int8 + 128), or s * (q @ x) for torch.int8 q; x [K] or [B, K]."""
    N, K = q.shape
    _require(q.dtype in (torch.uint8, torch.int8) and q.is_contiguous(), "q must be a contiguous uint8/int8 [N, K] tensor")
    _require(K % 64 == 0, f"K={K} must be a multiple of 64")
    _require(s.dtype in (torch.float32, torch.float16) and s.is_contiguous() and s.numel() == N,
             f"s must be a contiguous fp32/fp16 tensor of {N} row scales")
    _require(q.device == x.device and s.device == x.device, "x, q and s must be on the same device")
    batch, ldx = _act(x, K)
    y = _out(x, N, out)
    ldy = N if y.dim() == 1 else y.stride(0)
    L = _lib.lib()
    with _on_device(x.device):
        st = L.rb_gemv_int8(x.data_ptr(), _lib.dtype_code(x.dtype), ldx, q.data_ptr(), int(q.dtype == torch.int8),
                            s.data_ptr(), _lib.dtype_code(s.dtype), y.data_ptr(), _lib.dtype_code(y.dtype), ldy,
                            N, K, batch, config.flags(), _lib.stream_ptr(x.device))
    _lib.check("rb_gemv_int8", st)
    return y
