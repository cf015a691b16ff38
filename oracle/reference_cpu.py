"""The reference's CPU path for the decode step, restated in torch - TEST AND BASELINE INFRASTRUCTURE ONLY.

rumik-fast checks and times its kernels against torch on fp32 dequantised weights:
  dequantize          kernels/int4_gemv.py:27-30  (codes unpacked low nibble first, code * scale + min in fp32)
  gemv_int4_torch     kernels/bench_cuda.py:38    (dequantize(q, s, m) @ x.float())
  gemv_int8_torch     kernels/cuda_gemv.py:245-246 (((q.int() - 128).float() * s[:, None]) @ x.float())
bench.py's CPU-baseline leg and its reference arm time these on the host cores (torch.set_num_threads), one
decode step = the config-1 projection set plus the int8 head. Only tests/, __graft_entry__.smoke() and bench.py's
CPU legs may import this module; the product never calls it.
"""
import torch

G = 128


def dequantize(q, s, m, group=G):
    """uint8 [N, K/2] codes + fp16 [N, K/group] scale and min -> fp32 [N, K] weights."""
    n = q.shape[0]
    code = torch.stack([q & 0xF, q >> 4], -1).view(n, -1).float()
    return (code.view(n, -1, group) * s.float()[..., None] + m.float()[..., None]).view(n, -1)


def gemv_int4_torch(x, q, s, m):
    return dequantize(q, s, m) @ x.float()


def gemv_int8_torch(x, q, s, signed=True):
    """q int8 [N, K] (signed) or uint8 = int8 + 128; s per-row scale."""
    w = q.float() if signed else (q.int() - 128).float()
    return (w * s.float()[:, None]) @ x.float()
