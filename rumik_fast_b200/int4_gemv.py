"""Drop-in for the parts of rumik-fast kernels/int4_gemv.py that the engine imports.

    G = 128
    quantize(w, group=G) -> (qweight uint8 [N, K/2], scale fp16 [N, K/G], min fp16 [N, K/G])
        the reference's load-time quantiser (kernels/int4_gemv.py:16-24), same arithmetic, on w's device;
    gemv_int4(x, q, s, m, out=None) -> y in x's dtype
        the reference's Triton v1 contract (kernels/int4_gemv.py:84-96), served by the sm_100a CUDA GEMV.
"""
import torch

from .cuda_gemv import gemv_int4_cuda

G = 128


def quantize(w: torch.Tensor, group: int = G):
    n, k = w.shape
    g = w.float().view(n, k // group, group)
    mn, mx = g.amin(-1, keepdim=True), g.amax(-1, keepdim=True)
    scale = ((mx - mn) / 15).clamp(min=1e-8)
    code = ((g - mn) / scale).round().clamp(0, 15).to(torch.uint8).view(n, k)
    packed = (code[:, 0::2] | (code[:, 1::2] << 4)).contiguous()
    return packed, scale.half().view(n, -1).contiguous(), mn.half().view(n, -1).contiguous()


def gemv_int4(x, q, s, m, out=None):
    return gemv_int4_cuda(x, q, s, m, out=out)
