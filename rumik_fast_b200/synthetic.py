"""Seeded synthetic inputs with the distributions of the benchmark configurations (no dataset or checkpoint is
involved; the reference's own checks also use random weights, kernels/bench_cuda.py:36).

  int4 weights (configs 0, 1, 3): codes uniform 0..15 packed two per byte (low nibble = even column), which
      is the same as uniform random bytes; scale fp16 ~U(0.002, 0.02); min fp16 = -7.5 * scale + N(0, 1e-3).
  int8 head (config 2): codes uniform -127..127 (int8), fp16 row scale ~U(1e-4, 1e-3).
  activations: fp16 ~N(0, 1).
"""
import torch

G = 128

# 36-layer decode-step projection set (config 1): (name, N, K) per layer
LAYER_SHAPES = (("qkv", 5120, 3072), ("o_proj", 3072, 3072), ("gate_up", 16384, 3072), ("down", 3072, 8192))
HEAD_SHAPE = (16385, 3072)


def int4_bytes(N, K):
    """Algorithmic bytes of one int4 GEMV: codes + scale + min + x + y (fp16 activations)."""
    return N * K // 2 + 4 * N * (K // G) + 2 * K + 2 * N


def int8_bytes(N, K):
    """Algorithmic bytes of one int8 head GEMV with an fp16 row scale: codes + scale + x + y."""
    return N * K + 2 * N + 2 * K + 2 * N


def generator(seed, device):
    return torch.Generator(device=device).manual_seed(seed)


def int4_weights(N, K, gen, device):
    q = torch.randint(0, 256, (N, K // 2), generator=gen, device=device, dtype=torch.uint8)
    s = (torch.rand(N, K // G, generator=gen, device=device) * 0.018 + 0.002).to(torch.float16)
    m = (-7.5 * s.float() + torch.randn(N, K // G, generator=gen, device=device) * 1e-3).to(torch.float16)
    return q, s, m


def int8_weights(N, K, gen, device):
    q = torch.randint(-127, 128, (N, K), generator=gen, device=device, dtype=torch.int16).to(torch.int8)
    s = (torch.rand(N, generator=gen, device=device) * 9e-4 + 1e-4).to(torch.float16)
    return q, s


def activations(shape, gen, device, dtype=torch.float16):
    return torch.randn(shape, generator=gen, device=device).to(dtype)
