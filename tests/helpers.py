"""Shared helpers of the GPU parity tests: tensor <-> numpy for the oracle, and the acceptance check."""
import numpy as np
import torch

from oracle import oracle as O


def np_act(t):
    """Activation tensor -> (numpy array, oracle dtype tag)."""
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16), "bf16"
    return t.numpy(), "f16"


def np_f32(t):
    return t.detach().float().cpu().numpy()


def bf16_from_bits(u16):
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16).copy()).view(torch.bfloat16)


def assert_close(y, ref, what=""):
    rel, mab = O.errors(np_f32(y) if isinstance(y, torch.Tensor) else y, ref)
    assert rel <= O.REL_L2_TOL and mab <= O.MAX_ABS_TOL, f"{what}: rel-L2 {rel:.3e}, max-abs/max {mab:.3e}"
    return rel, mab


def int4_ref(x, q, s, m):
    xa, tag = np_act(x)
    return O.gemv_int4_ref(xa, q.cpu().numpy(), s.cpu().numpy(), m.cpu().numpy(), x_dtype=tag)


def int8_ref(x, q, s):
    xa, tag = np_act(x)
    signed = q.dtype == torch.int8
    qa = q.cpu().view(torch.uint8).numpy() if signed else q.cpu().numpy()
    return O.gemv_int8_ref(xa, qa, s.float().cpu().numpy(), signed=signed, x_dtype=tag)
