"""Host-side behaviour of the drop-in Python modules that needs no GPU."""
import os

import numpy as np
import pytest
import torch

import rumik_fast_b200 as rb
from rumik_fast_b200 import config, cuda_gemv, int4_gemv, synthetic

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def bf16_from_bits(u16):
    return torch.from_numpy(u16.view(np.int16).copy()).view(torch.bfloat16)


def test_reference_names_present():
    for name in ("gemv_int4_cuda", "gemv_int8_cuda", "quantize_int8_rows", "SHAPE"):
        assert hasattr(cuda_gemv, name)
    from rumik_fast_b200 import mm_int4 as mm
    assert callable(mm.mm_int4) and callable(mm.warmup) and mm.G == 128
    assert int4_gemv.G == 128 and callable(int4_gemv.quantize) and callable(int4_gemv.gemv_int4)


def test_cpu_tensors_are_rejected_not_computed():
    q = torch.zeros(16, 64, dtype=torch.uint8)
    s = torch.zeros(16, 1, dtype=torch.float16)
    x = torch.zeros(128, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA"):
        rb.gemv_int4_cuda(x, q, s, s)
    with pytest.raises(RuntimeError):
        rb.gemv_int8_cuda(x, torch.zeros(16, 128, dtype=torch.uint8), torch.zeros(16))
    with pytest.raises(RuntimeError, match="CUDA"):
        rb.mm_int4.mm_int4(torch.zeros(4, 128, dtype=torch.float16), q, s, s)


def test_shape_errors_raise_runtime_error():
    q = torch.zeros(16, 60, dtype=torch.uint8)   # K = 120, not a multiple of 128
    s = torch.zeros(16, 1, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="multiple of 128"):
        rb.gemv_int4_cuda(torch.zeros(120, dtype=torch.float16), q, s, s)


def test_quantize_matches_reference_fixture():
    g = np.load(os.path.join(GOLD, "golden_int4.npz"))
    for tag in ("a", "b", "c", "d"):
        q, s, m = int4_gemv.quantize(bf16_from_bits(g[f"{tag}_w"]))
        assert np.array_equal(q.numpy(), g[f"{tag}_q"])
        assert np.array_equal(s.numpy().view(np.uint16), g[f"{tag}_s"].view(np.uint16))
        assert np.array_equal(m.numpy().view(np.uint16), g[f"{tag}_m"].view(np.uint16))


def test_quantize_int8_rows_matches_reference_fixture():
    g = np.load(os.path.join(GOLD, "golden_int8.npz"))
    for tag in ("a", "b"):
        q, s = cuda_gemv.quantize_int8_rows(bf16_from_bits(g[f"{tag}_w"]))
        assert np.array_equal(q.numpy(), g[f"{tag}_q"])
        assert np.array_equal(s.numpy().view(np.uint32), g[f"{tag}_s"].view(np.uint32))


def test_launch_flags():
    with config.weight_prefetch(True):
        assert config.flags() == 3
    assert config.flags() == (1 if config.PDL else 0)


def test_synthetic_byte_counts():
    assert synthetic.int4_bytes(8192, 3072) == 13_391_872                          # config 0
    step = sum(synthetic.int4_bytes(n, k) for _, n, k in synthetic.LAYER_SHAPES) * 36
    assert step == 1_928_429_568                                                   # config 1
    assert synthetic.int8_bytes(*synthetic.HEAD_SHAPE) == 50_406_404               # config 2
