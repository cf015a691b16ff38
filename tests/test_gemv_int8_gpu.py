"""int8 per-row head GEMV on the GPU against the CPU oracle and the reference's golden outputs."""
import os

import numpy as np
import pytest
import torch

import rumik_fast_b200 as rb
from rumik_fast_b200 import synthetic as syn
from tests.helpers import assert_close, bf16_from_bits, int8_ref

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _gpu(native_lib):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    yield
    assert rb.device_error() == 0


@pytest.mark.parametrize("tag", ["a", "b"])
def test_golden_reference_quantised_head(tag):
    """uint8 = int8 + 128 codes and fp32 row scales from the reference's quantize_int8_rows."""
    g = np.load(os.path.join(GOLD, "golden_int8.npz"))
    q = torch.from_numpy(g[f"{tag}_q"]).to(DEV)
    s = torch.from_numpy(g[f"{tag}_s"]).to(DEV)
    y = rb.gemv_int8_cuda(torch.from_numpy(g[f"{tag}_x16"]).to(DEV), q, s)
    assert_close(y, g[f"{tag}_y16"], f"golden {tag}")
    yb = rb.gemv_int8_cuda(bf16_from_bits(g[f"{tag}_xbf"]).to(DEV), q, s)
    assert yb.dtype == torch.bfloat16
    assert_close(yb, g[f"{tag}_ybf"], f"golden bf16 {tag}")


def test_golden_config_style_signed_and_offset_storage():
    g = np.load(os.path.join(GOLD, "golden_int8.npz"))
    x = torch.from_numpy(g["cfg_x16"]).to(DEV)
    s = torch.from_numpy(g["cfg_s16"]).to(DEV)
    y_signed = rb.gemv_int8_cuda(x, torch.from_numpy(g["cfg_wi8"]).to(DEV), s)
    y_u8 = rb.gemv_int8_cuda(x, torch.from_numpy(g["cfg_qu8"]).to(DEV), s)
    assert_close(y_signed, g["cfg_y16"], "signed int8")
    assert_close(y_u8, g["cfg_y16"], "uint8+128")
    assert torch.equal(y_signed, y_u8)


def test_config2_full_size():
    """Config 2: W int8 [16385, 3072] uniform -127..127, fp16 row scale ~U(1e-4, 1e-3), x fp16 ~N(0,1)."""
    q, s = syn.int8_weights(16385, 3072, syn.generator(0, "cpu"), "cpu")
    x = syn.activations((3072,), syn.generator(1, "cpu"), "cpu")
    ref = int8_ref(x, q, s)
    y = rb.gemv_int8_cuda(x.to(DEV), q.to(DEV), s.to(DEV))
    assert y.shape == (16385,)
    rel, _ = assert_close(y, ref, "config 2")
    assert rel < 5e-4


@pytest.mark.parametrize("N,K", [(1, 64), (5, 192), (16, 256), (17, 512), (1000, 1024), (16400, 2048), (333, 16384)])
def test_shapes(N, K):
    g = syn.generator(N + K, "cpu")
    q, s = syn.int8_weights(N, K, g, "cpu")
    x = syn.activations((K,), g, "cpu")
    y = rb.gemv_int8_cuda(x.to(DEV), q.to(DEV), s.float().to(DEV))
    assert_close(y, int8_ref(x, q, s.float()), f"N={N} K={K}")


@pytest.mark.parametrize("B", [2, 4, 7, 16, 20])
def test_batches(B):
    g = syn.generator(B, "cpu")
    q, s = syn.int8_weights(2000, 3072, g, "cpu")
    x = syn.activations((B, 3072), g, "cpu")
    y = rb.gemv_int8_cuda(x.to(DEV), q.to(DEV), s.to(DEV))
    assert y.shape == (B, 2000)
    assert_close(y, int8_ref(x, q, s), f"batch {B}")


def test_quantize_then_gemv_on_device():
    """The engine's load path: bf16 head rows -> quantize_int8_rows on the GPU -> gemv_int8_cuda."""
    g = syn.generator(3, "cpu")
    w = (torch.randn(777, 1024, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    q, s = rb.quantize_int8_rows(w)
    assert q.shape[0] == 784 and q.dtype == torch.uint8 and s.dtype == torch.float32
    x = torch.randn(1024, generator=g).to(torch.bfloat16).to(DEV)
    y = rb.gemv_int8_cuda(x, q, s)
    assert_close(y, int8_ref(x, q, s), "engine head path")


@pytest.mark.parametrize("N,K", [(65536, 3072), (20000, 8192)])
def test_long_row_bands(N, K):
    """Row bands with many more stages than ring slots (regression for early passes of a reused slot)."""
    g = syn.generator(N, "cpu")
    q, s = syn.int8_weights(N, K, g, "cpu")
    x = syn.activations((K,), g, "cpu")
    y1 = rb.gemv_int8_cuda(x.to(DEV), q.to(DEV), s.to(DEV))
    y2 = rb.gemv_int8_cuda(x.to(DEV), q.to(DEV), s.to(DEV))
    assert torch.equal(y1, y2)
    rows = torch.from_numpy(np.sort(np.random.default_rng(N).choice(N, 2048, replace=False)))
    assert_close(y1.cpu()[rows], int8_ref(x, q[rows], s[rows]), f"N={N} K={K}")
    assert rb.device_error() == 0
