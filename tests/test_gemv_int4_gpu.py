"""int4 group-128 GEMV on the GPU against the CPU oracle and the reference's golden outputs.

Tolerance (north star): relative L2 error <= 1e-3 and max-abs error <= 2e-3 * max|ref|, against the
reference's fp32 dequantise-then-matmul."""
import os

import numpy as np
import pytest
import torch

import rumik_fast_b200 as rb
from rumik_fast_b200 import synthetic as syn
from tests.helpers import assert_close, bf16_from_bits, int4_ref

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _gpu(native_lib):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.manual_seed(0)
    yield
    assert rb.device_error() == 0


def weights(N, K, seed=0):
    return syn.int4_weights(N, K, syn.generator(seed, "cpu"), "cpu")


def to_dev(*ts):
    return [t.to(DEV) for t in ts]


@pytest.mark.parametrize("tag", ["a", "b", "c", "d", "cfg"])
def test_golden_fp16(tag):
    g = np.load(os.path.join(GOLD, "golden_int4.npz"))
    q = torch.from_numpy(g[f"{tag}_q"]).to(DEV)
    s = torch.from_numpy(g[f"{tag}_s"]).to(DEV)
    m = torch.from_numpy(g[f"{tag}_m"]).to(DEV)
    x = torch.from_numpy(g[f"{tag}_x16"]).to(DEV)
    y = rb.gemv_int4_cuda(x, q, s, m)
    assert y.dtype == torch.float16 and y.shape == (q.shape[0],)
    assert_close(y, g[f"{tag}_y16"], f"golden {tag}")


@pytest.mark.parametrize("tag", ["a", "b", "c", "d"])
def test_golden_bf16_and_batched(tag):
    g = np.load(os.path.join(GOLD, "golden_int4.npz"))
    q, s, m = (torch.from_numpy(g[f"{tag}_{k}"]).to(DEV) for k in "qsm")
    xb = bf16_from_bits(g[f"{tag}_xbf"]).to(DEV)
    y = rb.gemv_int4_cuda(xb, q, s, m)          # bf16 in -> bf16 out, as the reference engine uses it
    assert y.dtype == torch.bfloat16
    assert_close(y, g[f"{tag}_ybf"], f"golden bf16 {tag}")
    xbat = torch.from_numpy(g[f"{tag}_xbat"]).to(DEV)
    yb = rb.gemv_int4_cuda(xbat, q, s, m)
    assert yb.shape == (3, q.shape[0])
    assert_close(yb, g[f"{tag}_ybat"], f"golden batch {tag}")


def test_config0_full_size():
    """Config 0: N=8192, K=3072, fp16 x ~N(0,1), codes uniform, scale ~U(0.002,0.02), min = -7.5 s + N(0,1e-3)."""
    q, s, m = weights(8192, 3072, seed=0)
    x = syn.activations((3072,), syn.generator(1, "cpu"), "cpu")
    ref = int4_ref(x, q, s, m)
    q, s, m, x = to_dev(q, s, m, x)
    y = rb.gemv_int4_cuda(x, q, s, m)
    rel, _ = assert_close(y, ref, "config 0")
    assert rel < 5e-4


@pytest.mark.parametrize("N,K", [(1, 128), (7, 256), (8, 384), (9, 128), (100, 1024), (1000, 2048), (3072, 3072),
                                 (5120, 3072), (16384, 3072), (3072, 8192), (2048, 11008), (300, 16384), (25088, 2048),
                                 (16400, 2048), (21504, 3072)])  # the last: the engine's fused [q|k|v|gate|up] w_in
def test_shapes(N, K):
    q, s, m = weights(N, K, seed=N * 7 + K)
    x = syn.activations((K,), syn.generator(K, "cpu"), "cpu")
    ref = int4_ref(x, q, s, m)
    y = rb.gemv_int4_cuda(*to_dev(x, q, s, m))
    assert_close(y, ref, f"N={N} K={K}")


@pytest.mark.parametrize("B", [2, 3, 4, 5, 8, 12, 16, 17, 40])
def test_batches(B):
    N, K = 1000, 3072
    q, s, m = weights(N, K, seed=B)
    x = syn.activations((B, K), syn.generator(100 + B, "cpu"), "cpu")
    ref = int4_ref(x, q, s, m)
    y = rb.gemv_int4_cuda(*to_dev(x, q, s, m))
    assert y.shape == (B, N)
    assert_close(y, ref, f"batch {B}")


def test_strided_rows_and_out_dtype():
    N, K, B = 520, 1024, 3
    q, s, m = to_dev(*weights(N, K, seed=5))
    xbig = syn.activations((B, K + 64), syn.generator(6, "cpu"), "cpu").to(DEV)
    x = xbig[:, :K]                                 # row stride K + 64
    out = torch.zeros(B, N + 8, device=DEV, dtype=torch.bfloat16)[:, :N]
    y = rb.gemv_int4_cuda(x, q, s, m, out=out)
    assert y.data_ptr() == out.data_ptr()
    assert_close(y, int4_ref(x, q, s, m), "strided")


def test_out_and_ignored_tuning_kwargs():
    N, K = 256, 512
    q, s, m = to_dev(*weights(N, K, seed=9))
    x = syn.activations((K,), syn.generator(9, "cpu"), "cpu").to(DEV)
    out = torch.empty(N, device=DEV, dtype=torch.float16)
    y = rb.gemv_int4_cuda(x, q, s, m, out=out, warps=4, rows=1)
    assert y is out
    assert_close(y, int4_ref(x, q, s, m), "out")


def test_deterministic():
    q, s, m = to_dev(*weights(5120, 3072, seed=11))
    x = syn.activations((3072,), syn.generator(12, "cpu"), "cpu").to(DEV)
    y1 = rb.gemv_int4_cuda(x, q, s, m)
    y2 = rb.gemv_int4_cuda(x, q, s, m)
    assert torch.equal(y1, y2)


def test_misaligned_weights_raise():
    q, s, m = to_dev(*weights(64, 256, seed=1))
    qq = torch.empty(q.numel() + 8, dtype=torch.uint8, device=DEV)[8:].view(64, 128)
    with pytest.raises(RuntimeError, match="aligned"):
        rb.gemv_int4_cuda(syn.activations((256,), syn.generator(1, "cpu"), "cpu").to(DEV), qq, s, m)


@pytest.mark.parametrize("prefetch", [False, True])
@pytest.mark.parametrize("graph", [False, True])
def test_dependent_chain(prefetch, graph):
    """x of each GEMV is the previous GEMV's output: with PDL (and weight prefetch) every kernel must still
    read its input only after the previous one finished. Each step is checked against the oracle applied
    to the GPU's own input of that step."""
    K = 3072
    L = 6
    g = syn.generator(21, "cpu")
    mats = []
    for i in range(L):
        q, s, m = syn.int4_weights(K, K, g, "cpu")
        s = (s.float() * 0.35).half()                    # keep |y| ~ |x| along the chain
        m = (-7.5 * s.float()).half()
        mats.append(to_dev(q, s, m))
    x0 = syn.activations((K,), g, "cpu").to(DEV)
    ys = [torch.empty(K, device=DEV, dtype=torch.float16) for _ in range(L)]

    def run():
        x = x0
        for i, (q, s, m) in enumerate(mats):
            rb.gemv_int4_cuda(x, q, s, m, out=ys[i])
            x = ys[i]

    with rb.weight_prefetch(prefetch):
        run()
        torch.cuda.synchronize()
        if graph:
            for y in ys:
                y.zero_()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                run()
            gr.replay()
            torch.cuda.synchronize()
    x = x0
    for i, (q, s, m) in enumerate(mats):
        assert_close(ys[i], int4_ref(x, q, s, m), f"chain step {i}")
        x = ys[i]


@pytest.mark.parametrize("N,K", [(65536, 3072), (24576, 8192), (40000, 1024), (32768, 16384)])
def test_long_row_bands(N, K):
    """Row bands of 20-56 eight-row stages with fewer ring slots than consumer warps (regression: a consumer
    warp running a full ring lap ahead must still wait for its own stage's data). Checked on a row sample,
    twice, to also catch races."""
    q, s, m = weights(N, K, seed=N + K)
    x = syn.activations((K,), syn.generator(K + 1, "cpu"), "cpu")
    qd, sd, md, xd = to_dev(q, s, m, x)
    y1 = rb.gemv_int4_cuda(xd, qd, sd, md)
    y2 = rb.gemv_int4_cuda(xd, qd, sd, md)
    assert torch.equal(y1, y2)
    rows = torch.from_numpy(np.sort(np.random.default_rng(N).choice(N, 2048, replace=False)))
    assert_close(y1.cpu()[rows], int4_ref(x, q[rows], s[rows], m[rows]), f"N={N} K={K}")
    assert rb.device_error() == 0
