"""int4-weight prefill matmul (tcgen05) on the GPU against the CPU oracle and the reference's golden outputs.

Tolerance (north star): rel-L2 <= 1e-3 and max-abs <= 2e-3 * max|ref| against X.float() @ dequantize(q,s,m).t()
(kernels/mm_int4.py:96); bf16 outputs are held to the correctly rounded bf16 result (tests/helpers.py)."""
import os

import numpy as np
import pytest
import torch

import rumik_fast_b200 as rb
from oracle import oracle as O
from rumik_fast_b200 import synthetic as syn
from rumik_fast_b200.mm_int4 import mm_int4
from tests.helpers import assert_close, np_act

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _gpu(native_lib):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    yield
    assert rb.device_error() == 0


def mm_ref(X, q, s, m, cols=None):
    """Oracle, optionally on a subset of output columns (weight rows) to keep big cases fast."""
    xa, tag = np_act(X)
    qn, sn, mn = q.cpu().numpy(), s.cpu().numpy(), m.cpu().numpy()
    if cols is not None:
        qn, sn, mn = qn[cols], sn[cols], mn[cols]
    return O.mm_int4_ref(xa, qn, sn, mn, x_dtype=tag)


@pytest.mark.parametrize("tag", ["a", "b"])
def test_golden(tag):
    g = np.load(os.path.join(GOLD, "golden_mm.npz"))
    q, s, m = (torch.from_numpy(g[f"{tag}_{k}"]).to(DEV) for k in "qsm")
    X = torch.from_numpy(g[f"{tag}_X"]).to(DEV)
    Y = mm_int4(X, q, s, m)
    assert Y.shape == (X.shape[0], q.shape[0]) and Y.dtype == torch.float16
    assert_close(Y, g[f"{tag}_Y"], f"golden mm {tag}")


# Chunks of up to 128 tokens, or 256 where the plan estimates it faster ((512, 3072, 3072), (700, 4000, 2048),
# (1024, 3072, 8192): one 256-column accumulator, plain stores); M <= 64: three accumulators, one MMA issuer each.
# Chunks of <= 128 tokens store each item's tile with a bulk-tensor copy (Y, or the split-K partials: (100, 3072,
# 3072) in two rounds of 64 tokens); (300, 1000, 1024) ends in a partial chunk after full ones.
@pytest.mark.parametrize("M,N,K", [(1, 128, 128), (17, 200, 256), (34, 5120, 3072), (64, 3072, 8192), (300, 1000, 1024),
                                   (256, 3072, 3072), (1024, 16384, 3072), (512, 3072, 3072), (700, 4000, 2048),
                                   (1024, 3072, 8192), (100, 3072, 3072)])
def test_shapes(M, N, K):
    g = syn.generator(M * 31 + N + K, "cpu")
    q, s, m = syn.int4_weights(N, K, g, "cpu")
    X = syn.activations((M, K), g, "cpu")
    Y = mm_int4(X.to(DEV), q.to(DEV), s.to(DEV), m.to(DEV)).cpu()
    cols = np.sort(np.random.default_rng(N).choice(N, min(N, 512), replace=False))
    assert_close(Y[:, cols], mm_ref(X, q, s, m, cols), f"M={M} N={N} K={K}")


def test_bf16_strided_input():
    g = syn.generator(7, "cpu")
    q, s, m = syn.int4_weights(384, 1024, g, "cpu")
    Xbig = syn.activations((40, 1024 + 64), g, "cpu", dtype=torch.bfloat16)
    X = Xbig.to(DEV)[:, :1024]
    Y = mm_int4(X, q.to(DEV), s.to(DEV), m.to(DEV))
    assert Y.dtype == torch.bfloat16
    assert_close(Y, mm_ref(Xbig[:, :1024], q, s, m), "bf16 strided")


def test_matches_gemv_rows():
    """Each row of the prefill product equals the decode GEMV of that token (same weights)."""
    g = syn.generator(9, "cpu")
    q, s, m = (t.to(DEV) for t in syn.int4_weights(3072, 3072, g, "cpu"))
    X = syn.activations((8, 3072), g, "cpu").to(DEV)
    Y = mm_int4(X, q, s, m).float()
    Yg = rb.gemv_int4_cuda(X, q, s, m).float()
    assert torch.allclose(Y, Yg, rtol=2e-3, atol=2e-3 * Yg.abs().max().item())


def test_deterministic():
    g = syn.generator(11, "cpu")
    q, s, m = (t.to(DEV) for t in syn.int4_weights(1024, 2048, g, "cpu"))
    X = syn.activations((100, 2048), g, "cpu").to(DEV)
    assert torch.equal(mm_int4(X, q, s, m), mm_int4(X, q, s, m))


@pytest.mark.parametrize("M,N,K", [(34, 5120, 3072), (34, 3072, 8192), (256, 3072, 3072), (1024, 16384, 3072),
                                   (512, 3072, 3072)])
def test_bf16_x_through_the_c_abi(M, N, K):
    """The engine's bf16 activations straight into rb_mm_int4 (no split) and rb_mm_int4_ws (split K where the
    plan splits): converted to fp16 inside the kernel, so the result equals the fp16-X call bit for bit (the
    conversion is exact) and matches the oracle."""
    import ctypes
    from rumik_fast_b200 import _lib
    L = _lib.lib()
    g = syn.generator(M + N + K, "cpu")
    q, s, m = (t.to(DEV) for t in syn.int4_weights(N, K, g, "cpu"))
    Xb = syn.activations((M, K), g, "cpu", dtype=torch.bfloat16).to(DEV)
    Xh = Xb.to(torch.float16)
    ws_bytes = L.rb_mm_int4_workspace(M, N, K)
    ws = torch.empty(max(ws_bytes // 4, 1), device=DEV, dtype=torch.float32)
    out = {}
    for name, X in (("bf16", Xb), ("f16", Xh)):
        for split in (False, True):
            Y = torch.full((M, N), float("nan"), device=DEV, dtype=torch.float16)
            args = [X.data_ptr(), _lib.dtype_code(X.dtype), K, q.data_ptr(), s.data_ptr(), m.data_ptr(), Y.data_ptr(),
                    _lib.F16, N, M, N, K]
            stream = _lib.stream_ptr(torch.device(DEV))
            if split:
                st = L.rb_mm_int4_ws(*args, ctypes.c_void_p(ws.data_ptr()), ws_bytes, 0, stream)
            else:
                st = L.rb_mm_int4(*args, 0, stream)
            assert st == 0
            out[(name, split)] = Y
    torch.cuda.synchronize()
    assert torch.equal(out[("bf16", False)], out[("f16", False)])
    assert torch.equal(out[("bf16", True)], out[("f16", True)])
    cols = np.sort(np.random.default_rng(K).choice(N, 512, replace=False))
    assert_close(out[("bf16", True)].cpu()[:, cols], mm_ref(Xb.cpu(), q.cpu(), s.cpu(), m.cpu(), cols), "bf16 X")


def test_wrapper_launches_only_the_library_kernels():
    """mm_int4 with a bf16 X launches the prefill kernel (and its split-K reduction) and no torch op."""
    from torch.profiler import ProfilerActivity, profile
    g = syn.generator(13, "cpu")
    q, s, m = (t.to(DEV) for t in syn.int4_weights(3072, 8192, g, "cpu"))
    X = syn.activations((34, 8192), g, "cpu", dtype=torch.bfloat16).to(DEV)
    Y = torch.empty(34, 3072, device=DEV, dtype=torch.bfloat16)
    mm_int4(X, q, s, m, out=Y)  # first call: the workspace is allocated
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        mm_int4(X, q, s, m, out=Y)
        torch.cuda.synchronize()
    names = {e.name for e in prof.events() if e.device_type.name == "CUDA"}
    assert names and all("mm_int4" in n for n in names), names


@pytest.mark.parametrize("M", [34, 256, 700])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_list(M, dtype):
    """rb_mm_int4_list / MmInt4Set: a config-1 layer's four products (QKV, o_proj, gate_up with one X, down with
    another) plus a ragged one, in one persistent launch, against the oracle; two calls give the same bits."""
    from rumik_fast_b200.mm_int4 import MmInt4Set
    g = syn.generator(M * 7 + 1, "cpu")
    xs = {k: syn.activations((M, k), g, "cpu", dtype=dtype) for k in (3072, 8192, 1024)}
    shapes = [(n, k) for _, n, k in syn.LAYER_SHAPES] + [(1000, 1024)]
    host, ent = [], []
    for n, k in shapes:
        q, s, m = syn.int4_weights(n, k, g, "cpu")
        host.append((xs[k], q, s, m))
        ent.append((None, q.to(DEV), s.to(DEV), m.to(DEV), torch.full((M, n), float("nan"), device=DEV, dtype=dtype)))
    xd = {k: v.to(DEV) for k, v in xs.items()}
    ent = [(xd[q.shape[1] * 2], q, s, m, y) for _, q, s, m, y in ent]
    st = MmInt4Set(ent)
    st()
    torch.cuda.synchronize()
    for i, ((X, q, s, m), e) in enumerate(zip(host, ent)):
        n = q.shape[0]
        cols = np.sort(np.random.default_rng(n + i).choice(n, min(n, 256), replace=False))
        assert_close(e[4].cpu()[:, cols], mm_ref(X, q, s, m, cols), f"list M={M} entry {i} (N={n}, K={X.shape[1]})")
    first = [e[4].clone() for e in ent]
    st()
    torch.cuda.synchronize()
    assert all(torch.equal(a, e[4]) for a, e in zip(first, ent))


def test_list_longer_than_one_launch_and_graph():
    """60 products (more than the 52 of one launch): two launches; replayed from a CUDA graph."""
    from rumik_fast_b200.mm_int4 import MmInt4Set
    M = 48
    g = syn.generator(99, "cpu")
    X = syn.activations((M, 256), g, "cpu")
    host, ent = [], []
    xd = X.to(DEV)
    for i in range(60):
        n = 64 + 40 * (i % 5)
        q, s, m = syn.int4_weights(n, 256, g, "cpu")
        host.append((q, s, m))
        ent.append((xd, q.to(DEV), s.to(DEV), m.to(DEV), torch.full((M, n), float("nan"), device=DEV,
                                                                   dtype=torch.float16)))
    st = MmInt4Set(ent)
    st()
    torch.cuda.synchronize()
    for e in ent:
        e[4].fill_(float("nan"))
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        st()
    gr.replay()
    torch.cuda.synchronize()
    for i, ((q, s, m), e) in enumerate(zip(host, ent)):
        assert_close(e[4].cpu(), mm_ref(X, q, s, m), f"list entry {i}")
