"""One-launch list of independent int4 GEMVs (Int4GemvSet / rb_gemv_int4_multi) against the CPU oracle."""
import numpy as np
import pytest
import torch

import rumik_fast_b200 as rb
from rumik_fast_b200 import synthetic as syn
from tests.helpers import assert_close, int4_ref, int8_ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _gpu(native_lib):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    yield
    assert rb.device_error() == 0


def build(shapes, nx=2, seed=0, dtype=torch.float16):
    g = syn.generator(seed, "cpu")
    xs = {}
    host = []
    for i, (n, k) in enumerate(shapes):
        key = (i % nx, k)
        if key not in xs:
            xs[key] = syn.activations((k,), g, "cpu", dtype=dtype)
        q, s, m = syn.int4_weights(n, k, g, "cpu")
        host.append((xs[key], q, s, m))
    dev_x = {key: v.to(DEV) for key, v in xs.items()}
    out = []
    for i, ((x, q, s, m), (n, k)) in enumerate(zip(host, shapes)):
        key = (i % nx, k)
        y = torch.full((n,), float("nan"), device=DEV, dtype=dtype)
        out.append((dev_x[key], q.to(DEV), s.to(DEV), m.to(DEV), y))
    return host, out


def check(host, dev_entries, what):
    for i, ((x, q, s, m), e) in enumerate(zip(host, dev_entries)):
        assert_close(e[4], int4_ref(x, q, s, m), f"{what} entry {i}")


@pytest.mark.parametrize("kernel", ["tc", "mma"])
def test_layer_set(kernel):
    """Two layers of the config-1 projection set (QKV, o, gate_up with x_h; down with x_i), on each kernel
    explicitly: ~100 MB of codes is below the size at which the default choice moves to the tcgen05 kernel."""
    shapes = [(n, k) for _ in range(2) for _, n, k in syn.LAYER_SHAPES]
    host, ent = build(shapes, nx=1)
    rb.Int4GemvSet(ent, kernel=kernel)()
    check(host, ent, f"layers ({kernel})")


def test_ragged_and_mixed_k():
    shapes = [(1, 128), (7, 256), (9, 3072), (100, 11008), (1000, 2048), (25088, 2048), (300, 16384), (5, 8192)]
    host, ent = build(shapes, nx=3, seed=1)
    rb.Int4GemvSet(ent)()
    check(host, ent, "ragged")


def test_many_entries_and_slots_split_launches():
    """More than 256 entries and more than 8 distinct activation vectors: several launches."""
    shapes = [(16 + (i % 5) * 8, 128 * (1 + i % 3)) for i in range(300)]
    host, ent = build(shapes, nx=11, seed=2)
    rb.Int4GemvSet(ent)()
    check(host, ent, "split")


def test_bf16_and_graph_replay():
    shapes = [(3072, 3072), (640, 1024), (2000, 8192)]
    host, ent = build(shapes, nx=2, seed=3, dtype=torch.bfloat16)
    st = rb.Int4GemvSet(ent)
    st()
    torch.cuda.synchronize()
    for e in ent:
        e[4].fill_(float("nan"))
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        st()
    gr.replay()
    torch.cuda.synchronize()
    check(host, ent, "bf16 graph")


def test_matches_single_gemv_bitwise():
    g = syn.generator(4, "cpu")
    q, s, m = (t.to(DEV) for t in syn.int4_weights(5120, 3072, g, "cpu"))
    x = syn.activations((3072,), g, "cpu").to(DEV)
    y1 = rb.gemv_int4_cuda(x, q, s, m)
    y2 = torch.empty_like(y1)
    rb.Int4GemvSet([(x, q, s, m, y2)])()
    assert torch.allclose(y1.float(), y2.float(), rtol=1e-3, atol=1e-3 * y1.float().abs().max().item())


def _plain(ent):
    """The same list through rb_gemv_int4_multi (no workspace: never split)."""
    import ctypes  # noqa: F401
    from rumik_fast_b200 import _lib
    set_ = rb.Int4GemvSet(ent)
    L = _lib.lib()
    st = L.rb_gemv_int4_multi(set_._descs, len(ent), _lib.dtype_code(set_.x_dtype), _lib.dtype_code(set_.y_dtype),
                              rb.config.flags(), _lib.stream_ptr(torch.device(DEV)))
    _lib.check("rb_gemv_int4_multi", st)


@pytest.mark.parametrize("shapes", [
    [(3072, 3072), (3072, 8192)],                    # a decode layer's o_proj + down_proj: 48 blocks
    [(5120, 3072), (16384, 3072)],                   # QKV + gate_up: 168 blocks
    [(1000, 384), (130, 640), (7, 1152), (256, 16384)],  # odd group counts (G = 3, 5, 9), ragged N, long K
])
def test_split_k_lists(shapes):
    """On the tcgen05 kernel, lists with fewer blocks than 3 x the SM count run with K split over converter
    sets: the result matches the oracle, is the same on every call, and the per-block counters are zero again
    afterwards. The same list on the default kernel choice (warp-MMA for lists this small) agrees too."""
    host, ent = build(shapes, nx=2, seed=7)
    st = rb.Int4GemvSet(ent, kernel="tc")
    assert st.ws is not None                         # these lists do split
    st()
    torch.cuda.synchronize()
    check(host, ent, "split-K")
    first = [e[4].clone() for e in ent]
    for _ in range(3):
        st()
    torch.cuda.synchronize()
    assert all(torch.equal(a, e[4]) for a, e in zip(first, ent))
    n_blocks = sum((n + 127) // 128 for n, _ in shapes)
    assert torch.count_nonzero(st.ws[:4 * n_blocks]) == 0
    for e in ent:                                    # unsplit launch of the same list: the same GEMVs
        e[4].fill_(float("nan"))
    _plain(ent)
    torch.cuda.synchronize()
    check(host, ent, "unsplit")


def _int8_rows(N, K, seed, offset, s_dtype):
    """int8 rows [N, K] (torch.int8, or the uint8 = int8 + 128 storage of quantize_int8_rows) and row scales."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int16)
    q = (q + 128).to(torch.uint8) if offset else q.to(torch.int8)
    s = (torch.rand(N, generator=g) * 9e-4 + 1e-4).to(s_dtype)
    return q, s


@pytest.mark.parametrize("offset,s_dtype", [(False, torch.float16), (True, torch.float32)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("split", [False, True])
def test_int8_rows_in_the_list(offset, s_dtype, dtype, split):
    """The int8 head streamed as more rows of a tcgen05 list launch (rb_gemv_desc::w8): y = s * (q @ x) against
    the oracle's gemv_int8_ref, beside int4 entries that stay correct, with a ragged last block (N = 16385);
    split: few enough blocks that K is split over converter sets (partials and ticket); unsplit: the whole
    config-1 layers' projections plus the head. Two calls give the same bits; the tickets end zeroed."""
    # split: 56 blocks; unsplit: two config-1 layers (432 blocks) + the head (129) > 3 x 148 converter sets
    shapes = [(3072, 3072), (3072, 8192)] if split else [(n, k) for _ in range(2) for _, n, k in syn.LAYER_SHAPES]
    host, ent = build(shapes, nx=2, seed=11, dtype=dtype)
    q8, s8 = _int8_rows(16385 if not split else 1000, 3072, 12, offset, s_dtype)
    xh = syn.activations((3072,), syn.generator(13, "cpu"), "cpu", dtype=dtype)
    yh = torch.full((q8.shape[0],), float("nan"), device=DEV, dtype=dtype)
    head = (xh.to(DEV), q8.to(DEV), s8.to(DEV), None, yh)
    st = rb.Int4GemvSet([head] + ent, kernel="tc")
    assert (st.ws is not None) == split
    st()
    torch.cuda.synchronize()
    assert rb.device_error() == 0
    assert_close(yh, int8_ref(xh, q8, s8), "int8 rows")
    check(host, ent, "int4 entries beside the int8 rows")
    first = [yh.clone()] + [e[4].clone() for e in ent]
    st()
    torch.cuda.synchronize()
    assert all(torch.equal(a, b) for a, b in zip(first, [yh] + [e[4] for e in ent]))
    if split:  # the per-block tickets (the partials after them are not cleared)
        n_blocks = sum((n + 127) // 128 for n, _ in shapes) + (q8.shape[0] + 127) // 128
        assert int(torch.count_nonzero(st.ws[:4 * n_blocks])) == 0


def test_int8_rows_refused_off_the_tc_kernel():
    host, ent = build([(256, 1024)], nx=1, seed=14)
    q8, s8 = _int8_rows(64, 1024, 15, False, torch.float16)
    head = (ent[0][0], q8.to(DEV), s8.to(DEV), None, torch.empty(64, device=DEV, dtype=torch.float16))
    with pytest.raises(RuntimeError):
        rb.Int4GemvSet([head] + ent, kernel="mma")()
