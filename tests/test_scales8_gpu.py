"""GEMV lists with 8-bit double-quantised scales (Int4GemvSet entries (x, q, Scales8, None, y) on the tcgen05
kernel) against the CPU oracle of the weights those scales decode to."""
import numpy as np
import pytest
import torch

import rumik_fast_b200 as rb
from oracle import oracle as O
from rumik_fast_b200 import scales8
from rumik_fast_b200 import synthetic as syn
from tests.helpers import assert_close, int4_ref, np_act

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _gpu(native_lib):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    yield
    assert rb.device_error() == 0


def build(shapes, eight, seed=0, dtype=torch.float16, nx=2):
    """eight[i]: entry i carries 8-bit scales. Returns (host oracle inputs, device entries)."""
    g = syn.generator(seed, "cpu")
    xs, host, ent = {}, [], []
    for i, (n, k) in enumerate(shapes):
        key = (i % nx, k)
        if key not in xs:
            xs[key] = syn.activations((k,), g, "cpu", dtype=dtype)
        q, s, m = syn.int4_weights(n, k, g, "cpu")
        y = torch.full((n,), float("nan"), device=DEV, dtype=dtype)
        x = xs[key].to(DEV)
        if eight[i]:
            sc = scales8.pack(s.to(DEV), m.to(DEV))
            host.append((xs[key], q, sc.sz.cpu(), sc.s_row.cpu()))
            ent.append((x, q.to(DEV), sc, None, y))
        else:
            host.append((xs[key], q, s, m))
            ent.append((x, q.to(DEV), s.to(DEV), m.to(DEV), y))
    return host, ent


def ref8(x, q, sz, s_row):
    xa, tag = np_act(x)
    return O.gemv_int4_s8_ref(xa, q.numpy(), sz.numpy().view(np.uint16), s_row.numpy(), x_dtype=tag)


def check(host, ent, what):
    for i, (h, e) in enumerate(zip(host, ent)):
        ref = ref8(*h) if isinstance(e[2], scales8.Scales8) else int4_ref(*h)
        assert_close(e[4], ref, f"{what} entry {i}")


def test_device_pack_matches_oracle():
    g = syn.generator(3, "cpu")
    _, s, m = syn.int4_weights(4096, 3072, g, "cpu")
    sc = scales8.pack(s.to(DEV), m.to(DEV))
    sz, row = O.pack_scales8(s.numpy(), m.numpy())
    assert np.array_equal(sc.s_row.cpu().numpy(), row)
    assert np.array_equal(sc.sz.cpu().numpy().view(np.uint16), sz)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_whole_step_set(dtype):
    """Two layers of the config-1 projection set, all with 8-bit scales, as the step's long list (tc)."""
    shapes = [(n, k) for _ in range(2) for _, n, k in syn.LAYER_SHAPES]
    host, ent = build(shapes, [True] * len(shapes), seed=1, dtype=dtype, nx=1)
    rb.Int4GemvSet(ent, kernel="tc")()
    torch.cuda.synchronize()
    check(host, ent, "s8 set")


def test_mixed_ragged_odd_groups_split_k():
    """fp16 and 8-bit entries in one list; odd group counts (G = 3, 5, 9: the one-pair-at-a-time path), ragged N;
    a short list, so that the default choice is the tcgen05 kernel with K split over converter sets."""
    shapes = [(1000, 384), (130, 640), (7, 1152), (256, 16384), (3072, 3072), (640, 1024)]
    eight = [True, False, True, True, False, True]
    host, ent = build(shapes, eight, seed=2, nx=3)
    st = rb.Int4GemvSet(ent)
    assert st.ws is not None
    st()
    torch.cuda.synchronize()
    check(host, ent, "mixed")
    first = [e[4].clone() for e in ent]
    st()
    torch.cuda.synchronize()
    assert all(torch.equal(a, e[4]) for a, e in zip(first, ent))


def test_same_result_as_fp16_scales_it_decodes_to():
    """The 8-bit entry and an fp16 entry holding the decoded scale / min give the same GEMV (same kernel)."""
    g = syn.generator(4, "cpu")
    q, s, m = (t.to(DEV) for t in syn.int4_weights(5120, 3072, g, "cpu"))
    x = syn.activations((3072,), g, "cpu").to(DEV)
    sc = scales8.pack(s, m)
    s16, m16 = scales8.unpack(sc)
    y8, y16 = (torch.empty(5120, device=DEV, dtype=torch.float16) for _ in range(2))
    rb.Int4GemvSet([(x, q, sc, None, y8), (x, q, s16.contiguous(), m16.contiguous(), y16)], kernel="tc")()
    torch.cuda.synchronize()
    assert torch.equal(y8, y16)


def test_rejected_where_unsupported():
    g = syn.generator(5, "cpu")
    q, s, m = (t.to(DEV) for t in syn.int4_weights(256, 1024, g, "cpu"))
    x = syn.activations((1024,), g, "cpu").to(DEV)
    y = torch.empty(256, device=DEV, dtype=torch.float16)
    sc = scales8.pack(s, m)
    with pytest.raises(RuntimeError):                 # the warp-MMA kernel has no 8-bit scales
        rb.Int4GemvSet([(x, q, sc, None, y)], kernel="mma")()
    with pytest.raises(RuntimeError):                 # m must be None with 8-bit scales
        rb.Int4GemvSet([(x, q, sc, m, y)])
    bad = scales8.Scales8(sc.sz[:, :4].contiguous(), sc.s_row)
    with pytest.raises(RuntimeError):
        rb.Int4GemvSet([(x, q, bad, None, y)])
