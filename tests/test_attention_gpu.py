"""Decode attention (rb_attn_decode) on the GPU against the CPU oracle (engine/rumik_int4.py:163-171)."""
import numpy as np
import pytest
import torch

import rumik_fast_b200 as rb
from oracle import oracle as O
from rumik_fast_b200 import _lib
from rumik_fast_b200.attention import DecodeAttention
from tests.helpers import assert_close, np_act

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _gpu(native_lib):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    rb.device_error()
    yield
    assert rb.device_error() == 0


def setup(nq, nkv, S, dt, seed=0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(nq * 128, generator=g).to(dt)
    kc = torch.randn(nkv, S, 128, generator=g).to(dt)
    vc = torch.randn(nkv, S, 128, generator=g).to(dt)
    return q, kc, vc


def oracle(q, kc, vc, pos, nq, nkv):
    qa, t = np_act(q)
    return O.attention_ref(qa, np_act(kc)[0], np_act(vc)[0], pos, nq, nkv, 128, 128 ** -0.5, t)


@pytest.mark.parametrize("merge", ["auto", "ticket"])
@pytest.mark.parametrize("early", [False, True])
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("nq,nkv", [(24, 8), (16, 4), (8, 8), (16, 2), (64, 8)])
def test_attention_matches_oracle(dt, nq, nkv, early, merge):
    """early: with weight prefetch on, the position and the earlier slots' K/V rows are read before the wait.
    merge: the cluster form (distributed shared memory) or the ticket form (global partials)."""
    from rumik_fast_b200 import config
    S = 2048
    q, kc, vc = setup(nq, nkv, S, dt, seed=nq + nkv)
    qd, kd, vd = q.to(DEV), kc.to(DEV), vc.to(DEV)
    pos = torch.zeros(1, dtype=torch.int64, device=DEV)
    out = torch.full((nq * 128,), float("nan"), device=DEV, dtype=dt)
    attn = DecodeAttention(qd, kd, vd, pos, out, nq, nkv, merge=merge)
    for p in (0, 1, 31, 33, 200, 511, 512, 1500, S - 1):
        pos.fill_(p)
        with config.weight_prefetch(early):
            attn()
        torch.cuda.synchronize()
        assert_close(out, oracle(q, kc, vc, p, nq, nkv), f"attention at position {p}")


@pytest.mark.parametrize("merge", ["auto", "ticket"])
def test_attention_is_deterministic_and_reusable(merge):
    dt, nq, nkv, S = torch.float16, 24, 8, 512
    q, kc, vc = (t.to(DEV) for t in setup(nq, nkv, S, dt, seed=3))
    pos = torch.tensor([300], dtype=torch.int64, device=DEV)
    out = torch.empty(nq * 128, device=DEV, dtype=dt)
    attn = DecodeAttention(q, kc, vc, pos, out, nq, nkv, merge=merge)
    attn()
    first = out.clone()
    for _ in range(5):          # the completion counters reset themselves after every call
        attn()
    torch.cuda.synchronize()
    assert torch.equal(out, first)
    assert torch.count_nonzero(attn.ws[:256]) == 0


def test_attention_in_a_cuda_graph_follows_the_position():
    dt, nq, nkv, S = torch.bfloat16, 16, 4, 256
    q, kc, vc = setup(nq, nkv, S, dt, seed=4)
    qd, kd, vd = q.to(DEV), kc.to(DEV), vc.to(DEV)
    pos = torch.zeros(1, dtype=torch.int64, device=DEV)
    out = torch.empty(nq * 128, device=DEV, dtype=dt)
    outs = torch.empty(4, nq * 128, device=DEV, dtype=dt)
    attn = DecodeAttention(qd, kd, vd, pos, out, nq, nkv)
    attn()
    torch.cuda.synchronize()
    idx = torch.zeros(1, dtype=torch.int64, device=DEV)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        attn()
        outs.index_copy_(0, idx, out.view(1, -1))
        pos.add_(37)
        idx.add_(1)
    pos.fill_(5)
    idx.zero_()
    for _ in range(4):
        graph.replay()
    torch.cuda.synchronize()
    for i in range(4):
        assert_close(outs[i], oracle(q, kc, vc, 5 + 37 * i, nq, nkv), f"replay {i}")


def test_position_outside_the_cache_writes_nothing():
    dt, nq, nkv, S = torch.float16, 8, 2, 64
    q, kc, vc = (t.to(DEV) for t in setup(nq, nkv, S, dt, seed=5))
    out = torch.zeros(nq * 128, device=DEV, dtype=dt)
    for bad in (S, -3):
        pos = torch.tensor([bad], dtype=torch.int64, device=DEV)
        DecodeAttention(q, kc, vc, pos, out, nq, nkv)()
        assert rb.device_error() & _lib.DEVERR_ARG
        assert torch.count_nonzero(out) == 0


def output_side(nq, nkv, S, dt, seed, inter=1024, H=3072):
    """Attention inputs plus an o_proj [H, nq * 128] and a down_proj [H, inter] with its input vector."""
    from rumik_fast_b200 import synthetic as syn
    q, kc, vc = setup(nq, nkv, S, dt, seed=seed)
    g = syn.generator(seed + 100, "cpu")
    wo = syn.int4_weights(H, nq * 128, g, "cpu")
    wd = syn.int4_weights(H, inter, g, "cpu")
    act = syn.activations((inter,), g, "cpu", dtype=dt)
    return q, kc, vc, wo, wd, act


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("nq,nkv", [(24, 8), (16, 4), (8, 8)])
def test_attention_fused_into_the_output_gemvs(dt, nq, nkv):
    """AttnGemvSet: the attention computed inside the o_proj/down_proj launch (warp-MMA kernel) matches the
    oracle, o_proj multiplies exactly what it computed, down_proj is unaffected, the counters return to zero
    and repeated calls give the same bits."""
    from rumik_fast_b200 import fused
    from tests.helpers import int4_ref
    S, H = 2048, 3072
    q, kc, vc, wo, wd, act = output_side(nq, nkv, S, dt, seed=nq + 7 * nkv)
    qd, kd, vd, actd = q.to(DEV), kc.to(DEV), vc.to(DEV), act.to(DEV)
    wod, wdd = tuple(t.to(DEV) for t in wo), tuple(t.to(DEV) for t in wd)
    pos = torch.zeros(1, dtype=torch.int64, device=DEV)
    ob = torch.full((nq * 128,), float("nan"), device=DEV, dtype=dt)
    bo = torch.empty(H, device=DEV, dtype=dt)
    bd = torch.empty(H, device=DEV, dtype=dt)
    layer = fused.AttnGemvSet([(ob, *wod, bo), (actd, *wdd, bd)], q=qd, k_cache=kd, v_cache=vd, pos=pos, out=ob,
                              n_q_heads=nq, n_kv_heads=nkv)
    for p in (0, 40, 511, S - 1):
        pos.fill_(p)
        layer()
        torch.cuda.synchronize()
        assert_close(ob, oracle(q, kc, vc, p, nq, nkv), f"fused attention at position {p}")
        assert_close(bo, int4_ref(ob.cpu(), *wo), f"o_proj of the fused attention at {p}")
        assert_close(bd, int4_ref(act, *wd), f"down_proj beside the attention at {p}")
        assert torch.count_nonzero(layer.ws[:512]) == 0
        first = (ob.clone(), bo.clone(), bd.clone())
        layer()
        torch.cuda.synchronize()
        assert torch.equal(ob, first[0]) and torch.equal(bo, first[1]) and torch.equal(bd, first[2])


def test_fused_attention_in_a_cuda_graph_and_out_of_range():
    from rumik_fast_b200 import fused
    from tests.helpers import int4_ref
    dt, nq, nkv, S, H = torch.float16, 16, 4, 256, 3072
    q, kc, vc, wo, wd, act = output_side(nq, nkv, S, dt, seed=9)
    qd, kd, vd, actd = q.to(DEV), kc.to(DEV), vc.to(DEV), act.to(DEV)
    wod, wdd = tuple(t.to(DEV) for t in wo), tuple(t.to(DEV) for t in wd)
    pos = torch.zeros(1, dtype=torch.int64, device=DEV)
    ob = torch.empty(nq * 128, device=DEV, dtype=dt)
    bo = torch.empty(H, device=DEV, dtype=dt)
    bd = torch.empty(H, device=DEV, dtype=dt)
    outs = torch.empty(3, H, device=DEV, dtype=dt)
    idx = torch.zeros(1, dtype=torch.int64, device=DEV)
    layer = fused.AttnGemvSet([(actd, *wdd, bd), (ob, *wod, bo)], q=qd, k_cache=kd, v_cache=vd, pos=pos, out=ob,
                              n_q_heads=nq, n_kv_heads=nkv)
    layer()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        layer()
        outs.index_copy_(0, idx, bo.view(1, -1))
        pos.add_(50)
        idx.add_(1)
    pos.fill_(3)
    idx.zero_()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    for i in range(3):
        o_ref = oracle(q, kc, vc, 3 + 50 * i, nq, nkv)
        assert_close(outs[i], int4_ref(torch.from_numpy(o_ref).to(dt), *wo), f"graph replay {i}")
    # a position outside the cache: the attention writes nothing and the launch does not wait for it
    pos.fill_(S)
    layer()
    torch.cuda.synchronize()
    assert rb.device_error() & _lib.DEVERR_ARG
    assert torch.count_nonzero(layer.ws[:512]) == 0


@pytest.mark.parametrize("merge", ["auto", "ticket"])
@pytest.mark.parametrize("p", [0, 40, 511, 2047])
@pytest.mark.parametrize("graph", [False, True])
def test_early_loads_wait_for_the_producer_of_q_and_the_slot(p, graph, merge):
    """With weight prefetch on, the attention launch reads the position and the K/V rows of the slots before it
    ahead of its dependency wait. Here the launch just before it (a GEMV list launched with programmatic
    dependent launch) writes q and the token's K/V slot of every key-value head, which hold NaN until then: the
    output must match the oracle on the values that launch wrote, so no early load may have seen the stale ones."""
    from rumik_fast_b200 import config, synthetic as syn
    dt, nq, nkv, S, K = torch.float16, 24, 8, 2048, 1024
    q, kc, vc = (t.to(DEV) for t in setup(nq, nkv, S, dt, seed=11 + p))
    g = syn.generator(p, "cpu")
    x = syn.activations((K,), g, "cpu").to(DEV)
    wq = tuple(t.to(DEV) for t in syn.int4_weights(nq * 128, K, g, "cpu"))
    wk = [tuple(t.to(DEV) for t in syn.int4_weights(128, K, g, "cpu")) for _ in range(2 * nkv)]
    entries = [(x, *wq, q)] + [(x, *wk[h], kc[h, p]) for h in range(nkv)] + \
              [(x, *wk[nkv + h], vc[h, p]) for h in range(nkv)]
    pos = torch.tensor([p], dtype=torch.int64, device=DEV)
    out = torch.empty(nq * 128, device=DEV, dtype=dt)
    with config.weight_prefetch(True):
        producer = rb.Int4GemvSet(entries, kernel="mma")
        attn = DecodeAttention(q, kc, vc, pos, out, nq, nkv, merge=merge)

        def run():
            producer()
            attn()

        def stale():
            q.fill_(float("nan"))
            kc[:, p].fill_(float("nan"))
            vc[:, p].fill_(float("nan"))
            out.fill_(float("nan"))

        if graph:
            run()
            torch.cuda.synchronize()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                run()
            for _ in range(3):
                stale()
                gr.replay()
        else:
            for _ in range(3):
                stale()
                run()
    torch.cuda.synchronize()
    assert not torch.isnan(q).any() and not torch.isnan(kc[:, p]).any() and not torch.isnan(vc[:, p]).any()
    assert_close(out, oracle(q.cpu(), kc.cpu(), vc.cpu(), p, nq, nkv), f"early loads at position {p}")
