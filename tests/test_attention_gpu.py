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


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("nq,nkv", [(24, 8), (16, 4), (8, 8), (16, 2)])
def test_attention_matches_oracle(dt, nq, nkv):
    S = 2048
    q, kc, vc = setup(nq, nkv, S, dt, seed=nq + nkv)
    qd, kd, vd = q.to(DEV), kc.to(DEV), vc.to(DEV)
    pos = torch.zeros(1, dtype=torch.int64, device=DEV)
    out = torch.full((nq * 128,), float("nan"), device=DEV, dtype=dt)
    attn = DecodeAttention(qd, kd, vd, pos, out, nq, nkv)
    for p in (0, 1, 31, 33, 200, 1500, S - 1):
        pos.fill_(p)
        attn()
        torch.cuda.synchronize()
        assert_close(out, oracle(q, kc, vc, p, nq, nkv), f"attention at position {p}")


def test_attention_is_deterministic_and_reusable():
    dt, nq, nkv, S = torch.float16, 24, 8, 512
    q, kc, vc = (t.to(DEV) for t in setup(nq, nkv, S, dt, seed=3))
    pos = torch.tensor([300], dtype=torch.int64, device=DEV)
    out = torch.empty(nq * 128, device=DEV, dtype=dt)
    attn = DecodeAttention(q, kc, vc, pos, out, nq, nkv)
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
