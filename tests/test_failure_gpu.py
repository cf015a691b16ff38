"""The failure path of the bounded waits, shown without a GPU fault.

Every wait in the library's kernels gives up after a limit (rb_set_wait_limit; 4 s by default), sets its bit in
the device error word, skips the work that depended on it and returns, so the context stays usable. These tests
lower the limit to 10 ms and give two waits something that never arrives:
  * the tensor-parallel reduction at world 2 on one GPU, whose second "rank" is a local buffer nobody publishes
    into: the wait for that rank's flag runs out (ERR_TP_WAIT);
  * the fused attention + o_proj/down_proj launch with its heads-done counter left below zero in the workspace
    (as a caller that did not zero it would): the wait for all key-value heads runs out (ERR_ATT_WAIT).
Each then reads and clears the error word, restores the limit, and checks that the next call succeeds with the
right result.
"""
import ctypes

import numpy as np
import pytest
import torch

import rumik_fast_b200 as rb
from oracle import oracle as O
from rumik_fast_b200 import _lib
from rumik_fast_b200 import synthetic as syn
from tests.helpers import assert_close, int4_ref

pytestmark = pytest.mark.gpu
DEV = "cuda"
SHORT_NS = 10_000_000  # 10 ms


@pytest.fixture(autouse=True)
def _gpu(native_lib):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    rb.device_error()
    yield
    _lib.set_wait_limit(0)
    assert rb.device_error() == 0


def _allreduce(a, b, out, bufs, rank, world, flag_off, counter_off):
    arr = (ctypes.c_void_p * len(bufs))(*[t.data_ptr() for t in bufs])
    st = _lib.lib().rb_tp_allreduce_f16(a.data_ptr(), b.data_ptr(), out.data_ptr(), a.numel(), arr, rank, world,
                                        flag_off, counter_off, 0, _lib.stream_ptr(torch.device(DEV)))
    _lib.check("rb_tp_allreduce_f16", st)


def test_tp_peer_that_never_arrives():
    n, world = 3072, 2
    flag_off = 2 * world * n * 4
    counter_off = flag_off + 64
    bufs = [torch.zeros(counter_off + 64, dtype=torch.uint8, device=DEV) for _ in range(world)]
    g = torch.Generator().manual_seed(0)
    a, b = (torch.randn(n, generator=g).half().to(DEV) for _ in range(2))
    out = torch.empty(n, dtype=torch.float16, device=DEV)
    _lib.set_wait_limit(SHORT_NS)
    _allreduce(a, b, out, bufs, 0, world, flag_off, counter_off)   # "rank 1" never publishes its flag
    torch.cuda.synchronize()
    err = rb.device_error()
    assert err & _lib.DEVERR_TP_WAIT, hex(err)
    assert rb.device_error() == 0                                   # read and cleared
    _lib.set_wait_limit(0)
    fresh = torch.zeros(counter_off + 64, dtype=torch.uint8, device=DEV)
    _allreduce(a, b, out, [fresh], 0, 1, flag_off, counter_off)    # the next call works
    torch.cuda.synchronize()
    assert rb.device_error() == 0
    ref = (a.float() + b.float()).half()
    assert torch.equal(out, ref)


def test_fused_attention_heads_that_never_complete():
    from rumik_fast_b200 import fused
    nq, nkv, hd, S, pos = 8, 2, 128, 64, 40
    g = torch.Generator().manual_seed(1)
    q = torch.randn(nq * hd, generator=g).half()
    kc, vc = (torch.randn(nkv, S, hd, generator=g).half() for _ in range(2))
    ob = torch.empty(nq * hd, dtype=torch.float16, device=DEV)
    act = syn.activations((2048,), syn.generator(2, "cpu"), "cpu")
    wo = syn.int4_weights(512, nq * hd, syn.generator(3, "cpu"), "cpu")
    wd = syn.int4_weights(512, 2048, syn.generator(4, "cpu"), "cpu")
    yo, yd = (torch.full((512,), float("nan"), dtype=torch.float16, device=DEV) for _ in range(2))
    pos_t = torch.tensor([pos], dtype=torch.int64, device=DEV)
    st = fused.AttnGemvSet([(act.to(DEV), *(t.to(DEV) for t in wd), yd), (ob, *(t.to(DEV) for t in wo), yo)],
                           q=q.to(DEV), k_cache=kc.to(DEV), v_cache=vc.to(DEV), pos=pos_t, out=ob, n_q_heads=nq,
                           n_kv_heads=nkv)
    heads_done = st.ws.view(torch.int32)[64]                        # the heads-done counter (after 64 tickets)
    heads_done.fill_(-1000)                                         # never reaches n_kv_heads
    _lib.set_wait_limit(SHORT_NS)
    st()
    torch.cuda.synchronize()
    err = rb.device_error()
    assert err & _lib.DEVERR_ATT_WAIT, hex(err)
    assert rb.device_error() == 0
    assert int(st.ws.view(torch.int32)[64]) == 0                    # the launch reset its counters
    _lib.set_wait_limit(0)
    yo.fill_(float("nan"))
    st()                                                            # the next call works
    torch.cuda.synchronize()
    assert rb.device_error() == 0
    ref_att = O.attention_ref(q.numpy(), kc.numpy(), vc.numpy(), pos, nq, nkv, hd, hd ** -0.5, "f16")
    assert_close(ob, ref_att, "attention output")
    assert_close(yo, int4_ref(ob.cpu(), *wo), "o_proj of the attention output")
    assert_close(yd, int4_ref(act, *wd), "down_proj")
