"""The fused decode-layer glue (rb_gemv_int4_fused, rb_add_layernorm) on the GPU against the CPU oracle.

Each stage is checked on the stage's own inputs so that a difference points at one place:
  * the add + LayerNorm prologue: the new residual bit for bit, h within one unit in the last place (the mean
    and variance are fp32 sums in another order), and the GEMVs of h against the oracle GEMV of the GPU's h;
  * the epilogues on the GPU's own GEMV results (stored alongside): rope / KV routing and silu(gate) * up
    within one unit in the last place of the oracle applied to those results, and untouched cache slots;
  * the whole layer-input launch at the benchmark shapes against the oracle's unfused chain.
"""
import ctypes

import numpy as np
import pytest
import torch

import rumik_fast_b200 as rb
from oracle import oracle as O
from rumik_fast_b200 import _lib, fused
from rumik_fast_b200 import synthetic as syn
from rumik_fast_b200.gemv_set import _ws_len, _ws_ptr, workspace
from tests.helpers import assert_close, int4_ref, np_act, np_f32

pytestmark = pytest.mark.gpu
DEV = "cuda"
DTYPES = [torch.float16, torch.bfloat16]


@pytest.fixture(scope="module", autouse=True)
def _gpu(native_lib):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    rb.device_error()
    yield
    assert rb.device_error() == 0


def tag(dt):
    return "bf16" if dt == torch.bfloat16 else "f16"


def vals(t):
    """A 16-bit tensor -> float32 numpy values."""
    return np_f32(t)


def weights(n, k, g):
    q, s, m = syn.int4_weights(n, k, g, "cpu")
    return (q, s, m), tuple(t.to(DEV) for t in (q, s, m))


def rand(shape, g, dt, scale=1.0, shift=0.0):
    return (torch.randn(shape, generator=g) * scale + shift).to(dt)


def ln_inputs(H, g, dt):
    x = rand(H, g, dt, 4.0)
    a = rand(H, g, dt)
    b = rand(H, g, dt, 0.5)
    w = rand(H, g, dt, 0.1, 1.0)
    return x, a, b, w


KERNELS = ["tc", "mma"]  # the glue runs in both GEMV kernels (tcgen05 with split K, and warp-MMA)


def run_fused(entries, epis=None, ln=None, x_dtype=torch.float16, y_dtype=torch.float16, kernel="tc"):
    """One rb_gemv_int4_fused call on the given kernel (tc: through the split-K workspace the list uses)."""
    kf = _lib.KERNEL_FLAGS[kernel]
    d = (_lib.GemvDesc * len(entries))(*entries)
    e = (_lib.GemvEpi * len(entries))(*epis) if epis else None
    ws = workspace(d, len(entries), torch.device(DEV), kf)
    st = _lib.lib().rb_gemv_int4_fused(d, e, len(entries), ctypes.byref(ln.c) if ln else None, None, _ws_ptr(ws),
                                       _ws_len(ws), _lib.dtype_code(x_dtype), _lib.dtype_code(y_dtype),
                                       rb.config.flags() | kf, _lib.stream_ptr(torch.device(DEV)))
    _lib.check("rb_gemv_int4_fused", st)
    return ws


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("dt", DTYPES)
def test_add_ln_prologue_then_gemvs(dt, kernel):
    g = syn.generator(1, "cpu")
    H = 3072
    x, a, b, w = ln_inputs(H, g, dt)
    xd, ad, bd, wd = (t.to(DEV) for t in (x, a, b, w))
    x_out = torch.full((H,), float("nan"), device=DEV, dtype=dt)
    h_out = torch.full((H,), float("nan"), device=DEV, dtype=dt)
    ln = fused.AddLn(xd, ad, bd, wd, x_out, eps=1e-5, h_out=h_out)
    shapes = [(384, H), (1000, H)]   # 1000: a partial last block
    W = [weights(n, k, g) for n, k in shapes]
    ys = [torch.full((n,), float("nan"), device=DEV, dtype=dt) for n, _ in shapes]
    run_fused([_lib.GemvDesc(None, y.data_ptr(), *(t.data_ptr() for t in wd), n, H)
               for (n, _), (_, wd), y in zip(shapes, W, ys)], ln=ln, x_dtype=dt, y_dtype=dt, kernel=kernel)
    torch.cuda.synchronize()
    s_ref, h_ref = O.add_ln_ref(np_act(x)[0], np_act(a)[0], np_act(b)[0], np_act(w)[0], 1e-5, tag(dt))
    assert np.array_equal(vals(x_out), s_ref)
    assert O.ulp_diff(vals(h_out), h_ref, tag(dt)).max() <= 1
    for (wh, _), y in zip(W, ys):
        assert_close(y, int4_ref(h_out.cpu(), *wh), "GEMV of the normalised vector")
    # the standalone add + LayerNorm gives the same bits as the prologue
    x2 = torch.empty_like(x_out)
    h2 = torch.empty_like(h_out)
    fused.add_layernorm(fused.AddLn(xd, ad, bd, wd, x2, eps=1e-5, h_out=h2))
    torch.cuda.synchronize()
    assert torch.equal(x2, x_out) and torch.equal(h2, h_out)


@pytest.mark.parametrize("dt", DTYPES)
def test_add_ln_without_added_terms(dt):
    g = syn.generator(2, "cpu")
    H = 2048                               # the engine's hidden size
    x, _, _, w = ln_inputs(H, g, dt)
    xd, wd = x.to(DEV), w.to(DEV)
    h = torch.empty(H, device=DEV, dtype=dt)
    fused.add_layernorm(fused.AddLn(xd, None, None, wd, None, eps=1e-5, h_out=h))
    torch.cuda.synchronize()
    _, h_ref = O.add_ln_ref(np_act(x)[0], None, None, np_act(w)[0], 1e-5, tag(dt))
    assert O.ulp_diff(vals(h), h_ref, tag(dt)).max() <= 1


def rope_setup(dt, nq, nkv, hd, S, g):
    cos_n, sin_n = O.rope_tables(S, hd, 10000.0, tag(dt))
    to_t = (lambda a: torch.from_numpy(a.view(np.int16)).view(torch.bfloat16)) if dt == torch.bfloat16 else \
        (lambda a: torch.from_numpy(a))
    cos, sin = to_t(cos_n).to(DEV), to_t(sin_n).to(DEV)
    kc = rand((nkv, S, hd), g, dt).to(DEV)          # arbitrary prior cache contents: must survive
    vc = rand((nkv, S, hd), g, dt).to(DEV)
    return cos_n, sin_n, cos, sin, kc, vc


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("hd,rope", [(128, True), (128, False), (64, True)])
def test_rope_kv_epilogue(dt, hd, rope, kernel):
    g = syn.generator(3, "cpu")
    nq, nkv, S, pos, K = 4, 2, 48, 37, 1024
    N = (nq + 2 * nkv) * hd
    (wh, wd) = weights(N, K, g)
    xin = rand(K, g, dt).to(DEV)
    cos_n, sin_n, cos, sin, kc, vc = rope_setup(dt, nq, nkv, hd, S, g)
    kc0, vc0 = kc.clone(), vc.clone()
    q_out = torch.full((nq * hd,), float("nan"), device=DEV, dtype=dt)
    y = torch.empty(N, device=DEV, dtype=dt)
    pos_t = torch.tensor([pos], device=DEV, dtype=torch.int64)
    epi = _lib.GemvEpi(_lib.EPI_ROPE_KV, int(rope), nq, nkv, hd, S, pos_t.data_ptr(), cos.data_ptr(), sin.data_ptr(),
                       q_out.data_ptr(), kc.data_ptr(), vc.data_ptr(), None)
    run_fused([_lib.GemvDesc(xin.data_ptr(), y.data_ptr(), *(t.data_ptr() for t in wd), N, K)], [epi],
              x_dtype=dt, y_dtype=dt, kernel=kernel)
    torch.cuda.synchronize()
    assert_close(y, int4_ref(xin.cpu(), *wh), "QKV GEMV")
    q_ref, k_ref, v_ref = O.rope_kv_ref(vals(y), pos, cos_n, sin_n, nq, nkv, hd, rope, tag(dt))
    assert O.ulp_diff(vals(q_out), q_ref, tag(dt)).max() <= 1
    assert O.ulp_diff(vals(kc[:, pos]), k_ref, tag(dt)).max() <= 1
    assert np.array_equal(vals(vc[:, pos]), v_ref)                       # values are copied
    others = [p for p in range(S) if p != pos]
    assert torch.equal(kc[:, others], kc0[:, others]) and torch.equal(vc[:, others], vc0[:, others])


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("dt", DTYPES)
def test_swiglu_epilogue(dt, kernel):
    g = syn.generator(4, "cpu")
    inter, K = 640, 1024
    q, s, m = syn.int4_weights(2 * inter, K, g, "cpu")           # rows [gate (inter) | up (inter)]
    gq, gs, gm = (t.to(DEV) for t in fused.interleave_gate_up(q, s, m))
    xin = rand(K, g, dt).to(DEV)
    act = torch.full((inter,), float("nan"), device=DEV, dtype=dt)
    y = torch.empty(2 * inter, device=DEV, dtype=dt)
    epi = _lib.GemvEpi(_lib.EPI_SWIGLU, 0, 0, 0, 0, 0, None, None, None, None, None, None, act.data_ptr())
    run_fused([_lib.GemvDesc(xin.data_ptr(), y.data_ptr(), gq.data_ptr(), gs.data_ptr(), gm.data_ptr(), 2 * inter,
                             K)], [epi], x_dtype=dt, y_dtype=dt, kernel=kernel)
    torch.cuda.synchronize()
    order = O.gate_up_order(inter)
    y_nat = np.empty(2 * inter, np.float32)
    y_nat[order] = vals(y)                                         # back to [gate | up]
    assert_close(torch.from_numpy(y_nat).to(dt), int4_ref(xin.cpu(), q, s, m), "gate_up GEMV")
    act_ref = O.swiglu_ref(y_nat[:inter], y_nat[inter:], tag(dt))
    assert O.ulp_diff(vals(act), act_ref, tag(dt)).max() <= 1


@pytest.mark.parametrize("kernel", [None, "tc"])
@pytest.mark.parametrize("dt", DTYPES)
def test_layer_input_launch_at_benchmark_shapes(dt, kernel):
    """add_ln + QKV (24 query / 8 key-value heads of 128) + gate_up (2 x 8192) + post as ONE launch, against the
    oracle's unfused chain add_ln -> fp32 GEMV -> round -> rope / KV / silu * up."""
    g = syn.generator(5, "cpu")
    H, nq, nkv, hd, inter, S, pos = 3072, 24, 8, 128, 8192, 64, 5
    x, a, b, w = ln_inputs(H, g, dt)
    xd, ad, bd, wd = (t.to(DEV) for t in (x, a, b, w))
    qkv_h, qkv_d = weights((nq + 2 * nkv) * hd, H, g)
    gu_h = syn.int4_weights(2 * inter, H, g, "cpu")
    gu_d = tuple(t.to(DEV) for t in fused.interleave_gate_up(*gu_h))
    cos_n, sin_n, cos, sin, kc, vc = rope_setup(dt, nq, nkv, hd, S, g)
    x_out = torch.empty(H, device=DEV, dtype=dt)
    q_out = torch.empty(nq * hd, device=DEV, dtype=dt)
    act = torch.empty(inter, device=DEV, dtype=dt)
    pos_t = torch.tensor([pos], device=DEV, dtype=torch.int64)
    layer = fused.AddLnGemvPost(qkv_d, gu_d, add_ln=fused.AddLn(xd, ad, bd, wd, x_out, eps=1e-5), pos=pos_t,
                                cos=cos, sin=sin, k_cache=kc, v_cache=vc, q_out=q_out, act=act, n_q_heads=nq,
                                n_kv_heads=nkv, rope=True, kernel=kernel)
    layer()
    torch.cuda.synchronize()
    t = tag(dt)
    s_ref, h_ref = O.add_ln_ref(np_act(x)[0], np_act(a)[0], np_act(b)[0], np_act(w)[0], 1e-5, t)
    assert np.array_equal(vals(x_out), s_ref)
    h_st = O.from_f32(h_ref, t)
    y_qkv = O.round_act(O.gemv_int4_ref(h_st, *(u.numpy() for u in qkv_h), x_dtype=t), t)
    q_ref, k_ref, v_ref = O.rope_kv_ref(y_qkv, pos, cos_n, sin_n, nq, nkv, hd, True, t)
    y_gu = O.round_act(O.gemv_int4_ref(h_st, *(u.numpy() for u in gu_h), x_dtype=t), t)
    act_ref = O.swiglu_ref(y_gu[:inter], y_gu[inter:], t)
    for got, ref, what in ((q_out, q_ref, "q"), (kc[:, pos], k_ref, "k"), (vc[:, pos], v_ref, "v"),
                           (act, act_ref, "act")):
        assert_close(got, ref, what)


@pytest.mark.parametrize("dt", DTYPES)
def test_layer_input_launch_with_8bit_scales(dt):
    """The same layer-input launch with both weight sets carrying 8-bit double-quantised scales (the launch runs
    on the tcgen05 kernel), against the oracle's unfused chain on the fp16 scale / min those scales decode to."""
    from rumik_fast_b200 import scales8
    g = syn.generator(15, "cpu")
    H, nq, nkv, hd, inter, S, pos = 3072, 24, 8, 128, 8192, 64, 9
    x, a, b, w = ln_inputs(H, g, dt)
    xd, ad, bd, wd = (t.to(DEV) for t in (x, a, b, w))
    qkv_q, qkv_s, qkv_m = syn.int4_weights((nq + 2 * nkv) * hd, H, g, "cpu")
    gu_q, gu_s, gu_m = fused.interleave_gate_up(*syn.int4_weights(2 * inter, H, g, "cpu"))
    sc_qkv, sc_gu = scales8.pack(qkv_s, qkv_m), scales8.pack(gu_s, gu_m)
    cos_n, sin_n, cos, sin, kc, vc = rope_setup(dt, nq, nkv, hd, S, g)
    x_out = torch.empty(H, device=DEV, dtype=dt)
    q_out = torch.empty(nq * hd, device=DEV, dtype=dt)
    act = torch.empty(inter, device=DEV, dtype=dt)
    pos_t = torch.tensor([pos], device=DEV, dtype=torch.int64)
    on_dev = lambda sc: scales8.Scales8(sc.sz.to(DEV), sc.s_row.to(DEV))  # noqa: E731
    layer = fused.AddLnGemvPost((qkv_q.to(DEV), on_dev(sc_qkv), None), (gu_q.to(DEV), on_dev(sc_gu), None),
                                add_ln=fused.AddLn(xd, ad, bd, wd, x_out, eps=1e-5), pos=pos_t, cos=cos, sin=sin,
                                k_cache=kc, v_cache=vc, q_out=q_out, act=act, n_q_heads=nq, n_kv_heads=nkv,
                                rope=True)
    layer()
    torch.cuda.synchronize()
    t = tag(dt)
    s_ref, h_ref = O.add_ln_ref(np_act(x)[0], np_act(a)[0], np_act(b)[0], np_act(w)[0], 1e-5, t)
    assert np.array_equal(vals(x_out), s_ref)
    h_st = O.from_f32(h_ref, t)

    def gemv(q, sc):
        s16, m16 = O.unpack_scales8(sc.sz.numpy().view(np.uint16), sc.s_row.numpy())
        return O.round_act(O.gemv_int4_ref(h_st, q.numpy(), s16, m16, x_dtype=t), t)
    y_qkv = gemv(qkv_q, sc_qkv)
    q_ref, k_ref, v_ref = O.rope_kv_ref(y_qkv, pos, cos_n, sin_n, nq, nkv, hd, True, t)
    y_gu = gemv(gu_q, sc_gu)                          # interleaved rows: gate c at 2c, up c at 2c + 1
    act_ref = O.swiglu_ref(y_gu[0::2], y_gu[1::2], t)
    for got, ref, what in ((q_out, q_ref, "q"), (kc[:, pos], k_ref, "k"), (vc[:, pos], v_ref, "v"),
                           (act, act_ref, "act")):
        assert_close(got, ref, what)


def test_layer_input_in_a_cuda_graph_follows_the_position():
    """Captured once, replayed with pos advanced on the device: each replay writes the next cache slot."""
    dt = torch.float16
    g = syn.generator(6, "cpu")
    H, nq, nkv, hd, inter, S = 1024, 2, 1, 128, 256, 8
    h = rand(H, g, dt).to(DEV)
    _, qkv_d = weights((nq + 2 * nkv) * hd, H, g)
    gu_d = tuple(t.to(DEV) for t in fused.interleave_gate_up(*syn.int4_weights(2 * inter, H, g, "cpu")))
    _, _, cos, sin, _, _ = rope_setup(dt, nq, nkv, hd, S, g)
    kc = torch.zeros((nkv, S, hd), device=DEV, dtype=dt)
    vc = torch.zeros_like(kc)
    q_out = torch.empty(nq * hd, device=DEV, dtype=dt)
    act = torch.empty(inter, device=DEV, dtype=dt)
    pos = torch.zeros(1, device=DEV, dtype=torch.int64)
    layer = fused.AddLnGemvPost(qkv_d, gu_d, h=h, pos=pos, cos=cos, sin=sin, k_cache=kc, v_cache=vc, q_out=q_out,
                                act=act, n_q_heads=nq, n_kv_heads=nkv, rope=False)
    layer()                                     # warm-up outside the capture (sets the smem limit once)
    torch.cuda.synchronize()
    v0 = vc[:, 0].clone()
    kc.zero_()
    vc.zero_()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        layer()
        pos.add_(1)
    pos.zero_()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert pos.item() == 3
    for p in range(3):                          # same input every step: the same values in slots 0, 1, 2
        assert torch.equal(vc[:, p], v0)
    assert torch.count_nonzero(vc[:, 3:]) == 0 and torch.count_nonzero(kc[:, 3:]) == 0


@pytest.mark.parametrize("kernel", KERNELS)
def test_position_outside_the_cache_stores_nothing(kernel):
    dt = torch.float16
    g = syn.generator(7, "cpu")
    nq, nkv, hd, S, K = 2, 1, 128, 16, 512
    N = (nq + 2 * nkv) * hd
    _, wd = weights(N, K, g)
    xin = rand(K, g, dt).to(DEV)
    kc = torch.zeros((nkv, S, hd), device=DEV, dtype=dt)
    vc = torch.zeros_like(kc)
    q_out = torch.zeros(nq * hd, device=DEV, dtype=dt)
    for bad in (S, -1):
        pos = torch.tensor([bad], device=DEV, dtype=torch.int64)
        epi = _lib.GemvEpi(_lib.EPI_ROPE_KV, 0, nq, nkv, hd, S, pos.data_ptr(), None, None, q_out.data_ptr(),
                           kc.data_ptr(), vc.data_ptr(), None)
        run_fused([_lib.GemvDesc(xin.data_ptr(), None, *(t.data_ptr() for t in wd), N, K)], [epi], kernel=kernel)
        assert rb.device_error() & _lib.DEVERR_ARG
        assert torch.count_nonzero(kc) == 0 and torch.count_nonzero(vc) == 0 and torch.count_nonzero(q_out) == 0


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("dt", DTYPES)
def test_embedding_prologue(dt, kernel):
    """Layer 0: the residual is the token's int8 embedding row times its scale (engine/fused.py:18-27), read on the
    device from the token id; then the LayerNorm and the GEMVs, and the standalone kernel gives the same bits."""
    g = syn.generator(8, "cpu")
    vocab, H = 1000, 3072
    emb_q = torch.randint(-127, 128, (vocab, H), generator=g, dtype=torch.int16).to(torch.int8)
    emb_s = torch.rand(vocab, generator=g) * 0.02 + 0.001
    w = rand(H, g, dt, 0.1, 1.0)
    eq, es, wd = emb_q.to(DEV), emb_s.to(DEV), w.to(DEV)
    tok = torch.tensor([731], device=DEV, dtype=torch.int64)
    x_out = torch.empty(H, device=DEV, dtype=dt)
    h_out = torch.empty(H, device=DEV, dtype=dt)
    ln = fused.AddLn.from_embedding(eq, es, tok, wd, x_out, eps=1e-5, h_out=h_out)
    (wh, wdd) = weights(640, H, g)
    y = torch.empty(640, device=DEV, dtype=dt)
    run_fused([_lib.GemvDesc(None, y.data_ptr(), *(t.data_ptr() for t in wdd), 640, H)], ln=ln, x_dtype=dt,
              y_dtype=dt, kernel=kernel)
    torch.cuda.synchronize()
    s_ref, h_ref = O.embed_ln_ref(731, emb_q.numpy(), emb_s.numpy(), np_act(w)[0], 1e-5, tag(dt))
    assert np.array_equal(vals(x_out), s_ref)
    assert O.ulp_diff(vals(h_out), h_ref, tag(dt)).max() <= 1
    assert_close(y, int4_ref(h_out.cpu(), *wh), "GEMV of the embedded, normalised token")
    x2, h2 = torch.empty_like(x_out), torch.empty_like(h_out)
    fused.add_layernorm(fused.AddLn.from_embedding(eq, es, tok, wd, x2, eps=1e-5, h_out=h2))
    torch.cuda.synchronize()
    assert torch.equal(x2, x_out) and torch.equal(h2, h_out)
    tok.fill_(vocab)                                   # outside the table: row 0, error bit set
    fused.add_layernorm(fused.AddLn.from_embedding(eq, es, tok, wd, x2, eps=1e-5, h_out=h2))
    assert rb.device_error() & _lib.DEVERR_ARG
    s0, _ = O.embed_ln_ref(0, emb_q.numpy(), emb_s.numpy(), np_act(w)[0], 1e-5, tag(dt))
    assert np.array_equal(vals(x2), s0)
