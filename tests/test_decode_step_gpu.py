"""The whole-step kernel (rb_decode_layers, DecodeLayers) against the CPU oracle, stage by stage.

Three layers at the config-1 shapes (3072 hidden, 24 query / 8 key-value heads of 128, MLP 8192) run as one
launch; layer 0 reads the token's int8 embedding row, layers 1 and 2 the residual path, and layer 2 reuses the
buffer copies of layer 0. Each stage is checked on the GPU's own inputs to that stage, so a difference points at
one place (the same method as the per-launch glue tests):
  * the residual bit for bit (engine/fused.py:18-40's fp32 sum rounded once);
  * q (rotated), the k and v cache slot at pos, and silu(gate) * up against rope_kv_ref / swiglu_ref of the
    oracle GEMVs of the oracle's LayerNorm of that residual; the other cache slots untouched;
  * the attention output against attention_ref of the GPU's q and caches;
  * o_proj and down_proj against the oracle GEMVs of the GPU's attention output and activation.
Then: two calls give the same bits, and the workspace is left zeroed.
"""
import numpy as np
import pytest
import torch

import rumik_fast_b200 as rb
from oracle import oracle as O
from rumik_fast_b200 import _lib, fused
from rumik_fast_b200 import synthetic as syn
from rumik_fast_b200.decode_step import DecodeLayers
from tests.helpers import assert_close, np_act, np_f32

pytestmark = pytest.mark.gpu
DEV = "cuda"
H, NQ, NKV, HD, I, S = 3072, 24, 8, 128, 8192, 1024
EPS = 1e-5
# workspace bytes that hold the counters, split-K tickets and attention tickets at these shapes (1-3 layers)
COUNTER_BYTES = 1792


@pytest.fixture(autouse=True)
def _gpu(native_lib):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    rb.device_error()
    _lib.set_wait_limit(500_000_000)  # a wait that cannot finish gives up in 0.5 s here
    yield
    _lib.set_wait_limit(0)
    assert rb.device_error() == 0


def tag(dt):
    return "bf16" if dt == torch.bfloat16 else "f16"


def build(nl, pos, dt, seed=0):
    g = torch.Generator().manual_seed(seed)
    gs = syn.generator(seed + 1, "cpu")
    host = []
    for l in range(nl):
        qkv = syn.int4_weights((NQ + 2 * NKV) * HD, H, gs, "cpu")
        gu = fused.interleave_gate_up(*syn.int4_weights(2 * I, H, gs, "cpu"))
        wo = syn.int4_weights(H, NQ * HD, gs, "cpu")
        wd = syn.int4_weights(H, I, gs, "cpu")
        ln_w = (1 + 0.1 * torch.randn(H, generator=g)).to(dt)
        kc = torch.randn(NKV, S, HD, generator=g).to(dt)
        vc = torch.randn(NKV, S, HD, generator=g).to(dt)
        host.append(dict(qkv=qkv, gate_up=gu, o_proj=wo, down=wd, ln_w=ln_w, k_cache=kc, v_cache=vc, rope=l % 4 != 3))
    dev = [dict((k, tuple(t.to(DEV) for t in v) if isinstance(v, tuple) else (v.to(DEV) if torch.is_tensor(v) else v))
                for k, v in L.items()) for L in host]
    vocab = 4096
    emb_q = torch.randint(-127, 128, (vocab, H), generator=g, dtype=torch.int16).to(torch.int8)
    emb_s = torch.rand(vocab, generator=g) * 0.02 + 0.001
    tok = torch.tensor([1234], dtype=torch.int64)
    cos, sin = O.rope_tables(S, HD, 10000.0, tag(dt))
    to_t = (lambda a: torch.from_numpy(a.astype(np.float16))) if dt == torch.float16 else (
        lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16))
    cos_t, sin_t = to_t(cos), to_t(sin)
    pos_t = torch.tensor([pos], dtype=torch.int64)
    step = DecodeLayers(dev, pos=pos_t.to(DEV), cos=cos_t.to(DEV), sin=sin_t.to(DEV), emb_q=emb_q.to(DEV),
                        emb_s=emb_s.to(DEV), tok=tok.to(DEV), n_q_heads=NQ, n_kv_heads=NKV, eps=EPS)
    return step, host, dev, dict(emb_q=emb_q, emb_s=emb_s, tok=1234, cos=cos, sin=sin)


def gemv(x, w):
    xa, t = np_act(x)
    return O.gemv_int4_ref(xa, *(a.numpy() for a in w), x_dtype=t)


def check_layer(step, host, dev, aux, l, pos, dt, inputs_kept=True):
    """inputs_kept: the buffers layer l read (copy (l - 1) & 1) still hold what layer l - 1 wrote; otherwise
    (a later layer reused them) the residual sum is not checked and h is the LayerNorm of the stored residual."""
    t = tag(dt)
    par = l & 1
    L, D = host[l], dev[l]
    # residual (bit for bit) and the oracle's LayerNorm of it
    if l == 0:
        s_ref, h_ref = O.embed_ln_ref(aux["tok"], aux["emb_q"].numpy(), aux["emb_s"].numpy(), np_act(L["ln_w"])[0],
                                      EPS, t)
    elif inputs_kept:
        s_ref, h_ref = O.add_ln_ref(np_act(step.resid[par ^ 1])[0], np_act(step.o_out[par ^ 1])[0],
                                    np_act(step.down_out[par ^ 1])[0], np_act(L["ln_w"])[0], EPS, t)
    else:
        s_ref, h_ref = O.add_ln_ref(np_act(step.resid[par])[0], None, None, np_act(L["ln_w"])[0], EPS, t)
    assert np.array_equal(np_f32(step.resid[par]), s_ref), f"layer {l}: residual"
    h_in = torch.from_numpy(O.from_f32(h_ref, t).view(np.int16)).view(dt) if dt == torch.bfloat16 else \
        torch.from_numpy(h_ref.astype(np.float16))
    # QKV -> rope -> q and the cache slot
    y = O.round_act(gemv(h_in, L["qkv"]), t)
    q_ref, k_ref, v_ref = O.rope_kv_ref(y, pos, aux["cos"], aux["sin"], NQ, NKV, HD, L["rope"], t)
    assert_close(step.q_out[par], q_ref, f"layer {l}: q")
    assert_close(D["k_cache"][:, pos], k_ref, f"layer {l}: k slot")
    assert_close(D["v_cache"][:, pos], v_ref, f"layer {l}: v slot")
    others = torch.ones(S, dtype=torch.bool)
    others[pos] = False
    assert torch.equal(D["k_cache"][:, others].cpu(), L["k_cache"][:, others])
    assert torch.equal(D["v_cache"][:, others].cpu(), L["v_cache"][:, others])
    # gate_up -> silu(gate) * up
    yg = O.round_act(gemv(h_in, L["gate_up"]), t)
    assert_close(step.act[par], O.swiglu_ref(yg[0::2], yg[1::2], t), f"layer {l}: act")
    # attention of the GPU's q and caches
    qa = np_act(step.q_out[par])[0]
    ref_att = O.attention_ref(qa, np_act(D["k_cache"])[0], np_act(D["v_cache"])[0], pos, NQ, NKV, HD, HD ** -0.5, t)
    assert_close(step.attn_out[par], ref_att, f"layer {l}: attention")
    # o_proj, down_proj of the GPU's inputs
    assert_close(step.o_out[par], gemv(step.attn_out[par].cpu(), L["o_proj"]), f"layer {l}: o_proj")
    assert_close(step.down_out[par], gemv(step.act[par].cpu(), L["down"]), f"layer {l}: down_proj")


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_three_layers_stage_by_stage(dt):
    pos = 511
    step, host, dev, aux = build(3, pos, dt)
    step()
    torch.cuda.synchronize()
    assert rb.device_error() == 0
    # layer 2 wrote copy 0 over layer 0's outputs: check layer 2 (its inputs, copy 1, are layer 1's) and layer 1
    # (its outputs in copy 1; its inputs are gone)
    check_layer(step, host, dev, aux, 2, pos, dt)
    check_layer(step, host, dev, aux, 1, pos, dt, inputs_kept=False)
    assert int(torch.count_nonzero(step.ws[:COUNTER_BYTES])) == 0, "counters and tickets left set"


def test_layer0_from_the_embedding_and_repeatable():
    dt, pos = torch.float16, 40
    step, host, dev, aux = build(1, pos, dt, seed=3)
    step()
    torch.cuda.synchronize()
    check_layer(step, host, dev, aux, 0, pos, dt)
    first = [t.clone() for t in (step.resid[0], step.q_out[0], step.attn_out[0], step.act[0], step.o_out[0],
                                 step.down_out[0])]
    step()
    torch.cuda.synchronize()
    again = (step.resid[0], step.q_out[0], step.attn_out[0], step.act[0], step.o_out[0], step.down_out[0])
    assert all(torch.equal(a, b) for a, b in zip(first, again))
    assert int(torch.count_nonzero(step.ws[:COUNTER_BYTES])) == 0


def test_position_out_of_range_stores_nothing():
    dt = torch.float16
    step, host, dev, aux = build(1, 0, dt, seed=4)
    step._keep[0].fill_(S)             # pos = cache_len: out of range
    before = dev[0]["k_cache"].clone()
    step.resid[0].fill_(0)
    step()
    torch.cuda.synchronize()
    assert rb.device_error() & _lib.DEVERR_ARG
    assert torch.equal(dev[0]["k_cache"], before)
    assert int(torch.count_nonzero(step.resid[0])) == 0
