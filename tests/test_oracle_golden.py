"""Pin the CPU oracle to the reference: its functions must reproduce the outputs that the reference's own
code produced for the committed fixtures (tests/golden/make_golden.py)."""
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def g4():
    return np.load(os.path.join(GOLD, "golden_int4.npz"))


@pytest.fixture(scope="module")
def g8():
    return np.load(os.path.join(GOLD, "golden_int8.npz"))


@pytest.fixture(scope="module")
def gm():
    return np.load(os.path.join(GOLD, "golden_mm.npz"))


@pytest.mark.parametrize("tag", ["a", "b", "c", "d"])
def test_quantize_int4_bit_exact(g4, tag):
    w = O.bf16_bits_to_f32(g4[f"{tag}_w"])
    q, s, m = O.quantize_int4(w)
    assert np.array_equal(q, g4[f"{tag}_q"])
    assert np.array_equal(s.view(np.uint16), g4[f"{tag}_s"].view(np.uint16))
    assert np.array_equal(m.view(np.uint16), g4[f"{tag}_m"].view(np.uint16))


@pytest.mark.parametrize("tag", ["a", "b", "c", "d", "cfg"])
def test_dequantize_int4_bit_exact(g4, tag):
    deq = O.dequantize_int4(g4[f"{tag}_q"], g4[f"{tag}_s"], g4[f"{tag}_m"])
    assert np.array_equal(deq.view(np.uint32), g4[f"{tag}_deq"].view(np.uint32))


@pytest.mark.parametrize("tag", ["a", "b", "c", "d"])
def test_gemv_int4_ref_matches_reference(g4, tag):
    q, s, m = g4[f"{tag}_q"], g4[f"{tag}_s"], g4[f"{tag}_m"]
    np.testing.assert_allclose(O.gemv_int4_ref(g4[f"{tag}_x16"], q, s, m), g4[f"{tag}_y16"], rtol=2e-5, atol=2e-6)
    np.testing.assert_allclose(O.gemv_int4_ref(g4[f"{tag}_xbf"], q, s, m, x_dtype="bf16"), g4[f"{tag}_ybf"],
                               rtol=2e-5, atol=2e-6)
    np.testing.assert_allclose(O.gemv_int4_ref(g4[f"{tag}_xbat"], q, s, m), g4[f"{tag}_ybat"], rtol=2e-5, atol=2e-6)


def test_gemv_int4_ref_config_style(g4):
    y = O.gemv_int4_ref(g4["cfg_x16"], g4["cfg_q"], g4["cfg_s"], g4["cfg_m"])
    np.testing.assert_allclose(y, g4["cfg_y16"], rtol=2e-5, atol=2e-5)


@pytest.mark.parametrize("tag", ["a", "b"])
def test_quantize_int8_rows_bit_exact(g8, tag):
    q, s = O.quantize_int8_rows(O.bf16_bits_to_f32(g8[f"{tag}_w"]))
    assert np.array_equal(q, g8[f"{tag}_q"])
    assert np.array_equal(s.view(np.uint32), g8[f"{tag}_s"].view(np.uint32))
    assert q.shape[0] % 16 == 0


@pytest.mark.parametrize("tag", ["a", "b"])
def test_gemv_int8_ref_matches_reference(g8, tag):
    q, s = g8[f"{tag}_q"], g8[f"{tag}_s"]
    np.testing.assert_allclose(O.gemv_int8_ref(g8[f"{tag}_x16"], q, s), g8[f"{tag}_y16"], rtol=2e-5, atol=2e-6)
    np.testing.assert_allclose(O.gemv_int8_ref(g8[f"{tag}_xbf"], q, s, x_dtype="bf16"), g8[f"{tag}_ybf"],
                               rtol=2e-5, atol=2e-6)


def test_gemv_int8_signed_storage_equals_offset_storage(g8):
    y_signed = O.gemv_int8_ref(g8["cfg_x16"], g8["cfg_wi8"], g8["cfg_s16"], signed=True)
    y_u8 = O.gemv_int8_ref(g8["cfg_x16"], g8["cfg_qu8"], g8["cfg_s16"])
    np.testing.assert_allclose(y_signed, g8["cfg_y16"], rtol=2e-5, atol=2e-6)
    np.testing.assert_allclose(y_u8, g8["cfg_y16"], rtol=2e-5, atol=2e-6)


@pytest.mark.parametrize("tag", ["a", "b"])
def test_mm_int4_ref_matches_reference(gm, tag):
    Y = O.mm_int4_ref(gm[f"{tag}_X"], gm[f"{tag}_q"], gm[f"{tag}_s"], gm[f"{tag}_m"])
    np.testing.assert_allclose(Y, gm[f"{tag}_Y"], rtol=2e-5, atol=2e-6)


def test_tolerance_check_detects_planted_error(g4):
    """A mistake planted in the oracle's output must fail the acceptance criterion."""
    ref = g4["a_y16"].astype(np.float64)
    assert O.within_tolerance(ref, ref)
    bad = ref.copy()
    bad[3] += 0.01 * np.abs(ref).max()
    assert not O.within_tolerance(bad, ref)
    drift = ref * (1 + 3e-3)
    assert not O.within_tolerance(drift, ref)


def test_bf16_round_trip():
    f = np.array([1.0, -2.5, 3.14159, 1e-3, 65504.0], np.float32)
    b = O.f32_to_bf16_bits(f)
    back = O.bf16_bits_to_f32(b)
    assert np.all(np.abs(back - f) <= np.abs(f) * 2 ** -8)


# ---- decode-layer glue (engine/fused.py add_ln / post), pinned to the reference's cohere_ln and rope ----
@pytest.fixture(scope="module")
def gg():
    return np.load(os.path.join(GOLD, "golden_glue.npz"))


def _stored(a, dt):
    """Fixture storage (bf16 bit patterns or float16) -> float32 values."""
    return O.act_to_f32(a, dt)


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_add_ln_matches_reference(gg, dt):
    s, h = O.add_ln_ref(gg[f"{dt}_ln_x"], gg[f"{dt}_ln_a"], gg[f"{dt}_ln_b"], gg[f"{dt}_ln_w"], 1e-5, dt)
    assert np.array_equal(s, _stored(gg[f"{dt}_ln_s"], dt))           # one fp32 sum, one rounding: exact
    # the mean and variance are fp32 sums in another order than torch's: at most one unit in the last place
    assert O.ulp_diff(h, _stored(gg[f"{dt}_ln_h"], dt), dt).max() <= 1
    _, hn = O.add_ln_ref(gg[f"{dt}_ln_x"], None, None, gg[f"{dt}_ln_w"], 1e-5, dt)
    assert O.ulp_diff(hn, _stored(gg[f"{dt}_ln_hn"], dt), dt).max() <= 1


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_rope_kv_matches_reference(gg, dt):
    nq, nkv, hd, S, pos, theta = (int(v) if i < 5 else float(v) for i, v in enumerate(gg[f"{dt}_rope_meta"]))
    cos, sin = O.rope_tables(S, hd, theta, dt)
    # the oracle's tables against the reference's: fp32 cos/sin of the same angles, rounded to 16 bits
    assert O.ulp_diff(_stored(cos, dt), _stored(gg[f"{dt}_rope_cos"], dt), dt).max() <= 1
    assert O.ulp_diff(_stored(sin, dt), _stored(gg[f"{dt}_rope_sin"], dt), dt).max() <= 1
    y = _stored(gg[f"{dt}_rope_y"], dt)
    q, k, v = O.rope_kv_ref(y, pos, gg[f"{dt}_rope_cos"], gg[f"{dt}_rope_sin"], nq, nkv, hd, True, dt)
    assert np.array_equal(q, _stored(gg[f"{dt}_rope_q"], dt))
    assert np.array_equal(k, _stored(gg[f"{dt}_rope_k"], dt).reshape(nkv, hd))
    assert np.array_equal(v, y[(nq + nkv) * hd:].reshape(nkv, hd))
    q0, k0, _ = O.rope_kv_ref(y, pos, None, None, nq, nkv, hd, False, dt)   # no position embedding: a copy
    assert np.array_equal(q0, y[:nq * hd]) and np.array_equal(k0.reshape(-1), y[nq * hd:(nq + nkv) * hd])


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_swiglu_matches_reference(gg, dt):
    act = O.swiglu_ref(_stored(gg[f"{dt}_sw_g"], dt), _stored(gg[f"{dt}_sw_u"], dt), dt)
    assert O.ulp_diff(act, _stored(gg[f"{dt}_sw_act"], dt), dt).max() <= 1


def test_gate_up_order_pairs_each_gate_with_its_up_channel():
    order = O.gate_up_order(256)
    assert sorted(order.tolist()) == list(range(512))
    assert order[0::2].tolist() == list(range(256)) and order[1::2].tolist() == list(range(256, 512))


def test_attention_matches_reference(gg):
    nq, nkv, hd, S, pos = (int(v) for v in gg["attn_meta"])
    o = O.attention_ref(gg["attn_q"], gg["attn_k"], gg["attn_v"], pos, nq, nkv, hd, hd ** -0.5, "bf16")
    assert O.ulp_diff(o, _stored(gg["attn_o"], "bf16"), "bf16").max() <= 1


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_embed_ln_matches_reference(gg, dt):
    for i, tok in enumerate(gg["emb_ids"]):
        s, h = O.embed_ln_ref(int(tok), gg["emb_q"], gg["emb_s"], gg[f"{dt}_emb_w"], 1e-5, dt)
        assert np.array_equal(s, _stored(gg[f"{dt}_emb_x"][i], dt))     # one product, one rounding: exact
        assert O.ulp_diff(h, _stored(gg[f"{dt}_emb_h"][i], dt), dt).max() <= 1


@pytest.mark.parametrize("case", [0, 1, 2])
def test_sampling_tail_matches_reference(gg, case):
    """The stop predictor and the top-k / Gumbel-max pick against the reference's own eager functions
    (engine/rumik_int4.py:174-191) on the real head size, with the same uniforms."""
    m = gg[f"smp{case}_meta"]
    step, min_new, top_k, end_idx, end_id = (int(v) for v in m)
    s = O.stop_logit_ref(gg[f"smp{case}_hn"], gg[f"smp{case}_lnw"], gg[f"smp{case}_lnb"],
                         O.bf16_bits_to_f32(gg[f"smp{case}_w1"]), gg[f"smp{case}_b1"], gg[f"smp{case}_w2"],
                         gg[f"smp{case}_b2"], "bf16")
    assert (s > 0) == bool(gg[f"smp{case}_stop"])
    logits = O.bf16_bits_to_f32(gg[f"smp{case}_logits"])
    nxt = O.pick_ref(logits, step, min_new, end_idx, gg[f"smp{case}_u"], top_k, 1 / 0.8, gg["smp_ids"], s, end_id)
    assert nxt == int(gg[f"smp{case}_next"])


@pytest.mark.parametrize("tag", ["a", "b", "c", "d", "cfg"])
def test_torch_cpu_path_matches_reference(g4, tag):
    """The torch restatement timed as the CPU baseline (oracle/reference_cpu.py) gives the reference's own
    dequantised weights bit for bit and its GEMV to fp32 round-off."""
    import torch
    from oracle import reference_cpu as R
    q, s, m = (torch.from_numpy(np.ascontiguousarray(g4[f"{tag}_{k}"])) for k in "qsm")
    deq = R.dequantize(q, s, m)
    assert np.array_equal(deq.numpy().view(np.uint32), g4[f"{tag}_deq"].view(np.uint32))
    y = R.gemv_int4_torch(torch.from_numpy(g4[f"{tag}_x16"]), q, s, m)
    np.testing.assert_allclose(y.numpy(), g4[f"{tag}_y16"], rtol=2e-5, atol=2e-5)


def test_torch_cpu_int8_matches_reference(g8):
    import torch
    from oracle import reference_cpu as R
    x = torch.from_numpy(g8["cfg_x16"])
    s = torch.from_numpy(g8["cfg_s16"])
    y_signed = R.gemv_int8_torch(x, torch.from_numpy(g8["cfg_wi8"]), s, signed=True)
    y_u8 = R.gemv_int8_torch(x, torch.from_numpy(g8["cfg_qu8"]), s, signed=False)
    np.testing.assert_allclose(y_signed.numpy(), g8["cfg_y16"], rtol=2e-5, atol=2e-6)
    np.testing.assert_allclose(y_u8.numpy(), g8["cfg_y16"], rtol=2e-5, atol=2e-6)
