"""Generate the golden fixtures of this directory from the reference's OWN functions.

Run in a container where the rumik-fast reference is mounted (it is not needed anywhere else):

    python tests/golden/make_golden.py --ref /path/to/rumik-fast

It imports kernels/int4_gemv.py (quantize, dequantize) and kernels/cuda_gemv.py (quantize_int8_rows) from the
reference on the CPU and records, for small seeded inputs, the reference's outputs:
  * golden_int4.npz : bf16 weights -> reference quantize() -> (q, s, m); reference dequantize(); and
                      y = dequantize(q, s, m) @ x.float() (kernels/bench_cuda.py:38) for fp16/bf16 x,
                      batched x, and benchmark-config-style codes/scales/mins.
  * golden_int8.npz : bf16 head rows -> reference quantize_int8_rows(w, pad_to=16) -> (q, s); and
                      y = ((q - 128) * s) @ x (kernels/cuda_gemv.py:245-246).
  * golden_mm.npz   : Y = X.float() @ dequantize(q, s, m).t() (kernels/mm_int4.py:96).
  * golden_glue.npz : the decode-layer glue around the GEMVs, with engine/rumik_int4.py's own cohere_ln
                      (:38-43) and rope (:46-52): add_ln's residual sum (engine/fused.py:35-36, restated: an fp32
                      sum rounded once) then cohere_ln; rope of query/key heads at one position with the rotary
                      tables built as engine/rumik_int4.py:107-109; silu(gate) * up in fp32 (engine/fused.py:83,
                      with torch's silu), for bf16 (the engine's type) and fp16; decode attention with the
                      reference's _attend (engine/rumik_int4.py:163-171) and its decode mask (:204), bf16.
bf16 tensors are stored as uint16 bit patterns.  `--which glue` (or int4, int8, mm) regenerates one file.
"""
import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def bits(t):
    """bf16 tensor -> uint16 numpy bit pattern; fp16 -> numpy float16; others as is."""
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("RUMIK_REFERENCE"), required="RUMIK_REFERENCE" not in os.environ,
                    help="root of the rumik-fast checkout (or set RUMIK_REFERENCE)")
    ap.add_argument("--which", default="all", choices=["all", "int4", "int8", "mm", "glue"])
    a = ap.parse_args()
    sys.path.insert(0, os.path.join(a.ref, "kernels"))
    if a.which in ("all", "glue"):
        make_glue(a.ref)
    if a.which == "glue":
        return
    import int4_gemv as ref4  # noqa: E402  (reference module)
    import cuda_gemv as refc  # noqa: E402  (reference module; load_inline is only called lazily)

    out4 = {}
    # (A) reference-style weights: randn * 0.02 in bf16 (kernels/bench_cuda.py:36), several shapes
    for tag, (n, k, seed) in {"a": (64, 256, 0), "b": (24, 384, 1), "c": (8, 128, 2), "d": (40, 1024, 3)}.items():
        g = torch.Generator().manual_seed(seed)
        w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
        q, s, m = ref4.quantize(w)
        deq = ref4.dequantize(q, s, m)
        x16 = torch.randn(k, generator=g).to(torch.float16)
        xb = torch.randn(k, generator=g).to(torch.bfloat16)
        xbat = torch.randn(3, k, generator=g).to(torch.float16)
        out4.update({f"{tag}_w": bits(w), f"{tag}_q": bits(q), f"{tag}_s": bits(s), f"{tag}_m": bits(m),
                     f"{tag}_deq": deq.numpy(),
                     f"{tag}_x16": bits(x16), f"{tag}_y16": (deq @ x16.float()).numpy(),
                     f"{tag}_xbf": bits(xb), f"{tag}_ybf": (deq @ xb.float()).numpy(),
                     f"{tag}_xbat": bits(xbat), f"{tag}_ybat": (xbat.float() @ deq.t()).numpy()})
    # (B) benchmark config-0 style: codes uniform 0..15, scale ~U(0.002, 0.02), min = -7.5 scale + N(0, 1e-3)
    g = torch.Generator().manual_seed(10)
    n, k = 48, 512
    codes = torch.randint(0, 16, (n, k), generator=g, dtype=torch.uint8)
    q = (codes[:, 0::2] | (codes[:, 1::2] << 4)).contiguous()
    s = (torch.rand(n, k // 128, generator=g) * 0.018 + 0.002).to(torch.float16)
    m = (-7.5 * s.float() + torch.randn(n, k // 128, generator=g) * 1e-3).to(torch.float16)
    x = torch.randn(k, generator=g).to(torch.float16)
    deq = ref4.dequantize(q, s, m)
    out4.update({"cfg_q": bits(q), "cfg_s": bits(s), "cfg_m": bits(m), "cfg_deq": deq.numpy(),
                 "cfg_x16": bits(x), "cfg_y16": (deq @ x.float()).numpy()})
    np.savez_compressed(os.path.join(HERE, "golden_int4.npz"), **out4)

    out8 = {}
    for tag, (n, k, seed) in {"a": (13, 256, 20), "b": (33, 192, 21)}.items():
        g = torch.Generator().manual_seed(seed)
        w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
        q, s = refc.quantize_int8_rows(w)
        x16 = torch.randn(k, generator=g).to(torch.float16)
        xb = torch.randn(k, generator=g).to(torch.bfloat16)
        wq = (q.int() - 128).float() * s[:, None]
        out8.update({f"{tag}_w": bits(w), f"{tag}_q": bits(q), f"{tag}_s": bits(s),
                     f"{tag}_x16": bits(x16), f"{tag}_y16": (wq @ x16.float()).numpy(),
                     f"{tag}_xbf": bits(xb), f"{tag}_ybf": (wq @ xb.float()).numpy()})
    # benchmark config-2 style: W int8 uniform -127..127, fp16 row scale ~U(1e-4, 1e-3), unpadded N
    g = torch.Generator().manual_seed(22)
    n, k = 37, 320
    wi8 = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int16).to(torch.int8)
    s16 = (torch.rand(n, generator=g) * 9e-4 + 1e-4).to(torch.float16)
    x = torch.randn(k, generator=g).to(torch.float16)
    qu8 = (wi8.to(torch.int16) + 128).to(torch.uint8)          # the reference's storage of the same weights
    y = (((qu8.int() - 128).float() * s16.float()[:, None]) @ x.float())
    out8.update({"cfg_wi8": wi8.numpy(), "cfg_qu8": bits(qu8), "cfg_s16": bits(s16), "cfg_x16": bits(x),
                 "cfg_y16": y.numpy()})
    np.savez_compressed(os.path.join(HERE, "golden_int8.npz"), **out8)

    outm = {}
    for tag, (t, n, k, seed) in {"a": (5, 64, 256, 30), "b": (37, 80, 384, 31)}.items():
        g = torch.Generator().manual_seed(seed)
        w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
        q, s, m = ref4.quantize(w)
        X = torch.randn(t, k, generator=g).to(torch.float16)
        outm.update({f"{tag}_q": bits(q), f"{tag}_s": bits(s), f"{tag}_m": bits(m), f"{tag}_X": bits(X),
                     f"{tag}_Y": (X.float() @ ref4.dequantize(q, s, m).t()).numpy()})
    np.savez_compressed(os.path.join(HERE, "golden_mm.npz"), **outm)
    for f in ("golden_int4.npz", "golden_int8.npz", "golden_mm.npz"):
        print(f, os.path.getsize(os.path.join(HERE, f)), "bytes")


def make_glue(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "engine"))
    import rumik_int4 as refe  # noqa: E402  (reference module: cohere_ln, rope)
    import torch.nn.functional as F

    out = {}
    for dname, dt in (("bf16", torch.bfloat16), ("f16", torch.float16)):
        g = torch.Generator().manual_seed(40 if dt == torch.bfloat16 else 41)
        H, eps = 384, 1e-5
        x = (torch.randn(H, generator=g) * 4).to(dt)
        a_ = torch.randn(H, generator=g).to(dt)
        b_ = (torch.randn(H, generator=g) * 0.5).to(dt)
        w = (1 + 0.1 * torch.randn(H, generator=g)).to(dt)
        s = (x.float() + a_.float() + b_.float()).to(dt)          # engine/fused.py:35-36
        h = refe.cohere_ln(s, w, eps)
        hn = refe.cohere_ln(x, w, eps)                            # no added terms
        out.update({f"{dname}_ln_x": bits(x), f"{dname}_ln_a": bits(a_), f"{dname}_ln_b": bits(b_),
                    f"{dname}_ln_w": bits(w), f"{dname}_ln_s": bits(s), f"{dname}_ln_h": bits(h),
                    f"{dname}_ln_hn": bits(hn)})
        nq, nkv, hd, S, pos, theta = 3, 2, 64, 40, 17, 10000.0
        inv = 1.0 / (theta ** (torch.arange(0, hd, 2).float() / hd))   # engine/rumik_int4.py:107-109
        ang = torch.outer(torch.arange(S).float(), inv).repeat_interleave(2, -1)
        cos, sin = ang.cos().to(dt), ang.sin().to(dt)
        y = torch.randn((nq + 2 * nkv) * hd, generator=g).to(dt)
        qh = y[:nq * hd].view(nq, 1, hd)
        kh = y[nq * hd:(nq + nkv) * hd].view(nkv, 1, hd)
        out.update({f"{dname}_rope_y": bits(y), f"{dname}_rope_cos": bits(cos), f"{dname}_rope_sin": bits(sin),
                    f"{dname}_rope_q": bits(refe.rope(qh, cos[pos:pos + 1], sin[pos:pos + 1]).reshape(-1)),
                    f"{dname}_rope_k": bits(refe.rope(kh, cos[pos:pos + 1], sin[pos:pos + 1]).reshape(nkv, hd)),
                    f"{dname}_rope_meta": np.array([nq, nkv, hd, S, pos, theta])})
        inter = 256
        gt = (torch.randn(inter, generator=g) * 2).to(dt)
        up = torch.randn(inter, generator=g).to(dt)
        out.update({f"{dname}_sw_g": bits(gt), f"{dname}_sw_u": bits(up),
                    f"{dname}_sw_act": bits((F.silu(gt.float()) * up.float()).to(dt))})
    # layer-0 input: the reference's embed (int8 row x scale, rounded) then cohere_ln, bf16 and fp16 outputs
    import types
    g = torch.Generator().manual_seed(43)
    vocab, H = 37, 256
    emb_q = torch.randint(-127, 128, (vocab, H), generator=g, dtype=torch.int16).to(torch.int8)
    emb_s = torch.rand(vocab, generator=g) * 0.02 + 0.001
    ids = torch.tensor([5, 36, 0])
    for dname, dt in (("bf16", torch.bfloat16), ("f16", torch.float16)):
        w = (1 + 0.1 * torch.randn(H, generator=g)).to(dt)
        if dt == torch.bfloat16:   # the reference's own embed (engine/rumik_int4.py:134-135), bf16 by design
            e = refe.RumikInt4.embed(types.SimpleNamespace(emb_q=emb_q, emb_s=emb_s), ids)
        else:                      # the same product rounded to fp16
            e = (emb_q[ids].float() * emb_s[ids, None].float()).to(dt)
        out.update({f"{dname}_emb_w": bits(w), f"{dname}_emb_x": bits(e),
                    f"{dname}_emb_h": bits(torch.stack([refe.cohere_ln(r, w, 1e-5) for r in e]))})
    out.update({"emb_q": emb_q.numpy(), "emb_s": emb_s.numpy(), "emb_ids": ids.numpy()})
    # decode attention: 6 query heads on 2 key-value heads, 50 cache slots, position 33
    g = torch.Generator().manual_seed(42)
    nq, nkv, hd, S, pos = 6, 2, 128, 50, 33
    q = torch.randn(nq * hd, generator=g).to(torch.bfloat16)
    kc = torch.randn(nkv, S, hd, generator=g).to(torch.bfloat16)
    vc = torch.randn(nkv, S, hd, generator=g).to(torch.bfloat16)
    bias = torch.where(torch.arange(S) <= pos, 0.0, float("-inf"))
    o = refe.RumikInt4._attend(types.SimpleNamespace(hd=hd), q.view(nq, 1, hd), kc, vc, bias)[0]
    out.update({"attn_q": bits(q), "attn_k": bits(kc), "attn_v": bits(vc), "attn_o": bits(o),
                "attn_meta": np.array([nq, nkv, hd, S, pos])})
    # the sampling tail with the reference's eager _logits_and_stop / _pick (engine/rumik_int4.py:174-191) at the
    # real head size; torch.rand inside _pick is reproduced by re-seeding
    nv, hs, nz, top_k, temp, min_new = 16385, 256, 64, 30, 0.8, 8
    ids = (1000 + 3 * torch.arange(nv)).to(torch.int64)
    for case, (seed, step, b2) in enumerate(((50, 3, 5.0), (51, 20, -5.0), (52, 20, 5.0))):
        g = torch.Generator().manual_seed(seed)
        stop = {"0.weight": 1 + 0.1 * torch.randn(hs, generator=g), "0.bias": 0.1 * torch.randn(hs, generator=g),
                "1.weight": (0.05 * torch.randn(nz, hs, generator=g)).to(torch.bfloat16),
                "1.bias": 0.1 * torch.randn(nz, generator=g), "3.weight": 0.1 * torch.randn(1, nz, generator=g),
                "3.bias": torch.tensor([b2])}
        ns = types.SimpleNamespace(
            head_w=(0.05 * torch.randn(nv, hs, generator=g)).to(torch.bfloat16),
            hn=torch.randn(hs, generator=g).to(torch.bfloat16), stop=stop, H=hs, dev="cpu",
            step_i=torch.tensor(step), min_new=min_new, is_end=ids == ids[-1], top_k=top_k, temperature=temp,
            audio_ids=ids, end_id=int(ids[-1]))
        logits, st = refe.RumikInt4._logits_and_stop(ns)
        torch.manual_seed(1000 + case)
        nxt = refe.RumikInt4._pick(ns, logits, st)
        torch.manual_seed(1000 + case)
        u = torch.rand(top_k)
        out.update({f"smp{case}_logits": bits(logits.to(torch.bfloat16)), f"smp{case}_hn": bits(ns.hn),
                    f"smp{case}_lnw": stop["0.weight"].numpy(), f"smp{case}_lnb": stop["0.bias"].numpy(),
                    f"smp{case}_w1": bits(stop["1.weight"]), f"smp{case}_b1": stop["1.bias"].numpy(),
                    f"smp{case}_w2": stop["3.weight"].reshape(-1).numpy(), f"smp{case}_b2": stop["3.bias"].numpy(),
                    f"smp{case}_u": u.numpy(), f"smp{case}_stop": np.array(bool(st)),
                    f"smp{case}_meta": np.array([step, min_new, top_k, nv - 1, int(ids[-1])]),
                    f"smp{case}_next": np.array(int(nxt))})
    out["smp_ids"] = ids.numpy()
    np.savez_compressed(os.path.join(HERE, "golden_glue.npz"), **out)
    print("golden_glue.npz", os.path.getsize(os.path.join(HERE, "golden_glue.npz")), "bytes")


if __name__ == "__main__":
    main()
