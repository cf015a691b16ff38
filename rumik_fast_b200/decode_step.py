"""A decode step's transformer layers as ONE persistent launch (rb_decode_layers).

rumik-fast's decode step launches, per layer, the input GEMV, the post kernel, the attention and the output
GEMVs (engine/rumik_fused.py:97-121); fused.AddLnGemvPost / attention.DecodeAttention / Int4GemvSet bring that
to three launches per layer. DecodeLayers runs all the layers of the step in one cooperative launch of one CTA
per SM, whose weight stream never stops at a layer or phase boundary (rumik_fast_b200/csrc/decode_step.cu):

    layers = [dict(qkv=(q, s, m), gate_up=interleave_gate_up(q, s, m), o_proj=(q, s, m), down=(q, s, m),
                   ln_w=w, k_cache=kc, v_cache=vc, rope=True), ...]
    step = DecodeLayers(layers, pos=pos, cos=cos, sin=sin, emb_q=emb_q, emb_s=emb_s, tok=tok, n_q_heads=24,
                        n_kv_heads=8, eps=1e-5)
    step()                       # every layer; then add_layernorm(step.final_add_ln(w, h_out)) and the head

The buffers the layers pass on (residual, queries, attention output, MLP activation, o_proj and down_proj
outputs) are held here, two copies each (a layer writes copy l & 1). Built once; graph-capture safe to call;
every tensor must stay alive. Layers beyond 36 run as further launches of the same kernel.
"""
import ctypes

import torch

from . import _lib, config
from .cuda_gemv import _on_device, _require

G = 128
MAX_LAYERS_PER_LAUNCH = 36
_c = ctypes
_vp, _i64, _int = _c.c_void_p, _c.c_int64, _c.c_int


class DecodeLayer(ctypes.Structure):
    """struct rb_decode_layer (include/rumik_b200.h)."""
    _fields_ = [("qkv", _lib.GemvDesc), ("gate_up", _lib.GemvDesc), ("o_proj", _lib.GemvDesc), ("down", _lib.GemvDesc),
                ("ln_w", _vp), ("k_cache", _vp), ("v_cache", _vp), ("rope", _int)]


class DecodeStepC(ctypes.Structure):
    """struct rb_decode_step (include/rumik_b200.h)."""
    _fields_ = [("layers", _c.POINTER(DecodeLayer)), ("n_layers", _int), ("first_layer", _int), ("H", _i64),
                ("I", _i64), ("n_q_heads", _int), ("n_kv_heads", _int), ("head_dim", _int), ("cache_len", _i64),
                ("eps", _c.c_float), ("attn_scale", _c.c_float), ("pos", _vp), ("cos", _vp), ("sin", _vp),
                ("emb_q", _vp), ("emb_s", _vp), ("emb_s_dtype", _int), ("tok", _vp), ("vocab", _i64),
                ("resid", _vp * 2), ("q_out", _vp * 2), ("attn_out", _vp * 2), ("act", _vp * 2), ("o_out", _vp * 2),
                ("down_out", _vp * 2), ("ws", _vp), ("ws_bytes", _i64)]


def _desc(w, N, K, name):
    q, s, m = w
    _require(q.dtype == torch.uint8 and q.is_contiguous() and tuple(q.shape) == (N, K // 2),
             f"{name}: q must be a contiguous uint8 [{N}, {K // 2}] tensor")
    for t, nm in ((s, "s"), (m, "m")):
        _require(isinstance(t, torch.Tensor) and t.dtype == torch.float16 and t.is_contiguous()
                 and tuple(t.shape) == (N, K // G), f"{name}: {nm} must be a contiguous fp16 [{N}, {K // G}] tensor")
    return _lib.GemvDesc(None, None, q.data_ptr(), s.data_ptr(), m.data_ptr(), N, K)


class DecodeLayers:
    """layers: dicts with qkv, gate_up (interleave_gate_up order), o_proj, down as (q, s, m), ln_w [H], k_cache and
    v_cache [n_kv_heads, cache_len, head_dim], rope (bool). pos, tok: int64 [1] device tensors. emb_q int8
    [vocab, H] and emb_s [vocab] (fp32 or fp16): layer 0's input is the token's embedding row."""

    def __init__(self, layers, *, pos, cos, sin, emb_q, emb_s, tok, n_q_heads, n_kv_heads, eps=1e-5, scale=None):
        _require(len(layers) >= 1, "no layers")
        L0 = layers[0]
        self.dtype = L0["ln_w"].dtype
        _require(self.dtype in (torch.float16, torch.bfloat16), "activations must be fp16 or bf16")
        self.device = L0["ln_w"].device
        H = L0["ln_w"].numel()
        I = L0["down"][0].shape[1] * 2
        nkv, S, hd = L0["k_cache"].shape
        _require(nkv == n_kv_heads, "caches must be [n_kv_heads, cache_len, head_dim]")
        _require(emb_s.dtype in (torch.float32, torch.float16), "emb_s must be fp32 or fp16")
        dt, dev = self.dtype, self.device
        QD = n_q_heads * hd

        def pair(n):
            return [torch.zeros(n, device=dev, dtype=dt) for _ in range(2)]
        self.resid, self.q_out, self.attn_out = pair(H), pair(QD), pair(QD)
        self.act, self.o_out, self.down_out = pair(I), pair(H), pair(H)
        self._keep = [pos, cos, sin, emb_q, emb_s, tok, layers]
        scale = float(hd ** -0.5 if scale is None else scale)
        self.n_layers = len(layers)
        self._calls = []
        for first in range(0, len(layers), MAX_LAYERS_PER_LAUNCH):
            chunk = layers[first:first + MAX_LAYERS_PER_LAUNCH]
            arr = (DecodeLayer * len(chunk))()
            for i, Ly in enumerate(chunk):
                for t, nm in ((Ly["ln_w"], "ln_w"), (Ly["k_cache"], "k_cache"), (Ly["v_cache"], "v_cache")):
                    _require(t.dtype == dt and t.is_contiguous() and t.device == dev, f"layer {first + i}: {nm}")
                arr[i] = DecodeLayer(_desc(Ly["qkv"], (n_q_heads + 2 * n_kv_heads) * hd, H, "qkv"),
                                     _desc(Ly["gate_up"], 2 * I, H, "gate_up"), _desc(Ly["o_proj"], H, QD, "o_proj"),
                                     _desc(Ly["down"], H, I, "down"), Ly["ln_w"].data_ptr(),
                                     Ly["k_cache"].data_ptr(), Ly["v_cache"].data_ptr(), int(bool(Ly["rope"])))
            c = DecodeStepC()
            c.layers = arr
            c.n_layers = len(chunk)
            c.first_layer = first
            c.H, c.I, c.n_q_heads, c.n_kv_heads, c.head_dim, c.cache_len = H, I, n_q_heads, n_kv_heads, hd, S
            c.eps, c.attn_scale = float(eps), scale
            c.pos, c.cos, c.sin = pos.data_ptr(), cos.data_ptr(), sin.data_ptr()
            c.emb_q, c.emb_s, c.tok, c.vocab = emb_q.data_ptr(), emb_s.data_ptr(), tok.data_ptr(), emb_q.shape[0]
            c.emb_s_dtype = _lib.dtype_code(emb_s.dtype)
            for nm in ("resid", "q_out", "attn_out", "act", "o_out", "down_out"):
                bufs = getattr(self, nm)
                getattr(c, nm)[0], getattr(c, nm)[1] = bufs[0].data_ptr(), bufs[1].data_ptr()
            with _on_device(dev):
                need = _lib.lib().rb_decode_layers_workspace(ctypes.byref(c))
            if need < 0:
                _lib.check("rb_decode_layers_workspace", -need)
            ws = torch.zeros(need, dtype=torch.uint8, device=dev)
            c.ws, c.ws_bytes = ws.data_ptr(), need
            self._calls.append((c, arr, ws))
        self.ws = self._calls[0][2]

    def __call__(self):
        L = _lib.lib()
        with _on_device(self.device):
            for c, _, _ in self._calls:
                st = L.rb_decode_layers(ctypes.byref(c), _lib.dtype_code(self.dtype), config.flags(),
                                        _lib.stream_ptr(self.device))
                _lib.check("rb_decode_layers", st)

    def last(self):
        """(residual, o_proj output, down_proj output) of the last layer: the final add + LayerNorm's inputs."""
        p = (self.n_layers - 1) & 1
        return self.resid[p], self.o_out[p], self.down_out[p]
