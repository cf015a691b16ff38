"""Decode attention over the KV cache in one launch (rb_attn_decode).

Replaces rumik-fast's flash-decoding pair attn_split + attn_combine (engine/fused.py:120-200, launched at
engine/rumik_fused.py:88-94): out[h] = softmax(q[h] . K[h / rep, 0..pos] * scale) V[h / rep, 0..pos] for every
query head, with the position read on the device so that one CUDA graph serves every step.

    attn = DecodeAttention(q, k_cache, v_cache, pos, out, n_q_heads=24, n_kv_heads=8)   # built once
    attn()                                                                                 # every step
"""
import torch

from . import _lib, config
from .cuda_gemv import _on_device, _require


class DecodeAttention:
    """q [n_q_heads * 128], k_cache / v_cache [n_kv_heads, cache_len, 128], out [n_q_heads * 128] (one dtype,
    fp16 or bf16), pos an int64 [1] device tensor. Owns its workspace (per-head completion counters + fp32
    partials); calls sharing one object must be issued on one stream. merge: "auto" (a thread-block cluster
    per key-value head merging through distributed shared memory where the device can schedule it) or
    "ticket" (fp32 partials in the workspace and a per-head ticket)."""

    def __init__(self, q, k_cache, v_cache, pos, out, n_q_heads, n_kv_heads, scale=None, merge="auto"):
        _require(merge in ("auto", "ticket"), f"merge must be 'auto' or 'ticket', got {merge!r}")
        self.extra_flags = _lib.FLAG_ATTN_TICKET if merge == "ticket" else 0
        dt = q.dtype
        _require(dt in (torch.float16, torch.bfloat16), "q must be fp16 or bf16")
        nkv, S, hd = k_cache.shape
        _require(nkv == n_kv_heads and tuple(v_cache.shape) == (nkv, S, hd), "caches must be [n_kv_heads, S, 128]")
        for t, nm in ((q, "q"), (k_cache, "k_cache"), (v_cache, "v_cache"), (out, "out")):
            _require(t.is_cuda and t.device == q.device and t.dtype == dt and t.is_contiguous(),
                     f"{nm} must be a contiguous {dt} CUDA tensor on {q.device}")
        _require(q.numel() == n_q_heads * hd and out.numel() == n_q_heads * hd, "q/out must be [n_q_heads * 128]")
        _require(pos.dtype == torch.int64 and pos.device == q.device, "pos must be an int64 tensor on the device")
        need = _lib.lib().rb_attn_decode_workspace(n_q_heads, n_kv_heads, hd)
        _require(need > 0, f"unsupported heads {n_q_heads}/{n_kv_heads} x {hd} (head_dim 128, rep 1..8)")
        self.ws = torch.zeros(need, dtype=torch.uint8, device=q.device)
        self.args = (q, k_cache, v_cache, pos, out)
        self.nq, self.nkv, self.hd, self.S = n_q_heads, n_kv_heads, hd, S
        self.scale = float(hd ** -0.5 if scale is None else scale)
        self.dtype, self.device = dt, q.device

    def __call__(self):
        q, k, v, pos, out = self.args
        with _on_device(self.device):
            st = _lib.lib().rb_attn_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), pos.data_ptr(), out.data_ptr(),
                                           self.nq, self.nkv, self.hd, self.S, self.scale, self.ws.data_ptr(),
                                           self.ws.numel(), _lib.dtype_code(self.dtype),
                                           config.flags() | self.extra_flags,
                                           _lib.stream_ptr(self.device))
        _lib.check("rb_attn_decode", st)

    def bytes_read(self, pos):
        """Algorithmic bytes of one call at position pos: K and V of slots 0..pos, q, out."""
        return 2 * self.nkv * (pos + 1) * self.hd * 2 + 2 * self.nq * self.hd * 2
